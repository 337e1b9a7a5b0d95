"""Torch-tensor front end of the C-ABI kernels.

Each function validates shapes on the host, passes raw device pointers and the
current CUDA stream to libmlxz_b200.so, and returns without synchronising.
Kernels report out-of-range block ids, slots and context lengths through a
per-device int32 error word instead of trapping; ``check_device_errors`` reads
and clears it (``MLXZ_B200_DEBUG=1`` makes every call check it).
"""
from __future__ import annotations

import ctypes
import math
import os
from collections import OrderedDict

import torch

from . import _native as nat

_DTYPES = {torch.float16: nat.MZ_DTYPE_F16, torch.bfloat16: nat.MZ_DTYPE_BF16,
           torch.float32: nat.MZ_DTYPE_F32}
_DEBUG = os.environ.get("MLXZ_B200_DEBUG", "0") not in ("", "0")

_err_words: dict[int, torch.Tensor] = {}
# Decode workspaces handed out when the caller passes none, one per exact
# problem layout.  The kernels need the arrival counters and scheduler words at
# the front of a workspace to be zero at launch (each launch leaves them zero),
# and where those words sit depends on the problem sizes: a workspace last used
# with other sizes may hold partials there.  So a workspace is never shared
# between layouts.  A few layouts are kept, least recently used dropped first.
_WS_KEEP = 16
_workspaces: "OrderedDict[tuple, torch.Tensor]" = OrderedDict()
_qworkspaces: "OrderedDict[tuple, torch.Tensor]" = OrderedDict()


def _layout_workspace(cache, key: tuple, need: int, device: int, shared: bool) -> torch.Tensor:
    if not shared:
        return torch.zeros(max(need, 256), dtype=torch.uint8, device=f"cuda:{device}")
    ws = cache.get(key)
    if ws is None:
        ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=f"cuda:{device}")
        cache[key] = ws
        while len(cache) > _WS_KEEP:
            cache.popitem(last=False)
    else:
        cache.move_to_end(key)
    return ws


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPES[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}") from None


def _dev_index(t: torch.Tensor) -> int:
    if t.device.type != "cuda":
        raise ValueError(f"expected a CUDA tensor, got one on {t.device}")
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def _stream(device: int) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def error_word(device: int) -> torch.Tensor:
    """The int32 device error word kernels on `device` report into."""
    w = _err_words.get(device)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=f"cuda:{device}")
        _err_words[device] = w
    return w


def check_device_errors(device: int | None = None, clear: bool = True) -> int:
    """Synchronise with `device`'s error word; raise DeviceError if a bit is set."""
    device = torch.cuda.current_device() if device is None else device
    w = _err_words.get(device)
    if w is None:
        return 0
    bits = int(w.item())
    if bits and clear:
        w.zero_()
    if bits:
        raise nat.DeviceError(bits)
    return 0


def _after(device: int) -> None:
    if _DEBUG:
        check_device_errors(device)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _check_pools(k_pool: torch.Tensor, v_pool: torch.Tensor) -> tuple[int, int, int, int]:
    if k_pool.shape != v_pool.shape or k_pool.dtype != v_pool.dtype:
        raise ValueError("k_pool and v_pool must have the same shape and dtype")
    if k_pool.dim() != 4 or not k_pool.is_contiguous() or not v_pool.is_contiguous():
        raise ValueError("pools must be contiguous [n_blocks, n_kv_heads, block_size, head_dim]")
    if k_pool.device != v_pool.device:
        raise ValueError("pools must be on the same device")
    n, h, bs, d = k_pool.shape
    return n, h, bs, d


def _as_i32(t: torch.Tensor, device: torch.device, name: str) -> torch.Tensor:
    if t.dtype != torch.int32 or t.device != device or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous int32 tensor on {device}")
    return t


# ---------------------------------------------------------------------------
# Append / gather
# ---------------------------------------------------------------------------

def kv_append(k_pool: torch.Tensor, v_pool: torch.Tensor, keys: torch.Tensor,
              values: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """Write keys/values ``(1, H, n, D)`` (or ``(H, n, D)``) to pool slots.

    slot_mapping: int64 ``[n]`` on the pools' device; a negative slot skips.
    """
    n_blocks, H, bs, D = _check_pools(k_pool, v_pool)
    if keys.shape != values.shape or keys.dtype != k_pool.dtype or values.dtype != k_pool.dtype:
        raise ValueError("keys/values must match each other and the pool dtype")
    kk, vv = keys, values
    if kk.dim() == 4:
        if kk.shape[0] != 1:
            raise ValueError("keys must have batch size 1: (1, H, n, D)")
        kk, vv = kk[0], vv[0]
    if kk.dim() != 3 or kk.shape[0] != H or kk.shape[2] != D:
        raise ValueError(f"keys must be (1, {H}, n, {D}), got {tuple(keys.shape)}")
    if kk.stride(2) != 1 or vv.stride(2) != 1 or kk.stride() != vv.stride():
        kk, vv = kk.contiguous(), vv.contiguous()
    n = kk.shape[1]
    if slot_mapping.dtype != torch.int64 or slot_mapping.numel() != n or \
            slot_mapping.device != k_pool.device:
        raise ValueError("slot_mapping must be int64 [n] on the pool device")
    if n == 0:
        return
    dev = _dev_index(k_pool)
    nat.call("mz_kv_append", k_pool.data_ptr(), v_pool.data_ptr(), kk.data_ptr(), vv.data_ptr(),
             kk.stride(1), kk.stride(0), slot_mapping.data_ptr(), n, H, D, bs, n_blocks,
             dtype_code(k_pool.dtype), error_word(dev).data_ptr(), _stream(dev))
    _after(dev)


def kv_append_paged(k_pool: torch.Tensor, v_pool: torch.Tensor, keys: torch.Tensor,
                    values: torch.Tensor, block_tables: torch.Tensor,
                    positions: torch.Tensor) -> None:
    """Decode-step append: keys/values ``[B, H, D]`` (or ``[B, H, 1, D]``), one
    token per sequence at ``positions[b]`` through ``block_tables[b]``."""
    n_blocks, H, bs, D = _check_pools(k_pool, v_pool)
    kk, vv = keys, values
    if kk.dim() == 4:
        kk, vv = kk[:, :, 0, :], vv[:, :, 0, :]
    if kk.dim() != 3 or kk.shape[1:] != (H, D) or kk.shape != vv.shape:
        raise ValueError(f"keys must be [B, {H}, D={D}], got {tuple(keys.shape)}")
    if kk.dtype != k_pool.dtype or vv.dtype != k_pool.dtype:
        raise ValueError("keys/values dtype must match the pool")
    if kk.stride(2) != 1 or vv.stride(2) != 1 or kk.stride() != vv.stride():
        kk, vv = kk.contiguous(), vv.contiguous()
    B = kk.shape[0]
    _as_i32(block_tables, k_pool.device, "block_tables")
    _as_i32(positions, k_pool.device, "positions")
    if block_tables.dim() != 2 or block_tables.shape[0] < B or positions.numel() < B:
        raise ValueError("block_tables must be [>=B, max_blocks] and positions [>=B]")
    if B == 0:
        return
    dev = _dev_index(k_pool)
    nat.call("mz_kv_append_paged", k_pool.data_ptr(), v_pool.data_ptr(), kk.data_ptr(),
             vv.data_ptr(), kk.stride(0), kk.stride(1), block_tables.data_ptr(),
             block_tables.shape[1], positions.data_ptr(), B, H, D, bs, n_blocks,
             dtype_code(k_pool.dtype), error_word(dev).data_ptr(), _stream(dev))
    _after(dev)


def kv_gather(k_pool: torch.Tensor, v_pool: torch.Tensor, block_tables: torch.Tensor,
              ctx_lens: torch.Tensor, ctx_lens_host: list[int]) -> tuple[torch.Tensor, torch.Tensor]:
    """Gather each sequence's KV into contiguous ``[H, ctx_b, D]`` pieces.

    Returns (K, V) as flat tensors ``[sum_b H*ctx_b*D]`` viewed per sequence by
    the caller; with one sequence they are shaped ``(1, H, T, D)``.
    """
    n_blocks, H, bs, D = _check_pools(k_pool, v_pool)
    _as_i32(block_tables, k_pool.device, "block_tables")
    _as_i32(ctx_lens, k_pool.device, "ctx_lens")
    B = len(ctx_lens_host)
    offs = [0] * B
    tot = 0
    for i, c in enumerate(ctx_lens_host):
        offs[i] = tot
        tot += c
    out_k = torch.empty(tot * H * D, dtype=k_pool.dtype, device=k_pool.device)
    out_v = torch.empty_like(out_k)
    if B == 1:
        out_k = out_k.view(1, H, tot, D)
        out_v = out_v.view(1, H, tot, D)
    if B == 0 or tot == 0:
        return out_k, out_v
    off_t = torch.tensor(offs, dtype=torch.int64).to(k_pool.device, non_blocking=True)
    dev = _dev_index(k_pool)
    nat.call("mz_kv_gather", out_k.data_ptr(), out_v.data_ptr(), k_pool.data_ptr(),
             v_pool.data_ptr(), block_tables.data_ptr(), block_tables.shape[1],
             ctx_lens.data_ptr(), off_t.data_ptr(), B, max(ctx_lens_host), H, D, bs, n_blocks,
             dtype_code(k_pool.dtype), error_word(dev).data_ptr(), _stream(dev))
    _after(dev)
    return out_k, out_v


# ---------------------------------------------------------------------------
# Decode attention
# ---------------------------------------------------------------------------

def decode_workspace(n_seqs: int, n_kv_heads: int, rows: int, head_dim: int, device: int,
                     num_warps: int = 0, shared: bool = True, batch_invariant: bool = False,
                     max_blocks: int = 0, block_size: int = 16) -> torch.Tensor:
    """A zero-initialised decode workspace for exactly these sizes: the one
    kept for this layout (``shared``), or a new one the caller owns.  A
    batch-invariant launch needs room for the pieces of tables ``max_blocks``
    wide (of ``block_size``-token blocks)."""
    size = ctypes.c_size_t(0)
    if batch_invariant:
        if max_blocks <= 0:
            raise ValueError("a batch-invariant workspace needs max_blocks")
        nat.call("mz_paged_decode_workspace_size_ex", n_seqs, n_kv_heads, rows, head_dim,
                 num_warps, max_blocks, block_size, nat.MZ_DECODE_BATCH_INVARIANT, device,
                 ctypes.byref(size))
    else:
        nat.call("mz_paged_decode_workspace_size", n_seqs, n_kv_heads, rows, head_dim,
                 num_warps, device, ctypes.byref(size))
    key = (device, n_seqs, n_kv_heads, rows, head_dim, num_warps,
           (max_blocks, block_size) if batch_invariant else None)
    return _layout_workspace(_workspaces, key, int(size.value), device, shared)


def reset_workspaces() -> None:
    """Zero every cached workspace (needed after a call that reported an error)."""
    for ws in list(_workspaces.values()) + list(_qworkspaces.values()):
        ws.zero_()


def paged_decode(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                 block_tables: torch.Tensor, ctx_lens: torch.Tensor, scale: float | None = None,
                 out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
                 num_warps: int = 0, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Fused GQA paged decode attention.

    q: ``[B, Hq, D]`` (one query token per sequence) or ``[B, n_q, Hq, D]``.
    Returns ``out`` with q's shape, dtype ``out_dtype`` (default q.dtype).
    """
    n_blocks, Hkv, bs, D = _check_pools(k_pool, v_pool)
    if q.dtype != k_pool.dtype:
        raise ValueError("q dtype must match the pools")
    if q.dim() == 3:
        B, Hq, Dq = q.shape
        nq = 1
        q_sb, q_st, q_sh = q.stride(0), 0, q.stride(1)
    elif q.dim() == 4:
        B, nq, Hq, Dq = q.shape
        q_sb, q_st, q_sh = q.stride(0), q.stride(1), q.stride(2)
    else:
        raise ValueError("q must be [B, Hq, D] or [B, n_q, Hq, D]")
    if Dq != D or q.stride(-1) != 1:
        raise ValueError(f"q head_dim must be {D} with unit stride")
    if Hq % Hkv:
        raise ValueError(f"n_heads {Hq} is not a multiple of n_kv_heads {Hkv}")
    _as_i32(block_tables, k_pool.device, "block_tables")
    _as_i32(ctx_lens, k_pool.device, "ctx_lens")
    if block_tables.dim() != 2 or block_tables.shape[0] < B or ctx_lens.numel() < B:
        raise ValueError("block_tables must be [>=B, max_blocks] and ctx_lens [>=B]")
    out_dtype = out_dtype or q.dtype
    if out is None:
        out = torch.empty(q.shape, dtype=out_dtype, device=q.device)
    if out.shape != q.shape or out.dtype != out_dtype or out.stride(-1) != 1:
        raise ValueError("out must match q's shape with unit last stride")
    if q.dim() == 3:
        o_sb, o_st, o_sh = out.stride(0), 0, out.stride(1)
    else:
        o_sb, o_st, o_sh = out.stride(0), out.stride(1), out.stride(2)
    if scale is None:
        scale = D ** -0.5
    if B == 0:
        return out
    dev = _dev_index(q)
    rows = nq * (Hq // Hkv)
    if workspace is None:
        workspace = decode_workspace(B, Hkv, rows, D, dev, num_warps)
    nat.call("mz_paged_decode", out.data_ptr(), dtype_code(out_dtype), o_sb, o_st, o_sh,
             q.data_ptr(), q_sb, q_st, q_sh, nq, k_pool.data_ptr(), v_pool.data_ptr(),
             block_tables.data_ptr(), block_tables.shape[1], ctx_lens.data_ptr(), B, Hq, Hkv,
             D, bs, n_blocks, float(scale), dtype_code(q.dtype), num_warps,
             workspace.data_ptr(), workspace.numel(), error_word(dev).data_ptr(), _stream(dev))
    _after(dev)
    return out


def paged_append_decode(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                        k_new: torch.Tensor, v_new: torch.Tensor, block_tables: torch.Tensor,
                        ctx_lens: torch.Tensor, scale: float | None = None,
                        out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
                        num_warps: int = 0, workspace: torch.Tensor | None = None,
                        overlap_previous: bool = False,
                        batch_invariant: bool = False) -> torch.Tensor:
    """Fused decode step for one layer: write ``k_new/v_new [B, Hkv, D]`` at
    position ``ctx_lens[b] - 1`` of each sequence, then attend ``q [B, Hq, D]``
    over the first ``ctx_lens[b]`` tokens (one launch).  ``overlap_previous``:
    the launch may start while the kernel ahead of it on the stream runs
    (MZ_LAUNCH_OVERLAP_PREVIOUS) -- only when that kernel writes none of the
    pools, ``block_tables`` or ``ctx_lens``.  ``batch_invariant``: each
    sequence's output bytes are independent of the rest of the batch
    (MZ_DECODE_BATCH_INVARIANT)."""
    n_blocks, Hkv, bs, D = _check_pools(k_pool, v_pool)
    if q.dim() != 3 or q.shape[2] != D or q.stride(-1) != 1 or q.dtype != k_pool.dtype:
        raise ValueError(f"q must be [B, Hq, {D}] of the pool dtype with unit last stride")
    B, Hq, _ = q.shape
    if k_new.shape != (B, Hkv, D) or v_new.shape != (B, Hkv, D):
        raise ValueError(f"k_new/v_new must be [{B}, {Hkv}, {D}]")
    if k_new.dtype != k_pool.dtype or v_new.dtype != k_pool.dtype:
        raise ValueError("k_new/v_new dtype must match the pools")
    if k_new.stride() != v_new.stride() or k_new.stride(2) != 1:
        k_new, v_new = k_new.contiguous(), v_new.contiguous()
    _as_i32(block_tables, k_pool.device, "block_tables")
    _as_i32(ctx_lens, k_pool.device, "ctx_lens")
    out_dtype = out_dtype or q.dtype
    if out is None:
        out = torch.empty(q.shape, dtype=out_dtype, device=q.device)
    if out.shape != q.shape or out.dtype != out_dtype or out.stride(-1) != 1:
        raise ValueError("out must match q's shape with unit last stride")
    if scale is None:
        scale = D ** -0.5
    if B == 0:
        return out
    dev = _dev_index(q)
    if workspace is None:
        workspace = decode_workspace(B, Hkv, Hq // Hkv, D, dev, num_warps,
                                     batch_invariant=batch_invariant,
                                     max_blocks=block_tables.shape[1], block_size=bs)
    nat.call("mz_paged_append_decode_ex", out.data_ptr(), dtype_code(out_dtype), out.stride(0),
             out.stride(1), q.data_ptr(), q.stride(0), q.stride(1), k_pool.data_ptr(),
             v_pool.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0),
             k_new.stride(1), block_tables.data_ptr(), block_tables.shape[1],
             ctx_lens.data_ptr(), B, Hq, Hkv, D, bs, n_blocks, float(scale),
             dtype_code(q.dtype), num_warps,
             (nat.MZ_LAUNCH_OVERLAP_PREVIOUS if overlap_previous else 0)
             | (nat.MZ_DECODE_BATCH_INVARIANT if batch_invariant else 0),
             workspace.data_ptr(), workspace.numel(), error_word(dev).data_ptr(), _stream(dev))
    _after(dev)
    return out


def paged_prefill(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                  block_tables: torch.Tensor, q_start: torch.Tensor, q_len: torch.Tensor,
                  ctx_lens: torch.Tensor, max_q_len: int, scale: float | None = None,
                  out: torch.Tensor | None = None,
                  out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Chunked prefill attention (mz_paged_prefill): ``q [T, Hq, D]`` holds
    sequence b's ``q_len[b]`` query tokens at rows ``q_start[b]...``; they sit
    at the last ``q_len[b]`` of the sequence's ``ctx_lens[b]`` positions (their
    K/V already appended) and attend causally."""
    n_blocks, Hkv, bs, D = _check_pools(k_pool, v_pool)
    if q.dim() != 3 or q.shape[2] != D or q.stride(-1) != 1 or q.dtype != k_pool.dtype:
        raise ValueError(f"q must be [T, Hq, {D}] of the pool dtype with unit last stride")
    T, Hq, _ = q.shape
    B = block_tables.shape[0]
    for t, name in ((q_start, "q_start"), (q_len, "q_len"), (ctx_lens, "ctx_lens")):
        _as_i32(t, k_pool.device, name)
        if t.numel() != B:
            raise ValueError(f"{name} must hold one entry per sequence ({B})")
    _as_i32(block_tables, k_pool.device, "block_tables")
    out_dtype = out_dtype or q.dtype
    if out is None:
        out = torch.empty(q.shape, dtype=out_dtype, device=q.device)
    if out.shape != q.shape or out.dtype != out_dtype or out.stride(-1) != 1:
        raise ValueError("out must match q's shape with unit last stride")
    if scale is None:
        scale = D ** -0.5
    if B == 0 or T == 0 or max_q_len == 0:
        return out
    dev = _dev_index(q)
    nat.call("mz_paged_prefill", out.data_ptr(), dtype_code(out_dtype), out.stride(0),
             out.stride(1), q.data_ptr(), q.stride(0), q.stride(1), T, q_start.data_ptr(),
             q_len.data_ptr(), int(max_q_len), k_pool.data_ptr(), v_pool.data_ptr(),
             block_tables.data_ptr(), block_tables.shape[1], ctx_lens.data_ptr(), B, Hq, Hkv,
             D, bs, n_blocks, float(scale), dtype_code(q.dtype), error_word(dev).data_ptr(),
             _stream(dev))
    _after(dev)
    return out


def paged_append_decode_allgather(peers: "nat.PeerOutputs", q: torch.Tensor,
                                  k_pool: torch.Tensor, v_pool: torch.Tensor,
                                  k_new: torch.Tensor, v_new: torch.Tensor,
                                  block_tables: torch.Tensor, ctx_lens: torch.Tensor,
                                  out_seq_stride: int, out_head_stride: int,
                                  out_dtype: torch.dtype, scale: float | None = None,
                                  num_warps: int = 0,
                                  workspace: torch.Tensor | None = None,
                                  overlap_previous: bool = False,
                                  wait_previous: bool = False) -> None:
    """paged_append_decode whose output rows go to every rank's gathered
    buffer (``peers.out[r]``: this rank's head block there) and whose last
    warp signals the peers (mz_paged_append_decode_allgather); follow it with
    ``peer_wait``, or with a next launch made with ``wait_previous``, before
    reading the gathered buffer.  ``wait_previous`` (MZ_LAUNCH_WAIT_PREVIOUS):
    the launch first waits, on the device and bounded, for the peers' rows of
    this rank's previous launch."""
    n_blocks, Hkv, bs, D = _check_pools(k_pool, v_pool)
    if q.dim() != 3 or q.shape[2] != D or q.stride(-1) != 1 or q.dtype != k_pool.dtype:
        raise ValueError(f"q must be [B, Hq, {D}] of the pool dtype with unit last stride")
    B, Hq, _ = q.shape
    if B == 0:
        raise ValueError("an all-gather launch needs at least one sequence")
    if k_new.shape != (B, Hkv, D) or v_new.shape != (B, Hkv, D):
        raise ValueError(f"k_new/v_new must be [{B}, {Hkv}, {D}]")
    if k_new.dtype != k_pool.dtype or v_new.dtype != k_pool.dtype:
        raise ValueError("k_new/v_new dtype must match the pools")
    if k_new.stride() != v_new.stride() or k_new.stride(2) != 1:
        k_new, v_new = k_new.contiguous(), v_new.contiguous()
    _as_i32(block_tables, k_pool.device, "block_tables")
    _as_i32(ctx_lens, k_pool.device, "ctx_lens")
    if scale is None:
        scale = D ** -0.5
    dev = _dev_index(q)
    if workspace is None:
        workspace = decode_workspace(B, Hkv, Hq // Hkv, D, dev, num_warps)
    nat.call("mz_paged_append_decode_allgather", ctypes.byref(peers), dtype_code(out_dtype),
             out_seq_stride, out_head_stride, q.data_ptr(), q.stride(0), q.stride(1),
             k_pool.data_ptr(), v_pool.data_ptr(), k_new.data_ptr(), v_new.data_ptr(),
             k_new.stride(0), k_new.stride(1), block_tables.data_ptr(), block_tables.shape[1],
             ctx_lens.data_ptr(), B, Hq, Hkv, D, bs, n_blocks, float(scale),
             dtype_code(q.dtype), num_warps,
             (nat.MZ_LAUNCH_OVERLAP_PREVIOUS if overlap_previous else 0)
             | (nat.MZ_LAUNCH_WAIT_PREVIOUS if wait_previous else 0),
             workspace.data_ptr(), workspace.numel(), error_word(dev).data_ptr(), _stream(dev))
    _after(dev)


def peer_wait(signal: torch.Tensor, n_ranks: int, rank: int, epoch: int,
              timeout_s: float = 2.0) -> None:
    """Enqueue the bounded wait for every peer's signal word to reach
    ``epoch`` (mz_peer_wait); a timeout shows up as a device error."""
    if signal.dtype != torch.int32 or signal.numel() < n_ranks or not signal.is_cuda:
        raise ValueError(f"signal must be a CUDA int32 tensor of at least {n_ranks} words")
    dev = _dev_index(signal)
    nat.call("mz_peer_wait", signal.data_ptr(), n_ranks, rank, epoch & 0xFFFFFFFF,
             int(timeout_s * 1e9), error_word(dev).data_ptr(), _stream(dev))
    _after(dev)


def ipc_export(t: torch.Tensor) -> tuple[bytes, int]:
    """(handle, byte offset) of the device allocation holding ``t``'s data."""
    h = ctypes.create_string_buffer(nat.MZ_IPC_HANDLE_BYTES)
    off = ctypes.c_uint64()
    nat.call("mz_ipc_export", t.data_ptr(), h, ctypes.byref(off))
    return h.raw, int(off.value)


def ipc_open(handle: bytes, offset: int) -> tuple[int, int]:
    """Map a peer's exported allocation on the current device: (base, ptr)."""
    if len(handle) != nat.MZ_IPC_HANDLE_BYTES:
        raise ValueError("bad IPC handle length")
    base, ptr = ctypes.c_void_p(), ctypes.c_void_p()
    nat.call("mz_ipc_open", handle, offset, ctypes.byref(base), ctypes.byref(ptr))
    return int(base.value), int(ptr.value)


def ipc_close(base: int) -> None:
    nat.call("mz_ipc_close", base)


# ---------------------------------------------------------------------------
# Quantised KV
# ---------------------------------------------------------------------------

def _check_qpools(pools) -> tuple[int, int, int, int, int]:
    """(n_blocks, H, bs, D, bits) of a 6-tuple (k_codes, k_scales, k_biases,
    v_codes, v_scales, v_biases): codes int32 [N, H, bs, D*bits/32], scales and
    biases fp16 [N, H, bs, D/64]."""
    if len(pools) != 6:
        raise ValueError("quantised pools: (k_codes, k_scales, k_biases, v_codes, v_scales, v_biases)")
    kc, ks, kb, vc, vs, vb = pools
    for t in pools:
        if not t.is_contiguous() or t.device != kc.device or t.dim() != 4:
            raise ValueError("quantised pools must be contiguous 4-D tensors on one device")
    if kc.dtype != torch.int32 or vc.dtype != torch.int32 or kc.shape != vc.shape:
        raise ValueError("codes must be int32 [N, H, bs, words] (same for K and V)")
    for t in (ks, kb, vs, vb):
        if t.dtype != torch.float16 or t.shape != ks.shape:
            raise ValueError("scales/biases must be fp16 [N, H, bs, D/64]")
    n, h, bs, words = kc.shape
    D = ks.shape[3] * 64
    bits = words * 32 // D
    if bits not in (4, 8) or ks.shape[:3] != kc.shape[:3]:
        raise ValueError("codes/scales shapes do not describe 4- or 8-bit groups of 64")
    return n, h, bs, D, bits


def _qptrs(pools):
    return [t.data_ptr() for t in pools]


def kv_quant_append(pools, keys: torch.Tensor, values: torch.Tensor,
                    slot_mapping: torch.Tensor) -> None:
    """Quantise keys/values ``(1, H, n, D)`` (or ``(H, n, D)``) into pool slots."""
    n_blocks, H, bs, D, bits = _check_qpools(pools)
    kk, vv = (keys[0], values[0]) if keys.dim() == 4 else (keys, values)
    if kk.shape != vv.shape or kk.dim() != 3 or kk.shape[0] != H or kk.shape[2] != D:
        raise ValueError(f"keys must be (1, {H}, n, {D})")
    if kk.stride(2) != 1 or vv.stride(2) != 1 or kk.stride() != vv.stride():
        kk, vv = kk.contiguous(), vv.contiguous()
    n = kk.shape[1]
    if slot_mapping.dtype != torch.int64 or slot_mapping.numel() != n:
        raise ValueError("slot_mapping must be int64 [n]")
    if n == 0:
        return
    dev = _dev_index(pools[0])
    nat.call("mz_kv_quant_append", *_qptrs(pools), kk.data_ptr(), vv.data_ptr(), kk.stride(1),
             kk.stride(0), slot_mapping.data_ptr(), n, H, D, bs, n_blocks, bits, 64,
             dtype_code(kk.dtype), error_word(dev).data_ptr(), _stream(dev))
    _after(dev)


def kv_quant_append_paged(pools, keys: torch.Tensor, values: torch.Tensor,
                          block_tables: torch.Tensor, positions: torch.Tensor) -> None:
    """Decode-step quantise-append: keys/values ``[B, H, D]``, one token per
    sequence at ``positions[b]`` through ``block_tables[b]``."""
    n_blocks, H, bs, D, bits = _check_qpools(pools)
    kk, vv = keys, values
    if kk.dim() == 4:
        kk, vv = kk[:, :, 0, :], vv[:, :, 0, :]
    if kk.dim() != 3 or kk.shape[1:] != (H, D) or kk.shape != vv.shape:
        raise ValueError(f"keys must be [B, {H}, {D}]")
    if kk.stride(2) != 1 or vv.stride(2) != 1 or kk.stride() != vv.stride():
        kk, vv = kk.contiguous(), vv.contiguous()
    _as_i32(block_tables, pools[0].device, "block_tables")
    _as_i32(positions, pools[0].device, "positions")
    B = kk.shape[0]
    if B == 0:
        return
    dev = _dev_index(pools[0])
    nat.call("mz_kv_quant_append_paged", *_qptrs(pools), kk.data_ptr(), vv.data_ptr(),
             kk.stride(0), kk.stride(1), block_tables.data_ptr(), block_tables.shape[1],
             positions.data_ptr(), B, H, D, bs, n_blocks, bits, 64, dtype_code(kk.dtype),
             error_word(dev).data_ptr(), _stream(dev))
    _after(dev)


def kv_dequant_blocks(pools, block_ids: torch.Tensor, k_out: torch.Tensor,
                      v_out: torch.Tensor) -> None:
    """Dequantise quantised blocks ``block_ids`` (int32 on the pools' device)
    of the 6-tuple ``pools`` into ``k_out`` / ``v_out`` ``[n, H, bs, D]``
    (fp16 or bf16): block ``block_ids[i]`` becomes block ``i``."""
    n_blocks, H, bs, D, bits = _check_qpools(pools)
    _as_i32(block_ids, pools[0].device, "block_ids")
    n = block_ids.numel()
    for t in (k_out, v_out):
        if (t.shape != (n, H, bs, D) or t.dtype not in (torch.float16, torch.bfloat16)
                or not t.is_contiguous() or t.device != pools[0].device):
            raise ValueError(f"outputs must be contiguous fp16/bf16 [{n}, {H}, {bs}, {D}]")
    if k_out.dtype != v_out.dtype:
        raise ValueError("k_out and v_out must have the same dtype")
    if n == 0:
        return
    dev = _dev_index(pools[0])
    nat.call("mz_kv_dequant_blocks", k_out.data_ptr(), v_out.data_ptr(), dtype_code(k_out.dtype),
             *_qptrs(pools), block_ids.data_ptr(), n, H, D, bs, n_blocks, bits,
             error_word(dev).data_ptr(), _stream(dev))
    _after(dev)


def decode_q_workspace(n_seqs: int, n_kv_heads: int, rows: int, head_dim: int, bits: int,
                       device: int, num_warps: int = 0, shared: bool = True) -> torch.Tensor:
    """As ``decode_workspace``, for the quantised decode."""
    size = ctypes.c_size_t(0)
    nat.call("mz_paged_decode_q_workspace_size", n_seqs, n_kv_heads, rows, head_dim, bits,
             num_warps, device, ctypes.byref(size))
    key = (device, n_seqs, n_kv_heads, rows, head_dim, bits, num_warps)
    return _layout_workspace(_qworkspaces, key, int(size.value), device, shared)


def paged_decode_q(q: torch.Tensor, pools, block_tables: torch.Tensor, ctx_lens: torch.Tensor,
                   scale: float | None = None, out: torch.Tensor | None = None,
                   out_dtype: torch.dtype | None = None, num_warps: int = 0,
                   workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Decode attention over quantised K/V (dequantisation fused in).
    q: ``[B, Hq, D]`` or ``[B, n_q, Hq, D]`` (bf16/fp16)."""
    n_blocks, Hkv, bs, D, bits = _check_qpools(pools)
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("q must be fp16 or bf16")
    if q.dim() == 3:
        B, Hq, Dq = q.shape
        nq, q_sb, q_st, q_sh = 1, q.stride(0), 0, q.stride(1)
    elif q.dim() == 4:
        B, nq, Hq, Dq = q.shape
        q_sb, q_st, q_sh = q.stride(0), q.stride(1), q.stride(2)
    else:
        raise ValueError("q must be [B, Hq, D] or [B, n_q, Hq, D]")
    if Dq != D or q.stride(-1) != 1 or Hq % Hkv:
        raise ValueError("q shape does not match the pools")
    _as_i32(block_tables, q.device, "block_tables")
    _as_i32(ctx_lens, q.device, "ctx_lens")
    out_dtype = out_dtype or q.dtype
    if out is None:
        out = torch.empty(q.shape, dtype=out_dtype, device=q.device)
    if q.dim() == 3:
        o_sb, o_st, o_sh = out.stride(0), 0, out.stride(1)
    else:
        o_sb, o_st, o_sh = out.stride(0), out.stride(1), out.stride(2)
    if scale is None:
        scale = D ** -0.5
    if B == 0:
        return out
    dev = _dev_index(q)
    rows = nq * (Hq // Hkv)
    if workspace is None:
        workspace = decode_q_workspace(B, Hkv, rows, D, bits, dev, num_warps)
    nat.call("mz_paged_decode_q", out.data_ptr(), dtype_code(out_dtype), o_sb, o_st, o_sh,
             q.data_ptr(), q_sb, q_st, q_sh, nq, *_qptrs(pools), block_tables.data_ptr(),
             block_tables.shape[1], ctx_lens.data_ptr(), B, Hq, Hkv, D, bs, n_blocks, bits, 64,
             float(scale), dtype_code(q.dtype), num_warps, workspace.data_ptr(),
             workspace.numel(), error_word(dev).data_ptr(), _stream(dev))
    _after(dev)
    return out


# ---------------------------------------------------------------------------
# Block movement
# ---------------------------------------------------------------------------

def _pool_geometry(pools: torch.Tensor) -> tuple[int, int, int]:
    """(n_pools, n_blocks, block_bytes) of a contiguous ``[P, n_blocks, ...]``
    stack of pools (or a single pool ``[n_blocks, ...]``)."""
    if not pools.is_contiguous():
        raise ValueError("pools must be contiguous")
    return pools.shape[0], pools.shape[1], pools[0, 0].numel() * pools.element_size()


def block_copy(pools: torch.Tensor, src_ids: torch.Tensor, dst_ids: torch.Tensor) -> None:
    """Copy block src_ids[i] -> dst_ids[i] in every pool of ``pools``
    (a contiguous ``[P, n_blocks, ...]`` stack)."""
    P, N, bb = _pool_geometry(pools)
    _as_i32(src_ids, pools.device, "src_ids")
    _as_i32(dst_ids, pools.device, "dst_ids")
    if src_ids.numel() != dst_ids.numel():
        raise ValueError("src_ids and dst_ids must have the same length")
    n = src_ids.numel()
    if n == 0:
        return
    dev = _dev_index(pools)
    nat.call("mz_block_copy", pools.data_ptr(), N * bb, P, bb, src_ids.data_ptr(),
             dst_ids.data_ptr(), n, N, error_word(dev).data_ptr(), _stream(dev))
    _after(dev)


def block_pack(pools: torch.Tensor, ids: torch.Tensor, staging: torch.Tensor | None = None
               ) -> torch.Tensor:
    """Gather blocks ``ids`` of every pool into ``staging[n, P, block_bytes]`` (uint8)."""
    P, N, bb = _pool_geometry(pools)
    _as_i32(ids, pools.device, "ids")
    n = ids.numel()
    if staging is None:
        staging = torch.empty((n, P, bb), dtype=torch.uint8, device=pools.device)
    if staging.numel() < n * P * bb or not staging.is_contiguous():
        raise ValueError("staging too small or not contiguous")
    if n:
        dev = _dev_index(pools)
        nat.call("mz_block_pack", staging.data_ptr(), pools.data_ptr(), N * bb, P, bb,
                 ids.data_ptr(), n, N, error_word(dev).data_ptr(), _stream(dev))
        _after(dev)
    return staging


def block_unpack(pools: torch.Tensor, ids: torch.Tensor, staging: torch.Tensor) -> None:
    """Scatter ``staging[n, P, block_bytes]`` into blocks ``ids`` of every pool."""
    P, N, bb = _pool_geometry(pools)
    _as_i32(ids, pools.device, "ids")
    n = ids.numel()
    if staging.numel() < n * P * bb or not staging.is_contiguous() or \
            staging.device != pools.device:
        raise ValueError("staging must be a contiguous device buffer of n*P*block_bytes")
    if n:
        dev = _dev_index(pools)
        nat.call("mz_block_unpack", pools.data_ptr(), N * bb, P, bb, staging.data_ptr(),
                 ids.data_ptr(), n, N, error_word(dev).data_ptr(), _stream(dev))
        _after(dev)


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
