"""KV-head sharding of the decode step across GPUs (one process per GPU).

Attention for different KV heads is independent, so rank r of N owns KV heads
``[r*Hkv/N, (r+1)*Hkv/N)`` and the ``G = Hq/Hkv`` query heads of each: its
pools, appends and decode launches touch only that slice, with no exchange of
inputs.  The block tables are replicated (host-managed, identical on every
rank).  The only collective is the per-layer all-gather of the head-sharded
attention outputs ``[B, Hq/N, D]`` into the full ``[B, Hq, D]`` (NCCL over
NVLink on GPUs; any backend with ``all_gather_into_tensor``).

The reference has no multi-device path (its engine runs one MLX stream on one
device, src/mlxz/engine/thread_boundary.py:220-265); the sharding follows the
GQA head mapping of src/mlxz/paged_attention/attention.py:30-36 (query head h
reads KV head h // G), which keeps every query head on the rank holding its
KV head.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    """The KV-head and query-head ranges rank ``rank`` of ``world`` owns."""

    rank: int
    world: int
    n_kv_heads: int
    n_q_heads: int

    def __post_init__(self) -> None:
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} out of range for world size {self.world}")
        if self.n_kv_heads % self.world:
            raise ValueError(f"world size {self.world} must divide {self.n_kv_heads} KV heads")
        if self.n_q_heads % self.n_kv_heads:
            raise ValueError(f"{self.n_q_heads} query heads are not a multiple of "
                             f"{self.n_kv_heads} KV heads")

    @property
    def kv_local(self) -> int:
        return self.n_kv_heads // self.world

    @property
    def q_local(self) -> int:
        return self.n_q_heads // self.world

    @property
    def kv_range(self) -> tuple[int, int]:
        return self.rank * self.kv_local, (self.rank + 1) * self.kv_local

    @property
    def q_range(self) -> tuple[int, int]:
        return self.rank * self.q_local, (self.rank + 1) * self.q_local

    def kv_slice(self, t: torch.Tensor, dim: int) -> torch.Tensor:
        """This rank's KV heads of ``t`` along ``dim`` (a view)."""
        lo, _ = self.kv_range
        return t.narrow(dim, lo, self.kv_local)

    def q_slice(self, t: torch.Tensor, dim: int) -> torch.Tensor:
        """This rank's query heads of ``t`` along ``dim`` (a view)."""
        lo, _ = self.q_range
        return t.narrow(dim, lo, self.q_local)


class HeadAllGather:
    """Per-layer gather of head-sharded outputs ``[B, Hq/N, D]`` into
    ``[B, Hq, D]``.

    ``gather(local)`` all-gathers into a ``[N, B, Hq/N, D]`` staging buffer
    (each rank's slice contiguous, as the collective needs) and returns it;
    ``full(local)`` also lays it out as ``[B, Hq, D]`` (rank-major heads, so
    head r*Hq/N + j is rank r's local head j).  With world size 1 both return
    the input.
    """

    def __init__(self, shard: HeadShard, batch: int, head_dim: int, dtype: torch.dtype,
                 device, group=None) -> None:
        self.shard = shard
        self.group = group
        self.staging = None
        if shard.world > 1:
            self.staging = torch.empty((shard.world, batch, shard.q_local, head_dim),
                                       dtype=dtype, device=device)

    def gather(self, local: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if self.shard.world == 1:
            return local
        import torch.distributed as dist

        dst = self.staging if out is None else out
        N, B, hq, D = dst.shape
        # rank chunks stacked along dim 0 (the form every backend accepts)
        dist.all_gather_into_tensor(dst.view(N * B, hq, D), local.contiguous(), group=self.group)
        return dst

    def full(self, local: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        g = self.gather(local)
        if self.shard.world == 1:
            return local if out is None else out.copy_(local)
        N, B, hq, D = g.shape
        view = g.permute(1, 0, 2, 3)
        if out is None:
            return view.reshape(B, N * hq, D)
        out.view(B, N, hq, D).copy_(view)
        return out


# Mappings of peers' allocations opened in this process, shared by every
# PeerAllGather (an allocation is mapped once however many buffers it holds):
# handle -> [base address, users].
_opened: dict[bytes, list[int]] = {}


def _open(handle: bytes) -> int:
    from .. import ops

    ent = _opened.get(handle)
    if ent is None:
        base, _ = ops.ipc_open(handle, 0)
        ent = _opened[handle] = [base, 0]
    ent[1] += 1
    return ent[0]


def _close(handle: bytes) -> None:
    from .. import ops

    ent = _opened[handle]
    ent[1] -= 1
    if ent[1] == 0:
        ops.ipc_close(ent[0])
        del _opened[handle]


class PeerAllGather:
    """Head-sharded decode with the all-gather fused into the decode launch.

    Every rank keeps ``n_slots`` gathered buffers ``[B, Hq, D]`` and ``N``
    signal words in one device allocation, exchanged once with CUDA IPC.
    ``launch`` runs mz_paged_append_decode_allgather: each output row is
    stored into the slot of every rank's buffer as soon as it is final, the
    peers' over NVLink, and the launch's last block then signals the peers.
    No separate collective and no layout copy.  A launch's gathered buffer is
    complete for work queued after either

    * ``wait()`` (a small bounded-wait launch), or
    * the next ``launch(..., wait_previous=True)``, which waits for the peers'
      rows of the launch before it inside its own prologue (after its first
      K/V copies have started), so consecutive layers need no launch between
      them and keep their overlap.

    ``layer`` is ``launch`` + ``wait``.  Every launch must be followed by one
    of the two before the next plain launch (enforced), and all ranks must make
    the same sequence of launches (the epochs must agree).

    Slot reuse: peers store into a slot again as soon as this rank's launch
    before that one has completed, so the readers of a slot must be queued
    before that launch.  With readers queued right where the slot becomes
    complete, that means a slot is never reused by the next launch, nor, when
    the next launch is a ``wait_previous`` one (whose slot is then complete
    only after the launch after it), by the launch after that; both are
    checked.  Hence at least 2 slots for ``layer`` and 3 for chained launches.
    ``close`` (collective) ends the mappings.
    """

    def __init__(self, shard: HeadShard, batch: int, head_dim: int, dtype: torch.dtype,
                 device, n_slots: int = 3, group=None, timeout_s: float = 2.0) -> None:
        from .. import _native as nat
        from .. import ops

        if batch < 1 or n_slots < 2:
            raise ValueError("batch must be positive and n_slots at least 2")
        if shard.world > nat.MZ_MAX_RANKS:
            raise ValueError(f"at most {nat.MZ_MAX_RANKS} ranks")
        self.shard = shard
        self.group = group
        self.timeout_s = timeout_s
        self.device = torch.device(device)
        self.dtype = dtype
        N, r = shard.world, shard.rank
        Hq = shard.n_q_heads
        elem = torch.empty((), dtype=dtype).element_size()
        self.slot_elems = batch * Hq * head_dim
        full_bytes = n_slots * self.slot_elems * elem
        sig_off = -(-full_bytes // 256) * 256
        self.arena = torch.zeros(sig_off + 4 * N, dtype=torch.uint8, device=self.device)
        self.full = self.arena[:full_bytes].view(dtype).view(n_slots, batch, Hq, head_dim)
        self.signal = self.arena[sig_off:sig_off + 4 * N].view(torch.int32)
        self.arrivals = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.epoch = 0
        self.out_seq_stride = Hq * head_dim
        self.out_head_stride = head_dim
        self._handles: list[bytes] = []
        # (slot, chained) of the last two launches, and whether the last one
        # still needs wait() or a chained launch
        self._recent: list[tuple[int, bool]] = []
        self._pending = False
        bases = [self.arena.data_ptr()] * N
        if N > 1:
            import torch.distributed as dist

            torch.cuda.synchronize(self.device)  # the zeroed words are in place before peers map them
            mine = ops.ipc_export(self.arena)
            everyone: list = [None] * N
            dist.all_gather_object(everyone, mine, group=group)
            for s in range(N):
                if s == r:
                    continue
                handle, off = everyone[s]
                bases[s] = _open(handle) + off
                self._handles.append(handle)
        self._peers = []
        head_off = r * shard.q_local * head_dim * elem
        for k in range(n_slots):
            pe = nat.PeerOutputs()
            pe.n_ranks, pe.rank = N, r
            for s in range(N):
                pe.out[s] = bases[s] + k * self.slot_elems * elem + head_off
                pe.signal[s] = bases[s] + sig_off  # signal[r]: this rank's own words
            pe.arrivals = self.arrivals.data_ptr()
            self._peers.append(pe)

    def _check_slot(self, slot: int, wait_previous: bool) -> None:
        if not 0 <= slot < len(self._peers):
            raise ValueError(f"slot {slot} out of range (n_slots {len(self._peers)})")
        if self._pending and not wait_previous:
            raise RuntimeError("the previous launch was neither waited for nor followed by a "
                               "wait_previous launch")
        if self._recent and self._recent[-1][0] == slot:
            raise ValueError(f"slot {slot} is the previous launch's: peers could overwrite it "
                             "before this rank has read it")
        if len(self._recent) == 2 and self._recent[1][1] and self._recent[0][0] == slot:
            raise ValueError(f"slot {slot} was used two launches ago and the launch after it "
                             "waited for it (wait_previous): peers could overwrite it before "
                             "this rank has read it")

    def launch(self, step, l: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
               slot: int = 0, num_warps: int = 0, wait_previous: bool = False) -> None:
        """Queue layer ``l`` of a PagedDecodeStep on this rank's heads (append +
        attention), its rows stored into ``full[slot]`` of every rank.  With
        ``wait_previous`` the launch first waits (on the device, bounded) for
        every peer's rows of this rank's previous launch, which then completes
        that launch's slot for work queued after this one."""
        from .. import ops

        self._check_slot(slot, wait_previous)
        self.epoch = self.epoch % 0xFFFFFFFF + 1  # 1, 2, ..., 2^32 - 1, 1, ...
        pe = self._peers[slot]
        pe.epoch = self.epoch
        st = step.store
        # layers after the first may start while the previous layer drains
        ops.paged_append_decode_allgather(pe, q, st.k_pool(l), st.v_pool(l), k_new, v_new,
                                          step.tables, step.lengths, self.out_seq_stride,
                                          self.out_head_stride, self.dtype, scale=step.scale,
                                          num_warps=num_warps, workspace=step.workspace,
                                          overlap_previous=l > 0,
                                          wait_previous=wait_previous and self.epoch > 1)
        self._recent = (self._recent + [(slot, wait_previous)])[-2:]
        self._pending = True

    def wait(self) -> None:
        """Queue the bounded wait for every peer's rows of the last launch."""
        from .. import ops

        ops.peer_wait(self.signal, self.shard.world, self.shard.rank, self.epoch, self.timeout_s)
        self._pending = False

    def layer(self, step, l: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
              slot: int = 0, num_warps: int = 0) -> torch.Tensor:
        """``launch`` then ``wait``: returns ``full[slot]``, complete for work
        queued after it on the current stream."""
        self.launch(step, l, q, k_new, v_new, slot, num_warps)
        self.wait()
        return self.full[slot]

    def close(self) -> None:
        """Collective: wait for every rank's launches, then unmap the peers."""
        torch.cuda.synchronize(self.device)
        if self.shard.world > 1:
            import torch.distributed as dist

            dist.barrier(group=self.group)
        for h in self._handles:
            _close(h)
        self._handles = []
