"""Continuous-batching decode step over paged KV (the KV side of one step).

The reference batches only requests whose caches have the same offset
(ContinuousBatchingEngine._process_decodes, src/mlxz/engine/continuous.py:386-388),
concatenates their per-layer caches along the batch axis before the forward
and splits them back afterwards (_build_batched_cache / _scatter_batched_cache,
:804-832): two full KV copies per step.  Here every live sequence of any
length runs in one ragged launch per layer, straight from the block pools:

    per layer l:  mz_paged_append_decode  (new token -> its pool slot through
                  the block table, then fused GQA attention over ctx + 1 tokens,
                  in one launch)

``PagedKVStore`` holds all layers' pools with one block table per sequence
(the paged form of the per-request cache list built at continuous.py:195-200).
"""
from __future__ import annotations

import torch

from .. import ops
from ..paged_attention.block_manager import BlockManager


class PagedKVStore:
    """K/V pools of every layer, ``pools[l, 0]`` = K and ``pools[l, 1]`` = V,
    each ``[n_blocks, n_kv_heads, block_size, head_dim]``, sharing one
    BlockManager (one block id addresses the same slot range in every layer)."""

    def __init__(self, n_layers: int, n_blocks: int, n_kv_heads: int, head_dim: int,
                 block_size: int = 16, dtype: torch.dtype = torch.bfloat16, device=None,
                 init: str = "zeros") -> None:
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.n_layers, self.n_blocks = n_layers, n_blocks
        self.n_kv_heads, self.head_dim, self.block_size, self.dtype = (n_kv_heads, head_dim,
                                                                       block_size, dtype)
        shape = (n_layers, 2, n_blocks, n_kv_heads, block_size, head_dim)
        if init == "zeros":
            self.pools = torch.zeros(shape, dtype=dtype, device=self.device)
        elif init == "empty":
            self.pools = torch.empty(shape, dtype=dtype, device=self.device)
        else:
            raise ValueError(init)
        self.bm = BlockManager(n_blocks, block_size)
        self.tables: dict[str, list[int]] = {}
        self.offsets: dict[str, int] = {}

    def k_pool(self, layer: int) -> torch.Tensor:
        return self.pools[layer, 0]

    def v_pool(self, layer: int) -> torch.Tensor:
        return self.pools[layer, 1]

    @property
    def block_bytes(self) -> int:
        """Bytes of one block in one pool (one layer's K or V)."""
        return self.n_kv_heads * self.block_size * self.head_dim * self.pools.element_size()

    @property
    def bytes_per_token(self) -> int:
        """Bytes of one token over all layers, K and V."""
        return self.n_layers * 2 * self.n_kv_heads * self.head_dim * self.pools.element_size()

    def pool_stack(self) -> torch.Tensor:
        """All pools as one ``[2 * n_layers, n_blocks, ...]`` stack (block moves)."""
        return self.pools.view(2 * self.n_layers, self.n_blocks, self.n_kv_heads,
                               self.block_size, self.head_dim)

    def pool_stacks(self) -> list[torch.Tensor]:
        """Every tensor family a block lives in, as ``[P, n_blocks, ...]`` stacks."""
        return [self.pool_stack()]

    def add_sequence(self, seq_id: str, n_tokens: int = 0, blocks: list[int] | None = None) -> None:
        """Register a sequence holding `n_tokens` tokens, allocating blocks from
        the BlockManager unless an explicit block list is given."""
        need = -(-n_tokens // self.block_size)
        if blocks is None:
            blocks = self.bm.allocate(need)
        elif len(blocks) < need:
            raise ValueError("block list too short for n_tokens")
        self.tables[seq_id] = list(blocks)
        self.offsets[seq_id] = n_tokens

    def free_sequence(self, seq_id: str) -> None:
        if seq_id in self.tables:
            self.bm.free(self.tables.pop(seq_id))
            self.offsets.pop(seq_id, None)

    def make_writable(self, seq_id: str, position: int) -> tuple[int, int] | None:
        """Copy-on-write the block that will hold `position` if another table
        or the prefix cache shares it: the sequence gets a fresh block
        (BlockManager.copy_on_write) and the caller must copy the data.
        Returns (old, new) block ids, or None when the block is private."""
        t = self.tables[seq_id]
        bi = position // self.block_size
        if bi >= len(t):
            return None
        blk = t[bi]
        if self.bm.get_refcount(blk) <= 1:
            return None
        new = self.bm.copy_on_write(blk)
        t[bi] = new
        return blk, new

    def copy_blocks(self, pairs: list[tuple[int, int]]) -> None:
        """Copy block src -> dst in every layer's K and V (one mz_block_copy)."""
        if not pairs:
            return
        src = torch.tensor([a for a, _ in pairs], dtype=torch.int32).to(self.device, non_blocking=True)
        dst = torch.tensor([b for _, b in pairs], dtype=torch.int32).to(self.device, non_blocking=True)
        for stack in self.pool_stacks():
            ops.block_copy(stack, src, dst)

    def append_tokens(self, seq_id: str, keys: torch.Tensor, values: torch.Tensor) -> None:
        """Prefill-style append of n tokens to every layer: keys/values
        ``[L, H, n, D]``.  Grows the table, copy-on-writes a shared first
        block, then one mz_kv_append per layer with the slots of the new tokens."""
        n = keys.shape[2]
        if n == 0:
            return
        off = self.offsets[seq_id]
        self.ensure_capacity(seq_id, n)
        cow = self.make_writable(seq_id, off)
        if cow:
            self.copy_blocks([cow])
        t = self.tables[seq_id]
        bs = self.block_size
        slots = torch.tensor([t[(off + i) // bs] * bs + (off + i) % bs for i in range(n)],
                             dtype=torch.int64).to(self.device, non_blocking=True)
        for l in range(self.n_layers):
            self._write_layer(l, keys[l], values[l], slots)
        self.offsets[seq_id] = off + n

    def _write_layer(self, l: int, keys: torch.Tensor, values: torch.Tensor,
                     slots: torch.Tensor) -> None:
        ops.kv_append(self.k_pool(l), self.v_pool(l), keys, values, slots)

    def ensure_capacity(self, seq_id: str, extra: int) -> bool:
        """Grow the table for `extra` more tokens; True if it changed."""
        t = self.tables[seq_id]
        need = -(-(self.offsets[seq_id] + extra) // self.block_size)
        grew = False
        while len(t) < need:
            t.extend(self.bm.allocate(1))
            grew = True
        return grew


def _copy_groups(n_layers: int) -> list[tuple[int, int]]:
    """[a, b) layer ranges with boundaries at 0, 1, 2, 4, ... from each end."""
    cuts, b = {0, n_layers}, 1
    while b < n_layers:
        cuts.update((b, n_layers - b))
        b *= 2
    edges = sorted(c for c in cuts if 0 <= c <= n_layers)
    return list(zip(edges[:-1], edges[1:]))


class PagedDecodeStep:
    """One decode step for a fixed set of sequences.

    Device state: int32 block tables ``[B, max_blocks]``, the write positions
    (= current offsets) and the attended lengths (offset + 1).  ``step``
    takes the step's per-layer q ``[L, B, Hq, D]`` and new K/V ``[L, B, Hkv, D]``
    already on the device; ``step_host`` is the end-to-end form that copies
    them from (pinned) host memory and copies the output back.
    ``batch_invariant``: every sequence's output bytes are independent of the
    batch (each (sequence, KV head) pair is computed whole by one warp).
    """

    def __init__(self, store: PagedKVStore, seq_ids: list[str], n_heads: int,
                 scale: float | None = None, max_blocks: int | None = None,
                 batch_invariant: bool = False) -> None:
        self.store = store
        self.batch_invariant = batch_invariant
        self.seq_ids = list(seq_ids)
        self.n_heads = n_heads
        self.scale = scale if scale is not None else store.head_dim ** -0.5
        self.B = len(seq_ids)
        for s in self.seq_ids:
            store.ensure_capacity(s, 1)
        width = max(len(store.tables[s]) for s in self.seq_ids)
        self.max_blocks = max(width, max_blocks or 0)
        dev = store.device
        self.tables = torch.full((self.B, self.max_blocks), -1, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(self.B, dtype=torch.int32, device=dev)
        self.lengths = torch.zeros(self.B, dtype=torch.int32, device=dev)
        self.sync_metadata()
        G = n_heads // store.n_kv_heads
        # a workspace of its own: a step's launches never share one with
        # launches of other sizes
        self.workspace = ops.decode_workspace(self.B, store.n_kv_heads, G, store.head_dim,
                                              dev.index if dev.index is not None else 0,
                                              shared=False, batch_invariant=batch_invariant,
                                              max_blocks=self.max_blocks,
                                              block_size=store.block_size)
        self._dev_in = None
        self._graph = None

    def sync_metadata(self) -> None:
        """Upload block tables and offsets from the host mirror."""
        host = torch.full((self.B, self.max_blocks), -1, dtype=torch.int32)
        for i, s in enumerate(self.seq_ids):
            t = self.store.tables[s]
            if len(t) > self.max_blocks:
                raise ValueError("a table outgrew max_blocks; rebuild the step")
            if t:
                host[i, : len(t)] = torch.tensor(t, dtype=torch.int32)
        offs = torch.tensor([self.store.offsets[s] for s in self.seq_ids], dtype=torch.int32)
        self.tables.copy_(host, non_blocking=False)
        self.positions.copy_(offs)
        self.lengths.copy_(offs + 1)

    def layer(self, l: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
              out: torch.Tensor, num_warps: int = 0) -> None:
        """Append this step's token of layer l and attend, one launch (device
        tensors).  Layers after the first may start while the previous layer's
        launch finishes (it writes none of this layer's pools, and the tables
        and lengths change only between steps)."""
        st = self.store
        ops.paged_append_decode(q, st.k_pool(l), st.v_pool(l), k_new, v_new, self.tables,
                                self.lengths, scale=self.scale, out=out,
                                workspace=self.workspace, num_warps=num_warps,
                                overlap_previous=l > 0, batch_invariant=self.batch_invariant)

    def prepare_writes(self) -> int:
        """Copy-on-write every block this step will write that is shared (a
        restored prefix's partial last block, say); one batched block copy.
        Returns the number of blocks copied."""
        pairs = []
        for s in self.seq_ids:
            cow = self.store.make_writable(s, self.store.offsets[s])
            if cow:
                pairs.append(cow)
        if pairs:
            self.store.copy_blocks(pairs)
            self.sync_metadata()
        return len(pairs)

    def step(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
             out: torch.Tensor | None = None, advance: bool = False) -> torch.Tensor:
        """All layers: q ``[L, B, Hq, D]``, k_new/v_new ``[L, B, Hkv, D]``."""
        if out is None:
            out = torch.empty_like(q)
        self.prepare_writes()
        for l in range(self.store.n_layers):
            self.layer(l, q[l], k_new[l], v_new[l], out[l])
        if advance:
            self.advance()
        return out

    def advance(self) -> None:
        """Commit the appended token: offsets += 1, growing tables as needed."""
        grew = False
        for s in self.seq_ids:
            self.store.offsets[s] += 1
            grew |= self.store.ensure_capacity(s, 1)
        if grew:
            self.sync_metadata()
        else:
            self.positions.add_(1)
            self.lengths.add_(1)

    def capture(self, q_dtype: torch.dtype | None = None) -> None:
        """Capture every layer's launch of one step into a CUDA graph over
        static buffers ``q_in [L, B, Hq, D]``, ``k_in``/``v_in [L, B, Hkv, D]``
        and ``out [L, B, Hq, D]``.  The block tables, positions and lengths are
        device tensors that ``advance`` / ``sync_metadata`` update in place, so
        each replay runs the step the host state describes.  Copy-on-write
        (``prepare_writes``) and table growth stay on the host, outside the
        graph; a table outgrowing ``max_blocks`` needs a new step."""
        st = self.store
        dev = st.device
        dt = q_dtype or st.dtype  # q and the new K/V rows (the source dtype of a quantised store)
        L, B = st.n_layers, self.B
        self.q_in = torch.zeros((L, B, self.n_heads, st.head_dim), dtype=dt, device=dev)
        self.k_in = torch.zeros((L, B, st.n_kv_heads, st.head_dim), dtype=dt, device=dev)
        self.v_in = torch.zeros_like(self.k_in)
        self.out = torch.empty_like(self.q_in)
        ops.error_word(dev.index if dev.index is not None else torch.cuda.current_device())
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(self._graph, stream=side):
                for l in range(L):
                    self.layer(l, self.q_in[l], self.k_in[l], self.v_in[l], self.out[l])
        torch.cuda.current_stream(dev).wait_stream(side)

    def replay(self, q: torch.Tensor | None = None, k_new: torch.Tensor | None = None,
               v_new: torch.Tensor | None = None, advance: bool = False) -> torch.Tensor:
        """One captured step: copy the given inputs into the static buffers
        (or leave what the caller wrote there), copy-on-write shared blocks,
        replay, and return ``out``."""
        if self._graph is None:
            raise RuntimeError("capture() first")
        for src, dst in ((q, self.q_in), (k_new, self.k_in), (v_new, self.v_in)):
            if src is not None:
                dst.copy_(src, non_blocking=True)
        self.prepare_writes()
        self._graph.replay()
        if advance:
            self.advance()
        return self.out

    def step_host(self, q_host: torch.Tensor, k_host: torch.Tensor, v_host: torch.Tensor,
                  out_host: torch.Tensor, advance: bool = False, layer_fn=None) -> torch.Tensor:
        """End-to-end step from host buffers (pinned for async copies).

        The copies are pipelined with the layers in groups that double in
        size from each end (1, 1, 2, 4, ... 4, 2, 1, 1 layers): a group's
        inputs go up on one copy stream (its launches wait only for their
        group), and its outputs come back on a second copy stream while later
        groups run, so only one layer's copies are exposed at either end.
        (Groups, not single layers: an event between two launches stops the
        later one from starting while the earlier drains.)  The current stream waits for the last copy, so
        synchronising it covers the whole step.  ``layer_fn(l, q, k, v, out)``,
        if given, runs layer l instead of ``layer`` and returns the tensor to
        copy back (a head-sharded step returns its gathered output)."""
        dev = self.store.device
        L = self.store.n_layers
        groups = _copy_groups(L)
        if self._dev_in is None or self._dev_in[0].shape != q_host.shape:
            self._dev_in = (torch.empty(q_host.shape, dtype=q_host.dtype, device=dev),
                            torch.empty(k_host.shape, dtype=k_host.dtype, device=dev),
                            torch.empty(v_host.shape, dtype=v_host.dtype, device=dev),
                            torch.empty(q_host.shape, dtype=q_host.dtype, device=dev))
            self._copy_streams = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
            self._in_ready = [torch.cuda.Event() for _ in groups]
            self._out_ready = [torch.cuda.Event() for _ in groups]
        q, k, v, o = self._dev_in
        up, down = self._copy_streams
        compute = torch.cuda.current_stream(dev)
        # the previous step's kernels and copies are done with these buffers
        up.wait_stream(compute)
        down.wait_stream(compute)
        with torch.cuda.stream(up):
            for gi, (a, b) in enumerate(groups):
                q[a:b].copy_(q_host[a:b], non_blocking=True)
                k[a:b].copy_(k_host[a:b], non_blocking=True)
                v[a:b].copy_(v_host[a:b], non_blocking=True)
                self._in_ready[gi].record(up)
        self.prepare_writes()
        results = []
        for gi, (a, b) in enumerate(groups):
            compute.wait_event(self._in_ready[gi])
            for l in range(a, b):
                if layer_fn is None:
                    self.layer(l, q[l], k[l], v[l], o[l])
                    results.append(o[l])
                else:
                    results.append(layer_fn(l, q[l], k[l], v[l], o[l]))
            self._out_ready[gi].record(compute)
        with torch.cuda.stream(down):
            for gi, (a, b) in enumerate(groups):
                down.wait_event(self._out_ready[gi])
                for l in range(a, b):
                    out_host[l].copy_(results[l], non_blocking=True)
        compute.wait_stream(down)
        if advance:
            self.advance()
        return out_host


class QuantizedPagedKVStore(PagedKVStore):
    """Paged KV store holding 4/8-bit group-64 quantised K/V: per layer and
    per K/V, int32 codes ``[n_blocks, H, bs, D*bits/32]`` and fp16 scales and
    biases ``[n_blocks, H, bs, D/64]`` (the layout of mz_kv_quant_append)."""

    def __init__(self, n_layers: int, n_blocks: int, n_kv_heads: int, head_dim: int,
                 block_size: int = 16, bits: int = 8, group_size: int = 64, device=None,
                 init: str = "zeros") -> None:
        if bits not in (4, 8) or group_size != 64 or head_dim % 64:
            raise ValueError("quantised store: bits 4 or 8, group 64, head_dim a multiple of 64")
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.n_layers, self.n_blocks = n_layers, n_blocks
        self.n_kv_heads, self.head_dim, self.block_size = n_kv_heads, head_dim, block_size
        self.bits, self.group_size = bits, group_size
        self.dtype = torch.float16
        alloc = torch.zeros if init == "zeros" else torch.empty
        base = (n_layers, 2, n_blocks, n_kv_heads, block_size)
        self.codes = alloc(base + (head_dim * bits // 32,), dtype=torch.int32, device=self.device)
        self.scales = alloc(base + (head_dim // 64,), dtype=torch.float16, device=self.device)
        self.biases = alloc(base + (head_dim // 64,), dtype=torch.float16, device=self.device)
        self.pools = self.codes  # element size used by callers that size per-token bytes
        self.bm = BlockManager(n_blocks, block_size)
        self.tables: dict[str, list[int]] = {}
        self.offsets: dict[str, int] = {}

    def qpools(self, layer: int) -> tuple[torch.Tensor, ...]:
        """(k_codes, k_scales, k_biases, v_codes, v_scales, v_biases) of a layer."""
        return (self.codes[layer, 0], self.scales[layer, 0], self.biases[layer, 0],
                self.codes[layer, 1], self.scales[layer, 1], self.biases[layer, 1])

    def k_pool(self, layer: int) -> torch.Tensor:
        raise TypeError("quantised store: use qpools(layer)")

    v_pool = k_pool

    @property
    def bytes_per_token(self) -> int:
        """Bytes of one token over all layers, K and V (codes + scales + biases)."""
        per_head = self.head_dim * self.bits // 8 + 2 * 2 * (self.head_dim // 64)
        return self.n_layers * 2 * self.n_kv_heads * per_head

    def pool_stack(self) -> torch.Tensor:
        raise TypeError("quantised store: use pool_stacks()")

    def pool_stacks(self) -> list[torch.Tensor]:
        L2 = 2 * self.n_layers
        return [t.view(L2, self.n_blocks, *t.shape[3:]) for t in (self.codes, self.scales,
                                                                  self.biases)]

    def _write_layer(self, l: int, keys: torch.Tensor, values: torch.Tensor,
                     slots: torch.Tensor) -> None:
        ops.kv_quant_append(self.qpools(l), keys, values, slots)


class QuantizedPagedDecodeStep(PagedDecodeStep):
    """Decode step over a QuantizedPagedKVStore: per layer, quantise-on-append
    of the new token (mz_kv_quant_append_paged), then attention with the
    dequantisation fused in (mz_paged_decode_q)."""

    def __init__(self, store: QuantizedPagedKVStore, seq_ids: list[str], n_heads: int,
                 scale: float | None = None, max_blocks: int | None = None) -> None:
        self.store = store
        self.seq_ids = list(seq_ids)
        self.n_heads = n_heads
        self.scale = scale if scale is not None else store.head_dim ** -0.5
        self.B = len(seq_ids)
        for s in self.seq_ids:
            store.ensure_capacity(s, 1)
        width = max(len(store.tables[s]) for s in self.seq_ids)
        self.max_blocks = max(width, max_blocks or 0)
        dev = store.device
        self.tables = torch.full((self.B, self.max_blocks), -1, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(self.B, dtype=torch.int32, device=dev)
        self.lengths = torch.zeros(self.B, dtype=torch.int32, device=dev)
        self.sync_metadata()
        G = n_heads // store.n_kv_heads
        self.workspace = ops.decode_q_workspace(self.B, store.n_kv_heads, G, store.head_dim,
                                                store.bits,
                                                dev.index if dev.index is not None else 0,
                                                shared=False)
        self._dev_in = None
        self._graph = None

    def layer(self, l: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
              out: torch.Tensor, num_warps: int = 0) -> None:
        pools = self.store.qpools(l)
        ops.kv_quant_append_paged(pools, k_new, v_new, self.tables, self.positions)
        ops.paged_decode_q(q, pools, self.tables, self.lengths, scale=self.scale, out=out,
                           workspace=self.workspace, num_warps=num_warps)
