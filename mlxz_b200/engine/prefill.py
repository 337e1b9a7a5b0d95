"""Chunked prefill over paged KV.

``ChunkedPrefillScheduler`` splits prompts into fixed-size chunks with the
reference's behaviour (src/mlxz/scheduler/chunker.py:24-80): one chunk per
call, progress kept per request, ``is_last`` on the final chunk.

``PagedPrefillStep`` runs the KV side of one prefill iteration for any number
of sequences' chunks at once (ragged chunk lengths, ragged cache offsets):

    per layer l:  mz_kv_append     (the chunk's K/V -> pool slots through the
                                    block tables)
                  mz_paged_prefill (causal GQA attention of the chunk's
                                    queries over cache + chunk, from the pools)

Queries and new K/V arrive as the model's projections lay them out: q
``[T, Hq, D]`` and k / v ``[T, Hkv, D]``, the sequences' chunks stacked along
T in the order given.

Over a QuantizedPagedKVStore the chunk is quantised on append
(mz_kv_quant_append) and the chunk attends over the quantised keys and values,
as a quantised cache's attention does: per layer the step's blocks are
dequantised once into a staging pool of q's dtype (mz_kv_dequant_blocks) and
mz_paged_prefill runs on it through block tables renumbered to that pool.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops
from .decode_step import PagedKVStore, QuantizedPagedKVStore


@dataclass(slots=True)
class PrefillChunk:
    """A chunk of a prompt: its tokens, where it starts, whether it is the last."""

    request_id: str
    tokens: list[int]
    start_pos: int
    is_last: bool
    total_prompt_tokens: int


class ChunkedPrefillScheduler:
    """Splits prefill requests into chunks of ``chunk_size`` tokens so that
    decode steps can run between them."""

    def __init__(self, chunk_size: int = 128) -> None:
        if chunk_size < 1:
            raise ValueError(f"chunk_size must be >= 1, got {chunk_size}")
        self._chunk_size = chunk_size
        self._progress: dict[str, int] = {}

    @property
    def chunk_size(self) -> int:
        return self._chunk_size

    def needs_chunking(self, prompt_tokens: list[int]) -> bool:
        return len(prompt_tokens) > self._chunk_size

    def get_next_chunk(self, request_id: str, prompt_tokens: list[int]) -> PrefillChunk:
        """The request's next chunk; call until ``is_last``."""
        start = self._progress.get(request_id, 0)
        end = min(start + self._chunk_size, len(prompt_tokens))
        self._progress[request_id] = end
        return PrefillChunk(request_id=request_id, tokens=prompt_tokens[start:end],
                            start_pos=start, is_last=end >= len(prompt_tokens),
                            total_prompt_tokens=len(prompt_tokens))

    def reset(self, request_id: str) -> None:
        self._progress.pop(request_id, None)

    def get_progress(self, request_id: str) -> int:
        return self._progress.get(request_id, 0)


class PagedPrefillStep:
    """One prefill iteration: ``chunks`` = [(seq_id, n_tokens), ...] appended
    at each sequence's current offset.  Construction grows the block tables
    (copy-on-write of a shared block at the offset) and uploads the step's
    tables, slots and lengths once; ``layer`` runs append + attention for one
    layer; ``finish`` advances the sequences' offsets."""

    def __init__(self, store: PagedKVStore, chunks: list[tuple[str, int]], n_heads: int,
                 scale: float | None = None) -> None:
        if not isinstance(store, PagedKVStore):
            raise TypeError("chunked prefill needs a PagedKVStore")
        self.quantized = isinstance(store, QuantizedPagedKVStore)
        if n_heads % store.n_kv_heads:
            raise ValueError("n_heads must be a multiple of n_kv_heads")
        self.store = store
        self.chunks = [(s, int(n)) for s, n in chunks]
        self.n_heads = n_heads
        self.scale = scale if scale is not None else store.head_dim ** -0.5
        bs = store.block_size
        cow = []
        for s, n in self.chunks:
            store.ensure_capacity(s, n)
            if n:
                pair = store.make_writable(s, store.offsets[s])
                if pair:
                    cow.append(pair)
        store.copy_blocks(cow)
        B = len(self.chunks)
        self.T = sum(n for _, n in self.chunks)
        width = max([1] + [len(store.tables[s]) for s, _ in self.chunks])
        tables = torch.full((B, width), -1, dtype=torch.int32)
        # quantised store: the attention reads a staging pool holding the
        # step's blocks in first-use order, through renumbered tables
        uniq = list(dict.fromkeys(blk for s, _ in self.chunks for blk in store.tables[s]))
        local = {blk: i for i, blk in enumerate(uniq)}
        q_start, q_len, ctx, slots = [], [], [], []
        row = 0
        for b, (s, n) in enumerate(self.chunks):
            t = store.tables[s]
            tt = [local[blk] for blk in t] if self.quantized else t
            if tt:
                tables[b, :len(tt)] = torch.tensor(tt, dtype=torch.int32)
            off = store.offsets[s]
            q_start.append(row)
            q_len.append(n)
            ctx.append(off + n)
            slots.extend(t[p // bs] * bs + p % bs for p in range(off, off + n))
            row += n
        dev = store.device
        self.max_q_len = max([0] + q_len)
        self.tables = tables.to(dev)
        self.q_start = torch.tensor(q_start, dtype=torch.int32).to(dev)
        self.q_len = torch.tensor(q_len, dtype=torch.int32).to(dev)
        self.ctx_lens = torch.tensor(ctx, dtype=torch.int32).to(dev)
        self.slots = torch.tensor(slots, dtype=torch.int64).to(dev)
        self._ids = torch.tensor(uniq, dtype=torch.int32).to(dev) if self.quantized else None
        self._stage = None
        self._done = False

    def layer(self, l: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
              out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None
              ) -> torch.Tensor:
        """Append layer l's chunk K/V ``[T, Hkv, D]`` and return the causal
        attention of q ``[T, n_heads, D]`` over each sequence's cache + chunk."""
        st = self.store
        if k.shape != (self.T, st.n_kv_heads, st.head_dim) or v.shape != k.shape:
            raise ValueError(f"k/v must be [{self.T}, {st.n_kv_heads}, {st.head_dim}]")
        if q.shape != (self.T, self.n_heads, st.head_dim):
            raise ValueError(f"q must be [{self.T}, {self.n_heads}, {st.head_dim}]")
        if self.quantized:
            pools = st.qpools(l)
            ops.kv_quant_append(pools, k.transpose(0, 1), v.transpose(0, 1), self.slots)
            shape = (self._ids.numel(), st.n_kv_heads, st.block_size, st.head_dim)
            if self._stage is None or self._stage[0].dtype != q.dtype:
                self._stage = tuple(torch.empty(shape, dtype=q.dtype, device=st.device)
                                    for _ in range(2))
            kp, vp = self._stage
            ops.kv_dequant_blocks(pools, self._ids, kp, vp)
        else:
            kp, vp = st.k_pool(l), st.v_pool(l)
            ops.kv_append(kp, vp, k.transpose(0, 1), v.transpose(0, 1), self.slots)
        return ops.paged_prefill(q, kp, vp, self.tables, self.q_start, self.q_len, self.ctx_lens,
                                 self.max_q_len, self.scale, out=out, out_dtype=out_dtype)

    def finish(self) -> None:
        """Advance every sequence's offset past its chunk (once all layers ran)."""
        if self._done:
            return
        for s, n in self.chunks:
            self.store.offsets[s] += n
        self._done = True
