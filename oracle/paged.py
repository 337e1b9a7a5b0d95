"""numpy restatement of the reference's paged KV append / gather / attention
and of the block moves used by the prefix cache (oracle; test infrastructure).

Pools are uint16 bit-pattern arrays ``[n_blocks, H_kv, block_size, D]`` so
that every copy is compared bit for bit; attention converts to float and
computes softmax(q.K^T * scale).V in float64.
"""
from __future__ import annotations

import numpy as np


class PagedKVOracle:
    """The data half of ``PagedKVCache`` (src/mlxz/paged_attention/paged_kv.py:12-154).

    Block tables are supplied by the caller (allocation is host policy and is
    pinned separately against the reference's BlockManager traces).
    """

    def __init__(self, n_blocks: int, n_kv_heads: int, block_size: int, head_dim: int) -> None:
        # paged_kv.py:33-44: zero-filled pools (total_blocks, H_kv, bs, D)
        self.k_pool = np.zeros((n_blocks, n_kv_heads, block_size, head_dim), dtype=np.uint16)
        self.v_pool = np.zeros_like(self.k_pool)
        self.bs = block_size
        self.tables: dict[str, list[int]] = {}
        self.offsets: dict[str, int] = {}

    def set_table(self, seq: str, blocks: list[int], offset: int = 0) -> None:
        self.tables[seq] = list(blocks)
        self.offsets[seq] = offset

    def append_kv(self, seq: str, keys: np.ndarray, values: np.ndarray) -> list[int]:
        """paged_kv.py:63-93.  keys/values: (H, n_new, D) uint16.  Returns the
        slots written.  Table growth is the caller's job here: the table must
        already cover the new positions."""
        n_new = keys.shape[1]
        offset = self.offsets[seq]
        blocks = self.tables[seq]
        slots = []
        for i in range(n_new):
            pos = offset + i
            blk = blocks[pos // self.bs]          # :75-80 block_idx_in_table / pos_in_block
            self.k_pool[blk, :, pos % self.bs, :] = keys[:, i, :]   # :85-86
            self.v_pool[blk, :, pos % self.bs, :] = values[:, i, :]
            slots.append(blk * self.bs + pos % self.bs)
        self.offsets[seq] = offset + n_new       # :93
        return slots

    def get_kv(self, seq: str) -> tuple[np.ndarray, np.ndarray]:
        """paged_kv.py:95-137: first `offset` tokens of the table's blocks,
        concatenated along the sequence axis -> (H, T, D) (the reference adds a
        leading batch axis of 1)."""
        return gather(self.k_pool, self.v_pool, self.tables[seq], self.offsets[seq], self.bs)


def gather(k_pool: np.ndarray, v_pool: np.ndarray, blocks: list[int], offset: int,
           bs: int) -> tuple[np.ndarray, np.ndarray]:
    """paged_kv.py:112-137 for one sequence: (H, offset, D) K and V."""
    H, D = k_pool.shape[1], k_pool.shape[3]
    if offset == 0:  # :101-110 empty result
        return (np.zeros((H, 0, D), dtype=k_pool.dtype), np.zeros((H, 0, D), dtype=v_pool.dtype))
    ks, vs = [], []
    remaining = offset
    for b in blocks:
        n = min(remaining, bs)
        ks.append(k_pool[b, :, :n, :])
        vs.append(v_pool[b, :, :n, :])
        remaining -= n
        if remaining <= 0:
            break
    return np.concatenate(ks, axis=1), np.concatenate(vs, axis=1)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float | None = None) -> np.ndarray:
    """paged_attention_forward's math, src/mlxz/paged_attention/attention.py:23-48.

    q: (Hq, n_q, D) float; k, v: (Hkv, T, D) float.  Query head h reads KV head
    h // (Hq // Hkv) (mx.repeat along axis 1, :30-36).  No mask (:40-42).
    scale defaults to D**-0.5 (:26-28).  Returns float64 (Hq, n_q, D); with
    T == 0 the result is zeros.
    """
    Hq, nq, D = q.shape
    Hkv, T, _ = k.shape
    if scale is None:
        scale = D ** -0.5
    if T == 0:
        return np.zeros((Hq, nq, D), dtype=np.float64)
    G = Hq // Hkv
    kk = np.repeat(np.asarray(k, dtype=np.float64), G, axis=0)
    vv = np.repeat(np.asarray(v, dtype=np.float64), G, axis=0)
    s = np.einsum("hqd,htd->hqt", np.asarray(q, dtype=np.float64), kk) * scale
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("hqt,htd->hqd", p, vv)


def paged_decode(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray, tables: np.ndarray,
                 ctx_lens: np.ndarray, dtype: str, scale: float | None = None) -> np.ndarray:
    """Batched form: for each sequence b, get_kv then attention.

    q: (B, Hq, D) or (B, n_q, Hq, D) uint16 bits of `dtype`; pools uint16 bits.
    Returns float64 with q's shape.
    """
    from .rng import to_f32

    bs = k_pool.shape[2]
    q4 = q[:, None] if q.ndim == 3 else q
    B, nq, Hq, D = q4.shape
    out = np.zeros((B, nq, Hq, D), dtype=np.float64)
    for b in range(B):
        kb, vb = gather(k_pool, v_pool, list(tables[b]), int(ctx_lens[b]), bs)
        qb = to_f32(q4[b], dtype).transpose(1, 0, 2)  # (Hq, nq, D)
        out[b] = attention(qb, to_f32(kb, dtype), to_f32(vb, dtype), scale).transpose(1, 0, 2)
    return out[:, 0] if q.ndim == 3 else out


def block_copy(pools: np.ndarray, src: list[int], dst: list[int]) -> None:
    """Copy-on-write data move: pools[:, dst[i]] = pools[:, src[i]] for a stack
    of pools [P, n_blocks, ...] (the copy BlockManager.copy_on_write leaves to
    its caller, src/mlxz/paged_attention/block_manager.py:118)."""
    for s, d in zip(src, dst):
        pools[:, d] = pools[:, s]


def block_pack(pools: np.ndarray, ids: list[int]) -> np.ndarray:
    """[n, P, block_bytes] staging image of blocks `ids` of every pool."""
    P = pools.shape[0]
    raw = pools.reshape(P, pools.shape[1], -1).view(np.uint8)
    return np.ascontiguousarray(raw[:, ids].transpose(1, 0, 2))


def block_unpack(pools: np.ndarray, ids: list[int], staging: np.ndarray) -> None:
    P = pools.shape[0]
    raw = pools.reshape(P, pools.shape[1], -1).view(np.uint8)
    for i, b in enumerate(ids):
        raw[:, b] = staging[i]


def prefill_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, start: int,
                      scale: float | None = None) -> np.ndarray:
    """Causal attention of a prompt chunk at cache offset ``start``.

    The reference runs a prompt (or a ChunkedPrefillScheduler chunk,
    src/mlxz/scheduler/chunker.py:53-76) through mlx_lm's model forward
    (mlx-lm >=0.21,<0.23, pyproject.toml:11; not vendored), whose attention is
    scaled_dot_product_attention with the causal mask of a chunk of n queries
    over a cache of ``start`` tokens: query i sees key j iff j <= start + i.

    q: (Hq, n, D) float; k, v: (Hkv, start + n, D) float.  Query token i sees
    keys [0, start + i]; query head h reads KV head h // (Hq // Hkv).  Float64.
    """
    Hq, n, D = q.shape
    Hkv = k.shape[0]
    G = Hq // Hkv
    scale = D ** -0.5 if scale is None else scale
    kk = np.repeat(k.astype(np.float64), G, axis=0)
    vv = np.repeat(v.astype(np.float64), G, axis=0)
    s = np.einsum("hqd,htd->hqt", q.astype(np.float64), kk) * scale
    T = k.shape[1]
    mask = np.arange(T)[None, :] > (start + np.arange(n))[:, None]
    s = np.where(mask[None], -np.inf, s)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("hqt,htd->hqd", p, vv)


def paged_prefill(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray, tables: np.ndarray,
                  q_start: np.ndarray, q_len: np.ndarray, ctx_lens: np.ndarray, dtype: str,
                  scale: float | None = None) -> np.ndarray:
    """Batched form: sequence b's q_len[b] query rows of q (T, Hq, D) uint16
    bits, from row q_start[b], sit at the last q_len[b] of its ctx_lens[b]
    tokens; gather its KV then prefill_attention.  Returns float64 (T, Hq, D);
    rows of no sequence stay zero."""
    from .rng import to_f32

    bs = k_pool.shape[2]
    out = np.zeros(q.shape, dtype=np.float64)
    for b in range(len(q_len)):
        n, c, r0 = int(q_len[b]), int(ctx_lens[b]), int(q_start[b])
        if n == 0:
            continue
        kb, vb = gather(k_pool, v_pool, list(tables[b]), c, bs)
        qb = to_f32(q[r0:r0 + n], dtype).transpose(1, 0, 2)  # (Hq, n, D)
        o = prefill_attention(qb, to_f32(kb, dtype), to_f32(vb, dtype), c - n, scale)
        out[r0:r0 + n] = o.transpose(1, 0, 2)
    return out
