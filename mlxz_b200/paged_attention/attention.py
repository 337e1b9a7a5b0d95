"""Paged attention entry points over the fused sm_100a decode kernel.

``paged_attention_forward`` keeps the reference signature
(src/mlxz/paged_attention/attention.py:9-49) but does not gather or repeat:
``mz_paged_decode`` reads the pool blocks through the block table directly,
query head h reading KV head h // (n_heads // n_kv_heads), with the same
default scale (head_dim ** -0.5, :26-28) and no mask (:40-42).
``paged_decode`` is the batched ragged form the continuous decode step uses.
"""
from __future__ import annotations

import torch

from .. import ops
from .paged_kv import PagedKVCache


def paged_attention_forward(query: torch.Tensor, paged_cache: PagedKVCache, seq_id: str,
                            scale: float | None = None) -> torch.Tensor:
    """Attention of ``query (1, n_heads, n_new, head_dim)`` over the cached KV
    of `seq_id`; returns ``(1, n_heads, n_new, head_dim)`` in query's dtype."""
    if query.dim() != 4 or query.shape[0] != 1:
        raise ValueError("query must be (1, n_heads, n_new_tokens, head_dim)")
    if scale is None:
        scale = query.shape[-1] ** -0.5
    q = query.to(paged_cache.device)
    n_heads, n_new = q.shape[1], q.shape[2]
    G = n_heads // paged_cache.n_kv_heads
    if G < 1 or n_heads % paged_cache.n_kv_heads:
        raise ValueError("n_heads must be a multiple of the cache's n_kv_heads")
    out = torch.empty_like(q)
    table = paged_cache.block_table_tensor([seq_id])
    ctx = paged_cache.ctx_tensor([seq_id])
    # The kernel takes up to 16 grouped query rows per KV head per launch.
    chunk = max(1, 16 // G)
    for s in range(0, n_new, chunk):
        e = min(n_new, s + chunk)
        qv = q[:, :, s:e].permute(0, 2, 1, 3)  # (1, n, H, D) view
        ov = out[:, :, s:e].permute(0, 2, 1, 3)
        ops.paged_decode(qv, paged_cache.k_pool, paged_cache.v_pool, table, ctx, scale=scale,
                         out=ov)
    return out


def paged_decode(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                 block_tables: torch.Tensor, ctx_lens: torch.Tensor, scale: float | None = None,
                 out: torch.Tensor | None = None, **kw) -> torch.Tensor:
    """Ragged batched decode: ``q [B, n_heads, D]`` against each sequence's
    first ``ctx_lens[b]`` tokens through ``block_tables[b]``."""
    return ops.paged_decode(q, k_pool, v_pool, block_tables, ctx_lens, scale=scale, out=out, **kw)
