"""The reference's decode path on the host cores, for the timed CPU baseline
(oracle side; used only by bench.py's cpu_baseline leg and --impl reference).

A vectorised torch-CPU restatement of what
src/mlxz/paged_attention/attention.py:23-48 does per sequence:
  * write the new token to its slot (paged_kv.py:85-86);
  * ``get_kv``: gather the table's blocks into contiguous (H_kv, T, D)
    (paged_kv.py:112-137) -- one index_select here;
  * GQA attention softmax(q.K^T * scale).V with query head h reading KV head
    h // G.  The reference materialises mx.repeat(K, G) (attention.py:30-36);
    here the G query heads of a KV head are batched against the un-repeated
    K/V, the same arithmetic without the G-fold copy, which makes this the
    faster (stronger) baseline.
torch runs its intra-op thread pool over all host threads it is given.
"""
from __future__ import annotations

import torch


def decode_layer(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                 tables: list[torch.Tensor], ctx: list[int], new_k: torch.Tensor,
                 new_v: torch.Tensor, scale: float) -> torch.Tensor:
    """One layer of the decode step on the CPU.

    q: (B, Hq, D) float32; pools: (n_blocks, Hkv, bs, D) (bf16/fp16);
    tables[b]: int64 block ids; new_k/new_v: (B, Hkv, D) written at position
    ctx[b]; attention covers ctx[b] + 1 tokens.  Returns (B, Hq, D) float32.
    """
    B, Hq, D = q.shape
    _, Hkv, bs, _ = k_pool.shape
    G = Hq // Hkv
    out = torch.empty(B, Hq, D, dtype=torch.float32)
    for b in range(B):
        pos = int(ctx[b])
        blk = int(tables[b][pos // bs])
        k_pool[blk, :, pos % bs] = new_k[b]
        v_pool[blk, :, pos % bs] = new_v[b]
        T = pos + 1
        idx = tables[b][: -(-T // bs)]
        K = k_pool.index_select(0, idx).permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :T].float()
        V = v_pool.index_select(0, idx).permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :T].float()
        s = torch.bmm(q[b].view(Hkv, G, D), K.transpose(1, 2)) * scale
        p = torch.softmax(s, dim=-1)
        out[b] = torch.bmm(p, V).reshape(Hq, D)
    return out
