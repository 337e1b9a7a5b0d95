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


def prefill_layer(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                  tables: list[torch.Tensor], ctx: list[int], q_len: list[int],
                  new_k: torch.Tensor, new_v: torch.Tensor, scale: float) -> torch.Tensor:
    """One layer of a chunked-prefill iteration on the CPU: what the reference
    does for a prompt chunk (ChunkedPrefillScheduler, chunker.py:53-76, then
    mlx_lm's causal attention over cache + chunk).

    q: (T, Hq, D) float32, sequences' chunks stacked; new_k/new_v: (T, Hkv, D)
    written at positions [ctx[b] - q_len[b], ctx[b]); query i of sequence b
    sees keys [0, ctx[b] - q_len[b] + i].  Returns (T, Hq, D) float32.
    """
    T, Hq, D = q.shape
    _, Hkv, bs, _ = k_pool.shape
    G = Hq // Hkv
    out = torch.empty(T, Hq, D, dtype=torch.float32)
    r = 0
    for b in range(len(ctx)):
        n, c = int(q_len[b]), int(ctx[b])
        start = c - n
        for i in range(n):
            pos = start + i
            blk = int(tables[b][pos // bs])
            k_pool[blk, :, pos % bs] = new_k[r + i]
            v_pool[blk, :, pos % bs] = new_v[r + i]
        idx = tables[b][: -(-c // bs)]
        K = k_pool.index_select(0, idx).permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :c].float()
        V = v_pool.index_select(0, idx).permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :c].float()
        qb = q[r:r + n].view(n, Hkv, G, D).permute(1, 0, 2, 3).reshape(Hkv, n * G, D)
        s = torch.bmm(qb, K.transpose(1, 2)) * scale                     # (Hkv, n*G, c)
        lim = (start + torch.arange(n)).repeat_interleave(G)             # row -> last key
        s.masked_fill_(torch.arange(c)[None, None, :] > lim[None, :, None], float("-inf"))
        p = torch.softmax(s, dim=-1)
        o = torch.bmm(p, V).view(Hkv, n, G, D).permute(1, 0, 2, 3).reshape(n, Hq, D)
        out[r:r + n] = o
        r += n
    return out
