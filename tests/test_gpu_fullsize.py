"""Parity at the benchmark sizes, against the numpy oracle, every sequence.

* C2: one layer of the 8B-shape decode step (64 sequences, ctx U[512, 8192],
  8 KV heads, GQA group 4, bf16), through the fused append + decode launch
  the step uses: the new tokens land bit-exactly in their pool slots and every
  sequence's attention is within 2e-3 of the float64 oracle (fp32 output).
* C4: one layer of the quantised step (batch 32, ctx U[4096, 16384]) at 8 and
  4 bits: pools quantised on the GPU from N(0, 1) bf16, a sample of blocks
  bit-exact to the quantisation oracle, every sequence's dequant-fused
  attention within 2e-3 of the oracle's attention over the dequantised codes.
* C5: the 70B shape as one rank of 8 holds it (1 KV head, GQA group 8, 256
  sequences, lognormal ctx up to 32768), fused append + decode, every
  sequence against the oracle.

Inputs are generated on the GPU (seeded) and copied back for the oracle.
Semantics followed: src/mlxz/paged_attention/paged_kv.py:95-137 (get_kv) and
attention.py:9-49 (GQA attention, no mask).
"""
import numpy as np
import pytest
import torch

from mlxz_b200 import ops
from oracle import paged as opaged
from oracle import quant as oq
from oracle import rng
from tests.gpu_util import attn_err, to_bits

pytestmark = pytest.mark.gpu
ATOL_REL = 2e-3
BS, D = 16, 128


def _tables(ctx_after, seed):
    """Random block tables over a pool of the blocks needed + 10 %."""
    need = [(int(c) + BS - 1) // BS for c in ctx_after]
    n_blocks = int(sum(need) * 1.1) + 2
    perm = np.random.default_rng(seed).permutation(n_blocks)
    tables = np.full((len(need), max(need)), -1, dtype=np.int32)
    used = 0
    for b, n in enumerate(need):
        tables[b, :n] = perm[used:used + n]
        used += n
    return tables, n_blocks


def _bf16(t):
    return to_bits(t)


def _decode_vs_oracle(cuda, ctx, Hkv, G, seed, invariant=False):
    """Fused append + decode of one layer; returns (worst error, pools ok)."""
    B = len(ctx)
    tables, n_blocks = _tables(ctx + 1, seed)
    g = torch.Generator(device=cuda).manual_seed(seed)
    kp = torch.randn(n_blocks, Hkv, BS, D, device=cuda, generator=g).to(torch.bfloat16)
    vp = torch.randn(n_blocks, Hkv, BS, D, device=cuda, generator=g).to(torch.bfloat16)
    q = torch.randn(B, Hkv * G, D, device=cuda, generator=g).to(torch.bfloat16)
    kn = torch.randn(B, Hkv, D, device=cuda, generator=g).to(torch.bfloat16)
    vn = torch.randn(B, Hkv, D, device=cuda, generator=g).to(torch.bfloat16)
    lens = torch.from_numpy((ctx + 1).astype(np.int32)).to(cuda)
    kp_bits, vp_bits = _bf16(kp), _bf16(vp)  # before the append
    out = ops.paged_append_decode(q, kp, vp, kn, vn, torch.from_numpy(tables).to(cuda), lens,
                                  out_dtype=torch.float32, batch_invariant=invariant)
    torch.cuda.synchronize()
    ops.check_device_errors(cuda.index or 0)
    # the oracle's append: the new token at position ctx[b] (paged_kv.py:63-93)
    kn_bits, vn_bits = _bf16(kn), _bf16(vn)
    for b in range(B):
        pos = int(ctx[b])
        blk = tables[b][pos // BS]
        kp_bits[blk, :, pos % BS] = kn_bits[b]
        vp_bits[blk, :, pos % BS] = vn_bits[b]
    pools_ok = np.array_equal(_bf16(kp), kp_bits) and np.array_equal(_bf16(vp), vp_bits)
    ref = opaged.paged_decode(_bf16(q), kp_bits, vp_bits, tables, ctx + 1, "bf16")
    o = out.cpu().numpy()
    worst = max(attn_err(torch.from_numpy(o[b]), ref[b]) for b in range(B))
    return worst, pools_ok


def test_c2_full_layer_every_sequence(cuda):
    ctx = np.random.default_rng(0).integers(512, 8193, size=64).astype(np.int64)
    worst, pools_ok = _decode_vs_oracle(cuda, ctx, Hkv=8, G=4, seed=11)
    assert pools_ok
    assert worst <= ATOL_REL, worst


def test_c2_batch_invariant_every_sequence(cuda):
    """The batch-invariant schedule (pairs cut every 512 tokens, pieces merged
    in order) at the benchmark batch."""
    ctx = np.random.default_rng(0).integers(512, 8193, size=64).astype(np.int64)
    worst, pools_ok = _decode_vs_oracle(cuda, ctx, Hkv=8, G=4, seed=13, invariant=True)
    assert pools_ok
    assert worst <= ATOL_REL, worst


def test_c5_rank_shard_every_sequence(cuda):
    z = np.random.default_rng(5).standard_normal(256)
    ctx = np.clip(np.rint(np.exp(np.log(4096) + z)), 256, 32768).astype(np.int64)
    assert ctx.max() > 16384  # the long tail is in the case
    worst, pools_ok = _decode_vs_oracle(cuda, ctx, Hkv=1, G=8, seed=12)
    assert pools_ok
    assert worst <= ATOL_REL, worst


@pytest.mark.parametrize("tc", ["1", "0"])
@pytest.mark.parametrize("bits", [8, 4])
def test_c4_quantised_full_layer_every_sequence(cuda, bits, tc, monkeypatch):
    """Both forms of the quantised decode (MLXZ_B200_QDECODE_TC: tcgen05 or
    mma.sync)."""
    monkeypatch.setenv("MLXZ_B200_QDECODE_TC", tc)
    B, Hkv, G = 32, 8, 4
    ctx = np.random.default_rng(bits).integers(4096, 16385, size=B).astype(np.int64)
    tables, n_blocks = _tables(ctx, 20 + bits)
    w = D * bits // 32
    dev = cuda
    pools = (torch.zeros(n_blocks, Hkv, BS, w, dtype=torch.int32, device=dev),
             torch.zeros(n_blocks, Hkv, BS, D // 64, dtype=torch.float16, device=dev),
             torch.zeros(n_blocks, Hkv, BS, D // 64, dtype=torch.float16, device=dev),
             torch.zeros(n_blocks, Hkv, BS, w, dtype=torch.int32, device=dev),
             torch.zeros(n_blocks, Hkv, BS, D // 64, dtype=torch.float16, device=dev),
             torch.zeros(n_blocks, Hkv, BS, D // 64, dtype=torch.float16, device=dev))
    g = torch.Generator(device=dev).manual_seed(30 + bits)
    chunk = 8192
    sample_src = {}
    check_blocks = set(int(x) for x in tables[:, 0]) | set(int(x) for x in tables[:, 7])
    for lo in range(0, n_blocks * BS, chunk):
        n = min(chunk, n_blocks * BS - lo)
        slots = torch.arange(lo, lo + n, dtype=torch.int64, device=dev)
        k = torch.randn(1, Hkv, n, D, device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn(1, Hkv, n, D, device=dev, generator=g).to(torch.bfloat16)
        ops.kv_quant_append(pools, k, v, slots)
        for blk in check_blocks:
            if lo <= blk * BS < lo + n:
                a = blk * BS - lo
                sample_src[blk] = (_bf16(k[0, :, a:a + BS]), _bf16(v[0, :, a:a + BS]))
    q = torch.randn(B, Hkv * G, D, device=dev, generator=g).to(torch.bfloat16)
    out = ops.paged_decode_q(q, pools, torch.from_numpy(tables).to(dev),
                             torch.from_numpy(ctx.astype(np.int32)).to(dev),
                             out_dtype=torch.float32)
    torch.cuda.synchronize()
    ops.check_device_errors(dev.index or 0)
    host = [p.cpu().numpy() for p in pools]
    host = [h.view(np.uint32) if h.dtype == np.int32 else h.view(np.uint16) for h in host]
    # quantise-on-append, bit-exact on a sample of blocks (whole blocks, K and V)
    for blk, (kb, vb) in sample_src.items():
        for src, base in ((kb, 0), (vb, 3)):
            qw, sc, bi = oq.quantize(src.transpose(1, 0, 2), "bf16", bits)  # [bs, H, ...]
            assert np.array_equal(host[base][blk], qw.transpose(1, 0, 2)), blk
            assert np.array_equal(host[base + 1][blk], sc.transpose(1, 0, 2)), blk
            assert np.array_equal(host[base + 2][blk], bi.transpose(1, 0, 2)), blk
    qf = rng.to_f32(_bf16(q), "bf16")
    o = out.cpu().numpy()
    worst = 0.0
    for b in range(B):
        c = int(ctx[b])
        blocks = tables[b][: (c + BS - 1) // BS]
        K = oq.dequantize(host[0][blocks], host[1][blocks], host[2][blocks], bits, D)
        V = oq.dequantize(host[3][blocks], host[4][blocks], host[5][blocks], bits, D)
        K = K.transpose(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :c]
        V = V.transpose(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :c]
        ref = opaged.attention(qf[b][:, None], K, V)[:, 0]
        worst = max(worst, attn_err(torch.from_numpy(o[b]), ref))
    assert worst <= ATOL_REL, worst
