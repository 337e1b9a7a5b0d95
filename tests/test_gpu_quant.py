"""GPU: 4/8-bit quantise-on-append (bit-exact against the oracle's stated
rules) and dequant-fused paged decode (attention over the dequantised values,
float64 oracle, same tolerance metric as the bf16 kernel)."""
import numpy as np
import pytest
import torch

from mlxz_b200 import ops
from oracle import paged as opaged
from oracle import quant as oq
from oracle import rng
from tests.gpu_util import attn_err, to_bits, to_dev

pytestmark = pytest.mark.gpu


def _pools(n_blocks, H, bs, D, bits, dev):
    w = D * bits // 32
    return (torch.zeros(n_blocks, H, bs, w, dtype=torch.int32, device=dev),
            torch.zeros(n_blocks, H, bs, D // 64, dtype=torch.float16, device=dev),
            torch.zeros(n_blocks, H, bs, D // 64, dtype=torch.float16, device=dev),
            torch.zeros(n_blocks, H, bs, w, dtype=torch.int32, device=dev),
            torch.zeros(n_blocks, H, bs, D // 64, dtype=torch.float16, device=dev),
            torch.zeros(n_blocks, H, bs, D // 64, dtype=torch.float16, device=dev))


def _np(t):
    t = t.detach().cpu()
    return t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.float16 else \
        t.numpy().view(np.uint32)


def _edge_rows(n, D, dtype):
    """Random rows plus rows with a constant group, a tiny range and large values."""
    x = rng.to_f32(rng.normal(17, (n, D), dtype), dtype).astype(np.float64)
    x[0, :64] = 0.3
    x[1, 64 % D:] = 1e-3 * np.linspace(0, 1, D - 64 % D)
    x[2] *= 1000.0
    x[3, :32] = -60000.0
    return rng.from_f64(x, dtype)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_quant_append_bit_exact(cuda, bits, D, dtype):
    H, bs, N, n = 4, 16, 12, 37
    pools = _pools(N, H, bs, D, bits, cuda)
    k = _edge_rows(H * n, D, dtype).reshape(H, n, D)
    v = rng.normal(18, (H, n, D), dtype)
    slots = rng.permutation(5, N * bs)[:n].copy()
    slots[7] = -1
    ops.kv_quant_append(pools, to_dev(k, dtype, cuda)[None], to_dev(v, dtype, cuda)[None],
                        torch.from_numpy(slots).to(cuda))
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    want = [np.zeros(tuple(t.shape), dtype=np.uint32 if t.dtype == torch.int32 else np.uint16)
            for t in pools]
    for src, base in ((k, 0), (v, 3)):
        qw, sc, bi = oq.quantize(src.transpose(1, 0, 2), dtype, bits)  # [n, H, ...]
        for i, sl in enumerate(slots):
            if sl < 0:
                continue
            want[base][sl // bs, :, sl % bs] = qw[i]
            want[base + 1][sl // bs, :, sl % bs] = sc[i]
            want[base + 2][sl // bs, :, sl % bs] = bi[i]
    for got, exp in zip(pools, want):
        assert np.array_equal(_np(got), exp)


def _quant_case(seed, ctx, Hkv, D, bits, dtype, G=4, nq=1, bs=16):
    need = [(c + bs - 1) // bs for c in ctx]
    N = max(1, int(sum(need) * 1.1) + 2)
    perm = rng.permutation(seed, N)
    tables = np.full((len(ctx), max([1] + need)), -1, dtype=np.int32)
    u = 0
    for b, nb in enumerate(need):
        tables[b, :nb] = perm[u:u + nb]
        u += nb
    kraw = rng.normal(seed, (N, Hkv, bs, D), dtype, stream=1)
    vraw = rng.normal(seed, (N, Hkv, bs, D), dtype, stream=2)
    kq, ks, kb = oq.quantize(kraw, dtype, bits)
    vq, vs, vb = oq.quantize(vraw, dtype, bits)
    q = rng.normal(seed, (len(ctx), nq, Hkv * G, D), dtype, stream=3)
    return dict(N=N, bs=bs, tables=tables, ctx=np.array(ctx, dtype=np.int32), q=q,
                host=(kq, ks, kb, vq, vs, vb),
                kdeq=oq.dequantize(kq, ks, kb, bits, D), vdeq=oq.dequantize(vq, vs, vb, bits, D))


def _dev_pools(host, dev):
    out = []
    for a in host:
        t = torch.from_numpy(a.view(np.int32) if a.dtype == np.uint32 else a.view(np.int16))
        out.append(t.view(torch.float16).to(dev) if a.dtype == np.uint16 else t.to(dev))
    return tuple(out)


def _oracle_decode(case, dtype):
    qf = rng.to_f32(case["q"], dtype)
    B, nq, Hq, D = qf.shape
    out = np.zeros((B, nq, Hq, D))
    bs = case["bs"]
    for b in range(B):
        c = int(case["ctx"][b])
        nb = (c + bs - 1) // bs
        blocks = case["tables"][b][:nb]
        K = case["kdeq"][blocks].transpose(1, 0, 2, 3).reshape(case["kdeq"].shape[1], -1, D)[:, :c]
        V = case["vdeq"][blocks].transpose(1, 0, 2, 3).reshape(case["vdeq"].shape[1], -1, D)[:, :c]
        out[b] = opaged.attention(qf[b].transpose(1, 0, 2), K, V).transpose(1, 0, 2)
    return out


QCASES = [
    (8, 128, 4, "bf16", [513, 1, 15, 16, 17, 300, 2048, 0], 0),
    (8, 128, 4, "bf16", [513, 1, 15, 16, 17, 300, 2048, 0], 12),
    (4, 128, 4, "bf16", [513, 1, 15, 16, 17, 300, 2048, 0], 0),
    (8, 128, 8, "bf16", [77, 1000, 3], 0),
    (4, 128, 1, "f16", [77, 1000, 3], 8),
    (8, 64, 4, "f16", [38, 129, 301, 512], 0),
    (4, 64, 16, "bf16", [50, 9], 0),
]


@pytest.mark.parametrize("bits,D,G,dtype,ctx,nw", QCASES)
@pytest.mark.parametrize("out32", [True, False])
@pytest.mark.parametrize("form", ["mma_sync", "tcgen05"])
def test_paged_decode_q_vs_oracle(cuda, bits, D, G, dtype, ctx, nw, out32, form, monkeypatch):
    """Every case through the default mma.sync kernel (integer Q.K^T, 1, 2 or
    4 groups of four query rows) and through the opt-in tcgen05 form (head_dim
    128; other shapes fall back to the mma.sync kernel)."""
    monkeypatch.setenv("MLXZ_B200_QDECODE_TC", "1" if form == "tcgen05" else "0")
    Hkv = 2 if G == 16 else 4
    case = _quant_case(40 + bits + D + G, ctx, Hkv, D, bits, dtype, G=G)
    pools = _dev_pools(case["host"], cuda)
    q = to_dev(case["q"][:, 0], dtype, cuda)
    out = ops.paged_decode_q(q, pools, torch.from_numpy(case["tables"]).to(cuda),
                             torch.from_numpy(case["ctx"]).to(cuda), num_warps=nw,
                             out_dtype=torch.float32 if out32 else None)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    ref = _oracle_decode(case, dtype)[:, 0]
    assert attn_err(out, ref) <= 2e-3
    for b, c in enumerate(ctx):
        if c == 0:
            assert torch.count_nonzero(out[b]) == 0


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("bs", [32, 64])
@pytest.mark.parametrize("form", ["mma_sync", "tcgen05"])
def test_paged_decode_q_block_sizes(cuda, bits, bs, form, monkeypatch):
    """Blocks of several 16-token tiles: a tile's pool row is the block's row
    plus the tile's offset inside the block, and ragged lengths end inside a
    block."""
    monkeypatch.setenv("MLXZ_B200_QDECODE_TC", "1" if form == "tcgen05" else "0")
    ctx = [1, 47, bs, bs + 1, 3 * bs - 5, 700]
    case = _quant_case(60 + bits + bs, ctx, 4, 128, bits, "bf16", bs=bs)
    pools = _dev_pools(case["host"], cuda)
    q = to_dev(case["q"][:, 0], "bf16", cuda)
    out = ops.paged_decode_q(q, pools, torch.from_numpy(case["tables"]).to(cuda),
                             torch.from_numpy(case["ctx"]).to(cuda), out_dtype=torch.float32)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    ref = _oracle_decode(case, "bf16")[:, 0]
    assert attn_err(out, ref) <= 2e-3


def test_paged_decode_q_multi_query_and_paged_append(cuda):
    """Decode-step append through block tables, then attend with 2 query
    tokens per sequence."""
    bits, D, G, Hkv, dtype = 8, 128, 4, 2, "bf16"
    ctx = [40, 200, 7]
    case = _quant_case(91, ctx, Hkv, D, bits, dtype, G=G, nq=2)
    pools = _dev_pools(case["host"], cuda)
    tables = torch.from_numpy(case["tables"]).to(cuda)
    # overwrite the last token of each sequence through the paged append
    nk = rng.normal(92, (3, Hkv, D), dtype, stream=1)
    nv = rng.normal(92, (3, Hkv, D), dtype, stream=2)
    pos = torch.tensor([c - 1 for c in ctx], dtype=torch.int32, device=cuda)
    ops.kv_quant_append_paged(pools, to_dev(nk, dtype, cuda), to_dev(nv, dtype, cuda), tables, pos)
    host = [a.copy() for a in case["host"]]
    for b, c in enumerate(ctx):
        blk = case["tables"][b][(c - 1) // 16]
        for src, base in ((nk, 0), (nv, 3)):
            qw, sc, bi = oq.quantize(src[b], dtype, bits)
            host[base][blk, :, (c - 1) % 16] = qw
            host[base + 1][blk, :, (c - 1) % 16] = sc
            host[base + 2][blk, :, (c - 1) % 16] = bi
    torch.cuda.synchronize()
    for got, exp in zip(pools, host):
        assert np.array_equal(_np(got), exp)
    case["kdeq"] = oq.dequantize(host[0], host[1], host[2], bits, D)
    case["vdeq"] = oq.dequantize(host[3], host[4], host[5], bits, D)
    q = to_dev(case["q"], dtype, cuda)
    out = ops.paged_decode_q(q, pools, tables, torch.from_numpy(case["ctx"]).to(cuda),
                             out_dtype=torch.float32)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    assert attn_err(out, _oracle_decode(case, dtype)) <= 2e-3


@pytest.mark.parametrize("bits", [8, 4])
def test_paged_decode_q_reads_any_affine_codes(cuda, bits):
    """The dequant-fused decode depends only on w = scale * q + bias, not on
    how a quantiser chose the pair: groups with negative scales and a group
    edge as the bias (the form another quantiser may write) decode like the
    oracle's dequantisation of the same codes."""
    ctx, Hkv, D, G, dtype = [700, 33, 2049, 1], 4, 128, 4, "bf16"
    case = _quant_case(77 + bits, ctx, Hkv, D, bits, dtype, G=G)
    g = np.random.default_rng(bits)
    top = 2 ** bits - 1
    host = list(case["host"])
    for base in (0, 3):
        shape = host[base + 1].shape
        mag = (np.abs(g.standard_normal(shape)) * 3.0 + 0.5) / top
        neg = g.random(shape) < 0.5
        scale = np.where(neg, -mag, mag).astype(np.float16)
        # bias: the group's max when the scale is negative (w = bias at q = 0
        # and falls as q grows), its min otherwise
        edge = np.where(neg, 1.0, -1.0) * np.abs(g.standard_normal(shape)) * 2.0
        host[base + 1] = scale.view(np.uint16)
        host[base + 2] = edge.astype(np.float16).view(np.uint16)
        host[base] = g.integers(0, 2 ** 32, size=host[base].shape, dtype=np.uint64
                                ).astype(np.uint32)
    case["host"] = tuple(host)
    case["kdeq"] = oq.dequantize(host[0], host[1], host[2], bits, D)
    case["vdeq"] = oq.dequantize(host[3], host[4], host[5], bits, D)
    pools = _dev_pools(case["host"], cuda)
    q = to_dev(case["q"][:, 0], dtype, cuda)
    out = ops.paged_decode_q(q, pools, torch.from_numpy(case["tables"]).to(cuda),
                             torch.from_numpy(case["ctx"]).to(cuda), out_dtype=torch.float32)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    assert attn_err(out, _oracle_decode(case, dtype)[:, 0]) <= 2e-3


# The tensor-core form (head_dim 128; 1, 2, 4, 8 or 16 query rows per KV head):
# query rows from several tokens, every row count it is built for, capped
# grids (many split pairs, merged by the last CTA), and the same inputs through
# the mma.sync kernel.
TC_CASES = [
    # bits, G, n_q, ctx, num_warps
    (8, 2, 1, [513, 1, 127, 128, 129, 300, 4095, 0], 0),
    (4, 2, 1, [513, 1, 127, 128, 129, 300, 4095, 0], 0),
    (8, 4, 2, [700, 33, 2049], 0),
    (4, 8, 2, [700, 33, 2049], 0),
    (8, 16, 1, [1000, 5], 0),
    (4, 16, 1, [1000, 5], 0),
    (8, 4, 1, [5000, 3000, 129, 1], 8),
    (4, 4, 1, [5000, 3000, 129, 1], 20),
]


@pytest.mark.parametrize("bits,G,nq,ctx,nw", TC_CASES)
def test_paged_decode_q_tensor_core_rows(cuda, bits, G, nq, ctx, nw, monkeypatch):
    monkeypatch.setenv("MLXZ_B200_QDECODE_TC", "1")
    Hkv = 2 if G * nq >= 16 else 4
    case = _quant_case(90 + bits + G + nq, ctx, Hkv, 128, bits, "bf16", G=G, nq=nq)
    pools = _dev_pools(case["host"], cuda)
    q = to_dev(case["q"], "bf16", cuda)  # [B, n_q, Hq, D]
    tables = torch.from_numpy(case["tables"]).to(cuda)
    lens = torch.from_numpy(case["ctx"]).to(cuda)
    out = ops.paged_decode_q(q, pools, tables, lens, num_warps=nw, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    assert attn_err(out, _oracle_decode(case, "bf16")) <= 2e-3
    for b, c in enumerate(ctx):
        if c == 0:
            assert torch.count_nonzero(out[b]) == 0


def test_paged_decode_q_tensor_core_matches_mma_sync_kernel(cuda, monkeypatch):
    """MLXZ_B200_QDECODE_TC selects the form (1: tcgen05, 0: mma.sync): both
    agree with each other within the attention tolerance on the same inputs."""
    ctx = [3000, 17, 129, 8000]
    case = _quant_case(123, ctx, 8, 128, 8, "bf16", G=4)
    pools = _dev_pools(case["host"], cuda)
    q = to_dev(case["q"][:, 0], "bf16", cuda)
    tables = torch.from_numpy(case["tables"]).to(cuda)
    lens = torch.from_numpy(case["ctx"]).to(cuda)
    monkeypatch.setenv("MLXZ_B200_QDECODE_TC", "1")
    tc = ops.paged_decode_q(q, pools, tables, lens, out_dtype=torch.float32)
    monkeypatch.setenv("MLXZ_B200_QDECODE_TC", "0")
    legacy = ops.paged_decode_q(q, pools, tables, lens, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    assert attn_err(tc, legacy.cpu().numpy()) <= 2e-3
    assert attn_err(tc, _oracle_decode(case, "bf16")[:, 0]) <= 2e-3
