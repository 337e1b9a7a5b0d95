"""GPU parity: append / gather / decode attention / block moves through the
C ABI, against the golden fixtures (the reference's own outputs) and the CPU
oracle on the same seeded inputs.

Tolerances: data movement is bit-exact (SHA-256 or array equality).
Attention: max(|out - ref| - u*|ref|, 0) / max|ref| <= 2e-3 against the
float64 oracle, u = unit roundoff of the output dtype (2^-8 bf16, 2^-11 fp16,
0 for fp32 outputs, which therefore meet 2e-3 outright).
"""
import hashlib
import json

import numpy as np
import pytest
import torch

from mlxz_b200 import ops
from mlxz_b200._native import DeviceError
from mlxz_b200.paged_attention import (BlockManager, OutOfBlocksError, PagedKVCache,
                                       paged_attention_forward)
from oracle import paged as opaged
from oracle import rng
from tests.conftest import GOLDEN
from tests.gpu_util import TORCH, attn_err, random_paged_case, sha_t, to_bits, to_dev
from tests.test_oracle_golden import c1_inputs

pytestmark = pytest.mark.gpu
ATOL_REL = 2e-3


def test_c1_golden_through_reference_api(cuda):
    """C1 (1B shape, fp16, 4 ragged sequences, random block tables): append,
    gather and attention through PagedKVCache / paged_attention_forward."""
    g = json.loads((GOLDEN / "c1_layer.json").read_text())
    gold_attn = np.load(GOLDEN / "c1_layer_attn.npy")
    inp = c1_inputs()
    bm = BlockManager(inp["n_blocks"], inp["bs"])
    cache = PagedKVCache(bm, inp["H"], inp["D"], dtype=torch.float16, device=cuda)
    for b in range(4):
        sid = f"seq{b}"
        cache._block_tables[sid] = list(inp["tables"][b])  # injected, as in the fixture
        cache._offsets[sid] = 0
        cache.append_kv(sid, to_dev(inp["pre_k"][b], "f16", cuda)[None],
                        to_dev(inp["pre_v"][b], "f16", cuda)[None])
    for b in range(4):
        sid = f"seq{b}"
        cache.append_kv(sid, to_dev(inp["new_k"][b], "f16", cuda)[None],
                        to_dev(inp["new_v"][b], "f16", cuda)[None])
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    assert sha_t(cache.k_pool) == g["k_pool_sha256"]
    assert sha_t(cache.v_pool) == g["v_pool_sha256"]
    for b in range(4):
        sid = f"seq{b}"
        k, v = cache.get_kv(sid)
        assert list(k.shape) == g["seqs"][b]["shape"]
        assert sha_t(k) == g["seqs"][b]["k_sha256"]
        assert sha_t(v) == g["seqs"][b]["v_sha256"]
        q = to_dev(inp["q"][b], "f16", cuda)[None]
        out = paged_attention_forward(q, cache, sid, scale=g["scale"])
        assert out.shape == (1, 32, 1, 64) and out.dtype == torch.float16
        assert attn_err(out[0], gold_attn[b]) <= ATOL_REL
        # fp32 output path of the same kernel
        out32 = ops.paged_decode(q[:, :, 0, :], cache.k_pool, cache.v_pool,
                                 cache.block_table_tensor([sid]), cache.ctx_tensor([sid]),
                                 scale=g["scale"], out_dtype=torch.float32)
        assert attn_err(out32[0], gold_attn[b][:, 0, :]) <= ATOL_REL
    ops.check_device_errors(0)


def test_bm_paged_replay_through_api(cuda):
    """The reference's BlockManager-driven scenario (block growth, free,
    reuse of freed blocks) replayed through the product API: identical block
    tables, offsets, stats and pool bytes after every operation."""
    g = json.loads((GOLDEN / "bm_paged.json").read_text())
    c = g["config"]
    dt = TORCH[c["dtype"]]
    bm = BlockManager(c["n_blocks"], c["bs"])
    cache = PagedKVCache(bm, c["H"], c["D"], dtype=dt, device=cuda)
    for rec in g["ops"]:
        sid = rec["seq"]
        if rec["op"] == "alloc":
            cache.allocate_sequence(sid, rec["n"])
        elif rec["op"] == "free":
            cache.free_sequence(sid)
        else:
            n = rec["n"]
            k = rng.normal(g["seeds"]["k"], (c["H"], n, c["D"]), c["dtype"], stream=rec["k_stream"])
            v = rng.normal(g["seeds"]["v"], (c["H"], n, c["D"]), c["dtype"], stream=rec["k_stream"])
            cache.append_kv(sid, to_dev(k, c["dtype"], cuda)[None], to_dev(v, c["dtype"], cuda)[None])
        assert {s: cache.get_block_table(s) for s in sorted(cache._block_tables)} == rec["tables"]
        assert {s: cache.get_offset(s) for s in sorted(cache._offsets)} == rec["offsets"]
        assert cache.stats == rec["stats"]
        assert sha_t(cache.k_pool) == rec["k_pool_sha256"]
        assert sha_t(cache.v_pool) == rec["v_pool_sha256"]
    attn = np.load(GOLDEN / "bm_paged_attn.npy")
    for i, sid in enumerate(g["attn_order"]):
        k, v = cache.get_kv(sid)
        gg = g["gathers"][sid]
        assert sha_t(k) == gg["k_sha256"] and sha_t(v) == gg["v_sha256"]
        q = rng.normal(g["seeds"]["q"], (c["Hq"], 1, c["D"]), c["dtype"], stream=gg["q_stream"])
        out = paged_attention_forward(to_dev(q, c["dtype"], cuda)[None], cache, sid)
        assert attn_err(out[0], attn[i]) <= ATOL_REL
    ops.check_device_errors(0)


def test_append_out_of_blocks_partial_effect(cuda):
    """Running out of blocks mid-append: earlier rows written, offset kept,
    OutOfBlocksError raised (reference loop semantics)."""
    bm = BlockManager(2, 16)
    cache = PagedKVCache(bm, 2, 64, dtype=torch.bfloat16, device=cuda)
    cache.allocate_sequence("s", 1)
    k = torch.randn(1, 2, 40, 64, device=cuda).to(torch.bfloat16)
    with pytest.raises(OutOfBlocksError):
        cache.append_kv("s", k, k)
    assert cache.get_offset("s") == 0
    tab = cache.get_block_table("s")
    assert len(tab) == 2
    torch.cuda.synchronize()
    got = cache.k_pool[tab].permute(1, 0, 2, 3).reshape(2, 32, 64)
    assert torch.equal(got, k[0, :, :32])


DECODE_CASES = [
    # dtype, D, G, bs, ctx list, num_warps
    ("bf16", 128, 4, 16, [513, 1, 15, 16, 17, 100, 2048, 777], 0),
    ("bf16", 128, 4, 16, [513, 1, 15, 16, 17, 100, 2048, 777], 8),
    ("bf16", 128, 4, 16, [513, 1, 15, 16, 17, 100, 2048, 777], 12),
    ("bf16", 128, 8, 16, [300, 4096, 5, 0, 33], 0),
    ("bf16", 128, 1, 32, [300, 64, 5, 1000], 4),
    ("bf16", 128, 2, 64, [129, 64, 1], 0),
    ("f16", 64, 4, 16, [38, 129, 301, 512], 0),
    ("f16", 64, 4, 16, [38, 129, 301, 512], 4),
    ("f16", 128, 16, 16, [70, 3], 0),
    ("bf16", 64, 8, 16, [0, 0, 45], 0),
]


@pytest.mark.parametrize("dtype,D,G,bs,ctx,nw", DECODE_CASES)
@pytest.mark.parametrize("out32", [False, True])
def test_paged_decode_vs_oracle(cuda, dtype, D, G, bs, ctx, nw, out32):
    Hkv = 2 if G == 16 else 4
    case = random_paged_case(7 + len(ctx) + D + G, len(ctx), Hkv, D, bs, ctx, dtype, G=G)
    kp, vp = to_dev(case["kp"], dtype, cuda), to_dev(case["vp"], dtype, cuda)
    q = to_dev(case["q"][:, 0], dtype, cuda)
    tables = torch.from_numpy(case["tables"]).to(cuda)
    ctx_t = torch.from_numpy(case["ctx"]).to(cuda)
    out = ops.paged_decode(q, kp, vp, tables, ctx_t, num_warps=nw,
                           out_dtype=torch.float32 if out32 else None)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    ref = opaged.paged_decode(case["q"][:, 0], case["kp"], case["vp"], case["tables"], case["ctx"],
                              dtype)
    assert attn_err(out, ref) <= ATOL_REL
    # zero-context sequences produce exact zeros
    for b, c in enumerate(ctx):
        if c == 0:
            assert torch.count_nonzero(out[b]) == 0


def test_paged_decode_multi_query_rows(cuda):
    """n_q query tokens per sequence (no mask) and the 16-row chunking of
    paged_attention_forward."""
    dtype, D, G, Hkv = "bf16", 128, 4, 2
    case = random_paged_case(99, 3, Hkv, D, 16, [40, 200, 7], dtype, nq=3, G=G)
    kp, vp = to_dev(case["kp"], dtype, cuda), to_dev(case["vp"], dtype, cuda)
    q = to_dev(case["q"], dtype, cuda)  # [B, 3, Hq, D]
    out = ops.paged_decode(q, kp, vp, torch.from_numpy(case["tables"]).to(cuda),
                           torch.from_numpy(case["ctx"]).to(cuda), out_dtype=torch.float32)
    ref = opaged.paged_decode(case["q"], case["kp"], case["vp"], case["tables"], case["ctx"], dtype)
    assert attn_err(out, ref) <= ATOL_REL
    # through the reference-shaped API with 5 query tokens (G=4 -> chunks of 4)
    bm = BlockManager(64, 16)
    cache = PagedKVCache(bm, Hkv, D, dtype=torch.bfloat16, device=cuda)
    cache.allocate_sequence("x")
    kk = torch.randn(1, Hkv, 150, D, device=cuda).to(torch.bfloat16)
    vv = torch.randn(1, Hkv, 150, D, device=cuda).to(torch.bfloat16)
    cache.append_kv("x", kk, vv)
    qq = torch.randn(1, Hkv * G, 5, D, device=cuda).to(torch.bfloat16)
    o = paged_attention_forward(qq, cache, "x")
    r = opaged.attention(qq[0].float().cpu().numpy(), kk[0].float().cpu().numpy(),
                         vv[0].float().cpu().numpy())
    assert attn_err(o[0], r) <= ATOL_REL


@pytest.mark.parametrize("dtype,H,D,bs", [("bf16", 8, 128, 16), ("f16", 8, 64, 16),
                                          ("bf16", 3, 24, 8), ("f16", 2, 7, 5)])
def test_batched_append_and_gather_bit_exact(cuda, dtype, H, D, bs):
    ctx = [0, 1, 15, 16, 33, 100]
    B = len(ctx)
    case = random_paged_case(31 + D, B, H, D, bs, [c + 1 for c in ctx], dtype, G=1)
    kp, vp = to_dev(case["kp"], dtype, cuda), to_dev(case["vp"], dtype, cuda)
    newk = rng.normal(41, (B, H, D), dtype, stream=1)
    newv = rng.normal(41, (B, H, D), dtype, stream=2)
    tables = torch.from_numpy(case["tables"]).to(cuda)
    pos = torch.tensor(ctx, dtype=torch.int32, device=cuda)
    ops.kv_append_paged(kp, vp, to_dev(newk, dtype, cuda), to_dev(newv, dtype, cuda), tables, pos)
    # oracle
    okp, ovp = case["kp"].copy(), case["vp"].copy()
    for b in range(B):
        blk = case["tables"][b][ctx[b] // bs]
        okp[blk, :, ctx[b] % bs] = newk[b]
        ovp[blk, :, ctx[b] % bs] = newv[b]
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    assert np.array_equal(to_bits(kp), okp) and np.array_equal(to_bits(vp), ovp)
    lens = [c + 1 for c in ctx]
    ok, ov = ops.kv_gather(kp, vp, tables, torch.tensor(lens, dtype=torch.int32, device=cuda), lens)
    ok, ov = to_bits(ok).reshape(-1), to_bits(ov).reshape(-1)
    off = 0
    for b in range(B):
        gk, gv = opaged.gather(okp, ovp, list(case["tables"][b]), lens[b], bs)
        n = gk.size
        assert np.array_equal(ok[off:off + n], gk.reshape(-1))
        assert np.array_equal(ov[off:off + n], gv.reshape(-1))
        off += n


def test_slot_append_strided_input(cuda):
    """mz_kv_append with a non-contiguous (1, H, n, D) view and skipped slots."""
    H, D, bs, N = 4, 64, 16, 10
    kp = torch.zeros(N, H, bs, D, dtype=torch.float16, device=cuda)
    vp = torch.zeros_like(kp)
    big = torch.randn(1, 2 * H, 12, D, device=cuda).half()
    k = big[:, ::2]  # strided head axis
    v = big[:, 1::2]
    slots = torch.tensor([5, 17, -1, 40, 41, 159, 0, 1, 2, 3, 100, 101], dtype=torch.int64,
                         device=cuda)
    ops.kv_append(kp, vp, k, v, slots)
    torch.cuda.synchronize()
    okp = np.zeros((N, H, bs, D), dtype=np.uint16)
    okv = okp.copy()
    kb, vb = to_bits(k[0]), to_bits(v[0])
    for i, s in enumerate(slots.tolist()):
        if s >= 0:
            okp[s // bs, :, s % bs] = kb[:, i]
            okv[s // bs, :, s % bs] = vb[:, i]
    assert np.array_equal(to_bits(kp), okp) and np.array_equal(to_bits(vp), okv)


def test_block_copy_pack_unpack_bit_exact(cuda):
    pools_np = rng.normal(3, (6, 20, 8, 16, 128), "bf16")  # 3 layers x (K, V)
    pools = to_dev(pools_np, "bf16", cuda)
    src = torch.tensor([1, 2, 3, 19], dtype=torch.int32, device=cuda)
    dst = torch.tensor([10, 11, 0, 12], dtype=torch.int32, device=cuda)
    ops.block_copy(pools, src, dst)
    opaged.block_copy(pools_np, [1, 2, 3, 19], [10, 11, 0, 12])
    torch.cuda.synchronize()
    assert np.array_equal(to_bits(pools), pools_np)
    ids = torch.tensor([4, 0, 17], dtype=torch.int32, device=cuda)
    st = ops.block_pack(pools, ids)
    torch.cuda.synchronize()
    assert np.array_equal(st.cpu().numpy(), opaged.block_pack(pools_np, [4, 0, 17]))
    fresh = torch.zeros_like(pools)
    ops.block_unpack(fresh, ids, st)
    torch.cuda.synchronize()
    for b in (4, 0, 17):
        assert torch.equal(fresh[:, b], pools[:, b])
    ops.check_device_errors(0)


def test_device_error_word_reports_bad_block_ids(cuda):
    """Out-of-range table entries are skipped by the kernels' own bounds
    checks and reported in the device error word (no trap)."""
    kp = torch.zeros(4, 2, 16, 64, dtype=torch.bfloat16, device=cuda)
    vp = torch.zeros_like(kp)
    tables = torch.tensor([[0, 9]], dtype=torch.int32, device=cuda)
    ctx = torch.tensor([20], dtype=torch.int32, device=cuda)
    q = torch.randn(1, 8, 64, device=cuda).to(torch.bfloat16)
    ops.paged_decode(q, kp, vp, tables, ctx)
    torch.cuda.synchronize()
    with pytest.raises(DeviceError):
        ops.check_device_errors(0)
    ops.reset_workspaces()
    pos = torch.tensor([200], dtype=torch.int32, device=cuda)
    ops.kv_append_paged(kp, vp, q[:, :2], q[:, :2], tables, pos)
    torch.cuda.synchronize()
    with pytest.raises(DeviceError):
        ops.check_device_errors(0)
    ops.check_device_errors(0)  # cleared


def test_decode_full_size_properties(cuda):
    """8B-shape layer at the benchmark batch (64 sequences, ctx in [512, 8192]):
    constant V gives exactly that constant; a sample of sequences matches a
    torch fp32 reference gathered through torch indexing."""
    B, Hkv, G, D, bs = 64, 8, 4, 128, 16
    gen = torch.Generator().manual_seed(0)
    ctx = torch.randint(512, 8193, (B,), generator=gen)
    need = (ctx + bs - 1) // bs
    n_blocks = int(need.sum().item() * 1.1)
    perm = torch.randperm(n_blocks, generator=gen)
    tables = torch.full((B, int(need.max())), -1, dtype=torch.int32)
    used = 0
    for b in range(B):
        tables[b, : need[b]] = perm[used:used + need[b]].int()
        used += int(need[b])
    kp = torch.randn(n_blocks, Hkv, bs, D, device=cuda).to(torch.bfloat16)
    vp = torch.full_like(kp, 0.375)
    q = torch.randn(B, Hkv * G, D, device=cuda).to(torch.bfloat16)
    tab_d, ctx_d = tables.to(cuda), ctx.int().to(cuda)
    out = ops.paged_decode(q, kp, vp, tab_d, ctx_d, out_dtype=torch.float32)
    # P.V carries P as a bf16 hi+lo pair (~16 significant bits) while the
    # normaliser sums fp32 P, so a constant V comes back within ~1e-5.
    dev_max = float((out - 0.375).abs().max())
    assert dev_max <= 0.375 * 1e-4, dev_max
    vp.normal_()
    out = ops.paged_decode(q, kp, vp, tab_d, ctx_d, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    for b in (0, 17, 63):
        blocks = tables[b, : need[b]].long().to(cuda)
        K = kp[blocks].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, : ctx[b]].float()
        V = vp[blocks].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, : ctx[b]].float()
        Kr, Vr = K.repeat_interleave(G, 0), V.repeat_interleave(G, 0)
        s = torch.einsum("hd,htd->ht", q[b].float(), Kr) * D ** -0.5
        ref = torch.einsum("ht,htd->hd", torch.softmax(s, -1), Vr)
        assert attn_err(out[b], ref.cpu().numpy()) <= ATOL_REL


@pytest.mark.parametrize("nw", [0, 4, 40, 400])
def test_fused_append_decode_matches_separate_launches(cuda, nw):
    """mz_paged_append_decode = mz_kv_append_paged then mz_paged_decode:
    identical pools (bit-exact) and attention within tolerance, for warp
    counts that make the schedule all-static, mixed, or all-dynamic."""
    B, Hkv, G, D, bs = 12, 8, 4, 128, 16
    lengths = [1, 15, 16, 17, 100, 511, 512, 513, 2000, 33, 7, 4095]
    case = random_paged_case(77, B, Hkv, D, bs, lengths, "bf16", G=G)
    kp, vp = to_dev(case["kp"], "bf16", cuda), to_dev(case["vp"], "bf16", cuda)
    kp2, vp2 = kp.clone(), vp.clone()
    nk_bits = rng.normal(78, (B, Hkv, D), "bf16", stream=1)
    nv_bits = rng.normal(78, (B, Hkv, D), "bf16", stream=2)
    nk, nv = to_dev(nk_bits, "bf16", cuda), to_dev(nv_bits, "bf16", cuda)
    q = to_dev(case["q"][:, 0], "bf16", cuda)
    tables = torch.from_numpy(case["tables"]).to(cuda)
    lens = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    out = ops.paged_append_decode(q, kp, vp, nk, nv, tables, lens, num_warps=nw,
                                  out_dtype=torch.float32)
    ops.kv_append_paged(kp2, vp2, nk, nv, tables, lens - 1)
    out2 = ops.paged_decode(q, kp2, vp2, tables, lens, num_warps=nw, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    assert torch.equal(kp, kp2) and torch.equal(vp, vp2)
    assert attn_err(out, out2.cpu().numpy()) <= ATOL_REL
    okp, ovp = case["kp"].copy(), case["vp"].copy()
    for b in range(B):
        pos = lengths[b] - 1
        blk = case["tables"][b][pos // bs]
        okp[blk, :, pos % bs] = nk_bits[b]
        ovp[blk, :, pos % bs] = nv_bits[b]
    ref = opaged.paged_decode(case["q"][:, 0], okp, ovp, case["tables"], np.array(lengths), "bf16")
    assert attn_err(out, ref) <= ATOL_REL


@pytest.mark.parametrize("nw,static_pct,min_chunk", [(0, 100, 16), (0, 85, 16), (8, 60, 4),
                                                     (1000, 70, 1), (40, 1, 16)])
def test_decode_many_ragged_sequences_dynamic_schedule(cuda, monkeypatch, nw, static_pct,
                                                       min_chunk):
    """Many short and long sequences (pairs cut by static shares and dynamic
    chunks claimed by ticket) against the oracle, twice in a row on the same
    workspace so the self-resetting counters are exercised."""
    monkeypatch.setenv("MLXZ_B200_DECODE_STATIC_PCT", str(static_pct))
    monkeypatch.setenv("MLXZ_B200_DECODE_MIN_CHUNK", str(min_chunk))
    dtype, D, G, Hkv, bs = "bf16", 128, 4, 2, 16
    ctx = [int(x) for x in rng.randint(21, 150, 0, 1200)]
    ctx[3] = 0
    ctx[10] = 1
    case = random_paged_case(21, len(ctx), Hkv, D, bs, ctx, dtype, G=G)
    kp, vp = to_dev(case["kp"], dtype, cuda), to_dev(case["vp"], dtype, cuda)
    q = to_dev(case["q"][:, 0], dtype, cuda)
    tables = torch.from_numpy(case["tables"]).to(cuda)
    ctx_t = torch.from_numpy(case["ctx"]).to(cuda)
    ref = opaged.paged_decode(case["q"][:, 0], case["kp"], case["vp"], case["tables"], case["ctx"],
                              dtype)
    for _ in range(2):
        out = ops.paged_decode(q, kp, vp, tables, ctx_t, num_warps=nw, out_dtype=torch.float32)
        torch.cuda.synchronize()
        ops.check_device_errors(0)
        assert attn_err(out, ref) <= ATOL_REL


@pytest.mark.parametrize("G,static_pct", [(8, 100), (8, 85), (16, 85), (4, 85)])
def test_decode_few_long_pairs_many_piece_merges(cuda, monkeypatch, G, static_pct):
    """Three sequences of up to 30k tokens on the full default grid: every
    pair is cut into hundreds of pieces, so a merge stages its pieces into the
    stage ring over many rounds (up to 16 rows per piece); the dynamic split
    falls back to static here (pairs far longer than a warp's share)."""
    monkeypatch.setenv("MLXZ_B200_DECODE_STATIC_PCT", str(static_pct))
    dtype, D, Hkv, bs = "bf16", 128, 1, 16
    ctx = [30000, 20011, 5]
    case = random_paged_case(71, len(ctx), Hkv, D, bs, ctx, dtype, G=G)
    kp, vp = to_dev(case["kp"], dtype, cuda), to_dev(case["vp"], dtype, cuda)
    q = to_dev(case["q"][:, 0], dtype, cuda)
    tables = torch.from_numpy(case["tables"]).to(cuda)
    ctx_t = torch.from_numpy(case["ctx"]).to(cuda)
    ref = opaged.paged_decode(case["q"][:, 0], case["kp"], case["vp"], case["tables"], case["ctx"],
                              dtype)
    for _ in range(2):
        out = ops.paged_decode(q, kp, vp, tables, ctx_t, out_dtype=torch.float32)
        torch.cuda.synchronize()
        ops.check_device_errors(0)
        assert attn_err(out, ref) <= ATOL_REL


def test_workspaces_of_different_sizes_do_not_mix(cuda):
    """Calls with different pair counts and group sizes, interleaved, each
    against the oracle: the workspaces handed out are per layout, so one
    call's partials never sit where another expects zeroed counters."""
    shapes = [(3, 1, 8, [30000, 77, 4100]), (40, 4, 4, None), (9, 8, 2, None)]
    cases = []
    for i, (B, Hkv, G, ctx) in enumerate(shapes):
        ctx = ctx or [int(x) for x in rng.randint(90 + i, B, 1, 3000)]
        case = random_paged_case(91 + i, B, Hkv, 128, 16, ctx, "bf16", G=G)
        ref = opaged.paged_decode(case["q"][:, 0], case["kp"], case["vp"], case["tables"],
                                  case["ctx"], "bf16")
        dev = [to_dev(case[k], "bf16", cuda) for k in ("kp", "vp")]
        cases.append((to_dev(case["q"][:, 0], "bf16", cuda), *dev,
                      torch.from_numpy(case["tables"]).to(cuda),
                      torch.from_numpy(case["ctx"]).to(cuda), ref))
    for rnd in range(2):
        for q, kp, vp, tables, ctx_t, ref in (cases if rnd == 0 else cases[::-1]):
            out = ops.paged_decode(q, kp, vp, tables, ctx_t, out_dtype=torch.float32)
            torch.cuda.synchronize()
            ops.check_device_errors(0)
            assert attn_err(out, ref) <= ATOL_REL


def test_decode_step_multi_layer_with_table_growth(cuda):
    """PagedDecodeStep over 2 layers for 20 steps with advance(): appends cross
    block boundaries (tables grow through the BlockManager) and every step's
    output matches the oracle replaying the same appends."""
    from mlxz_b200.engine import PagedDecodeStep, PagedKVStore

    L, Hkv, G, D, bs = 2, 2, 4, 128, 16
    Hq = Hkv * G
    offsets = [0, 15, 16, 31, 100, 5]
    store = PagedKVStore(L, 64, Hkv, D, bs, torch.bfloat16, cuda, init="zeros")
    init = rng.normal(61, tuple(store.pools.shape), "bf16")
    store.pools.copy_(to_dev(init, "bf16", cuda))
    for i, o in enumerate(offsets):
        store.add_sequence(f"r{i}", o)
    ids = [f"r{i}" for i in range(len(offsets))]
    step = PagedDecodeStep(store, ids, Hq, max_blocks=16)
    mirror = init.copy()
    B = len(ids)
    for it in range(20):
        qb = rng.normal(62, (L, B, Hq, D), "bf16", stream=it)
        kb = rng.normal(63, (L, B, Hkv, D), "bf16", stream=it)
        vb = rng.normal(64, (L, B, Hkv, D), "bf16", stream=it)
        out = step.step(to_dev(qb, "bf16", cuda), to_dev(kb, "bf16", cuda),
                        to_dev(vb, "bf16", cuda))
        torch.cuda.synchronize()
        ops.check_device_errors(0)
        tabs = np.full((B, 16), -1, dtype=np.int32)
        for b, s in enumerate(ids):
            t = store.tables[s]
            tabs[b, : len(t)] = t
            pos = store.offsets[s]
            for l in range(L):
                mirror[l, 0, t[pos // bs], :, pos % bs] = kb[l, b]
                mirror[l, 1, t[pos // bs], :, pos % bs] = vb[l, b]
        lens = np.array([store.offsets[s] + 1 for s in ids])
        for l in range(L):
            ref = opaged.paged_decode(qb[l], mirror[l, 0], mirror[l, 1], tabs, lens, "bf16")
            assert attn_err(out[l], ref) <= ATOL_REL, (it, l)
        step.advance()
    assert np.array_equal(to_bits(store.pools), mirror)


def test_step_host_pipelined_matches_device_step(cuda):
    """step_host (inputs up and outputs down on copy streams, per layer,
    overlapped with the layers) gives bit-for-bit the outputs and pools of the
    device-side step, over steps that advance and grow the tables."""
    from mlxz_b200.engine import PagedDecodeStep, PagedKVStore

    L, Hkv, G, D, bs = 3, 2, 4, 128, 16
    Hq = Hkv * G
    offsets = [0, 15, 31, 200]
    stores, steps = [], []
    for _ in range(2):
        st = PagedKVStore(L, 64, Hkv, D, bs, torch.bfloat16, cuda, init="zeros")
        st.pools.copy_(to_dev(rng.normal(71, tuple(st.pools.shape), "bf16"), "bf16", cuda))
        for i, o in enumerate(offsets):
            st.add_sequence(f"r{i}", o)
        stores.append(st)
        steps.append(PagedDecodeStep(st, [f"r{i}" for i in range(len(offsets))], Hq,
                                     max_blocks=16))
    B = len(offsets)
    out_h = torch.empty((L, B, Hq, D), dtype=torch.bfloat16).pin_memory()
    for it in range(4):
        qb = rng.normal(72, (L, B, Hq, D), "bf16", stream=it)
        kb = rng.normal(73, (L, B, Hkv, D), "bf16", stream=it)
        vb = rng.normal(74, (L, B, Hkv, D), "bf16", stream=it)
        host = [to_dev(x, "bf16", "cpu").pin_memory() for x in (qb, kb, vb)]
        ref = steps[0].step(*(h.to(cuda) for h in host), advance=True)
        steps[1].step_host(*host, out_h, advance=True)
        torch.cuda.synchronize()
        ops.check_device_errors(0)
        assert torch.equal(out_h, ref.cpu()), it
    assert torch.equal(stores[0].pools, stores[1].pools)


@pytest.mark.parametrize("quantized", [False, True])
def test_captured_step_matches_eager_step(cuda, quantized):
    """A step captured once into a CUDA graph and replayed (tables and lengths
    advanced in place, blocks appended as tables grow) gives bit-for-bit the
    outputs and pools of eager steps on the same inputs."""
    from mlxz_b200.engine import (PagedDecodeStep, PagedKVStore, QuantizedPagedDecodeStep,
                                  QuantizedPagedKVStore)

    L, Hkv, G, D, bs = 2, 2, 4, 128, 16
    Hq = Hkv * G
    offsets = [3, 15, 30, 200]
    stores, steps = [], []
    for _ in range(2):
        if quantized:
            st = QuantizedPagedKVStore(L, 64, Hkv, D, bs, bits=8, device=cuda)
        else:
            st = PagedKVStore(L, 64, Hkv, D, bs, torch.bfloat16, cuda, init="zeros")
            st.pools.copy_(to_dev(rng.normal(81, tuple(st.pools.shape), "bf16"), "bf16", cuda))
        for i, o in enumerate(offsets):
            st.add_sequence(f"r{i}", 0)
        ids = [f"r{i}" for i in range(len(offsets))]
        # fill the prefixes through the store's own append path
        for i, o in enumerate(offsets):
            if o:
                kk = to_dev(rng.normal(82 + i, (L, Hkv, o, D), "bf16"), "bf16", cuda)
                st.append_tokens(f"r{i}", kk, kk)
        cls = QuantizedPagedDecodeStep if quantized else PagedDecodeStep
        stores.append(st)
        steps.append(cls(st, ids, Hq, max_blocks=16))
    steps[1].capture(torch.bfloat16)
    B = len(offsets)
    for it in range(5):
        q = to_dev(rng.normal(83, (L, B, Hq, D), "bf16", stream=it), "bf16", cuda)
        k = to_dev(rng.normal(84, (L, B, Hkv, D), "bf16", stream=it), "bf16", cuda)
        v = to_dev(rng.normal(85, (L, B, Hkv, D), "bf16", stream=it), "bf16", cuda)
        ref = steps[0].step(q, k, v, advance=True)
        got = steps[1].replay(q, k, v, advance=True)
        torch.cuda.synchronize()
        ops.check_device_errors(0)
        assert torch.equal(got, ref), it
    for a, b in zip(stores[0].pool_stacks(), stores[1].pool_stacks()):
        assert torch.equal(a, b)


def test_overlapped_launch_waits_for_the_kernel_ahead(cuda):
    """MZ_LAUNCH_OVERLAP_PREVIOUS: q and k_new/v_new written by a long kernel
    right ahead of the launch (the last elements of a 512 MiB elementwise op)
    are what the launch reads: its result equals a plain launch's bit for bit."""
    B, Hkv, G, D, bs = 16, 4, 4, 128, 16
    lengths = [int(x) for x in rng.randint(12, B, 1, 3000)]
    case = random_paged_case(13, B, Hkv, D, bs, lengths, "bf16", G=G)
    tables = torch.from_numpy(case["tables"]).to(cuda)
    lens = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    q = to_dev(case["q"][:, 0], "bf16", cuda)
    kn = to_dev(rng.normal(14, (B, Hkv, D), "bf16"), "bf16", cuda)
    vn = to_dev(rng.normal(15, (B, Hkv, D), "bf16"), "bf16", cuda)
    pools = [to_dev(case[k], "bf16", cuda) for k in ("kp", "vp")]
    ref = ops.paged_append_decode(q, pools[0].clone(), pools[1].clone(), kn, vn, tables, lens)
    pad = 256 << 20  # elements ahead of the inputs in the buffer the kernel ahead writes
    src = torch.cat([torch.ones(pad, dtype=torch.bfloat16, device=cuda), q.flatten(),
                     kn.flatten(), vn.flatten()])
    big = torch.zeros_like(src)
    nq, nk = q.numel(), kn.numel()
    q_in = big[pad:pad + nq].view(q.shape)
    k_in = big[pad + nq:pad + nq + nk].view(kn.shape)
    v_in = big[pad + nq + nk:].view(vn.shape)
    kp, vp = pools[0].clone(), pools[1].clone()
    torch.cuda.synchronize()
    torch.mul(src, 1.0, out=big)  # the kernel ahead: writes q / k_new / v_new last
    out = ops.paged_append_decode(q_in, kp, vp, k_in, v_in, tables, lens,
                                  overlap_previous=True)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    assert torch.equal(out, ref)
