"""GPU parity: chunked prefill attention over paged KV (mz_paged_prefill) and
the PagedPrefillStep (append + attention per layer) against the float64 causal
oracle on the same seeded inputs.

Tolerance: max(|out - ref| - u*|ref|, 0) / max|ref| <= 2e-3, u = unit roundoff
of the output dtype (0 for fp32 outputs).  Pool writes are bit-exact.
"""
import numpy as np
import pytest
import torch

from mlxz_b200 import ops
from mlxz_b200._native import DeviceError, NativeError
from oracle import paged as opaged
from oracle import rng
from tests.gpu_util import TORCH, attn_err, random_paged_case, to_bits, to_dev

pytestmark = pytest.mark.gpu
ATOL_REL = 2e-3


def _prefill_case(seed, ctx, qlen, dtype, D, G, bs, Hkv):
    case = random_paged_case(seed, len(ctx), Hkv, D, bs, ctx, dtype, G=G)
    T = sum(qlen)
    case["qp"] = rng.normal(seed, (max(T, 1), Hkv * G, D), dtype, stream=9)[:T]
    case["q_start"] = np.cumsum([0] + qlen[:-1]).astype(np.int32)
    case["q_len"] = np.array(qlen, dtype=np.int32)
    return case


def _run(case, dtype, cuda, out_dtype=None, max_q_len=None, q_dev=None):
    kp, vp = to_dev(case["kp"], dtype, cuda), to_dev(case["vp"], dtype, cuda)
    q = q_dev if q_dev is not None else to_dev(case["qp"], dtype, cuda)
    dev = {k: torch.from_numpy(case[k]).to(cuda) for k in ("tables", "q_start", "q_len", "ctx")}
    mq = max_q_len if max_q_len is not None else int(case["q_len"].max(initial=0))
    out = ops.paged_prefill(q, kp, vp, dev["tables"], dev["q_start"], dev["q_len"], dev["ctx"],
                            mq, out_dtype=out_dtype)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    return out


PREFILL_CASES = [
    # dtype, D, G, bs, ctx (chunk included), q_len
    ("bf16", 128, 8, 16, [100, 300, 17, 64], [100, 37, 1, 0]),
    ("f16", 64, 1, 16, [1000, 129], [513, 129]),
    ("bf16", 64, 16, 32, [77, 40], [30, 40]),
    ("f16", 128, 4, 64, [2000, 5], [200, 5]),
    ("bf16", 128, 2, 16, [16, 33, 1], [16, 33, 1]),
    ("bf16", 128, 1, 16, [4096], [128]),
    ("f16", 128, 32, 128, [700, 260], [300, 260]),
    ("bf16", 64, 4, 48, [1000, 333, 47], [513, 1, 47]),
]


@pytest.mark.parametrize("dtype,D,G,bs,ctx,qlen", PREFILL_CASES)
@pytest.mark.parametrize("out32", [False, True])
@pytest.mark.parametrize("form", ["persistent", "per_block"])
def test_paged_prefill_vs_oracle(cuda, dtype, D, G, bs, ctx, qlen, out32, form, monkeypatch):
    """Every case through the persistent kernel (the default: one CTA per SM
    over all query blocks) and the one-CTA-per-block kernel."""
    monkeypatch.setenv("MLXZ_B200_PREFILL_PERSIST", "1" if form == "persistent" else "0")
    Hkv = 2 if G == 16 else 4
    case = _prefill_case(5 + D + G + len(ctx), ctx, qlen, dtype, D, G, bs, Hkv)
    out = _run(case, dtype, cuda, torch.float32 if out32 else None)
    ref = opaged.paged_prefill(case["qp"], case["kp"], case["vp"], case["tables"],
                               case["q_start"], case["q_len"], case["ctx"], dtype)
    assert attn_err(out, ref) <= ATOL_REL


def test_prefill_long_context(cuda):
    """32K-token caches: 256 key tiles per CTA, so every ring slot and S buffer
    wraps its mbarrier phases many times; chunks end mid-block."""
    dtype, D, G, bs, Hkv = "bf16", 128, 8, 16, 1
    ctx, qlen = [32768, 20000], [72, 33]
    case = _prefill_case(123, ctx, qlen, dtype, D, G, bs, Hkv)
    out = _run(case, dtype, cuda, torch.float32)
    ref = opaged.paged_prefill(case["qp"], case["kp"], case["vp"], case["tables"],
                               case["q_start"], case["q_len"], case["ctx"], dtype)
    assert attn_err(out, ref) <= ATOL_REL


def test_prefill_strided_q_and_oversized_grid(cuda):
    """q as the query slice of a packed [T, Hq + 2 Hkv, D] projection, and a
    max_q_len above every chunk (the extra query blocks do nothing)."""
    dtype, D, G, bs, Hkv = "bf16", 128, 4, 16, 2
    ctx, qlen = [90, 47], [50, 47]
    case = _prefill_case(77, ctx, qlen, dtype, D, G, bs, Hkv)
    T, Hq = sum(qlen), Hkv * G
    packed = torch.zeros(T, Hq + 2 * Hkv, D, dtype=TORCH[dtype], device=cuda)
    packed[:, :Hq] = to_dev(case["qp"], dtype, cuda)
    out = _run(case, dtype, cuda, max_q_len=300, q_dev=packed[:, :Hq])
    ref = opaged.paged_prefill(case["qp"], case["kp"], case["vp"], case["tables"],
                               case["q_start"], case["q_len"], case["ctx"], dtype)
    assert attn_err(out, ref) <= ATOL_REL


def test_prefill_last_row_equals_decode(cuda):
    """The last query of a chunk sees the whole context: the prefill row and the
    decode kernel on the same query agree to the attention tolerance."""
    dtype, D, G, bs, Hkv = "f16", 128, 8, 16, 1
    ctx, qlen = [700, 250], [64, 9]
    case = _prefill_case(91, ctx, qlen, dtype, D, G, bs, Hkv)
    out = _run(case, dtype, cuda, torch.float32)
    last = case["q_start"] + case["q_len"] - 1
    q = to_dev(case["qp"][last], dtype, cuda)
    kp, vp = to_dev(case["kp"], dtype, cuda), to_dev(case["vp"], dtype, cuda)
    dec = ops.paged_decode(q, kp, vp, torch.from_numpy(case["tables"]).to(cuda),
                           torch.from_numpy(case["ctx"]).to(cuda), out_dtype=torch.float32)
    torch.cuda.synchronize()
    ref = opaged.paged_decode(case["qp"][last], case["kp"], case["vp"], case["tables"],
                              case["ctx"], dtype)
    assert attn_err(out[torch.from_numpy(last).long()], ref) <= ATOL_REL
    assert attn_err(dec, ref) <= ATOL_REL


def test_prefill_rejects_bad_inputs(cuda):
    dtype, D, bs = "bf16", 64, 16
    case = _prefill_case(3, [20], [10], dtype, D, 4, bs, 2)
    # a chunk longer than its context is reported on the device error word
    bad = dict(case, ctx=np.array([5], dtype=np.int32))
    with pytest.raises(DeviceError):
        _run(bad, dtype, cuda)
    # query rows past the end of q (q_start + q_len > rows of q)
    bad = dict(case, q_start=np.array([3], dtype=np.int32))
    with pytest.raises(DeviceError, match="query rows"):
        _run(bad, dtype, cuda)
    # a block id outside the pool
    bad = dict(case, tables=case["tables"].copy())
    bad["tables"][0, 0] = case["n_blocks"] + 3
    with pytest.raises(DeviceError):
        _run(bad, dtype, cuda)
    # unsupported group size (16 % G != 0) is refused on the host
    kp = to_dev(case["kp"], dtype, cuda)
    q = torch.zeros(10, 6, D, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(NativeError):
        ops.paged_prefill(q, kp, kp, torch.from_numpy(case["tables"]).to(cuda),
                          torch.zeros(1, dtype=torch.int32, device=cuda),
                          torch.full((1,), 10, dtype=torch.int32, device=cuda),
                          torch.full((1,), 20, dtype=torch.int32, device=cuda), 10)
    # the row max is taken on raw scores: a non-positive scale is refused
    q8 = torch.zeros(10, 8, D, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        ops.paged_prefill(q8, kp, kp, torch.from_numpy(case["tables"]).to(cuda),
                          torch.zeros(1, dtype=torch.int32, device=cuda),
                          torch.full((1,), 10, dtype=torch.int32, device=cuda),
                          torch.full((1,), 20, dtype=torch.int32, device=cuda), 10, scale=-0.1)
    torch.cuda.synchronize()


def test_chunked_prefill_step_matches_whole_prompt(cuda):
    """Three prompts (one sharing its first block with another through the
    BlockManager) prefilled in chunks of 48 by ChunkedPrefillScheduler +
    PagedPrefillStep over 2 layers: every chunk's output equals the causal
    attention of the whole prompt, the pools hold the prompt K/V bit for bit,
    and a decode step afterwards matches the oracle."""
    from mlxz_b200.engine import (ChunkedPrefillScheduler, PagedDecodeStep, PagedKVStore,
                                  PagedPrefillStep)

    L, Hkv, G, D, bs, dtype = 2, 2, 4, 128, 16, "bf16"
    Hq = Hkv * G
    prompts = {"a": 150, "b": 37, "c": 96}
    store = PagedKVStore(L, 64, Hkv, D, bs, torch.bfloat16, cuda, init="zeros")
    store.add_sequence("a")
    store.add_sequence("b")
    # "c" starts from a cached 20-token prefix held in a block shared with a
    # retired owner: its first chunk copy-on-writes that block
    shared = store.bm.allocate(2)
    store.bm.incref(shared)
    store.add_sequence("c", 20, blocks=list(shared))
    pre_k = rng.normal(70, (L, Hkv, 20, D), dtype, stream=1)
    pre_v = rng.normal(70, (L, Hkv, 20, D), dtype, stream=2)
    for l in range(L):
        for p in range(20):
            store.pools[l, 0, shared[p // bs], :, p % bs] = to_dev(pre_k[l, :, p], dtype, cuda)
            store.pools[l, 1, shared[p // bs], :, p % bs] = to_dev(pre_v[l, :, p], dtype, cuda)
    store.offsets["c"] = 20
    before_shared = to_bits(store.pools[:, :, shared[1]]).copy()

    full = {s: {"q": rng.normal(71, (L, n, Hq, D), dtype, stream=i),
                "k": rng.normal(72, (L, n, Hkv, D), dtype, stream=i),
                "v": rng.normal(73, (L, n, Hkv, D), dtype, stream=i)}
            for i, (s, n) in enumerate(prompts.items())}
    for l in range(L):
        full["c"]["k"][l, :20] = pre_k[l].transpose(1, 0, 2)
        full["c"]["v"][l, :20] = pre_v[l].transpose(1, 0, 2)
    outs = {s: np.zeros((L, n, Hq, D)) for s, n in prompts.items()}
    sched = ChunkedPrefillScheduler(chunk_size=48)
    base = {"a": 0, "b": 0, "c": 20}  # "c" prefills only the suffix after its cached prefix
    toks = {s: list(range(base[s], n)) for s, n in prompts.items()}
    live = set(prompts)
    while live:
        chunks = []
        for s in sorted(live):
            ch = sched.get_next_chunk(s, toks[s])
            chunks.append((s, base[s] + ch.start_pos, len(ch.tokens)))
            if ch.is_last:
                live.discard(s)
        step = PagedPrefillStep(store, [(s, n) for s, _, n in chunks], Hq)
        for l in range(L):
            q = np.concatenate([full[s]["q"][l, a:a + n] for s, a, n in chunks])
            k = np.concatenate([full[s]["k"][l, a:a + n] for s, a, n in chunks])
            v = np.concatenate([full[s]["v"][l, a:a + n] for s, a, n in chunks])
            out = step.layer(l, to_dev(q, dtype, cuda), to_dev(k, dtype, cuda),
                             to_dev(v, dtype, cuda), out_dtype=torch.float32)
            torch.cuda.synchronize()
            ops.check_device_errors(0)
            o = out.cpu().numpy()
            r = 0
            for s, a, n in chunks:
                outs[s][l, a:a + n] = o[r:r + n]
                r += n
        step.finish()
    # the full shared block is kept, the partly filled one was copied on write
    assert store.tables["c"][0] == shared[0] and store.tables["c"][1] != shared[1]
    assert np.array_equal(to_bits(store.pools[:, :, shared[1]]), before_shared)
    for s, n in prompts.items():
        assert store.offsets[s] == n
        t = store.tables[s]
        for l in range(L):
            kq = rng.to_f32(full[s]["q"][l], dtype).transpose(1, 0, 2)
            kk = rng.to_f32(full[s]["k"][l], dtype).transpose(1, 0, 2)
            vv = rng.to_f32(full[s]["v"][l], dtype).transpose(1, 0, 2)
            ref = opaged.prefill_attention(kq, kk, vv, 0).transpose(1, 0, 2)
            a0 = 20 if s == "c" else 0
            assert attn_err(torch.from_numpy(outs[s][l, a0:]).float(), ref[a0:]) <= ATOL_REL, (s, l)
            kb, vb = opaged.gather(to_bits(store.pools[l, 0]), to_bits(store.pools[l, 1]), t, n, bs)
            assert np.array_equal(kb, full[s]["k"][l].transpose(1, 0, 2))
            assert np.array_equal(vb, full[s]["v"][l].transpose(1, 0, 2))

    # decode continues from the prefilled caches
    ids = sorted(prompts)
    dec = PagedDecodeStep(store, ids, Hq)
    qd = rng.normal(74, (L, 3, Hq, D), dtype)
    kd = rng.normal(75, (L, 3, Hkv, D), dtype)
    vd = rng.normal(76, (L, 3, Hkv, D), dtype)
    out = dec.step(to_dev(qd, dtype, cuda), to_dev(kd, dtype, cuda), to_dev(vd, dtype, cuda))
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    for l in range(L):
        for b, s in enumerate(ids):
            kk = np.concatenate([full[s]["k"][l], kd[l, b][None]]).transpose(1, 0, 2)
            vv = np.concatenate([full[s]["v"][l], vd[l, b][None]]).transpose(1, 0, 2)
            ref = opaged.attention(rng.to_f32(qd[l, b][:, None], dtype), rng.to_f32(kk, dtype),
                                   rng.to_f32(vv, dtype))[:, 0]
            assert attn_err(out[l, b], ref) <= ATOL_REL, (s, l)
