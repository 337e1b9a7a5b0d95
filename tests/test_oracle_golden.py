"""Pins the CPU oracle against vectors produced by the reference's own code
(tests/golden/make_golden.py ran src/mlxz/paged_attention/*.py over a torch-CPU
stand-in for mlx.core)."""
import hashlib
import json

import numpy as np
import pytest

from oracle import paged, rng
from tests.conftest import GOLDEN


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def c1_inputs():
    ctx = (37, 128, 300, 511)
    H, D, Hq, n_blocks, bs, dtype = 8, 64, 32, 256, 16, "f16"
    perm = rng.permutation(1, n_blocks)
    tables, used = [], 0
    for c in ctx:
        nb = (c + 1 + bs - 1) // bs
        tables.append([int(x) for x in perm[used:used + nb]])
        used += nb
    return dict(
        ctx=list(ctx), H=H, D=D, Hq=Hq, n_blocks=n_blocks, bs=bs, dtype=dtype, tables=tables,
        pre_k=[rng.normal(2, (H, c, D), dtype, stream=b) for b, c in enumerate(ctx)],
        pre_v=[rng.normal(2, (H, c, D), dtype, stream=100 + b) for b, c in enumerate(ctx)],
        new_k=[rng.normal(3, (H, 1, D), dtype, stream=b) for b in range(len(ctx))],
        new_v=[rng.normal(3, (H, 1, D), dtype, stream=100 + b) for b in range(len(ctx))],
        q=[rng.normal(4, (Hq, 1, D), dtype, stream=b) for b in range(len(ctx))])


def inputs_digest(inp) -> str:
    h = hashlib.sha256()
    for key in ("pre_k", "pre_v", "new_k", "new_v", "q"):
        for a in inp[key]:
            h.update(np.ascontiguousarray(a).tobytes())
    h.update(json.dumps(inp["tables"]).encode())
    return h.hexdigest()


def test_rng_is_reproducible():
    a = rng.normal(9, (1000,), "bf16")
    b = rng.normal(9, (1000,), "bf16")
    assert np.array_equal(a, b)
    x = rng.to_f32(rng.normal(9, (200_000,), "f16"), "f16")
    assert abs(float(x.mean())) < 0.02 and abs(float(x.std()) - 1.0) < 0.02
    p = rng.permutation(3, 100)
    assert sorted(p.tolist()) == list(range(100))


def test_c1_layer_inputs_match_golden():
    g = json.loads((GOLDEN / "c1_layer.json").read_text())
    inp = c1_inputs()
    assert inp["tables"] == g["tables"]
    assert inputs_digest(inp) == g["inputs_sha256"]


def test_oracle_c1_layer_append_gather_attention():
    g = json.loads((GOLDEN / "c1_layer.json").read_text())
    gold_attn = np.load(GOLDEN / "c1_layer_attn.npy")
    inp = c1_inputs()
    o = paged.PagedKVOracle(inp["n_blocks"], inp["H"], inp["bs"], inp["D"])
    for b in range(4):
        o.set_table(f"seq{b}", inp["tables"][b])
        o.append_kv(f"seq{b}", inp["pre_k"][b], inp["pre_v"][b])
    for b in range(4):
        o.append_kv(f"seq{b}", inp["new_k"][b], inp["new_v"][b])
    assert _sha(o.k_pool) == g["k_pool_sha256"]
    assert _sha(o.v_pool) == g["v_pool_sha256"]
    for b in range(4):
        k, v = o.get_kv(f"seq{b}")
        assert _sha(k) == g["seqs"][b]["k_sha256"]
        assert _sha(v) == g["seqs"][b]["v_sha256"]
        assert o.offsets[f"seq{b}"] == g["seqs"][b]["offset"]
        out = paged.attention(rng.to_f32(inp["q"][b], "f16"), rng.to_f32(k, "f16"),
                              rng.to_f32(v, "f16"), g["scale"])
        np.testing.assert_allclose(out, gold_attn[b], rtol=0, atol=2e-6)


def test_oracle_bm_paged_replay():
    """Replays the BlockManager-driven scenario with the fixture's tables."""
    g = json.loads((GOLDEN / "bm_paged.json").read_text())
    c = g["config"]
    o = paged.PagedKVOracle(c["n_blocks"], c["H"], c["bs"], c["D"])
    digest = hashlib.sha256()
    for rec in g["ops"]:
        sid = rec["seq"]
        if rec["op"] == "alloc":
            o.set_table(sid, rec["tables"][sid])
        elif rec["op"] == "free":
            o.tables.pop(sid)
            o.offsets.pop(sid)
        else:
            n = rec["n"]
            k = rng.normal(g["seeds"]["k"], (c["H"], n, c["D"]), c["dtype"], stream=rec["k_stream"])
            v = rng.normal(g["seeds"]["v"], (c["H"], n, c["D"]), c["dtype"], stream=rec["k_stream"])
            digest.update(k.tobytes())
            digest.update(v.tobytes())
            o.tables[sid] = list(rec["tables"][sid])  # table growth is host policy
            o.append_kv(sid, k, v)
        assert {s: o.offsets[s] for s in sorted(o.offsets)} == rec["offsets"]
        assert _sha(o.k_pool) == rec["k_pool_sha256"]
        assert _sha(o.v_pool) == rec["v_pool_sha256"]
    attn = np.load(GOLDEN / "bm_paged_attn.npy")
    for i, sid in enumerate(g["attn_order"]):
        k, v = o.get_kv(sid)
        gg = g["gathers"][sid]
        assert _sha(k) == gg["k_sha256"] and _sha(v) == gg["v_sha256"]
        q = rng.normal(g["seeds"]["q"], (c["Hq"], 1, c["D"]), c["dtype"], stream=gg["q_stream"])
        digest.update(q.tobytes())
        out = paged.attention(rng.to_f32(q, c["dtype"]), rng.to_f32(k, c["dtype"]),
                              rng.to_f32(v, c["dtype"]))
        np.testing.assert_allclose(out, attn[i], rtol=0, atol=2e-6)
    assert digest.hexdigest() == g["inputs_sha256"]


def test_oracle_block_moves():
    pools = rng.normal(5, (3, 10, 2, 4, 8), "bf16")
    ref = pools.copy()
    paged.block_copy(pools, [1, 2], [7, 9])
    assert np.array_equal(pools[:, 7], ref[:, 1]) and np.array_equal(pools[:, 9], ref[:, 2])
    st = paged.block_pack(ref, [4, 0, 3])
    assert st.shape == (3, 3, 2 * 4 * 8 * 2)
    back = np.zeros_like(ref)
    paged.block_unpack(back, [4, 0, 3], st)
    for b in (4, 0, 3):
        assert np.array_equal(back[:, b], ref[:, b])


@pytest.mark.parametrize("G", [1, 4, 8])
def test_oracle_attention_gqa_mapping(G):
    """Query head h reads KV head h // G (mx.repeat semantics)."""
    Hkv, T, D = 2, 5, 8
    r = np.random.default_rng(0)
    q = r.standard_normal((Hkv * G, 1, D))
    k = r.standard_normal((Hkv, T, D))
    v = r.standard_normal((Hkv, T, D))
    out = paged.attention(q, k, v)
    for h in range(Hkv * G):
        s = q[h, 0] @ k[h // G].T * D ** -0.5
        p = np.exp(s - s.max())
        p /= p.sum()
        np.testing.assert_allclose(out[h, 0], p @ v[h // G], atol=1e-12)
