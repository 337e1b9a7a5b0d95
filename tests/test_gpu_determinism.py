"""GPU: the determinism gates of the reference's plan
(MLXZ_IMPLEMENTATION_PLAN.md:1058-1059) on the KV path's output.

* Batch-position determinism, bytewise: with MZ_DECODE_BATCH_INVARIANT a
  sequence's decode output has the same bytes at any batch position and with
  any other sequences around it.
* Prefix-cache drift max|O - O'| < 1e-4: a sequence whose prefix was restored
  from the paged prefix cache (shared blocks) and one that appended the same
  prefix itself decode to outputs within 1e-4 in the default schedule, and to
  identical bytes with MZ_DECODE_BATCH_INVARIANT.
"""
import numpy as np
import pytest
import torch

from mlxz_b200 import ops
from mlxz_b200.engine import PagedDecodeStep, PagedKVStore
from mlxz_b200.prefix_cache import PagedPrefixCache, RollingPrefixHasher
from oracle import paged as opaged
from oracle import rng
from tests.gpu_util import attn_err, to_bits, to_dev

pytestmark = pytest.mark.gpu
ATOL_REL = 2e-3


def _batch(cuda, kp, vp, tables_np, ctx_np, q_np, kn_np, vn_np, invariant):
    out = ops.paged_append_decode(to_dev(q_np, "bf16", cuda), kp, vp,
                                  to_dev(kn_np, "bf16", cuda), to_dev(vn_np, "bf16", cuda),
                                  torch.from_numpy(tables_np).to(cuda),
                                  torch.from_numpy(ctx_np).to(cuda), out_dtype=torch.float32,
                                  batch_invariant=invariant)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    return out.cpu()


@pytest.mark.parametrize("G", [4, 8])
def test_batch_position_bytewise(cuda, G):
    """Sequence X (3000 tokens) decoded inside two different batches -- other
    sequences, other sizes, X at another position -- gives the same bytes with
    batch_invariant; both batches also match the oracle."""
    Hkv, D, bs = 4, 128, 16
    n_blocks = 1400
    perm = rng.permutation(5, n_blocks)
    kp_np = rng.normal(5, (n_blocks, Hkv, bs, D), "bf16", stream=1)
    vp_np = rng.normal(5, (n_blocks, Hkv, bs, D), "bf16", stream=2)
    kp, vp = to_dev(kp_np, "bf16", cuda), to_dev(vp_np, "bf16", cuda)
    ctx_x = 3000
    lens = {"x": ctx_x, "a": 9000, "b": 40, "c": 2500, "d": 5000, "e": 17}
    tabs, used = {}, 0
    for s, c in lens.items():
        nb = -(-c // bs)
        tabs[s] = perm[used:used + nb]
        used += nb
    qs = {s: rng.normal(6, (Hkv * G, D), "bf16", stream=i) for i, s in enumerate(lens)}
    kns = {s: rng.normal(7, (Hkv, D), "bf16", stream=i) for i, s in enumerate(lens)}
    vns = {s: rng.normal(8, (Hkv, D), "bf16", stream=i) for i, s in enumerate(lens)}

    def run(order, invariant):
        width = max(len(tabs[s]) for s in order)
        t = np.full((len(order), width), -1, dtype=np.int32)
        for i, s in enumerate(order):
            t[i, :len(tabs[s])] = tabs[s]
        ctx = np.array([lens[s] for s in order], dtype=np.int32)
        q = np.stack([qs[s] for s in order])
        kn = np.stack([kns[s] for s in order])
        vn = np.stack([vns[s] for s in order])
        out = _batch(cuda, kp, vp, t, ctx, q, kn, vn, invariant)
        return out, t, ctx, q

    o1, t1, c1, q1 = run(["a", "x", "b", "c"], True)
    o2, t2, c2, q2 = run(["d", "e", "x"], True)
    assert torch.equal(o1[1], o2[2])
    # the appends wrote the same bytes to the same slots; compare with the oracle
    kpool, vpool = to_bits(kp), to_bits(vp)
    for o, t, c, q in ((o1, t1, c1, q1), (o2, t2, c2, q2)):
        ref = opaged.paged_decode(q, kpool, vpool, t, c, "bf16")
        assert attn_err(o, ref) <= ATOL_REL
    # the default schedule is correct too (its bytes may depend on the batch)
    o3, t3, c3, q3 = run(["a", "x", "b", "c"], False)
    assert attn_err(o3, opaged.paged_decode(q3, kpool, vpool, t3, c3, "bf16")) <= ATOL_REL


def test_prefix_hit_drift(cuda):
    """a appends a 1000-token prompt; b restores it from the prefix cache
    (zero copy); c appends the same prompt into its own blocks.  One decode
    step of all three with the same new token: max|O_b - O_a| and
    max|O_c - O_a| < 1e-4 by default, 0 with batch_invariant."""
    L, Hkv, G, D, bs = 2, 4, 4, 128, 16
    Hq = Hkv * G
    n = 1000
    store = PagedKVStore(L, 256, Hkv, D, bs, torch.bfloat16, cuda, init="zeros")
    cache = PagedPrefixCache(store, memory_budget_bytes=1 << 30)
    hasher = RollingPrefixHasher(bs)
    k = to_dev(rng.normal(9, (L, Hkv, n, D), "bf16", stream=1), "bf16", cuda)
    v = to_dev(rng.normal(9, (L, Hkv, n, D), "bf16", stream=2), "bf16", cuda)
    store.add_sequence("a")
    store.append_tokens("a", k, v)
    hashes = hasher.hash_chunks(list(range(n)))
    cache.store_sync(hashes, "a", block_size=bs)
    got, state, _ = cache.lookup_sync(hashes)
    assert got in (n, n - n % bs)
    cache.restore("b", state)
    if got < n:  # b appends the tail the cache does not hold
        store.append_tokens("b", k[:, :, got:], v[:, :, got:])
    store.add_sequence("c")
    store.append_tokens("c", k, v)
    assert store.tables["b"][0] == store.tables["a"][0]
    assert store.tables["c"][0] != store.tables["a"][0]
    q1 = rng.normal(10, (L, 1, Hq, D), "bf16")
    k1 = rng.normal(11, (L, 1, Hkv, D), "bf16")
    v1 = rng.normal(12, (L, 1, Hkv, D), "bf16")
    q3 = to_dev(np.repeat(q1, 3, axis=1), "bf16", cuda)
    k3 = to_dev(np.repeat(k1, 3, axis=1), "bf16", cuda)
    v3 = to_dev(np.repeat(v1, 3, axis=1), "bf16", cuda)
    for invariant in (False, True):
        # the step's appends copy-on-write the shared partial block first
        step = PagedDecodeStep(store, ["a", "b", "c"], Hq, batch_invariant=invariant)
        step.prepare_writes()
        out = step.step(q3, k3, v3).float().cpu()
        torch.cuda.synchronize()
        ops.check_device_errors(0)
        drift_b = (out[:, 1] - out[:, 0]).abs().max().item()
        drift_c = (out[:, 2] - out[:, 0]).abs().max().item()
        if invariant:
            assert drift_b == 0.0 and drift_c == 0.0
        else:
            assert drift_b < 1e-4 and drift_c < 1e-4
