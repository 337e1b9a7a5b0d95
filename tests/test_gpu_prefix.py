"""GPU: paged prefix cache data path -- zero-copy restore, copy-on-write of a
shared partial block, eviction to the pinned host tier and reload -- checked
bit-exactly against a CPU mirror of the pools, plus attention over restored
prefixes against the oracle."""
import numpy as np
import pytest
import torch

from mlxz_b200 import ops
from mlxz_b200.engine import PagedDecodeStep, PagedKVStore
from mlxz_b200.prefix_cache import PagedPrefixCache, PinnedHostTier, RollingPrefixHasher
from oracle import paged as opaged
from oracle import rng
from tests.gpu_util import attn_err, to_bits, to_dev

pytestmark = pytest.mark.gpu


def _seq_bits(mirror, table, n, bs):
    """[L, 2, H, n, D] uint16 of a sequence's first n tokens from the mirror."""
    L = mirror.shape[0]
    out = np.stack([np.stack([opaged.gather(mirror[l, 0], mirror[l, 1], table, n, bs)[kv]
                              for kv in (0, 1)]) for l in range(L)])
    return out


def _dev_seq(store, table, n):
    pools = to_bits(store.pools)
    return _seq_bits(pools, table, n, store.block_size)


def test_paged_prefix_restore_cow_evict_reload(cuda):
    L, H, D, bs, N = 2, 2, 128, 16, 64
    G = 4
    store = PagedKVStore(L, N, H, D, bs, torch.bfloat16, cuda, init="zeros")
    tier = PinnedHostTier(32, 2 * L, store.block_bytes, cuda, staging_bytes=4 * 2 * L * store.block_bytes)
    cache = PagedPrefixCache(store, memory_budget_bytes=1 << 30, host_tier=tier)
    hasher = RollingPrefixHasher(16)
    # sequence a: 70 prompt tokens
    store.add_sequence("a", 0)
    ka = rng.normal(1, (L, H, 70, D), "bf16", stream=1)
    va = rng.normal(1, (L, H, 70, D), "bf16", stream=2)
    store.append_tokens("a", to_dev(ka, "bf16", cuda), to_dev(va, "bf16", cuda))
    want_a = np.stack([ka, va], axis=1)  # [L, 2, H, 70, D]
    assert np.array_equal(_dev_seq(store, store.tables["a"], 70), want_a)
    hashes = hasher.hash_chunks(list(range(70)))
    cache.store_sync(hashes, "a", block_size=16)

    # zero-copy restore of the full 70-token prefix into c: same blocks
    n, state, _ = cache.lookup_sync(hashes)
    assert n == 70
    tab_c = cache.restore("c", state)
    assert tab_c == store.tables["a"][:5]
    # c appends one token: block 4 is shared (a, cache, c) -> copy-on-write
    kc = rng.normal(2, (L, H, 1, D), "bf16", stream=1)
    vc = rng.normal(2, (L, H, 1, D), "bf16", stream=2)
    store.append_tokens("c", to_dev(kc, "bf16", cuda), to_dev(vc, "bf16", cuda))
    assert store.tables["c"][:4] == store.tables["a"][:4]
    assert store.tables["c"][4] != store.tables["a"][4]
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    assert np.array_equal(_dev_seq(store, store.tables["a"], 70), want_a)  # a untouched
    want_c = np.concatenate([want_a, np.stack([kc, vc], axis=1)], axis=3)
    assert np.array_equal(_dev_seq(store, store.tables["c"], 71), want_c)

    # decode over restored prefixes: b restores 48 tokens, steps 3 times
    n, state48, _ = cache.lookup_sync(hashes[:3])
    assert n == 48
    cache.restore("b", state48)
    step = PagedDecodeStep(store, ["b", "c"], H * G, max_blocks=8)
    mirror = to_bits(store.pools)
    for it in range(3):
        q = rng.normal(3, (L, 2, H * G, D), "bf16", stream=it)
        kn = rng.normal(4, (L, 2, H, D), "bf16", stream=it)
        vn = rng.normal(5, (L, 2, H, D), "bf16", stream=it)
        out = step.step(to_dev(q, "bf16", cuda), to_dev(kn, "bf16", cuda), to_dev(vn, "bf16", cuda))
        torch.cuda.synchronize()
        ops.check_device_errors(0)
        mirror = to_bits(store.pools)  # append results are checked through attention below
        tabs = np.full((2, 8), -1, dtype=np.int32)
        lens = []
        for i, s in enumerate(["b", "c"]):
            t = store.tables[s]
            tabs[i, :len(t)] = t
            lens.append(store.offsets[s] + 1)
            pos = store.offsets[s]
            for l in range(L):
                assert np.array_equal(mirror[l, 0, t[pos // bs], :, pos % bs], kn[l, i])
        for l in range(L):
            ref = opaged.paged_decode(q[l], mirror[l, 0], mirror[l, 1], tabs, np.array(lens), "bf16")
            assert attn_err(out[l], ref) <= 2e-3
        step.advance()
    # a's prefix blocks still hold a's data after b and c wrote past them
    assert np.array_equal(_dev_seq(store, store.tables["a"], 70), want_a)

    # evict to host: drop the sequences, move the cache's blocks out, then
    # overwrite the freed device blocks before reloading
    for s in ("a", "b", "c"):
        store.free_sequence(s)
    held = cache.device_blocks()
    assert all(store.bm.get_refcount(b) == 1 for b in held)
    moved = cache.evict_to_host(len(held))
    assert moved == len(held) and cache.device_blocks() == []
    assert set(cache.entry_location(state)) == {"host"}
    store.add_sequence("junk", 0)
    junk = torch.full((L, H, 16 * store.bm.free_blocks, D), 7.0, dtype=torch.bfloat16, device=cuda)
    store.append_tokens("junk", junk, junk)
    store.free_sequence("junk")
    n, state, _ = cache.lookup_sync(hashes)
    tab_d = cache.restore("d", state)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    assert set(cache.entry_location(state)) == {"dev"}
    assert np.array_equal(_dev_seq(store, tab_d, 70), want_a)
    st = cache.stats()
    assert st.host_evicted_blocks == moved and st.host_reloaded_blocks == 5


def test_host_tier_roundtrip_many_chunks(cuda):
    """Pack/D2H and H2D/unpack across several staging chunks (ping-pong)."""
    pools = to_dev(rng.normal(9, (6, 40, 2, 16, 64), "bf16"), "bf16", cuda)
    bb = 2 * 16 * 64 * 2
    tier = PinnedHostTier(40, 6, bb, cuda, staging_bytes=3 * 6 * bb)
    ids = [5, 9, 0, 33, 12, 13, 14, 39, 2, 7, 21]
    before = to_bits(pools)
    slots = tier.evict(pools, ids)
    fresh = [1, 3, 4, 6, 8, 10, 11, 15, 16, 17, 18]
    tier.reload(pools, slots, fresh)
    tier.sync()
    after = to_bits(pools)
    for a, b in zip(ids, fresh):
        assert np.array_equal(after[:, b], before[:, a])
    ops.check_device_errors(0)


@pytest.mark.parametrize("quantized", [False, True])
def test_paged_entry_disk_round_trip(cuda, tmp_path, quantized):
    """A cached paged prefix spilled to the disk tier and loaded into a fresh
    store: the same K/V (codes, scales, biases) bit for bit, a restorable entry,
    and the file readable as the per-layer states of the reference's format."""
    from mlxz_b200.engine import PagedKVStore, QuantizedPagedKVStore
    from mlxz_b200.prefix_cache import PagedPrefixCache, PrefixCacheDisk

    L, H, D, bs, n = 2, 2, 128, 16, 37

    def make():
        if quantized:
            return QuantizedPagedKVStore(L, 16, H, D, bs, bits=8, device=cuda)
        return PagedKVStore(L, 16, H, D, bs, torch.bfloat16, cuda)

    a = make()
    a.add_sequence("s")
    kv = torch.randn(L, H, n, D, device=cuda).to(torch.bfloat16)
    a.append_tokens("s", kv, kv * 2)
    cache_a = PagedPrefixCache(a, 1 << 30)
    hashes = tuple(bytes([i]) * 32 for i in range(5))
    cache_a.store_sync(hashes, "s", n_tokens=n, block_size=8)
    disk = PrefixCacheDisk(tmp_path, 1 << 30, "model")
    assert cache_a.spill_to_disk(hashes, disk)

    b = make()
    cache_b = PagedPrefixCache(b, 1 << 30)
    assert cache_b.load_from_disk(hashes, disk, block_size=8) == n
    got, state, _ = cache_b.lookup_sync(hashes)
    assert got == n
    table_b = cache_b.restore("r", state)
    ta = torch.tensor(a.tables["s"][: -(-n // bs)], device=cuda)
    tb = torch.tensor(table_b, device=cuda)
    for sa, sb in zip(a.pool_stacks(), b.pool_stacks()):
        xa = sa.index_select(1, ta).permute(0, 2, 1, 3, 4).flatten(2, 3)[:, :, :n]
        xb = sb.index_select(1, tb).permute(0, 2, 1, 3, 4).flatten(2, 3)[:, :, :n]
        assert torch.equal(xa, xb)
    _, states, ctype = disk.lookup_sync(hashes)
    assert ctype == ("QuantizedKVCache" if quantized else "KVCache") and len(states) == L
    if not quantized:
        assert torch.equal(states[1][0].to(cuda)[0], kv[1])
        assert torch.equal(states[1][1].to(cuda)[0], kv[1] * 2)
