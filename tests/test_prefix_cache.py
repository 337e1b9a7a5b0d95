"""Prefix cache host policy: hasher digests and PrefixCacheMemory behaviour
replayed from the reference's own code (tests/golden), and the refcount
bookkeeping of the paged prefix cache (no kernels: CPU only)."""
import json
import types

import pytest
import torch

from mlxz_b200.paged_attention.block_manager import BlockManager
from mlxz_b200.prefix_cache import PagedPrefixCache, PrefixCacheMemory, RollingPrefixHasher
from tests.conftest import GOLDEN


def test_hasher_matches_reference_digests():
    cases = json.loads((GOLDEN / "hasher.json").read_text())
    for c in cases:
        got = RollingPrefixHasher(c["block_size"]).hash_chunks(c["tokens"])
        assert [d.hex() for d in got] == c["digests"]
    with pytest.raises(ValueError):
        RollingPrefixHasher(0)


class MockKVCache:
    """Tensor-state layer cache with trim (as the reference's tests use)."""

    def __init__(self, seq_len: int, head_dim: int, fill: float) -> None:
        self._keys = torch.full((1, 1, seq_len, head_dim), fill, dtype=torch.float32)
        self._values = torch.full((1, 1, seq_len, head_dim), fill + 1, dtype=torch.float32)

    @property
    def state(self):
        return (self._keys, self._values)

    def is_trimmable(self):
        return True

    def trim(self, n):
        if n <= 0:
            return 0
        self._keys = self._keys[:, :, :-n, :]
        self._values = self._values[:, :, :-n, :]
        return n


TRACES = json.loads((GOLDEN / "prefix_memory_traces.json").read_text())


@pytest.mark.parametrize("ti", range(len(TRACES)))
def test_prefix_memory_replays_reference_trace(ti):
    tr = TRACES[ti]
    cache = PrefixCacheMemory(memory_budget_bytes=tr["budget"])
    for rec in tr["ops"]:
        hashes = tuple(bytes([x]) * 32 for x in rec["key"])
        if rec["op"] == "store":
            layers = [MockKVCache(rec["seq_len"], 4, rec["fill"]) for _ in range(rec["n_layers"])]
            cache.store_sync(hashes, layers, n_tokens=rec["n_tokens"], block_size=rec["block_size"])
        else:
            n, states, ct = cache.lookup_sync(hashes, cache_type=rec["cache_type"])
            assert (n, ct, states is not None) == (rec["n"], rec["result_type"], rec["hit"])
            if states is not None:
                assert int(states[0][0].shape[2]) == rec["state_len"]
                assert len(states) == rec["n_layers"]
                if rec["state_fill"] is not None:
                    assert float(states[0][0].flatten()[0]) == rec["state_fill"]
        st = cache.stats()
        assert {"hits": st.hits, "misses": st.misses, "hit_bytes": st.hit_bytes,
                "evictions": st.evictions, "memory_used_bytes": st.memory_used_bytes} == rec["stats"]
        assert sorted([[h[0] for h in k] for k in cache._entries]) == rec["entries"]


def test_prefix_memory_deep_copy_independence():
    cache = PrefixCacheMemory(10_000_000)
    kv = [MockKVCache(2, 4, 0.0)]
    h = (bytes([1]) * 32,)
    cache.store_sync(h, kv)
    kv[0]._keys.fill_(999.0)
    _, states, _ = cache.lookup_sync(h)
    assert torch.all(states[0][0] == 0)


def _fake_store(n_blocks=64, bs=16, L=2, H=2, D=8):
    st = types.SimpleNamespace()
    st.bm = BlockManager(n_blocks, bs)
    st.block_size = bs
    st.n_layers, st.n_kv_heads, st.head_dim = L, H, D
    st.pools = torch.zeros(1, dtype=torch.bfloat16)
    st.tables, st.offsets = {}, {}
    return st


def test_paged_prefix_refcounts_store_restore_drop():
    st = _fake_store()
    st.tables["a"] = st.bm.allocate(5)  # 70 tokens -> 5 blocks
    st.offsets["a"] = 70
    bpt = 2 * 2 * 2 * 8 * 2  # layers * (K,V) * heads * dim * 2 bytes
    cache = PagedPrefixCache(st, memory_budget_bytes=10 ** 9)
    h = RollingPrefixHasher(16).hash_chunks(list(range(70)))
    cache.store_sync(h, "a", block_size=16)
    # entries at 16, 32, 48, 64, 70 tokens; the cache holds one ref per block
    assert len(cache._entries) == 5
    assert [st.bm.get_refcount(b) for b in st.tables["a"]] == [2] * 5
    assert cache.stats().memory_used_bytes == (16 + 32 + 48 + 64 + 70) * bpt
    n, state, ct = cache.lookup_sync(h[:3] + (b"x" * 32,))
    assert n == 48 and ct == "PagedKVCache"
    table = cache.restore("b", state)
    assert table == st.tables["a"][:3] and st.offsets["b"] == 48
    assert [st.bm.get_refcount(b) for b in table] == [3, 3, 3]
    # the request frees its table and the source sequence goes away
    st.bm.free(st.tables.pop("b"))
    st.bm.free(st.tables.pop("a"))
    assert [st.bm.get_refcount(b) for b in table] == [1, 1, 1]
    # a budget too small for anything drops every entry and every block
    cache._budget = 0
    cache._evict_until_room(1)
    assert not cache._entries and st.bm.free_blocks == st.bm.total_blocks
    assert cache.stats().evictions == 5


def test_paged_prefix_budget_lru_matches_reference_accounting():
    st = _fake_store()
    bpt = 2 * 2 * 2 * 8 * 2
    cache = PagedPrefixCache(st, memory_budget_bytes=20 * bpt)
    for name, n in (("a", 16), ("b", 16)):
        st.tables[name] = st.bm.allocate(1)
        st.offsets[name] = n
    ha = (b"a" * 32,)
    hb = (b"b" * 32,)
    cache.store_sync(ha, "a", block_size=16)
    cache.store_sync(hb, "b", block_size=16)  # evicts a (LRU), budget fits one
    assert cache.lookup_sync(ha)[0] == 0 and cache.lookup_sync(hb)[0] == 16
    assert st.bm.get_refcount(st.tables["a"][0]) == 1  # cache reference released
