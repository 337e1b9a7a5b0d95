"""Disk tier of the prefix cache (host side): the reference's own cases from
tests/unit/test_prefix_disk.py restated over torch tensors, plus the file
format (tensor names, sidecar fields, checksum) and quantised states."""
import json
import os
import time
from pathlib import Path

import pytest
import torch

from mlxz_b200.prefix_cache.disk import (PrefixCacheDisk, flatten_states, state_checksum,
                                         unflatten_states)


def _make_mock_kv_cache(n_layers=2, seq_len=4, head_dim=8, dtype=torch.float32):
    class MockKVCache:
        def __init__(self):
            self._keys = torch.zeros((1, 1, seq_len, head_dim), dtype=dtype)
            self._values = torch.ones((1, 1, seq_len, head_dim), dtype=dtype)

        @property
        def state(self):
            return (self._keys, self._values)

    return [MockKVCache() for _ in range(n_layers)]


def _make_hashes(n):
    return tuple(bytes([i] * 32) for i in range(n))


def test_store_and_lookup(tmp_path):
    cache = PrefixCacheDisk(tmp_path, disk_budget_bytes=100_000_000, model_hash="test")
    hashes = _make_hashes(2)
    cache.store_sync(hashes, _make_mock_kv_cache(), n_tokens=4)
    n, states, ctype = cache.lookup_sync(hashes)
    assert n == 4 and states is not None and ctype == "MockKVCache" and len(states) == 2
    assert torch.equal(states[1][0], torch.zeros(1, 1, 4, 8))
    assert torch.equal(states[1][1], torch.ones(1, 1, 4, 8))


def test_miss_returns_zero_none(tmp_path):
    cache = PrefixCacheDisk(tmp_path, disk_budget_bytes=100_000_000, model_hash="test")
    assert cache.lookup_sync(_make_hashes(3)) == (0, None, None)


def test_checksum_validation(tmp_path):
    cache = PrefixCacheDisk(tmp_path, disk_budget_bytes=100_000_000, model_hash="test")
    hashes = _make_hashes(1)
    cache.store_sync(hashes, _make_mock_kv_cache(), n_tokens=4)
    entry = cache._entry_path(hashes)
    meta_path = cache._meta_path(entry)
    meta = json.loads(meta_path.read_text())
    meta["checksum"] = "0" * 64
    meta_path.write_text(json.dumps(meta))
    assert cache.lookup_sync(hashes) == (0, None, None)
    assert not entry.exists() and not meta_path.exists()


def test_corrupt_tensor_bytes_are_caught(tmp_path):
    cache = PrefixCacheDisk(tmp_path, disk_budget_bytes=100_000_000, model_hash="test")
    hashes = _make_hashes(1)
    cache.store_sync(hashes, _make_mock_kv_cache(), n_tokens=4)
    entry = cache._entry_path(hashes)
    raw = bytearray(entry.read_bytes())
    raw[-1] ^= 0xFF  # flip a bit of the last tensor's data
    entry.write_bytes(bytes(raw))
    assert cache.lookup_sync(hashes) == (0, None, None)
    assert not entry.exists()


def test_graceful_io_failure(tmp_path):
    blocker = tmp_path / "file"
    blocker.write_text("x")  # a file where the directory would go
    cache = PrefixCacheDisk(blocker, disk_budget_bytes=100_000_000, model_hash="test")
    cache.store_sync(_make_hashes(1), _make_mock_kv_cache(), n_tokens=4)
    assert cache.lookup_sync(_make_hashes(1)) == (0, None, None)


def test_duplicate_store_is_noop(tmp_path):
    cache = PrefixCacheDisk(tmp_path, disk_budget_bytes=100_000_000, model_hash="test")
    hashes = _make_hashes(1)
    cache.store_sync(hashes, _make_mock_kv_cache(), n_tokens=4)
    cache.store_sync(hashes, _make_mock_kv_cache(), n_tokens=4)
    assert len(list((tmp_path / "test").glob("*.safetensors"))) == 1


def test_lru_eviction_by_mtime(tmp_path):
    kv = _make_mock_kv_cache()
    entry_size = sum(a.numel() * a.element_size() for layer in kv for a in layer.state)
    cache = PrefixCacheDisk(tmp_path, disk_budget_bytes=entry_size * 2 + 1000, model_hash="test")
    h1, h2, h3 = (bytes([1] * 32),), (bytes([2] * 32),), (bytes([3] * 32),)
    cache.store_sync(h1, _make_mock_kv_cache(), n_tokens=4)
    os.utime(cache._entry_path(h1), (time.time() - 20, time.time() - 20))
    cache.store_sync(h2, _make_mock_kv_cache(), n_tokens=4)
    os.utime(cache._entry_path(h2), (time.time() - 10, time.time() - 10))
    cache.store_sync(h3, _make_mock_kv_cache(), n_tokens=4)
    files = list((tmp_path / "test").glob("*.safetensors"))
    assert len(files) <= 2
    assert not cache._entry_path(h1).exists()  # the oldest went first
    assert cache.stats().evictions >= 1


def test_model_hash_isolation(tmp_path):
    a = PrefixCacheDisk(tmp_path, 100_000_000, model_hash="model_a")
    b = PrefixCacheDisk(tmp_path, 100_000_000, model_hash="model_b")
    hashes = _make_hashes(1)
    a.store_sync(hashes, _make_mock_kv_cache(), n_tokens=4)
    assert b.lookup_sync(hashes)[0] == 0
    assert a.lookup_sync(hashes)[0] == 4


def test_longest_prefix_and_cache_type_filter(tmp_path):
    cache = PrefixCacheDisk(tmp_path, 100_000_000, model_hash="m")
    h = _make_hashes(4)
    cache.store_sync(h[:2], _make_mock_kv_cache(seq_len=2), n_tokens=2)
    n, _, ctype = cache.lookup_sync(h)  # the longest stored prefix of 4 hashes
    assert (n, ctype) == (2, "MockKVCache")
    assert cache.lookup_sync(h, cache_type="QuantizedKVCache")[0] == 0


def test_file_format_fields(tmp_path):
    cache = PrefixCacheDisk(tmp_path, 100_000_000, model_hash="m")
    h = _make_hashes(1)
    cache.store_sync(h, _make_mock_kv_cache(n_layers=3, dtype=torch.bfloat16))
    meta = json.loads(cache._meta_path(cache._entry_path(h)).read_text())
    assert meta["format_version"] == "1" and meta["n_layers"] == 3 and meta["n_tokens"] == 4
    assert meta["tensor_keys"] == sorted(f"l{i}_t{j}" for i in range(3) for j in range(2))
    from safetensors.torch import load_file
    t = load_file(str(cache._entry_path(h)))
    assert meta["checksum"] == state_checksum(t) and t["l2_t1"].dtype == torch.bfloat16


def test_quantized_states_round_trip_names(tmp_path):
    g = torch.Generator().manual_seed(3)
    codes = torch.randint(-2**31, 2**31 - 1, (1, 2, 5, 32), dtype=torch.int32, generator=g)
    sc = torch.randn(1, 2, 5, 2, generator=g).half()
    states = [((codes, sc, sc + 1), (codes + 1, sc * 2, sc - 1)) for _ in range(2)]
    flat = flatten_states(states)
    assert sorted(flat) == sorted(f"l{i}_t{j}_q{k}" for i in range(2) for j in range(2)
                                  for k in range(3))
    back = unflatten_states(flat, 2)
    assert len(back[0]) == 6 and torch.equal(back[1][0], codes)
    cache = PrefixCacheDisk(tmp_path, 100_000_000, model_hash="m")
    cache.store_states(_make_hashes(1), states, 5, "QuantizedKVCache")
    n, got, ctype = cache.lookup_sync(_make_hashes(1), cache_type="QuantizedKVCache")
    assert (n, ctype) == (5, "QuantizedKVCache")
    assert all(torch.equal(a, b) for a, b in zip(got[1], back[1]))
