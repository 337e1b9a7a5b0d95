"""Cache construction helpers (host logic, no kernel calls): the reference's
own cases from tests/unit/test_cache_utils.py:21-57, restated for the CUDA
caches, plus state/offset/trim bookkeeping."""
import pytest
import torch

from mlxz_b200.config import KVConfig
from mlxz_b200.engine.cache_utils import (KVCache, QuantizedKVCache, RestoringQuantizedKVCache,
                                          _state_token_count, build_prompt_cache,
                                          cache_type_name, should_quantize_cache,
                                          trim_prompt_cache)


class _DummyModel:
    def __init__(self, n_layers: int = 2) -> None:
        self.layers = [object() for _ in range(n_layers)]


def test_should_quantize_cache_uses_total_requested_tokens():
    cfg = KVConfig(quantized_kv_start=256)
    assert not should_quantize_cache(cfg, 255)
    assert should_quantize_cache(cfg, 256)


def test_build_prompt_cache_keeps_short_requests_on_standard_kv():
    cache = build_prompt_cache(_DummyModel(), quantized=False)
    assert len(cache) == 2
    assert isinstance(cache[0], KVCache)
    assert not isinstance(cache[0], QuantizedKVCache)
    assert cache_type_name(cache) == "KVCache"


def test_build_prompt_cache_quantizes_long_requests():
    cache = build_prompt_cache(_DummyModel(), quantized=True, group_size=64, bits=8)
    assert len(cache) == 2
    assert isinstance(cache[0], RestoringQuantizedKVCache)
    assert cache_type_name(cache) == "QuantizedKVCache"
    assert cache[0].bits == 8 and cache[0].group_size == 64 and cache[0].offset == 0


def test_restoring_quantized_cache_state_restores_offset():
    cache = RestoringQuantizedKVCache(group_size=64, bits=8)
    keys = torch.zeros((1, 2, 3, 4), dtype=torch.float16)
    values = torch.zeros((1, 2, 3, 4), dtype=torch.float16)
    cache.state = (keys, values)
    assert cache.offset == 3
    assert cache.state[0].shape[2] == 3


def test_plain_quantized_cache_keeps_offset_on_restore():
    cache = QuantizedKVCache(group_size=64, bits=4)
    codes = torch.zeros((1, 2, 5, 16), dtype=torch.int32)
    sc = torch.zeros((1, 2, 5, 2), dtype=torch.float16)
    cache.state = ((codes, sc, sc), (codes, sc, sc))
    assert cache.offset == 0  # as mlx_lm's: the restoring subclass exists for this
    r = RestoringQuantizedKVCache(group_size=64, bits=4)
    r.state = ((codes, sc, sc), (codes, sc, sc))
    assert r.offset == 5
    assert r.trim(2) == 2 and r.offset == 3
    assert [t.shape[2] for t in r.state[0]] == [3, 3, 3]


def test_state_token_count_forms():
    t = torch.zeros(1, 2, 7, 4)
    assert _state_token_count((t, t)) == 7
    assert _state_token_count(((t, t, t), (t, t, t))) == 7
    assert _state_token_count((torch.zeros(9), None)) == 9
    assert _state_token_count(()) == 0
    assert _state_token_count(((), ())) == 0


def test_kv_cache_state_and_trim():
    c = KVCache()
    assert c.state == (None, None) and c.offset == 0
    k = torch.zeros(1, 2, 6, 8)
    c.state = (k, k)
    assert c.offset == 6
    assert trim_prompt_cache([c], 4) == 4 and c.offset == 2
    assert c.state[0].shape[2] == 2
    assert trim_prompt_cache([c], 0) == 0


@pytest.mark.parametrize("gs,bits", [(32, 8), (64, 3), (128, 4)])
def test_quantized_cache_rejects_unsupported_formats(gs, bits):
    with pytest.raises(ValueError):
        QuantizedKVCache(group_size=gs, bits=bits)


def test_rotating_cache_is_not_offered():
    with pytest.raises(NotImplementedError):
        build_prompt_cache(_DummyModel(), max_kv_size=128)
