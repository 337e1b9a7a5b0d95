"""The contiguous request caches on the GPU: KVCache appends bit-exact, the
quantised cache packs bit-exact to the quantisation oracle, conversion and
restore keep the data and the offset."""
import numpy as np
import pytest
import torch

from mlxz_b200.engine.cache_utils import (KVCache, QuantizedKVCache, RestoringQuantizedKVCache,
                                          _quantize_layer, build_prompt_cache)
from oracle import quant, rng
from tests.gpu_util import to_bits, to_dev

pytestmark = pytest.mark.gpu


def _chunks(seed, B, H, lens, D, dtype="bf16"):
    return [(to_dev(rng.normal(seed + i, (B, H, n, D), dtype, stream=1), dtype, "cuda"),
             to_dev(rng.normal(seed + i, (B, H, n, D), dtype, stream=2), dtype, "cuda"))
            for i, n in enumerate(lens)]


def test_kv_cache_appends_bit_exact_across_growth(cuda):
    B, H, D = 2, 4, 128
    parts = _chunks(3, B, H, [5, 1, 300, 1, 0, 17], D)
    c = KVCache()
    for k, v in parts:
        kk, vv = c.update_and_fetch(k, v)
    torch.cuda.synchronize()
    ref_k = torch.cat([k for k, _ in parts], dim=2)
    ref_v = torch.cat([v for _, v in parts], dim=2)
    assert c.offset == ref_k.shape[2] == 324
    assert c.keys.shape[2] == 512  # grown in steps of 256
    assert torch.equal(kk, ref_k) and torch.equal(vv, ref_v)


def _quant_ref(x: torch.Tensor, bits):
    """Oracle quantisation of [B, H, n, D] bf16 -> (codes, scales, biases) numpy."""
    B, H, n, D = x.shape
    q, s, b = quant.quantize(to_bits(x).reshape(-1, D), "bf16", bits)
    return (q.view(np.int32).reshape(B, H, n, -1), s.reshape(B, H, n, -1), b.reshape(B, H, n, -1))


@pytest.mark.parametrize("bits", [4, 8])
def test_quantized_cache_bit_exact_to_oracle(cuda, bits):
    B, H, D = 2, 2, 128
    parts = _chunks(11, B, H, [7, 1, 260], D)
    c = QuantizedKVCache(group_size=64, bits=bits)
    for k, v in parts:
        state = c.update_and_fetch(k, v)
    torch.cuda.synchronize()
    assert c.offset == 268
    for got, src in ((state[0], torch.cat([k for k, _ in parts], 2)),
                     (state[1], torch.cat([v for _, v in parts], 2))):
        rq, rs, rb = _quant_ref(src, bits)
        assert np.array_equal(got[0].cpu().numpy(), rq)
        assert np.array_equal(got[1].cpu().view(torch.int16).numpy().view(np.uint16), rs)
        assert np.array_equal(got[2].cpu().view(torch.int16).numpy().view(np.uint16), rb)


def test_to_quantized_and_restore_keep_offset(cuda):
    B, H, D = 1, 8, 128
    parts = _chunks(21, B, H, [40, 3], D)
    c = KVCache()
    for k, v in parts:
        c.update_and_fetch(k, v)
    q = _quantize_layer(c, group_size=64, bits=8)
    assert isinstance(q, RestoringQuantizedKVCache) and q.offset == 43
    # restore the quantised state into a fresh cache, then keep appending
    r = build_prompt_cache(type("M", (), {"layers": [0]})(), quantized=True)[0]
    r.state = q.state
    assert r.offset == 43
    k2, v2 = _chunks(22, B, H, [2], D)[0]
    st = r.update_and_fetch(k2, v2)
    torch.cuda.synchronize()
    assert r.offset == 45
    all_k = torch.cat([k for k, _ in parts] + [k2], 2)
    rq, rs, rb = _quant_ref(all_k, 8)
    assert np.array_equal(st[0][0].cpu().numpy(), rq)
    assert np.array_equal(st[0][1].cpu().view(torch.int16).numpy().view(np.uint16), rs)
