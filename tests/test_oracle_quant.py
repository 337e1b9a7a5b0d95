"""The quantisation oracle follows its stated rules (no reference vectors
exist for MLX's affine quantisation here: parity unpinned, rules pinned)."""
import numpy as np
import pytest

from oracle import quant, rng


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_roundtrip_error_within_half_step(bits, dtype):
    x = rng.normal(3, (50, 128), dtype)
    q, s, b = quant.quantize(x, dtype, bits)
    assert q.shape == (50, 128 * bits // 32) and s.shape == (50, 2) and b.shape == (50, 2)
    w = rng.to_f32(x, dtype).astype(np.float64)
    deq = quant.dequantize(q, s, b, bits, 128)
    step = np.repeat(s.view(np.float16).astype(np.float64), 64, axis=-1)
    bias = np.repeat(b.view(np.float16).astype(np.float64), 64, axis=-1)
    # rounding to the grid costs <= half a step (plus fp16 rounding of the bias
    # and of the scale over up to 2^bits steps)
    slack = 0.5 * step + np.abs(bias) * 2.0 ** -11 + step * (2 ** bits) * 2.0 ** -11
    assert np.all(np.abs(deq - w) <= slack + 1e-12)


def test_packing_is_lsb_first():
    x = np.array([[float(i % 16) for i in range(64)]], dtype=np.float64)
    bits16 = rng.from_f64(x, "f16")
    q, s, b = quant.quantize(bits16, "f16", 4)
    # min 0, max 15 -> scale 1, bias 0 -> codes equal the values
    assert s.view(np.float16)[0, 0] == 1.0 and b.view(np.float16)[0, 0] == 0.0
    assert q[0, 0] == sum(i << (4 * i) for i in range(8))
    assert np.array_equal(quant.unpack(q, 4, 64)[0], (np.arange(64) % 16).astype(np.uint32))


def test_constant_group_codes_are_zero():
    x = rng.from_f64(np.full((2, 64), 0.75), "bf16")
    q, s, b = quant.quantize(x, "bf16", 8)
    assert np.all(q == 0) and np.all(s.view(np.float16) == 0)
    assert np.all(quant.dequantize(q, s, b, 8, 64) == 0.75)


def test_rint_is_round_half_even():
    # values 0, 0.5, 1.5, 2.5 ... with scale 1 (max-min = 255 steps of 1 at 8 bits)
    vals = np.zeros(64)
    vals[0], vals[1] = 0.0, 255.0
    vals[2:6] = [0.5, 1.5, 2.5, 3.5]
    q, s, b = quant.quantize(rng.from_f64(vals[None], "f16"), "f16", 8)
    codes = quant.unpack(q, 8, 64)[0]
    assert list(codes[2:6]) == [0, 2, 2, 4]
