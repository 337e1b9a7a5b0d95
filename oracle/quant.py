"""Affine group quantisation of KV rows (oracle; test infrastructure).

The reference quantises KV through mlx_lm's QuantizedKVCache
(src/mlxz/engine/cache_utils.py:54-92, `KVCache.to_quantized(group_size,
bits)`), i.e. MLX's affine quantisation, whose published definition is, per
group of `group` consecutive values along the last axis,
    scale = (max - min) / (2^bits - 1),  bias = min,
    q = round((w - bias) / scale),  w ~ scale * q + bias,
with q packed little-end-first into uint32 words.  MLX itself cannot run in
this environment, so its own rounding is not pinned; this module writes the
rules down exactly, and the CUDA kernel must match it bit for bit:

  1. w is the fp16/bf16 input widened to float32 (exact);
  2. mn, mx = group min / max (float32);
  3. scale = fl32(fl32(mx - mn) / fl32(2^bits - 1)), IEEE round-to-nearest-even;
  4. scale16 = fp16(scale), bias16 = fp16(mn), both round-to-nearest-even;
  5. q = clamp(rint(fl32(fl32(w - f32(bias16)) / f32(scale16))), 0, 2^bits - 1)
     with rint = round half to even; if scale16 == 0 (a constant group or a
     range below fp16's smallest subnormal), q = 0;
  6. element i of a row goes to word i // (32 // bits), bits
     [bits * (i % (32 // bits)), ...) (least significant first);
  7. dequantised value: f32(scale16) * q + f32(bias16).
Scales and biases are stored as fp16 (the build's chosen format; MLX keeps
them in the input dtype).  Inputs must be finite with |w| <= 65504.

Standing of this rule (parity unpinned).  The rule above is this build's own
restatement of the documented affine form.  Nothing pins it to MLX 0.22.1 /
mlx-lm 0.22.1 (the reference's pins, pyproject.toml:10-11): MLX cannot run
here, and no reference test or fixture holds quantised values
(tests/unit/test_cache_utils.py:49-57 checks shapes and offsets only).  MLX's
implementation may choose the pair differently: for example, taking as the
bias whichever group edge (min or max) has the larger magnitude, with a
scale whose sign follows that edge, rescaled so that the edge itself is
exactly representable.  Where it does, the codes, scales and biases that
quantise-on-append writes differ from what mlx_lm's QuantizedKVCache would
hold for the same input, and "bit-exact quantised packing" holds against
this rule only.  The dequantisation w = scale * q + bias, the group size,
the packing and the layout do not depend on how the pair was chosen, so the
dequant-fused attention reads either kind of code (tested with negative
scales and edge biases).
"""
from __future__ import annotations

import numpy as np

from .rng import to_f32


def quantize(x_bits: np.ndarray, dtype: str, bits: int, group: int = 64
             ) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """x_bits: uint16 patterns [..., D] of `dtype` ('f16' | 'bf16').

    Returns (q uint32 [..., D*bits/32], scales uint16 fp16 bits [..., D/group],
    biases uint16 fp16 bits [..., D/group])."""
    x = to_f32(x_bits, dtype)
    D = x.shape[-1]
    assert D % group == 0 and 32 % bits == 0
    xg = x.reshape(*x.shape[:-1], D // group, group)
    mn = xg.min(axis=-1)
    mx = xg.max(axis=-1)
    nb = np.float32(2 ** bits - 1)
    scale = ((mx - mn).astype(np.float32) / nb).astype(np.float32)
    s16 = scale.astype(np.float16)
    b16 = mn.astype(np.float16)
    sf = s16.astype(np.float32)[..., None]
    bf = b16.astype(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        qf = np.rint(((xg - bf).astype(np.float32) / sf).astype(np.float32))
    qf = np.where(sf == 0, np.float32(0), qf)
    q = np.clip(qf, 0, 2 ** bits - 1).astype(np.uint32).reshape(x.shape)
    per = 32 // bits
    qw = q.reshape(*x.shape[:-1], D // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * np.uint32(bits))
    words = np.bitwise_or.reduce(qw << shifts, axis=-1).astype(np.uint32)
    return words, s16.view(np.uint16), b16.view(np.uint16)


def unpack(words: np.ndarray, bits: int, D: int) -> np.ndarray:
    """uint32 words [..., D*bits/32] -> integer codes [..., D] (uint32)."""
    per = 32 // bits
    shifts = np.arange(per, dtype=np.uint32) * np.uint32(bits)
    q = (words[..., None] >> shifts) & np.uint32(2 ** bits - 1)
    return q.reshape(*words.shape[:-1], D)


def dequantize(words: np.ndarray, scales: np.ndarray, biases: np.ndarray, bits: int,
               D: int, group: int = 64) -> np.ndarray:
    """Dequantised rows [..., D] as float64 (f32(scale16) * q + f32(bias16))."""
    q = unpack(words, bits, D).astype(np.float64)
    s = scales.view(np.float16).astype(np.float64)
    b = biases.view(np.float16).astype(np.float64)
    qg = q.reshape(*q.shape[:-1], D // group, group)
    return (qg * s[..., None] + b[..., None]).reshape(q.shape)
