"""Helpers shared by the GPU parity tests (uint16 bit patterns <-> torch)."""
import hashlib

import numpy as np
import torch

from oracle import rng

TORCH = {"f16": torch.float16, "bf16": torch.bfloat16}


def to_dev(bits: np.ndarray, dtype: str, device) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits).astype(np.int16)).view(TORCH[dtype])
    return t.to(device)


def to_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def sha_t(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def rel_err(out, ref) -> float:
    """max |out - ref| / max |ref| (the attention tolerance metric)."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30))


# Unit roundoff of the output element type: storing a result in bf16 (8-bit
# significand) or fp16 (11-bit) alone moves it by up to this fraction of its
# magnitude, so the 2e-3 attention bar is applied to the error beyond that.
UNIT_ROUNDOFF = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11, torch.float32: 0.0}


def attn_err(out: torch.Tensor, ref) -> float:
    """Attention error metric: max(|out - ref| - u*|ref|, 0) / max|ref|, with u
    the unit roundoff of out's dtype (0 for float32 outputs)."""
    u = UNIT_ROUNDOFF[out.dtype]
    o = out.detach().float().cpu().numpy().astype(np.float64)
    r = np.asarray(ref, dtype=np.float64)
    excess = np.maximum(np.abs(o - r) - u * np.abs(r), 0.0)
    return float(excess.max() / max(np.abs(r).max(), 1e-30))


def random_paged_case(seed, B, Hkv, D, bs, ctx, dtype, n_blocks=None, nq=1, G=4):
    """Seeded pools/tables/q for a ragged batch (oracle-side uint16 bits)."""
    need = [(c + bs - 1) // bs for c in ctx]
    n_blocks = n_blocks or max(1, int(sum(need) * 1.1) + 2)
    perm = rng.permutation(seed, n_blocks)
    maxb = max([1] + need)
    tables = np.full((B, maxb), -1, dtype=np.int32)
    used = 0
    for b in range(B):
        tables[b, :need[b]] = perm[used:used + need[b]]
        used += need[b]
    kp = rng.normal(seed, (n_blocks, Hkv, bs, D), dtype, stream=1)
    vp = rng.normal(seed, (n_blocks, Hkv, bs, D), dtype, stream=2)
    q = rng.normal(seed, (B, nq, Hkv * G, D), dtype, stream=3)
    return dict(kp=kp, vp=vp, q=q, tables=tables, ctx=np.array(ctx, dtype=np.int32),
                n_blocks=n_blocks)
