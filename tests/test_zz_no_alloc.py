"""The allocation-free decode entry point, mz_paged_decode_noalloc.

It serves callers that cannot allocate device memory when they call in (a
host whose own pool already owns the GPU, an FFI binding without a device
allocator, a latency-bound path that may not synchronise on cudaMalloc): its
scratch is a fixed array inside the library instead of a caller workspace.

Checked here through the C ABI (ctypes): two calls in a row give the same
result as mz_paged_decode with a workspace, within the attention tolerance
the other tests use; oversized problems are refused with MZ_ERR_TOO_LARGE.
This file sorts last so a run that stops at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from mlxz_b200 import _native, ops
from oracle import paged as opaged
from tests.gpu_util import attn_err, random_paged_case, to_dev

pytestmark = pytest.mark.gpu
ATOL_REL = 2e-3


def _noalloc(out, q, kp, vp, tables, ctx, n_heads, num_warps=0):
    """Call mz_paged_decode_noalloc for q [B, Hq, D] -> out [B, Hq, D]."""
    lib = _native.lib()
    B, Hq, D = q.shape
    _, Hkv, bs, _ = kp.shape
    err = ops.error_word(q.device.index)
    return lib.mz_paged_decode_noalloc(
        out.data_ptr(), ops.dtype_code(out.dtype), out.stride(0), 0, out.stride(1),
        q.data_ptr(), q.stride(0), 0, q.stride(1), 1, kp.data_ptr(), vp.data_ptr(),
        tables.data_ptr(), tables.shape[1], ctx.data_ptr(), B, n_heads, Hkv, D, bs, kp.shape[0],
        ctypes.c_float(D ** -0.5), ops.dtype_code(q.dtype), num_warps, err.data_ptr(),
        torch.cuda.current_stream(q.device).cuda_stream)


@pytest.mark.parametrize("dtype,D,G,ctx,nw", [
    ("bf16", 128, 4, [513, 1, 15, 16, 17, 100, 2048, 777, 0, 4000], 0),
    ("bf16", 128, 4, [513, 1, 15, 16, 17, 100, 2048, 777, 0, 4000], 8),
    ("f16", 64, 4, [38, 129, 301, 512], 0),
])
def test_noalloc_matches_workspace_entry_point(cuda, dtype, D, G, ctx, nw):
    Hkv = 4
    case = random_paged_case(123 + D, len(ctx), Hkv, D, 16, ctx, dtype, G=G)
    kp, vp = to_dev(case["kp"], dtype, cuda), to_dev(case["vp"], dtype, cuda)
    q = to_dev(case["q"][:, 0], dtype, cuda)
    tables = torch.from_numpy(case["tables"]).to(cuda)
    ctx_t = torch.from_numpy(case["ctx"]).to(cuda)
    # existing entry point (caller workspace), as the reference result
    want = ops.paged_decode(q, kp, vp, tables, ctx_t, num_warps=nw, out_dtype=torch.float32)
    oracle = opaged.paged_decode(case["q"][:, 0], case["kp"], case["vp"], case["tables"],
                                 case["ctx"], dtype)
    for call in range(2):
        out = torch.full_like(want, float("nan"))
        rc = _noalloc(out, q, kp, vp, tables, ctx_t, Hkv * G, num_warps=nw)
        assert rc == _native.MZ_OK, _native.last_error()
        torch.cuda.synchronize()
        ops.check_device_errors(cuda.index or 0)
        assert attn_err(out, want.cpu().numpy()) <= ATOL_REL, f"call {call}"
        assert attn_err(out, oracle) <= ATOL_REL, f"call {call}"
        for b, c in enumerate(ctx):
            if c == 0:
                assert torch.count_nonzero(out[b]) == 0


def test_noalloc_native_dtype_output_twice(cuda):
    """bf16 output, same buffers reused across two calls."""
    ctx = [700, 33, 4096]
    case = random_paged_case(5, len(ctx), 8, 128, 16, ctx, "bf16", G=4)
    kp, vp = to_dev(case["kp"], "bf16", cuda), to_dev(case["vp"], "bf16", cuda)
    q = to_dev(case["q"][:, 0], "bf16", cuda)
    tables = torch.from_numpy(case["tables"]).to(cuda)
    ctx_t = torch.from_numpy(case["ctx"]).to(cuda)
    want = ops.paged_decode(q, kp, vp, tables, ctx_t)
    out = torch.empty_like(want)
    for _ in range(2):
        out.fill_(0)
        assert _noalloc(out, q, kp, vp, tables, ctx_t, 32) == _native.MZ_OK
        torch.cuda.synchronize()
        assert attn_err(out.float(), want.float().cpu().numpy()) <= ATOL_REL


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    B, Hkv, D = 20000, 8, 128
    kp = torch.zeros(4, Hkv, 16, D, dtype=torch.bfloat16, device=cuda)
    q = torch.zeros(B, Hkv * 16, D, dtype=torch.bfloat16, device=cuda)
    tables = torch.zeros(B, 1, dtype=torch.int32, device=cuda)
    ctx = torch.ones(B, dtype=torch.int32, device=cuda)
    out = torch.empty_like(q)
    rc = _noalloc(out, q, kp, kp, tables, ctx, Hkv * 16)
    assert rc == _native.MZ_ERR_TOO_LARGE
    code, msg = _native.last_error()
    assert code == rc and "scratch" in msg
