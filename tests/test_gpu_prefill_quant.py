"""GPU: chunked prefill over a quantised paged store.

* mz_kv_dequant_blocks is bit-exact against the dequantisation rule written
  down in oracle/quant.py (f32(scale) * q + f32(bias), multiply and add
  rounded separately, then rounded to nearest in the output type).
* PagedPrefillStep over a QuantizedPagedKVStore (quantise-on-append of the
  chunk, attention over the dequantised cache + chunk) matches the float64
  causal oracle on those dequantised values within the attention tolerance:
  max(|out - ref| - u*|ref|, 0) / max|ref| <= 2e-3 (fp32 outputs, u = 0).
"""
import numpy as np
import pytest
import torch

from mlxz_b200 import ops
from oracle import paged as opaged
from oracle import quant as oquant
from oracle import rng
from tests.gpu_util import TORCH, attn_err, to_dev

pytestmark = pytest.mark.gpu
ATOL_REL = 2e-3


def _deq_ref(codes: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, bits: int,
             out_dtype: torch.dtype) -> torch.Tensor:
    """Dequantised rows [..., D] of out_dtype, computed on the CPU."""
    words = codes.cpu().numpy().view(np.uint32)
    D = scales.shape[-1] * 64
    q = oquant.unpack(words, bits, D).astype(np.float32)
    s = scales.cpu().float().numpy()[..., None]
    b = biases.cpu().float().numpy()[..., None]
    qg = q.reshape(*q.shape[:-1], D // 64, 64)
    v = (qg * s).astype(np.float32) + b
    return torch.from_numpy(v.astype(np.float32).reshape(q.shape)).to(out_dtype)


def _filled_store(cuda, bits, L=1, n_blocks=24, Hkv=2, D=128, bs=16, seed=1):
    from mlxz_b200.engine import QuantizedPagedKVStore

    st = QuantizedPagedKVStore(L, n_blocks, Hkv, D, bs, bits=bits, device=cuda)
    slots = torch.arange(n_blocks * bs, dtype=torch.int64, device=cuda)
    for l in range(L):
        k = to_dev(rng.normal(seed, (Hkv, n_blocks * bs, D), "bf16", stream=2 * l), "bf16", cuda)
        v = to_dev(rng.normal(seed, (Hkv, n_blocks * bs, D), "bf16", stream=2 * l + 1), "bf16",
                   cuda)
        ops.kv_quant_append(st.qpools(l), k, v, slots)
    torch.cuda.synchronize()
    return st


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
def test_dequant_blocks_bit_exact(cuda, bits, out_dtype):
    st = _filled_store(cuda, bits)
    pools = st.qpools(0)
    ids = [5, 0, 23, 5, 11]
    ids_t = torch.tensor(ids, dtype=torch.int32, device=cuda)
    shape = (len(ids), st.n_kv_heads, st.block_size, st.head_dim)
    ko = torch.empty(shape, dtype=out_dtype, device=cuda)
    vo = torch.empty_like(ko)
    ops.kv_dequant_blocks(pools, ids_t, ko, vo)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    kc, ks, kb, vc, vs, vb = pools
    idx = torch.tensor(ids)
    want_k = _deq_ref(kc.cpu()[idx], ks.cpu()[idx], kb.cpu()[idx], bits, out_dtype)
    want_v = _deq_ref(vc.cpu()[idx], vs.cpu()[idx], vb.cpu()[idx], bits, out_dtype)
    assert torch.equal(ko.cpu().view(torch.int16), want_k.view(torch.int16))
    assert torch.equal(vo.cpu().view(torch.int16), want_v.view(torch.int16))


@pytest.mark.parametrize("bits", [8, 4])
def test_quantized_chunked_prefill(cuda, bits):
    """Two sequences with quantised cached prefixes (70 and 0 tokens) prefill
    chunks of 45 and 33 tokens over 2 layers through PagedPrefillStep."""
    from mlxz_b200.engine import PagedPrefillStep, QuantizedPagedKVStore

    L, Hkv, G, D, bs, dtype = 2, 2, 4, 128, 16, "bf16"
    Hq = Hkv * G
    st = QuantizedPagedKVStore(L, 32, Hkv, D, bs, bits=bits, device=cuda)
    pre = {"a": 70, "b": 0}
    chunk = {"a": 45, "b": 33}
    for i, (s, n) in enumerate(pre.items()):
        st.add_sequence(s)
        if n:
            k = to_dev(rng.normal(20 + i, (L, Hkv, n, D), dtype, stream=1), dtype, cuda)
            v = to_dev(rng.normal(20 + i, (L, Hkv, n, D), dtype, stream=2), dtype, cuda)
            st.append_tokens(s, k, v)
    step = PagedPrefillStep(st, [(s, chunk[s]) for s in pre], Hq)
    T = sum(chunk.values())
    for l in range(L):
        q = rng.normal(30, (T, Hq, D), dtype, stream=l)
        k = rng.normal(31, (T, Hkv, D), dtype, stream=l)
        v = rng.normal(32, (T, Hkv, D), dtype, stream=l)
        out = step.layer(l, to_dev(q, dtype, cuda), to_dev(k, dtype, cuda),
                         to_dev(v, dtype, cuda), out_dtype=torch.float32)
        torch.cuda.synchronize()
        ops.check_device_errors(0)
        kc, ks, kb, vc, vs, vb = st.qpools(l)
        kdq = _deq_ref(kc, ks, kb, bits, TORCH[dtype]).float().numpy()  # [N, H, bs, D]
        vdq = _deq_ref(vc, vs, vb, bits, TORCH[dtype]).float().numpy()
        r = 0
        for s in pre:
            n, c = chunk[s], pre[s] + chunk[s]
            t = st.tables[s]
            kk, vv = opaged.gather(kdq, vdq, t, c, bs)  # (H, c, D)
            qb = rng.to_f32(q[r:r + n], dtype).transpose(1, 0, 2)
            ref = opaged.prefill_attention(qb, kk, vv, c - n).transpose(1, 0, 2)
            assert attn_err(out[r:r + n], ref) <= ATOL_REL, (s, l)
            r += n
    step.finish()
    assert st.offsets == {"a": 115, "b": 33}
