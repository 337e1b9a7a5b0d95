// Dequantisation of whole quantised KV blocks into a 16-bit staging pool: the
// prompt pass over a quantised cache attends over the dequantised values of
// the blocks its sequences use (what a quantised cache's attention over a
// prompt chunk computes), so the prefill kernel runs on them unchanged.
//
// HBM-bound elementwise work: each thread turns 8 codes of one row (one or two
// code words, one group's scale and bias) into 8 values, f32(scale) * q +
// f32(bias) with a separate multiply and add (no fused rounding), rounded to
// the output type, stored as one 16-byte vector.
#include "common.cuh"

namespace mz {
namespace {

template <int BITS, bool BF16>
__global__ void dequant_blocks_kernel(uint16_t *__restrict__ ko, uint16_t *__restrict__ vo,
                                      const uint32_t *__restrict__ kc,
                                      const __half *__restrict__ ks,
                                      const __half *__restrict__ kb,
                                      const uint32_t *__restrict__ vc,
                                      const __half *__restrict__ vs,
                                      const __half *__restrict__ vb,
                                      const int32_t *__restrict__ ids, int n_ids, int H, int D,
                                      int bs, int64_t n_blocks, int32_t *err) {
  const int oct = D / 8;                                   // 8-element units per row
  const int64_t rows_per_block = static_cast<int64_t>(H) * bs;
  const int64_t per_kv = static_cast<int64_t>(n_ids) * rows_per_block * oct;
  const int words = D * BITS / 32;                          // code words per row
  for (int64_t x = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; x < 2 * per_kv;
       x += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const bool isv = x >= per_kv;
    const int64_t y = isv ? x - per_kv : x;
    const int u = static_cast<int>(y % oct);
    const int64_t r = y / oct;                              // output row: i * H * bs + h * bs + t
    const int i = static_cast<int>(r / rows_per_block);
    const int64_t rem = r - static_cast<int64_t>(i) * rows_per_block;
    const int32_t blk = ids[i];
    if (blk < 0 || blk >= n_blocks) {
      if (u == 0 && rem == 0 && !isv) dev_error(err, MZ_DEVERR_BLOCK_ID);
      continue;
    }
    const int64_t src = static_cast<int64_t>(blk) * rows_per_block + rem;
    const uint32_t *cw = (isv ? vc : kc) + src * words;
    const int64_t gi = src * (D / 64) + (8 * u) / 64;
    const float s = __half2float((isv ? vs : ks)[gi]);
    const float b = __half2float((isv ? vb : kb)[gi]);
    uint32_t q[8];
    if constexpr (BITS == 8) {
      const uint32_t w0 = cw[2 * u], w1 = cw[2 * u + 1];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        q[j] = (w0 >> (8 * j)) & 0xFFu;
        q[4 + j] = (w1 >> (8 * j)) & 0xFFu;
      }
    } else {
      const uint32_t w = cw[u];
#pragma unroll
      for (int j = 0; j < 8; ++j) q[j] = (w >> (4 * j)) & 0xFu;
    }
    uint32_t packed[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = __fadd_rn(__fmul_rn(static_cast<float>(q[2 * j]), s), b);
      const float c = __fadd_rn(__fmul_rn(static_cast<float>(q[2 * j + 1]), s), b);
      packed[j] = pack2<BF16>(a, c);
    }
    *reinterpret_cast<uint4 *>((isv ? vo : ko) + r * D + 8 * u) =
        make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
}

}  // namespace
}  // namespace mz

using namespace mz;

extern "C" int mz_kv_dequant_blocks(void *k_out, void *v_out, int32_t out_dtype,
                                    const void *k_codes, const void *k_scales,
                                    const void *k_biases, const void *v_codes,
                                    const void *v_scales, const void *v_biases,
                                    const int32_t *block_ids, int32_t n_ids, int32_t n_kv_heads,
                                    int32_t head_dim, int32_t block_size, int64_t n_blocks,
                                    int32_t bits, int32_t *dev_err, mz_stream_t stream) {
  const char *fn = "mz_kv_dequant_blocks";
  if (out_dtype != MZ_DTYPE_F16 && out_dtype != MZ_DTYPE_BF16)
    return fail(MZ_ERR_UNSUPPORTED, "%s: out_dtype must be F16 or BF16", fn);
  if (bits != 4 && bits != 8) return fail(MZ_ERR_UNSUPPORTED, "%s: bits must be 4 or 8", fn);
  if (head_dim <= 0 || head_dim % 64)
    return fail(MZ_ERR_UNSUPPORTED, "%s: head_dim %d is not a multiple of 64", fn, head_dim);
  if (n_ids < 0 || n_kv_heads <= 0 || block_size <= 0 || n_blocks <= 0)
    return fail(MZ_ERR_INVALID_ARG, "%s: bad sizes", fn);
  if (n_ids == 0) return MZ_OK;
  if (!k_out || !v_out || !k_codes || !k_scales || !k_biases || !v_codes || !v_scales ||
      !v_biases || !block_ids)
    return fail(MZ_ERR_INVALID_ARG, "%s: null pointer", fn);
  if (!aligned(k_out, 16) || !aligned(v_out, 16) || !aligned(k_codes, 4) || !aligned(v_codes, 4) ||
      !aligned(k_scales, 2) || !aligned(k_biases, 2) || !aligned(v_scales, 2) ||
      !aligned(v_biases, 2))
    return fail(MZ_ERR_ALIGNMENT, "%s: outputs need 16-byte, codes 4-byte alignment", fn);
  const int64_t units = 2LL * n_ids * n_kv_heads * block_size * (head_dim / 8);
  // grid-stride kernel: at most 32 blocks of 256 threads per SM
  const int sms = sm_count(current_device());
  if (sms <= 0) return fail(MZ_ERR_CUDA, "%s: cannot query the device's SM count", fn);
  int64_t g = (units + 255) / 256;
  if (g > 32LL * sms) g = 32LL * sms;
  const unsigned grid = static_cast<unsigned>(g);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto *ko = static_cast<uint16_t *>(k_out);
  auto *vo = static_cast<uint16_t *>(v_out);
  auto *kc = static_cast<const uint32_t *>(k_codes);
  auto *vc = static_cast<const uint32_t *>(v_codes);
  auto *ks = static_cast<const __half *>(k_scales);
  auto *kb = static_cast<const __half *>(k_biases);
  auto *vs = static_cast<const __half *>(v_scales);
  auto *vb = static_cast<const __half *>(v_biases);
#define MZ_DQ(B_, BF_)                                                                      \
  dequant_blocks_kernel<B_, BF_><<<grid, 256, 0, s>>>(ko, vo, kc, ks, kb, vc, vs, vb,      \
                                                      block_ids, n_ids, n_kv_heads, head_dim, \
                                                      block_size, n_blocks, dev_err)
  const bool bf16 = out_dtype == MZ_DTYPE_BF16;
  if (bits == 8) {
    if (bf16) MZ_DQ(8, true); else MZ_DQ(8, false);
  } else {
    if (bf16) MZ_DQ(4, true); else MZ_DQ(4, false);
  }
#undef MZ_DQ
  MZ_CHECK_LAUNCH(fn);
  return MZ_OK;
}
