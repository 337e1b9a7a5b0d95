// Dequantisation of whole quantised KV blocks into a 16-bit staging pool: the
// prompt pass over a quantised cache attends over the dequantised values of
// the blocks its sequences use (what a quantised cache's attention over a
// prompt chunk computes), so the prefill kernel runs on them unchanged.
//
// HBM-bound elementwise work.  One CTA per (block id, K or V): the block's
// codes (H * bs rows) are contiguous, so its threads stream them with vector
// loads, 16 codes (one 16- or 8-byte piece of a row, inside one group of 64)
// per step, and turn each into f32(scale) * q + f32(bias) with a separate
// multiply and add (no fused rounding), rounded to the output type and stored
// as two 16-byte vectors.
#include "common.cuh"

namespace mz {
namespace {

template <int BITS>
__device__ __forceinline__ void load_codes(const uint8_t *p, bool vec, uint32_t (&w)[BITS / 2]) {
  // BITS / 2 words hold 16 codes: 4 words at 8-bit, 2 at 4-bit
  if constexpr (BITS == 8) {
    if (vec) {
      const uint4 x = *reinterpret_cast<const uint4 *>(p);
      w[0] = x.x, w[1] = x.y, w[2] = x.z, w[3] = x.w;
      return;
    }
  } else {
    if (vec) {
      const uint2 x = *reinterpret_cast<const uint2 *>(p);
      w[0] = x.x, w[1] = x.y;
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < BITS / 2; ++j) w[j] = reinterpret_cast<const uint32_t *>(p)[j];
}

template <int BITS, bool BF16>
__global__ void __launch_bounds__(256)
    dequant_blocks_kernel(uint16_t *__restrict__ ko, uint16_t *__restrict__ vo,
                          const uint32_t *__restrict__ kc, const __half *__restrict__ ks,
                          const __half *__restrict__ kb, const uint32_t *__restrict__ vc,
                          const __half *__restrict__ vs, const __half *__restrict__ vb,
                          const int32_t *__restrict__ ids, int H, int D, int bs, int64_t n_blocks,
                          bool vec, int32_t *err) {
  const int i = static_cast<int>(blockIdx.x >> 1);
  const bool isv = (blockIdx.x & 1) != 0;
  const int32_t blk = ids[i];
  if (blk < 0 || blk >= n_blocks) {
    if (threadIdx.x == 0 && !isv) dev_error(err, MZ_DEVERR_BLOCK_ID);
    return;
  }
  const int rows = H * bs;       // rows of one block
  const int per_row = D / 16;    // 16-code pieces per row
  const int row_bytes = D * BITS / 8;
  const int groups = D / 64;
  const uint8_t *codes = reinterpret_cast<const uint8_t *>(isv ? vc : kc) +
                         static_cast<int64_t>(blk) * rows * row_bytes;
  const int64_t g0 = static_cast<int64_t>(blk) * rows * groups;
  const __half *sc = (isv ? vs : ks) + g0;
  const __half *bi = (isv ? vb : kb) + g0;
  uint16_t *out = (isv ? vo : ko) + static_cast<int64_t>(i) * rows * D;
  const int units = rows * per_row;
  for (int u = threadIdx.x; u < units; u += blockDim.x) {
    const int row = u / per_row, c = u - row * per_row;
    const float s = __half2float(sc[row * groups + (c >> 2)]);
    const float b = __half2float(bi[row * groups + (c >> 2)]);
    uint32_t w[BITS / 2];
    load_codes<BITS>(codes + row * row_bytes + c * (16 * BITS / 8), vec, w);
    uint32_t packed[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t q0, q1;  // codes 2j and 2j + 1 (LSB-first fields)
      if constexpr (BITS == 8) {
        q0 = (w[j >> 1] >> (16 * (j & 1))) & 0xFFu;
        q1 = (w[j >> 1] >> (16 * (j & 1) + 8)) & 0xFFu;
      } else {
        q0 = (w[j >> 2] >> (8 * (j & 3))) & 0xFu;
        q1 = (w[j >> 2] >> (8 * (j & 3) + 4)) & 0xFu;
      }
      const float a = __fadd_rn(__fmul_rn(static_cast<float>(q0), s), b);
      const float e = __fadd_rn(__fmul_rn(static_cast<float>(q1), s), b);
      packed[j] = pack2<BF16>(a, e);
    }
    uint4 *o = reinterpret_cast<uint4 *>(out + static_cast<int64_t>(row) * D + 16 * c);
    o[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    o[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
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
  if (n_ids > (1 << 30)) return fail(MZ_ERR_UNSUPPORTED, "%s: more than 2^30 block ids", fn);
  if (!k_out || !v_out || !k_codes || !k_scales || !k_biases || !v_codes || !v_scales ||
      !v_biases || !block_ids)
    return fail(MZ_ERR_INVALID_ARG, "%s: null pointer", fn);
  if (!aligned(k_out, 16) || !aligned(v_out, 16) || !aligned(k_codes, 4) || !aligned(v_codes, 4) ||
      !aligned(k_scales, 2) || !aligned(k_biases, 2) || !aligned(v_scales, 2) ||
      !aligned(v_biases, 2))
    return fail(MZ_ERR_ALIGNMENT, "%s: outputs need 16-byte, codes 4-byte alignment", fn);
  // one CTA per (block id, K or V)
  const unsigned grid = static_cast<unsigned>(2 * static_cast<int64_t>(n_ids));
  // 16 codes are 16 (8-bit) or 8 (4-bit) bytes: vector loads when the code
  // pools are aligned to that (row pieces then are too), else word loads
  const bool vec = aligned(k_codes, bits * 2) && aligned(v_codes, bits * 2);
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
                                                      block_ids, n_kv_heads, head_dim,      \
                                                      block_size, n_blocks, vec, dev_err)
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
