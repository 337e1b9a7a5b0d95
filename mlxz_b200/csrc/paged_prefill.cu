// Paged prefill attention for sm_100a (chunked prefill over paged KV).
//
// A chunk of n_b query tokens of sequence b sits at positions
// [ctx_b - n_b, ctx_b) -- its own K/V already appended to the pools -- and
// token i attends causally to the sequence's first ctx_b - n_b + i + 1 tokens,
// as the causal SDPA of a prompt chunk over a cache of that offset does.
//
// One CTA per (query block, KV head, sequence): 4 warps, each with 16 query
// rows (16/G tokens x the G query heads of the KV head), so a CTA covers
// 64/G tokens and reads every K/V tile of its causal range once for all 64
// rows.  Thread 0 streams the tiles with 2-D bulk tensor copies (128-byte
// swizzle, no multicast) into a 4-stage ring shared by the warps: a stage's
// "full" mbarrier completes on the copy's bytes, its "empty" mbarrier on the
// four warps' release, after which thread 0 refills it.  Per warp and tile:
// S = Q.K^T with mma.sync.m16n8k16, the causal mask per row, an fp32 online
// softmax in the exp2 domain, O += P.V (bf16: P as hi + lo parts).  Every wait
// is bounded; a wait that gives up sets MZ_DEVERR_TIMEOUT and the CTA stops.
#include "decode_common.cuh"

namespace mz {
namespace prefill {

using decode::kTileTok;
using decode::kTimeoutNs;
using decode::make_row_map;

constexpr int kWarps = 4;
constexpr int kStages = 4;

struct PParams {
  void *out;
  int64_t o_st, o_sh;  // out element (row t of the call, head hq, dim d)
  int out_f32;
  const void *q;
  int64_t q_st, q_sh;
  int q_bf16;
  const int32_t *q_start;  // [B] first row of sequence b in q / out
  const int32_t *q_len;    // [B] query tokens of sequence b
  const int32_t *ctx;      // [B] tokens in the pools, the chunk included
  const int32_t *tables;
  int max_blocks;
  int B, Hkv, G, bs, tpb;
  int64_t n_blocks;
  float scale_log2;
  int tok_per_warp;  // 16 / G
  int32_t *err;
};

template <int D>
struct PCfg {
  static constexpr int kTileBytes = kTileTok * D * 2;  // one of K or V
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kSmemBytes = kStages * kStageBytes + 2 * kStages * 8 + 1024;
};

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kWarps * 32, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const PParams p) {
  using C = PCfg<D>;
  constexpr int S = kStages;
  constexpr int KS = D / 16;
  constexpr int NT = D / 8;
  const int b = blockIdx.z, h = blockIdx.y;
  const int tpc = kWarps * p.tok_per_warp;  // query tokens per CTA
  const int n = p.q_len[b];
  const int q0 = blockIdx.x * tpc;
  if (n <= 0 || q0 >= n) return;
  int ctx = p.ctx[b];
  const int cap = p.max_blocks * p.bs;
  if (ctx < n || ctx > cap) {
    if (threadIdx.x == 0) dev_error(p.err, MZ_DEVERR_CONTEXT);
    return;
  }
  const int start = ctx - n;              // position of query token 0
  const int q_hi = min(q0 + tpc, n);      // query tokens [q0, q_hi) in this CTA
  const int kv_len = start + q_hi;        // keys [0, kv_len) are needed
  const int ntiles = (kv_len + kTileTok - 1) / kTileTok;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  const uint32_t stage0 = smem_u32(smem);
  const uint32_t full0 = stage0 + S * C::kStageBytes;
  const uint32_t empty0 = full0 + 8 * S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, kWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const uint64_t pol = l2_policy_evict_first();
  auto issue = [&](int t) {  // thread 0: tile t into stage t % S
    const int s = t % S;
    int32_t blk = p.tables[(int64_t)b * p.max_blocks + t / p.tpb];
    if (blk < 0 || blk >= p.n_blocks) {
      dev_error(p.err, MZ_DEVERR_BLOCK_ID);
      blk = 0;
    }
    const int y = static_cast<int>(((int64_t)blk * p.Hkv + h) * p.bs + (t % p.tpb) * kTileTok);
    const uint32_t bar = full0 + 8 * s;
    const uint32_t dk = stage0 + s * C::kStageBytes;
    mbar_arrive_expect_tx(bar, C::kStageBytes);
#pragma unroll
    for (int c2 = 0; c2 < D / 64; ++c2) {
      tma_load_2d(dk + c2 * 2048, &tmK, c2 * 64, y, bar, pol);
      tma_load_2d(dk + C::kTileBytes + c2 * 2048, &tmV, c2 * 64, y, bar, pol);
    }
  };
  int issued = 0;  // tiles issued so far (thread 0's count)
  if (threadIdx.x == 0)
    for (; issued < S && issued < ntiles; ++issued) issue(issued);

  // This warp's rows: r = 0..15 <-> token q0 + warp*tpw + r / G, head h*G + r % G.
  const int g = lane >> 2, cq = lane & 3;
  const int mi = lane >> 3, r8 = lane & 7;
  const int tokK = r8 + 8 * (mi >> 1), subK = mi & 1;
  const int tokV = r8 + 8 * (mi & 1), subV = mi >> 1;
  const int tw0 = q0 + warp * p.tok_per_warp;  // first query token of the warp
  const int t_row0 = tw0 + g / p.G, t_row1 = tw0 + (g + 8) / p.G;
  const bool live0 = t_row0 < q_hi, live1 = t_row1 < q_hi;
  // causal limit (last visible key position); rows past the chunk reuse the
  // last live token's so that their (unstored) softmax stays finite
  const int lim0 = start + min(t_row0, q_hi - 1), lim1 = start + min(t_row1, q_hi - 1);

  uint32_t qa[KS][4];
  {
    const auto *q16 = static_cast<const uint16_t *>(p.q);
    const int64_t base0 = (int64_t)(p.q_start[b] + t_row0) * p.q_st + (int64_t)(h * p.G + g % p.G) * p.q_sh;
    const int64_t base1 =
        (int64_t)(p.q_start[b] + t_row1) * p.q_st + (int64_t)(h * p.G + (g + 8) % p.G) * p.q_sh;
#pragma unroll
    for (int j = 0; j < KS; ++j) {
      const int d = 16 * j + 2 * cq;
      qa[j][0] = live0 ? *reinterpret_cast<const uint32_t *>(q16 + base0 + d) : 0u;
      qa[j][1] = live1 ? *reinterpret_cast<const uint32_t *>(q16 + base1 + d) : 0u;
      qa[j][2] = live0 ? *reinterpret_cast<const uint32_t *>(q16 + base0 + d + 8) : 0u;
      qa[j][3] = live1 ? *reinterpret_cast<const uint32_t *>(q16 + base1 + d + 8) : 0u;
    }
  }
  float oacc[NT][4];
#pragma unroll
  for (int k = 0; k < NT; ++k) oacc[k][0] = oacc[k][1] = oacc[k][2] = oacc[k][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int i = 0; i < ntiles; ++i) {
    const int s = i % S;
    const uint32_t ph = (i / S) & 1;
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(full0 + 8 * s, ph, kTimeoutNs))) {
      if (lane == 0) dev_error(p.err, MZ_DEVERR_TIMEOUT);
      // the issuing thread waits (bounded) for its copies still in flight
      if (threadIdx.x == 0)
        for (int k = i + 1; k < issued; ++k)
          (void)mbar_wait_bounded(full0 + 8 * (k % S), (k / S) & 1, kTimeoutNs);
      return;
    }
    uint8_t *vt = smem + s * C::kStageBytes + C::kTileBytes;
    const uint32_t kb = stage0 + s * C::kStageBytes;
    const uint32_t vb = kb + C::kTileBytes;
    const int t0 = i * kTileTok;
    const int nvalid = min(kTileTok, kv_len - t0);
    if (nvalid < kTileTok) {
      // keys past kv_len may be stale: exact zeros so that 0 * V stays 0
      // (every warp writes the same zeros before it reads)
      for (int e = lane; e < (kTileTok - nvalid) * (D / 8); e += 32) {
        const int tok = nvalid + e / (D / 8), d = (e % (D / 8)) * 8;
        *reinterpret_cast<uint4 *>(vt + decode::swz128(tok, 2 * d)) = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }

    float sacc[2][4];
#pragma unroll
    for (int k = 0; k < 2; ++k) sacc[k][0] = sacc[k][1] = sacc[k][2] = sacc[k][3] = 0.f;
#pragma unroll
    for (int j = 0; j < KS; ++j) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(kb + decode::swz128(tokK, 2 * (16 * j + 8 * subK)), b0, b1, b2, b3);
      mma_16816<BF16>(sacc[0], qa[j], b0, b1);
      mma_16816<BF16>(sacc[1], qa[j], b2, b3);
    }

    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int k = 0; k < 2; ++k)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = t0 + k * 8 + 2 * cq + (e & 1);
        float x = sacc[k][e] * p.scale_log2;
        if (key >= kv_len || key > (e < 2 ? lim0 : lim1)) x = -INFINITY;
        sacc[k][e] = x;
        if (e < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    // a row whose keys in this tile are all masked keeps its running max
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float a0 = (mn0 == -INFINITY) ? 1.f : fast_exp2(m0 - mn0);
    const float a1 = (mn1 == -INFINITY) ? 1.f : fast_exp2(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      sacc[k][0] = (m0 == -INFINITY) ? 0.f : fast_exp2(sacc[k][0] - m0);
      sacc[k][1] = (m0 == -INFINITY) ? 0.f : fast_exp2(sacc[k][1] - m0);
      sacc[k][2] = (m1 == -INFINITY) ? 0.f : fast_exp2(sacc[k][2] - m1);
      sacc[k][3] = (m1 == -INFINITY) ? 0.f : fast_exp2(sacc[k][3] - m1);
      rs0 += sacc[k][0] + sacc[k][1];
      rs1 += sacc[k][2] + sacc[k][3];
    }
    l0 = l0 * a0 + rs0;
    l1 = l1 * a1 + rs1;
    if (__any_sync(0xffffffffu, a0 != 1.f || a1 != 1.f)) {
#pragma unroll
      for (int k = 0; k < NT; ++k) {
        oacc[k][0] *= a0;
        oacc[k][1] *= a0;
        oacc[k][2] *= a1;
        oacc[k][3] *= a1;
      }
    }

    uint32_t ph_[4], pl_[4];
    {
      float hi[2][4];
#pragma unroll
      for (int k = 0; k < 2; ++k)
#pragma unroll
        for (int e = 0; e < 4; ++e) hi[k][e] = round16<BF16>(sacc[k][e]);
      ph_[0] = pack2<BF16>(hi[0][0], hi[0][1]);
      ph_[1] = pack2<BF16>(hi[0][2], hi[0][3]);
      ph_[2] = pack2<BF16>(hi[1][0], hi[1][1]);
      ph_[3] = pack2<BF16>(hi[1][2], hi[1][3]);
      if constexpr (BF16) {
        pl_[0] = pack2<BF16>(sacc[0][0] - hi[0][0], sacc[0][1] - hi[0][1]);
        pl_[1] = pack2<BF16>(sacc[0][2] - hi[0][2], sacc[0][3] - hi[0][3]);
        pl_[2] = pack2<BF16>(sacc[1][0] - hi[1][0], sacc[1][1] - hi[1][1]);
        pl_[3] = pack2<BF16>(sacc[1][2] - hi[1][2], sacc[1][3] - hi[1][3]);
      }
    }
#pragma unroll
    for (int j = 0; j < KS; ++j) {
      uint32_t v0, v1, v2, v3;
      ldsm_x4_trans(vb + decode::swz128(tokV, 2 * (16 * j + 8 * subV)), v0, v1, v2, v3);
      mma_16816<BF16>(oacc[2 * j], ph_, v0, v1);
      mma_16816<BF16>(oacc[2 * j + 1], ph_, v2, v3);
      if constexpr (BF16) {
        mma_16816<BF16>(oacc[2 * j], pl_, v0, v1);
        mma_16816<BF16>(oacc[2 * j + 1], pl_, v2, v3);
      }
    }

    // release the stage; thread 0 refills it once all four warps have
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * s);
    if (threadIdx.x == 0 && i + S < ntiles) {
      if (!mbar_wait_bounded(empty0 + 8 * s, ph, kTimeoutNs)) {
        dev_error(p.err, MZ_DEVERR_TIMEOUT);
      } else {
        fence_proxy_async_smem();
        issue(i + S);
        ++issued;
      }
    }
  }

  // normalise and store the live rows
  float L0 = l0, L1 = l1;
  L0 += __shfl_xor_sync(0xffffffffu, L0, 1);
  L0 += __shfl_xor_sync(0xffffffffu, L0, 2);
  L1 += __shfl_xor_sync(0xffffffffu, L1, 1);
  L1 += __shfl_xor_sync(0xffffffffu, L1, 2);
  const float i0 = 1.f / L0, i1 = 1.f / L1;
  auto store = [&](int64_t off, float x, float y) {
    if (p.out_f32) {
      *reinterpret_cast<float2 *>(static_cast<float *>(p.out) + off) = make_float2(x, y);
    } else if (p.q_bf16) {
      *reinterpret_cast<__nv_bfloat162 *>(static_cast<__nv_bfloat16 *>(p.out) + off) =
          __floats2bfloat162_rn(x, y);
    } else {
      *reinterpret_cast<__half2 *>(static_cast<__half *>(p.out) + off) = __floats2half2_rn(x, y);
    }
  };
  if (live0) {
    const int64_t o = (int64_t)(p.q_start[b] + t_row0) * p.o_st + (int64_t)(h * p.G + g % p.G) * p.o_sh;
#pragma unroll
    for (int k = 0; k < NT; ++k) store(o + k * 8 + 2 * cq, oacc[k][0] * i0, oacc[k][1] * i0);
  }
  if (live1) {
    const int64_t o =
        (int64_t)(p.q_start[b] + t_row1) * p.o_st + (int64_t)(h * p.G + (g + 8) % p.G) * p.o_sh;
#pragma unroll
    for (int k = 0; k < NT; ++k) store(o + k * 8 + 2 * cq, oacc[k][2] * i1, oacc[k][3] * i1);
  }
}

template <int D, bool BF16>
int smem_attr() {
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, []() {
    err = cudaFuncSetAttribute(paged_prefill_kernel<D, BF16>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, PCfg<D>::kSmemBytes);
  });
  if (err != cudaSuccess) return cuda_fail(err, "mz_paged_prefill: shared memory attribute");
  return MZ_OK;
}

}  // namespace prefill
}  // namespace mz

using namespace mz;
using namespace mz::prefill;

extern "C" int mz_paged_prefill(void *out, int32_t out_dtype, int64_t out_tok_stride,
                                int64_t out_head_stride, const void *q, int64_t q_tok_stride,
                                int64_t q_head_stride, const int32_t *q_start,
                                const int32_t *q_len, int32_t max_q_len, const void *k_pool,
                                const void *v_pool, const int32_t *block_tables,
                                int32_t max_blocks_per_seq, const int32_t *ctx_lens,
                                int32_t n_seqs, int32_t n_heads, int32_t n_kv_heads,
                                int32_t head_dim, int32_t block_size, int64_t n_blocks,
                                float scale, int32_t dtype, int32_t *dev_err,
                                mz_stream_t stream) {
  const char *fn = "mz_paged_prefill";
  if (dtype != MZ_DTYPE_F16 && dtype != MZ_DTYPE_BF16)
    return fail(MZ_ERR_UNSUPPORTED, "%s: dtype must be F16 or BF16", fn);
  if (out_dtype != dtype && out_dtype != MZ_DTYPE_F32)
    return fail(MZ_ERR_UNSUPPORTED, "%s: out_dtype must equal dtype or be F32", fn);
  if (head_dim != 64 && head_dim != 128)
    return fail(MZ_ERR_UNSUPPORTED, "%s: head_dim %d (supported: 64, 128)", fn, head_dim);
  if (block_size <= 0 || block_size % kTileTok)
    return fail(MZ_ERR_UNSUPPORTED, "%s: block_size %d is not a multiple of 16", fn, block_size);
  if (n_seqs < 0 || n_kv_heads <= 0 || n_heads <= 0 || n_heads % n_kv_heads || max_q_len < 0 ||
      max_blocks_per_seq <= 0 || n_blocks <= 0)
    return fail(MZ_ERR_INVALID_ARG, "%s: bad sizes", fn);
  const int G = n_heads / n_kv_heads;
  if (16 % G)
    return fail(MZ_ERR_UNSUPPORTED, "%s: n_heads / n_kv_heads = %d does not divide 16", fn, G);
  if (!std::isfinite(scale)) return fail(MZ_ERR_INVALID_ARG, "%s: scale not finite", fn);
  if (n_seqs == 0 || max_q_len == 0) return MZ_OK;
  if (!out || !q || !q_start || !q_len || !k_pool || !v_pool || !block_tables || !ctx_lens)
    return fail(MZ_ERR_INVALID_ARG, "%s: null pointer", fn);
  if (!aligned(k_pool, 16) || !aligned(v_pool, 16) || !aligned(q, 4) || (q_tok_stride & 1) ||
      (q_head_stride & 1))
    return fail(MZ_ERR_ALIGNMENT,
                "%s: pools need 16-byte alignment, q 4-byte alignment and even strides", fn);
  const int ob = out_dtype == MZ_DTYPE_F32 ? 8 : 4;
  if (!aligned(out, ob) || (out_tok_stride & 1) || (out_head_stride & 1))
    return fail(MZ_ERR_ALIGNMENT, "%s: out needs %d-byte alignment and even strides", fn, ob);
  const int64_t rows_total = n_blocks * n_kv_heads * block_size;
  if (rows_total >= (int64_t(1) << 31))
    return fail(MZ_ERR_UNSUPPORTED, "%s: pool has >= 2^31 rows", fn);

  const bool bf16 = dtype == MZ_DTYPE_BF16;
  CUtensorMap tk, tv;
  const auto type = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (int rc = make_row_map(&tk, k_pool, rows_total, head_dim, type, 2, 64)) return rc;
  if (int rc = make_row_map(&tv, v_pool, rows_total, head_dim, type, 2, 64)) return rc;

  PParams p;
  p.out = out;
  p.o_st = out_tok_stride;
  p.o_sh = out_head_stride;
  p.out_f32 = out_dtype == MZ_DTYPE_F32;
  p.q = q;
  p.q_st = q_tok_stride;
  p.q_sh = q_head_stride;
  p.q_bf16 = bf16;
  p.q_start = q_start;
  p.q_len = q_len;
  p.ctx = ctx_lens;
  p.tables = block_tables;
  p.max_blocks = max_blocks_per_seq;
  p.B = n_seqs;
  p.Hkv = n_kv_heads;
  p.G = G;
  p.bs = block_size;
  p.tpb = block_size / kTileTok;
  p.n_blocks = n_blocks;
  p.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
  p.tok_per_warp = 16 / G;
  p.err = dev_err;

  const int tpc = kWarps * p.tok_per_warp;
  const dim3 grid((max_q_len + tpc - 1) / tpc, n_kv_heads, n_seqs);
  if (grid.x > 2147483647u || n_seqs > 65535 || n_kv_heads > 65535)
    return fail(MZ_ERR_UNSUPPORTED, "%s: grid too large", fn);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define MZ_PLAUNCH(D_, BF_)                                                                      \
  do {                                                                                           \
    if (int rc = smem_attr<D_, BF_>()) return rc;                                                \
    paged_prefill_kernel<D_, BF_><<<grid, kWarps * 32, PCfg<D_>::kSmemBytes, s>>>(tk, tv, p);     \
  } while (0)
  if (head_dim == 128) {
    if (bf16) MZ_PLAUNCH(128, true); else MZ_PLAUNCH(128, false);
  } else {
    if (bf16) MZ_PLAUNCH(64, true); else MZ_PLAUNCH(64, false);
  }
#undef MZ_PLAUNCH
  MZ_CHECK_LAUNCH(fn);
  return MZ_OK;
}
