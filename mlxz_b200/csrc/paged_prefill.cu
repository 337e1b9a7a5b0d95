// Paged prefill attention for sm_100a (chunked prefill over paged KV).
//
// A chunk of n_b query tokens of sequence b sits at positions
// [ctx_b - n_b, ctx_b) -- its own K/V already appended to the pools -- and
// token i attends causally to the sequence's first ctx_b - n_b + i + 1 tokens,
// as the causal SDPA of a prompt chunk over a cache of that offset does.
//
// Tensor-core form (tcgen05 + TMEM), see the kernel's own comment below.
// Shapes: head_dim 64 or 128, n_heads / n_kv_heads dividing 128, block_size a
// multiple of 16, scale > 0 (the row max is taken on the raw scores).
#include "decode_common.cuh"
#include "tcgen05.cuh"

namespace mz {
namespace prefill {

using decode::kTileTok;
using decode::kTimeoutNs;

struct PParams {
  void *out;
  int64_t o_st, o_sh;  // out element (row t of the call, head hq, dim d)
  int out_f32;
  const void *q;
  int64_t q_st, q_sh;
  int n_rows;              // rows of q / out
  const int32_t *q_start;  // [B] first row of sequence b in q / out
  const int32_t *q_len;    // [B] query tokens of sequence b
  const int32_t *ctx;      // [B] tokens in the pools, the chunk included
  const int32_t *tables;
  int max_blocks;
  int Hkv, G, bs;
  int64_t n_blocks;
  float scale_log2;
  int sub_log2;      // rows per bulk copy box: gcd(block_size, 128) = 1 << sub_log2
  int32_t *err;
  int n_seqs, qblocks;  // persistent form: sequences, query blocks per sequence
};

// 4-D bulk tensor copy (no multicast): box {64, 8, D / 64, rows / 8} of the
// grouped map at row group `grp`.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void *tmap, int grp, uint32_t bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %2, %2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(0), "r"(grp), "r"(bar), "l"(policy)
      : "memory");
}

// Pool [rows][D] viewed as 4-D: (64 columns, 8 rows, D / 64 chunks, rows / 8
// groups) with strides (row D*2 B, chunk 128 B, group 8*D*2 B), box {64, 8,
// D / 64, box_rows / 8}, 128-byte swizzle: one copy brings box_rows whole rows
// in the grouped layout the MMA descriptors read.
inline int make_group_map(CUtensorMap *m, const void *base, int64_t rows, int D,
                          CUtensorMapDataType type, int box_rows) {
  auto fn = decode::encode_fn();
  if (!fn) return fail(MZ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[4] = {64, 8, static_cast<cuuint64_t>(D / 64), static_cast<cuuint64_t>(rows / 8)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(D) * 2, 128, static_cast<cuuint64_t>(D) * 16};
  cuuint32_t box[4] = {64, 8, static_cast<cuuint32_t>(D / 64),
                       static_cast<cuuint32_t>(box_rows / 8)};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = fn(m, type, 4, const_cast<void *>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MZ_ERR_CUDA, "cuTensorMapEncodeTiled (grouped) failed (%d)", (int)r);
  return MZ_OK;
}


// Two fp32 values in one 64-bit register, for the packed fp32 instructions
// (fma / add / sub .f32x2): one instruction for both keys of a pair.
__device__ __forceinline__ uint64_t f2_pack(float x, float y) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float &x, float &y) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(x), "=f"(y) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// max(a, b, c) in one instruction (three-input max.f32 of sm_100)
__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// ---------------------------------------------------------------------------
// One CTA per (128 query rows, KV head, sequence): row m is
// token q0 + m / G, query head h*G + m % G.  Ten warps:
//   warps 0-7  softmax + epilogue; thread t owns row t % 128 (TMEM lane
//              t % 128) and half t / 128 of its keys (64 of each 128-key tile)
//              and of its O columns; the two halves of a row exchange their
//              maxima through shared memory (bounded mbarrier waits)
//   warp 8     streams 128-key K and V tiles (2-D bulk tensor copies of
//              gcd(block_size, 128)-row boxes, 128-byte swizzle, no
//              multicast) into a 3-stage K ring (a slot frees when its S MMA
//              completes) and a 2-stage V ring (when its PV MMA completes), K
//              running one tile ahead of V
//   warp 9     allocates TMEM and issues the MMAs (one elected lane)
// TMEM columns: O [0, D) fp32; three 128-column S buffers at 128, 256, 384.
// Per key tile i:  S_i = Q.K_i^T (SS MMA, M=128 N=128 K=16 steps) into buffer
// i % 3; softmax reads S_i, writes P_i over it (16-bit, two per column; each
// half of the keys over its own 64 S columns: bf16 hi in the first 32, lo in
// the last 32; fp16 in the first 32); O += P_i.V_i (TS MMA, A = P
// from TMEM, B = V MN-major, N = D).  S_{i+1} is issued before PV_i so the
// tensor core works on it during softmax_i.  The running max is only moved
// when a row's tile max exceeds it by more than 8 (log2 units): P then stays
// below 2^8 and O is rescaled in TMEM only on those tiles.
// Every wait is bounded; a wait that gives up sets MZ_DEVERR_TIMEOUT and the
// abort flag, every role leaves its loop, the issuing threads wait (bounded)
// for their copies / MMAs in flight, and warp 9 frees the TMEM.
namespace tcp {
constexpr int kM = 128;
constexpr int kN = 128;
constexpr int kKRing = 3;
constexpr int kVRing = 2;
constexpr int kSBufs = 3;
constexpr int kSoftWarps = 8;
constexpr int kProdWarp = 8, kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.f;

template <int D>
struct TCfg {
  // K / V tile layout in shared memory: 16 groups of 8 keys, each group the
  // D / 64 column chunks of 8 rows x 128 bytes (one 128-byte-swizzle atom per
  // chunk): key r, chunk c at (r / 8) * kGroup + c * 1024 + (r % 8) * 128.
  static constexpr int kGroup = 8 * D * 2;              // 8 keys x D
  static constexpr int kTile = (kN / 8) * kGroup;       // one K or V tile
  static constexpr int kQ = (D / 64) * kM * 128;        // 128 rows x D, chunk-major
  static constexpr int kK0 = kQ;                        // K slot s at kK0 + s kTile
  static constexpr int kV0 = kQ + kKRing * kTile;       // V slot s at kV0 + s kTile
  static constexpr int kBar = kV0 + kVRing * kTile;     // barriers after the tiles
  static constexpr int kXm = kBar + 256;                // [2 parity][2 half][128] maxima
  static constexpr int kXl = kXm + 2 * 2 * kM * 4;      // [2 half][128] row sums
  static constexpr int kSmemBytes = kXl + 2 * kM * 4 + 1024;
};

// barrier slots (8 bytes each) after the tiles
constexpr int kBarKFull = 0, kBarVFull = 3, kBarSFull = 5, kBarPFull = 8, kBarPvDone = 11,
              kBarDrain = 14, kBarXchg = 15 /* [parity][pair] */, kBarLx = 23 /* [pair] */,
              kNumBars = 27;
// persistent form only: Q of the next item loaded, O of the last item read
constexpr int kBarQReady = 27, kBarOFree = 28, kNumBarsPs = 29;
static_assert(8 * kNumBarsPs + 8 <= 256, "barrier area");
static_assert(kKRing == kSBufs, "K slots are released through the S barriers");
}  // namespace tcp

template <int D, bool BF16>
__global__ void __launch_bounds__(tcp::kThreads, 1)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const PParams p) {
  using namespace tcp;
  using C = TCfg<D>;
  const int b = blockIdx.z, h = blockIdx.y;
  const int tpc = kM / p.G;
  const int n = p.q_len[b];
  // last query block first: the blocks with the most key tiles start earliest
  const int q0 = (gridDim.x - 1 - blockIdx.x) * tpc;
  if (n <= 0 || q0 >= n) return;
  const int ctx = p.ctx[b];
  if (ctx < n || ctx > p.max_blocks * p.bs) {
    if (threadIdx.x == 0) dev_error(p.err, MZ_DEVERR_CONTEXT);
    return;
  }
  if (p.q_start[b] < 0 || (int64_t)p.q_start[b] + n > p.n_rows) {
    if (threadIdx.x == 0) dev_error(p.err, MZ_DEVERR_ROWS);
    return;
  }
  const int start = ctx - n;
  const int q_hi = min(q0 + tpc, n);
  const int kv_len = start + q_hi;
  const int ntiles = (kv_len + kN - 1) / kN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t qs = sbase;
  auto kst = [&](int s) { return sbase + C::kK0 + s * C::kTile; };
  auto vst = [&](int s) { return sbase + C::kV0 + s * C::kTile; };
  const uint32_t bars = sbase + C::kBar;
  auto bar = [&](int i) { return bars + 8 * i; };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::kBar + 8 * kNumBars);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::kBar + 8 * kNumBars + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // The copy warp sets up the barriers and starts its copies at once; the
  // other warps load Q and allocate TMEM meanwhile and meet it at named
  // barrier 1 (the copy warp only arrives there).
  if (warp == kProdWarp && lane == 0) {
    for (int s = 0; s < kKRing; ++s) mbar_init(bar(kBarKFull + s), 1);
    for (int s = 0; s < kVRing; ++s) mbar_init(bar(kBarVFull + s), 1);
    for (int s = 0; s < kSBufs; ++s) {
      mbar_init(bar(kBarSFull + s), 1);
      mbar_init(bar(kBarPFull + s), kSoftWarps);
      mbar_init(bar(kBarPvDone + s), 1);
    }
    mbar_init(bar(kBarDrain), 1);
    for (int x = 0; x < 8; ++x) mbar_init(bar(kBarXchg + x), 64);
    for (int x = 0; x < 4; ++x) mbar_init(bar(kBarLx + x), 64);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProdWarp) {
    __syncwarp();
    asm volatile("bar.arrive 1, %0;" ::"n"(kThreads) : "memory");
  }
  if (warp == kMmaWarp) tc::tmem_alloc(smem_u32(tmem_slot), kTmemCols);

  // this thread's row and half (softmax warps)
  const int row = threadIdx.x & (kM - 1), hf = threadIdx.x >> 7;
  const int tok = q0 + row / p.G;
  const int hq = h * p.G + row % p.G;
  const bool live = warp < kSoftWarps && tok < q_hi;
  const int lim = start + min(tok, q_hi - 1);  // last visible key of the row
  if (warp < kSoftWarps) {
    // half hf of the Q row -> shared memory (128-byte-swizzled K-major layout)
    const uint4 *src = reinterpret_cast<const uint4 *>(
        static_cast<const uint16_t *>(p.q) + (int64_t)(p.q_start[b] + tok) * p.q_st +
        (int64_t)hq * p.q_sh);
#pragma unroll
    for (int u = hf * (D / 16); u < (hf + 1) * (D / 16); ++u) {
      const uint4 v = live ? src[u] : make_uint4(0, 0, 0, 0);
      const int c = u >> 3, uu = u & 7;
      *reinterpret_cast<uint4 *>(smem + c * (kM * 128) + row * 128 + ((uu ^ (row & 7)) << 4)) = v;
    }
    fence_proxy_async_smem();
  }
  uint32_t tmem = 0;
  if (warp != kProdWarp) {
    tc::fence_before_sync();
    asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
    tc::fence_after_sync();
    tmem = *tmem_slot;
  }

  auto give_up = [&]() {
    dev_error(p.err, MZ_DEVERR_TIMEOUT);
    *abort_flag = 1;
  };

  if (warp == kProdWarp) {
    // ---------------- producer (whole warp) ----------------
    // A tile is nst = 128 / sub boxes of sub = gcd(block_size, 128) keys.
    // Block rows come in groups of four tiles: lane l < 4 nst covers box
    // l % nst of tile 4g + l / nst.  A group's block ids are loaded four steps
    // before use and only then checked and turned into pool rows, so the
    // loads' latency stays off the issue path; a shuffle hands each issuing
    // lane (lane < nst: box lane) the row it copies.
    const uint64_t pol = l2_policy_evict_last();
    const int sub = 1 << p.sub_log2, nst_log2 = 7 - p.sub_log2, nst = 1 << nst_log2;
    auto group_key = [&](int g) {
      return lane < 4 * nst ? (4 * g + (lane >> nst_log2)) * kN + (lane & (nst - 1)) * sub
                            : kv_len;
    };
    auto group_ids = [&](int g) -> int32_t {
      const int t = group_key(g);
      return t < kv_len ? p.tables[(int64_t)b * p.max_blocks + t / p.bs] : 0;
    };
    auto group_rows = [&](int g, int32_t blk) -> int {
      const int t = group_key(g);
      if (t >= kv_len) return 0;
      if (blk < 0 || blk >= p.n_blocks) {
        dev_error(p.err, MZ_DEVERR_BLOCK_ID);
        blk = 0;
      }
      return static_cast<int>(((int64_t)blk * p.Hkv + h) * p.bs + t % p.bs);
    };
    auto load = [&](const CUtensorMap *tm, uint32_t dst, uint32_t fbar, int j, int y) {
      const int nsub = min(nst, (kv_len - j * kN + sub - 1) >> p.sub_log2);
      if (lane == 0)
        mbar_arrive_expect_tx(fbar, static_cast<uint32_t>(nsub * (D / 64) * sub * 128));
      __syncwarp();
      if (lane < nsub) tma_load_4d(dst + lane * (sub / 8) * C::kGroup, tm, y >> 3, fbar, pol);
    };
    int k_issued = 0, v_issued = 0;
    int y_prv = 0, y_cur = group_rows(0, group_ids(0));
    int32_t id_nxt = group_ids(1);
    // step t: K_t, then V_{t-1}
    for (int t = 0; t <= ntiles; ++t) {
      if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
      if (t > 0 && (t & 3) == 0) {
        y_prv = y_cur;
        y_cur = group_rows(t >> 2, id_nxt);
        id_nxt = group_ids((t >> 2) + 1);
      }
      if (t < ntiles) {
        const int s = t % kKRing;
        const int y = __shfl_sync(0xffffffffu, y_cur, ((t & 3) << nst_log2) + (lane & (nst - 1)));
        // K slot s frees when S_{t-3} completed (kKRing == kSBufs)
        if (t >= kKRing &&
            !__all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarSFull + (t - kKRing) % kSBufs),
                                                        ((t - kKRing) / kSBufs) & 1, kTimeoutNs))) {
          if (lane == 0) give_up();
          break;
        }
        load(&tmK, kst(s), bar(kBarKFull + s), t, y);
        k_issued = t + 1;
      }
      if (t >= 1) {
        const int j = t - 1, s = j % kVRing;
        const int y = __shfl_sync(0xffffffffu, (j >> 2) == (t >> 2) ? y_cur : y_prv,
                                  ((j & 3) << nst_log2) + (lane & (nst - 1)));
        // V slot s frees when PV_{j-2} completed
        if (j >= kVRing &&
            !__all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarPvDone + (j - kVRing) % kSBufs),
                                                        ((j - kVRing) / kSBufs) & 1, kTimeoutNs))) {
          if (lane == 0) give_up();
          break;
        }
        load(&tmV, vst(s), bar(kBarVFull + s), j, y);
        v_issued = j + 1;
      }
    }
    // copies still in flight land before the CTA leaves
    if (lane == 0) {
      for (int j = max(0, k_issued - kKRing); j < k_issued; ++j)
        (void)mbar_wait_bounded(bar(kBarKFull + j % kKRing), (j / kKRing) & 1, kTimeoutNs);
      for (int j = max(0, v_issued - kVRing); j < v_issued; ++j)
        (void)mbar_wait_bounded(bar(kBarVFull + j % kVRing), (j / kVRing) & 1, kTimeoutNs);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issue (whole warp, one elected lane issues) ----------------
    constexpr uint32_t idS = tc::idesc_f16(BF16, kM, kN, false);
    constexpr uint32_t idPV = tc::idesc_f16(BF16, kM, D, true);
    const uint32_t tm0 = __shfl_sync(0xffffffffu, tmem, 0);
    auto issue_s = [&](int j) -> bool {
      const int s = j % kKRing, buf = j % kSBufs;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(bar(kBarKFull + s), (j / kKRing) & 1, kTimeoutNs)))
        return false;
      // buffer j % 3 is free once PV_{j-3} (which read P from it) completed
      if (j >= kSBufs &&
          !__all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarPvDone + buf),
                                                      ((j - kSBufs) / kSBufs) & 1, kTimeoutNs)))
        return false;
      tc::fence_after_sync();
      const uint32_t d = tm0 + 128 * (1 + buf);
#pragma unroll
      for (int k = 0; k < D / 16; ++k) {
        const uint32_t ko = (k & 3) * 32;  // 16-column step inside the chunk's atom
        tc::mma_ss_elect(d, tc::smem_desc_sw128(qs + (k >> 2) * (kM * 128) + ko, 16, 1024),
                         tc::smem_desc_sw128(kst(s) + (k >> 2) * 1024 + ko, 16, C::kGroup),
                         idS, k > 0);
      }
      tc::commit_elect(bar(kBarSFull + buf));  // also frees K slot s
      return true;
    };
    bool ok = issue_s(0);
    for (int i = 0; ok && i < ntiles; ++i) {
      if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
      if (i + 1 < ntiles && !issue_s(i + 1)) {
        ok = false;
        break;
      }
      const int s = i % kVRing, buf = i % kSBufs;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(bar(kBarPFull + buf), (i / kSBufs) & 1, kTimeoutNs) &&
                          mbar_wait_bounded(bar(kBarVFull + s), (i / kVRing) & 1, kTimeoutNs))) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const uint32_t pcol = tm0 + 128 * (1 + buf);
#pragma unroll
      for (int kk = 0; kk < kN / 16; ++kk) {
        // keys 16 kk .. : half kk / 4, its hi columns from 64 half, lo 32 further
        const uint32_t pa = pcol + 64 * (kk >> 2) + 8 * (kk & 3);
        const uint64_t dv = tc::smem_desc_sw128(vst(s) + kk * 2 * C::kGroup, 1024, C::kGroup);
        tc::mma_ts_elect(tm0, pa, dv, idPV, (i > 0 || kk > 0) ? 1u : 0u);
        if constexpr (BF16) tc::mma_ts_elect(tm0, pa + 32, dv, idPV, 1u);
      }
      tc::commit_elect(bar(kBarPvDone + buf));  // also frees V slot s
    }
    if (!ok && lane == 0) give_up();
    // every MMA issued has completed before the TMEM is freed
    tc::commit_elect(bar(kBarDrain));
    (void)mbar_wait_bounded(bar(kBarDrain), 0, kTimeoutNs);
    __syncwarp();
  } else {
    // ---------------- softmax + epilogue (warps 0-7) ----------------
    constexpr int kH = kN / 2;  // keys of a tile per half
    const uint32_t tl = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int pair = warp & 3;
    float *xm = reinterpret_cast<float *>(smem + C::kXm);  // [parity][half][row]
    float *xl = reinterpret_cast<float *>(smem + C::kXl);  // [half][row]
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < ntiles; ++i) {
      if (__any_sync(0xffffffffu, *abort_flag != 0)) {
        ok = false;
        break;
      }
      const int buf = i % kSBufs;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(bar(kBarSFull + buf), (i / kSBufs) & 1, kTimeoutNs))) {
        if (lane == 0) give_up();
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const uint32_t scol = tl + 128 * (1 + buf) + kH * hf;  // this half's 64 S columns
      float sv[kH];
      {
        uint32_t r[kH / 32][32];
#pragma unroll
        for (int c = 0; c < kH / 32; ++c) tc::ld32(scol + 32 * c, r[c]);
        tc::wait_ld();
#pragma unroll
        for (int c = 0; c < kH / 32; ++c)
#pragma unroll
          for (int j = 0; j < 32; ++j) sv[32 * c + j] = __uint_as_float(r[c][j]);
      }
      const int key0 = i * kN + kH * hf;
      if (key0 + kH - 1 > lim) {  // this half crosses the row's causal limit
#pragma unroll
        for (int j = 0; j < kH; ++j)
          if (key0 + j > lim) sv[j] = -INFINITY;
      }
      // max over the raw scores (scale > 0), eight independent chains, then
      // the other half's through shared memory
      float mx;
      {
        // four independent chains of three-input maxima over 16 scores each
        float m4[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float m = fmax3f(sv[k], sv[k + 4], sv[k + 8]);
#pragma unroll
          for (int t = 3; t + 1 < kH / 4; t += 2) m = fmax3f(m, sv[k + 4 * t], sv[k + 4 * (t + 1)]);
          m4[k] = fmaxf(m, sv[k + kH - 4]);
        }
        mx = fmax3f(m4[0], m4[1], fmaxf(m4[2], m4[3]));
        const int par = i & 1;
        xm[(par * 2 + hf) * kM + row] = mx;
        mbar_arrive(bar(kBarXchg + par * 4 + pair));
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarXchg + par * 4 + pair),
                                                        (i >> 1) & 1, kTimeoutNs))) {
          if (lane == 0) give_up();
          ok = false;
          break;
        }
        mx = fmaxf(xm[(par * 2) * kM + row], xm[(par * 2 + 1) * kM + row]) * p.scale_log2;
      }
      const bool need = mx > m_used + kRescaleLog2;
      const float m_new = need ? mx : m_used;
      const float alpha = need ? fast_exp2(m_used - m_new) : 1.f;
      if (i > 0 && __any_sync(0xffffffffu, need)) {
        const int pb = (i - 1) % kSBufs;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarPvDone + pb),
                                                        ((i - 1) / kSBufs) & 1, kTimeoutNs))) {
          if (lane == 0) give_up();
          ok = false;
          break;
        }
        tc::fence_after_sync();
#pragma unroll 1
        for (int c = hf * (D / 64); c < (hf + 1) * (D / 64); ++c) {  // this half's O columns
          uint32_t r[32];
          tc::ld32(tl + 32 * c, r);
          tc::wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * alpha);
          tc::st32(tl + 32 * c, r);
        }
        tc::wait_st();
      }
      m_used = m_new;
      const float neg_m = -m_used;
      // key pairs through the packed fp32 instructions: scale and shift, the
      // running sums (four pair accumulators) and the bf16 residual
      const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2), nm2 = f2_pack(neg_m, neg_m);
      uint64_t l2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
      for (int c = 0; c < kH / 32; ++c) {
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int w = 0; w < 16; ++w) {
          float xa, xe;
          f2_unpack(f2_fma(f2_pack(sv[32 * c + 2 * w], sv[32 * c + 2 * w + 1]), sc2, nm2), xa, xe);
          const float a = fast_exp2(xa), e = fast_exp2(xe);
          const uint64_t ae = f2_pack(a, e);
          l2[w & 3] = f2_add(l2[w & 3], ae);
          hi[w] = pack2<BF16>(a, e);
          if constexpr (BF16) {
            float ra, re;
            f2_unpack(f2_sub(ae, f2_pack(__uint_as_float(hi[w] << 16),
                                         __uint_as_float(hi[w] & 0xffff0000u))),
                      ra, re);
            lo[w] = pack2<BF16>(ra, re);
          }
        }
        // P over this half's own S columns: hi in the first 32, lo in the last
        tc::st16(scol + 16 * c, hi);
        if constexpr (BF16) tc::st16(scol + 32 + 16 * c, lo);
      }
      float l8[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) f2_unpack(l2[k], l8[2 * k], l8[2 * k + 1]);
      l = l * alpha + (((l8[0] + l8[1]) + (l8[2] + l8[3])) + ((l8[4] + l8[5]) + (l8[6] + l8[7])));
      const int nvalid = kv_len - i * kN;
      if (nvalid < kN) {
        // last tile: keys past kv_len hold stale smem / pool rows; their P is
        // 0 but 0 * NaN is not, so the V rows become exact zeros first
        const int s = i % kVRing;
        if (!__all_sync(0xffffffffu,
                        mbar_wait_bounded(bar(kBarVFull + s), (i / kVRing) & 1, kTimeoutNs))) {
          if (lane == 0) give_up();
          ok = false;
          break;
        }
        const int units = (kN - nvalid) * (D / 8);
        for (int e = threadIdx.x; e < units; e += 32 * kSoftWarps) {
          const int r = nvalid + e / (D / 8), u = e % (D / 8);
          const int c = u >> 3, uu = u & 7;
          *reinterpret_cast<uint4 *>(smem + C::kV0 + s * C::kTile + (r >> 3) * C::kGroup +
                                     c * 1024 + (r & 7) * 128 + ((uu ^ (r & 7)) << 4)) =
              make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
      }
      tc::wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kBarPFull + buf));
    }
    if (ok) {
      const int lb = (ntiles - 1) % kSBufs;
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarPvDone + lb),
                                                     ((ntiles - 1) / kSBufs) & 1, kTimeoutNs));
      if (!ok && lane == 0) give_up();
    }
    if (ok) {
      // row sum = the two halves' sums, added in a fixed order
      xl[hf * kM + row] = l;
      mbar_arrive(bar(kBarLx + pair));
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarLx + pair), 0, kTimeoutNs));
      if (!ok && lane == 0) give_up();
    }
    if (ok) {
      tc::fence_after_sync();
      const float inv = 1.f / (xl[row] + xl[kM + row]);
      const int64_t ob = (int64_t)(p.q_start[b] + tok) * p.o_st + (int64_t)hq * p.o_sh;
#pragma unroll
      for (int c = hf * (D / 64); c < (hf + 1) * (D / 64); ++c) {
        uint32_t r[32];
        tc::ld32(tl + 32 * c, r);
        tc::wait_ld();
        if (live) {
          if (p.out_f32) {
            float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.out) + ob + 32 * c);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              dst[j] = make_float4(__uint_as_float(r[4 * j]) * inv, __uint_as_float(r[4 * j + 1]) * inv,
                                   __uint_as_float(r[4 * j + 2]) * inv,
                                   __uint_as_float(r[4 * j + 3]) * inv);
          } else {
            uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.out) + ob + 32 * c);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              dst[j] = make_uint4(pack2<BF16>(__uint_as_float(r[8 * j]) * inv,
                                              __uint_as_float(r[8 * j + 1]) * inv),
                                  pack2<BF16>(__uint_as_float(r[8 * j + 2]) * inv,
                                              __uint_as_float(r[8 * j + 3]) * inv),
                                  pack2<BF16>(__uint_as_float(r[8 * j + 4]) * inv,
                                              __uint_as_float(r[8 * j + 5]) * inv),
                                  pack2<BF16>(__uint_as_float(r[8 * j + 6]) * inv,
                                              __uint_as_float(r[8 * j + 7]) * inv));
          }
        }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Persistent form: one CTA per SM takes work items -- (sequence, KV head,
// query block of 128 rows) -- in turn, the query blocks with the most key
// tiles first, and keeps its barriers, TMEM and copy rings across items.  Tile
// slots, buffers and barrier phases count the CTA's key tiles over all its
// items (global tile index g), so the copy warp streams the next item's K/V
// while the current one finishes.  Per item the softmax warps load Q (once the
// item before has no S left to issue) and signal it (kBarQReady); the first
// PV of an item, which starts O afresh, waits until the softmax warps have
// read the previous item's O (kBarOFree).  Everything else is the one-block
// kernel above.
template <int D, bool BF16>
__global__ void __launch_bounds__(tcp::kThreads, 1)
    paged_prefill_ps_kernel(const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const PParams p) {
  using namespace tcp;
  using C = TCfg<D>;
  const int tpc = kM / p.G;
  const int per_q = p.n_seqs * p.Hkv;
  const int n_items = per_q * p.qblocks;

  // item e: query block qblocks - 1 - e % qblocks (a pair's last, longest
  // blocks first) of pair e / qblocks = (sequence, KV head): neighbouring
  // items share their pair's K/V through L2
  struct Item {
    int b, h, q0, n, start, q_hi, kv_len, ntiles;
    bool ok;
  };
  auto item_at = [&](int e) {
    Item it{};
    const int rem = e / p.qblocks, jr = e - rem * p.qblocks;
    it.b = rem / p.Hkv;
    it.h = rem - it.b * p.Hkv;
    it.q0 = (p.qblocks - 1 - jr) * tpc;
    it.n = p.q_len[it.b];
    it.ok = false;
    if (it.n <= 0 || it.q0 >= it.n) return it;
    const int ctx = p.ctx[it.b];
    if (ctx < it.n || ctx > p.max_blocks * p.bs) {
      if (threadIdx.x == 0) dev_error(p.err, MZ_DEVERR_CONTEXT);
      return it;
    }
    if (p.q_start[it.b] < 0 || (int64_t)p.q_start[it.b] + it.n > p.n_rows) {
      if (threadIdx.x == 0) dev_error(p.err, MZ_DEVERR_ROWS);
      return it;
    }
    it.start = ctx - it.n;
    it.q_hi = min(it.q0 + tpc, it.n);
    it.kv_len = it.start + it.q_hi;
    it.ntiles = (it.kv_len + kN - 1) / kN;
    it.ok = true;
    return it;
  };

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t qs = sbase;
  auto kst = [&](int s) { return sbase + C::kK0 + s * C::kTile; };
  auto vst = [&](int s) { return sbase + C::kV0 + s * C::kTile; };
  const uint32_t bars = sbase + C::kBar;
  auto bar = [&](int i) { return bars + 8 * i; };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::kBar + 8 * kNumBarsPs);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::kBar + 8 * kNumBarsPs + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (warp == kProdWarp && lane == 0) {
    for (int s = 0; s < kKRing; ++s) mbar_init(bar(kBarKFull + s), 1);
    for (int s = 0; s < kVRing; ++s) mbar_init(bar(kBarVFull + s), 1);
    for (int s = 0; s < kSBufs; ++s) {
      mbar_init(bar(kBarSFull + s), 1);
      mbar_init(bar(kBarPFull + s), kSoftWarps);
      mbar_init(bar(kBarPvDone + s), 1);
    }
    mbar_init(bar(kBarDrain), 1);
    for (int x = 0; x < 8; ++x) mbar_init(bar(kBarXchg + x), 64);
    for (int x = 0; x < 4; ++x) mbar_init(bar(kBarLx + x), 64);
    mbar_init(bar(kBarQReady), kSoftWarps);
    mbar_init(bar(kBarOFree), kSoftWarps);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProdWarp) {
    __syncwarp();
    asm volatile("bar.arrive 1, %0;" ::"n"(kThreads) : "memory");
  }
  if (warp == kMmaWarp) tc::tmem_alloc(smem_u32(tmem_slot), kTmemCols);
  uint32_t tmem = 0;
  if (warp != kProdWarp) {
    tc::fence_before_sync();
    asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
    tc::fence_after_sync();
    tmem = *tmem_slot;
  }

  auto give_up = [&]() {
    dev_error(p.err, MZ_DEVERR_TIMEOUT);
    *abort_flag = 1;
  };

  if (warp == kProdWarp) {
    // ---------------- producer (whole warp) ----------------
    const uint64_t pol = l2_policy_evict_last();
    const int sub = 1 << p.sub_log2, nst_log2 = 7 - p.sub_log2, nst = 1 << nst_log2;
    int tg = 0, k_issued = 0, v_issued = 0;  // global tile counts
    bool ok = true;
    for (int e = blockIdx.x; ok && e < n_items; e += gridDim.x) {
      const Item it = item_at(e);
      if (!it.ok) continue;
      const int b = it.b, h = it.h, kv_len = it.kv_len, ntiles = it.ntiles;
      auto group_key = [&](int g) {
        return lane < 4 * nst ? (4 * g + (lane >> nst_log2)) * kN + (lane & (nst - 1)) * sub
                              : kv_len;
      };
      auto group_ids = [&](int g) -> int32_t {
        const int t = group_key(g);
        return t < kv_len ? p.tables[(int64_t)b * p.max_blocks + t / p.bs] : 0;
      };
      auto group_rows = [&](int g, int32_t blk) -> int {
        const int t = group_key(g);
        if (t >= kv_len) return 0;
        if (blk < 0 || blk >= p.n_blocks) {
          dev_error(p.err, MZ_DEVERR_BLOCK_ID);
          blk = 0;
        }
        return static_cast<int>(((int64_t)blk * p.Hkv + h) * p.bs + t % p.bs);
      };
      auto load = [&](const CUtensorMap *tm, uint32_t dst, uint32_t fbar, int j, int y) {
        const int nsub = min(nst, (kv_len - j * kN + sub - 1) >> p.sub_log2);
        if (lane == 0)
          mbar_arrive_expect_tx(fbar, static_cast<uint32_t>(nsub * (D / 64) * sub * 128));
        __syncwarp();
        if (lane < nsub) tma_load_4d(dst + lane * (sub / 8) * C::kGroup, tm, y >> 3, fbar, pol);
      };
      int y_prv = 0, y_cur = group_rows(0, group_ids(0));
      int32_t id_nxt = group_ids(1);
      // step t: K_t, then V_{t-1} (item-local t; slots by the global index)
      for (int t = 0; t <= ntiles; ++t) {
        if (__any_sync(0xffffffffu, *abort_flag != 0)) {
          ok = false;
          break;
        }
        if (t > 0 && (t & 3) == 0) {
          y_prv = y_cur;
          y_cur = group_rows(t >> 2, id_nxt);
          id_nxt = group_ids((t >> 2) + 1);
        }
        if (t < ntiles) {
          const int g = tg + t, s = g % kKRing;
          const int y = __shfl_sync(0xffffffffu, y_cur, ((t & 3) << nst_log2) + (lane & (nst - 1)));
          // K slot s frees when S of global tile g - 3 completed (kKRing == kSBufs)
          if (g >= kKRing &&
              !__all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarSFull + (g - kKRing) % kSBufs),
                                                          ((g - kKRing) / kSBufs) & 1, kTimeoutNs))) {
            if (lane == 0) give_up();
            ok = false;
            break;
          }
          load(&tmK, kst(s), bar(kBarKFull + s), t, y);
          k_issued = g + 1;
        }
        if (t >= 1) {
          const int j = t - 1, gj = tg + j, s = gj % kVRing;
          const int y = __shfl_sync(0xffffffffu, (j >> 2) == (t >> 2) ? y_cur : y_prv,
                                    ((j & 3) << nst_log2) + (lane & (nst - 1)));
          // V slot s frees when PV of global tile gj - 2 completed
          if (gj >= kVRing &&
              !__all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarPvDone + (gj - kVRing) % kSBufs),
                                                          ((gj - kVRing) / kSBufs) & 1, kTimeoutNs))) {
            if (lane == 0) give_up();
            ok = false;
            break;
          }
          load(&tmV, vst(s), bar(kBarVFull + s), j, y);
          v_issued = gj + 1;
        }
      }
      tg += ntiles;
    }
    // copies still in flight land before the CTA leaves
    if (lane == 0) {
      for (int j = max(0, k_issued - kKRing); j < k_issued; ++j)
        (void)mbar_wait_bounded(bar(kBarKFull + j % kKRing), (j / kKRing) & 1, kTimeoutNs);
      for (int j = max(0, v_issued - kVRing); j < v_issued; ++j)
        (void)mbar_wait_bounded(bar(kBarVFull + j % kVRing), (j / kVRing) & 1, kTimeoutNs);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issue (whole warp, one elected lane issues) ----------------
    constexpr uint32_t idS = tc::idesc_f16(BF16, kM, kN, false);
    constexpr uint32_t idPV = tc::idesc_f16(BF16, kM, D, true);
    const uint32_t tm0 = __shfl_sync(0xffffffffu, tmem, 0);
    // S of global tile j
    auto issue_s = [&](int j) -> bool {
      const int s = j % kKRing, buf = j % kSBufs;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(bar(kBarKFull + s), (j / kKRing) & 1, kTimeoutNs)))
        return false;
      // buffer j % 3 is free once PV of global tile j - 3 (which read P from it) completed
      if (j >= kSBufs &&
          !__all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarPvDone + buf),
                                                      ((j - kSBufs) / kSBufs) & 1, kTimeoutNs)))
        return false;
      tc::fence_after_sync();
      const uint32_t d = tm0 + 128 * (1 + buf);
#pragma unroll
      for (int k = 0; k < D / 16; ++k) {
        const uint32_t ko = (k & 3) * 32;  // 16-column step inside the chunk's atom
        tc::mma_ss_elect(d, tc::smem_desc_sw128(qs + (k >> 2) * (kM * 128) + ko, 16, 1024),
                         tc::smem_desc_sw128(kst(s) + (k >> 2) * 1024 + ko, 16, C::kGroup),
                         idS, k > 0);
      }
      tc::commit_elect(bar(kBarSFull + buf));  // also frees K slot s
      return true;
    };
    int tg = 0, nit = 0;
    bool ok = true;
    for (int e = blockIdx.x; ok && e < n_items; e += gridDim.x) {
      const Item it = item_at(e);
      if (!it.ok) continue;
      const int ntiles = it.ntiles;
      // this item's Q is in shared memory
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarQReady), nit & 1, kTimeoutNs)) ||
          !issue_s(tg)) {
        ok = false;
        break;
      }
      for (int i = 0; i < ntiles; ++i) {
        if (__any_sync(0xffffffffu, *abort_flag != 0)) {
          ok = false;
          break;
        }
        const int g = tg + i;
        if (i + 1 < ntiles && !issue_s(g + 1)) {
          ok = false;
          break;
        }
        const int s = g % kVRing, buf = g % kSBufs;
        if (!__all_sync(0xffffffffu,
                        mbar_wait_bounded(bar(kBarPFull + buf), (g / kSBufs) & 1, kTimeoutNs) &&
                            mbar_wait_bounded(bar(kBarVFull + s), (g / kVRing) & 1, kTimeoutNs))) {
          ok = false;
          break;
        }
        // the first PV of an item starts O afresh: the previous item's O has been read
        if (i == 0 && nit > 0 &&
            !__all_sync(0xffffffffu,
                        mbar_wait_bounded(bar(kBarOFree), (nit - 1) & 1, kTimeoutNs))) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t pcol = tm0 + 128 * (1 + buf);
#pragma unroll
        for (int kk = 0; kk < kN / 16; ++kk) {
          // keys 16 kk .. : half kk / 4, its hi columns from 64 half, lo 32 further
          const uint32_t pa = pcol + 64 * (kk >> 2) + 8 * (kk & 3);
          const uint64_t dv = tc::smem_desc_sw128(vst(s) + kk * 2 * C::kGroup, 1024, C::kGroup);
          tc::mma_ts_elect(tm0, pa, dv, idPV, (i > 0 || kk > 0) ? 1u : 0u);
          if constexpr (BF16) tc::mma_ts_elect(tm0, pa + 32, dv, idPV, 1u);
        }
        tc::commit_elect(bar(kBarPvDone + buf));  // also frees V slot s
      }
      tg += ntiles;
      ++nit;
    }
    if (!ok && lane == 0) give_up();
    // every MMA issued has completed before the TMEM is freed
    tc::commit_elect(bar(kBarDrain));
    (void)mbar_wait_bounded(bar(kBarDrain), 0, kTimeoutNs);
    __syncwarp();
  } else {
    // ---------------- softmax + epilogue (warps 0-7) ----------------
    constexpr int kH = kN / 2;  // keys of a tile per half
    const uint32_t tl = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int pair = warp & 3;
    float *xm = reinterpret_cast<float *>(smem + C::kXm);  // [parity][half][row]
    float *xl = reinterpret_cast<float *>(smem + C::kXl);  // [half][row]
    const int row = threadIdx.x & (kM - 1), hf = threadIdx.x >> 7;
    int tg = 0, nit = 0;
    bool ok = true;
    for (int e = blockIdx.x; ok && e < n_items; e += gridDim.x) {
      const Item it = item_at(e);
      if (!it.ok) continue;
      const int b = it.b, start = it.start, q_hi = it.q_hi, kv_len = it.kv_len, ntiles = it.ntiles;
      const int tok = it.q0 + row / p.G;
      const int hq = it.h * p.G + row % p.G;
      const bool live = tok < q_hi;
      const int lim = start + min(tok, q_hi - 1);  // last visible key of the row
      {
        // half hf of the Q row -> shared memory (128-byte-swizzled K-major
        // layout); every S of the item before has completed (this thread
        // waited for each)
        const uint4 *src = reinterpret_cast<const uint4 *>(
            static_cast<const uint16_t *>(p.q) + (int64_t)(p.q_start[b] + tok) * p.q_st +
            (int64_t)hq * p.q_sh);
#pragma unroll
        for (int u = hf * (D / 16); u < (hf + 1) * (D / 16); ++u) {
          const uint4 v = live ? src[u] : make_uint4(0, 0, 0, 0);
          const int c = u >> 3, uu = u & 7;
          *reinterpret_cast<uint4 *>(smem + c * (kM * 128) + row * 128 + ((uu ^ (row & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kBarQReady));
      }
      float m_used = -INFINITY, l = 0.f;
      for (int i = 0; i < ntiles; ++i) {
        const int g = tg + i;
        if (__any_sync(0xffffffffu, *abort_flag != 0)) {
          ok = false;
          break;
        }
        const int buf = g % kSBufs;
        if (!__all_sync(0xffffffffu,
                        mbar_wait_bounded(bar(kBarSFull + buf), (g / kSBufs) & 1, kTimeoutNs))) {
          if (lane == 0) give_up();
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t scol = tl + 128 * (1 + buf) + kH * hf;  // this half's 64 S columns
        float sv[kH];
        {
          uint32_t r[kH / 32][32];
  #pragma unroll
          for (int c = 0; c < kH / 32; ++c) tc::ld32(scol + 32 * c, r[c]);
          tc::wait_ld();
  #pragma unroll
          for (int c = 0; c < kH / 32; ++c)
  #pragma unroll
            for (int j = 0; j < 32; ++j) sv[32 * c + j] = __uint_as_float(r[c][j]);
        }
        const int key0 = i * kN + kH * hf;
        if (key0 + kH - 1 > lim) {  // this half crosses the row's causal limit
  #pragma unroll
          for (int j = 0; j < kH; ++j)
            if (key0 + j > lim) sv[j] = -INFINITY;
        }
        // max over the raw scores (scale > 0), eight independent chains, then
        // the other half's through shared memory
        float mx;
        {
          // four independent chains of three-input maxima over 16 scores each
          float m4[4];
  #pragma unroll
          for (int k = 0; k < 4; ++k) {
            float m = fmax3f(sv[k], sv[k + 4], sv[k + 8]);
  #pragma unroll
            for (int t = 3; t + 1 < kH / 4; t += 2) m = fmax3f(m, sv[k + 4 * t], sv[k + 4 * (t + 1)]);
            m4[k] = fmaxf(m, sv[k + kH - 4]);
          }
          mx = fmax3f(m4[0], m4[1], fmaxf(m4[2], m4[3]));
          const int par = g & 1;
          xm[(par * 2 + hf) * kM + row] = mx;
          mbar_arrive(bar(kBarXchg + par * 4 + pair));
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarXchg + par * 4 + pair),
                                                          (g >> 1) & 1, kTimeoutNs))) {
            if (lane == 0) give_up();
            ok = false;
            break;
          }
          mx = fmaxf(xm[(par * 2) * kM + row], xm[(par * 2 + 1) * kM + row]) * p.scale_log2;
        }
        const bool need = mx > m_used + kRescaleLog2;
        const float m_new = need ? mx : m_used;
        const float alpha = need ? fast_exp2(m_used - m_new) : 1.f;
        if (i > 0 && __any_sync(0xffffffffu, need)) {
          const int pb = (g - 1) % kSBufs;
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarPvDone + pb),
                                                          ((g - 1) / kSBufs) & 1, kTimeoutNs))) {
            if (lane == 0) give_up();
            ok = false;
            break;
          }
          tc::fence_after_sync();
  #pragma unroll 1
          for (int c = hf * (D / 64); c < (hf + 1) * (D / 64); ++c) {  // this half's O columns
            uint32_t r[32];
            tc::ld32(tl + 32 * c, r);
            tc::wait_ld();
  #pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * alpha);
            tc::st32(tl + 32 * c, r);
          }
          tc::wait_st();
        }
        m_used = m_new;
        const float neg_m = -m_used;
        // key pairs through the packed fp32 instructions: scale and shift, the
        // running sums (four pair accumulators) and the bf16 residual
        const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2), nm2 = f2_pack(neg_m, neg_m);
        uint64_t l2[4] = {0ull, 0ull, 0ull, 0ull};
  #pragma unroll
        for (int c = 0; c < kH / 32; ++c) {
          uint32_t hi[16], lo[16];
  #pragma unroll
          for (int w = 0; w < 16; ++w) {
            float xa, xe;
            f2_unpack(f2_fma(f2_pack(sv[32 * c + 2 * w], sv[32 * c + 2 * w + 1]), sc2, nm2), xa, xe);
            const float a = fast_exp2(xa), e = fast_exp2(xe);
            const uint64_t ae = f2_pack(a, e);
            l2[w & 3] = f2_add(l2[w & 3], ae);
            hi[w] = pack2<BF16>(a, e);
            if constexpr (BF16) {
              float ra, re;
              f2_unpack(f2_sub(ae, f2_pack(__uint_as_float(hi[w] << 16),
                                           __uint_as_float(hi[w] & 0xffff0000u))),
                        ra, re);
              lo[w] = pack2<BF16>(ra, re);
            }
          }
          // P over this half's own S columns: hi in the first 32, lo in the last
          tc::st16(scol + 16 * c, hi);
          if constexpr (BF16) tc::st16(scol + 32 + 16 * c, lo);
        }
        float l8[8];
  #pragma unroll
        for (int k = 0; k < 4; ++k) f2_unpack(l2[k], l8[2 * k], l8[2 * k + 1]);
        l = l * alpha + (((l8[0] + l8[1]) + (l8[2] + l8[3])) + ((l8[4] + l8[5]) + (l8[6] + l8[7])));
        const int nvalid = kv_len - i * kN;
        if (nvalid < kN) {
          // last tile: keys past kv_len hold stale smem / pool rows; their P is
          // 0 but 0 * NaN is not, so the V rows become exact zeros first
          const int s = g % kVRing;
          if (!__all_sync(0xffffffffu,
                          mbar_wait_bounded(bar(kBarVFull + s), (g / kVRing) & 1, kTimeoutNs))) {
            if (lane == 0) give_up();
            ok = false;
            break;
          }
          const int units = (kN - nvalid) * (D / 8);
          for (int e = threadIdx.x; e < units; e += 32 * kSoftWarps) {
            const int r = nvalid + e / (D / 8), u = e % (D / 8);
            const int c = u >> 3, uu = u & 7;
            *reinterpret_cast<uint4 *>(smem + C::kV0 + s * C::kTile + (r >> 3) * C::kGroup +
                                       c * 1024 + (r & 7) * 128 + ((uu ^ (r & 7)) << 4)) =
                make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();
        }
        tc::wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kBarPFull + buf));
      }
      if (ok) {
        const int lb = (tg + ntiles - 1) % kSBufs;
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarPvDone + lb),
                                                       ((tg + ntiles - 1) / kSBufs) & 1, kTimeoutNs));
        if (!ok && lane == 0) give_up();
      }
      if (ok) {
        // row sum = the two halves' sums, added in a fixed order
        xl[hf * kM + row] = l;
        mbar_arrive(bar(kBarLx + pair));
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarLx + pair), nit & 1, kTimeoutNs));
        if (!ok && lane == 0) give_up();
      }
      if (ok) {
        tc::fence_after_sync();
        const float inv = 1.f / (xl[row] + xl[kM + row]);
        const int64_t ob = (int64_t)(p.q_start[b] + tok) * p.o_st + (int64_t)hq * p.o_sh;
  #pragma unroll
        for (int c = hf * (D / 64); c < (hf + 1) * (D / 64); ++c) {
          uint32_t r[32];
          tc::ld32(tl + 32 * c, r);
          tc::wait_ld();
          if (live) {
            if (p.out_f32) {
              float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.out) + ob + 32 * c);
  #pragma unroll
              for (int j = 0; j < 8; ++j)
                dst[j] = make_float4(__uint_as_float(r[4 * j]) * inv, __uint_as_float(r[4 * j + 1]) * inv,
                                     __uint_as_float(r[4 * j + 2]) * inv,
                                     __uint_as_float(r[4 * j + 3]) * inv);
            } else {
              uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.out) + ob + 32 * c);
  #pragma unroll
              for (int j = 0; j < 4; ++j)
                dst[j] = make_uint4(pack2<BF16>(__uint_as_float(r[8 * j]) * inv,
                                                __uint_as_float(r[8 * j + 1]) * inv),
                                    pack2<BF16>(__uint_as_float(r[8 * j + 2]) * inv,
                                                __uint_as_float(r[8 * j + 3]) * inv),
                                    pack2<BF16>(__uint_as_float(r[8 * j + 4]) * inv,
                                                __uint_as_float(r[8 * j + 5]) * inv),
                                    pack2<BF16>(__uint_as_float(r[8 * j + 6]) * inv,
                                                __uint_as_float(r[8 * j + 7]) * inv));
            }
          }
        }
      }
      if (!ok) break;
      // this item's O has been read: the next item's first PV may overwrite it
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kBarOFree));
      tg += ntiles;
      ++nit;
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, bool BF16>
int smem_attr_ps() {
  static DeviceOnce once;
  return smem_optin(paged_prefill_ps_kernel<D, BF16>, tcp::TCfg<D>::kSmemBytes, once,
                    "mz_paged_prefill: shared memory attribute (persistent form)");
}

template <int D, bool BF16>
int smem_attr_tc() {
  static DeviceOnce once;
  return smem_optin(paged_prefill_tc_kernel<D, BF16>, tcp::TCfg<D>::kSmemBytes, once,
                    "mz_paged_prefill: shared memory attribute");
}

}  // namespace prefill
}  // namespace mz

using namespace mz;
using namespace mz::prefill;

extern "C" int mz_paged_prefill(void *out, int32_t out_dtype, int64_t out_tok_stride,
                                int64_t out_head_stride, const void *q, int64_t q_tok_stride,
                                int64_t q_head_stride, int32_t n_rows, const int32_t *q_start,
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
      max_blocks_per_seq <= 0 || n_blocks <= 0 || n_rows < 0)
    return fail(MZ_ERR_INVALID_ARG, "%s: bad sizes", fn);
  const int G = n_heads / n_kv_heads;
  if (tcp::kM % G)
    return fail(MZ_ERR_UNSUPPORTED, "%s: n_heads / n_kv_heads = %d does not divide %d", fn, G,
                tcp::kM);
  if (!std::isfinite(scale) || !(scale > 0.f))
    return fail(MZ_ERR_INVALID_ARG, "%s: scale must be finite and positive", fn);
  if (n_seqs == 0 || max_q_len == 0) return MZ_OK;
  if (!out || !q || !q_start || !q_len || !k_pool || !v_pool || !block_tables || !ctx_lens)
    return fail(MZ_ERR_INVALID_ARG, "%s: null pointer", fn);
  // rows move as 16-byte vectors: q and out 16-byte aligned, strides whole vectors
  const int oe = out_dtype == MZ_DTYPE_F32 ? 4 : 8;
  if (!aligned(k_pool, 16) || !aligned(v_pool, 16) || !aligned(q, 16) || (q_tok_stride % 8) ||
      (q_head_stride % 8) || !aligned(out, 16) || (out_tok_stride % oe) || (out_head_stride % oe))
    return fail(MZ_ERR_ALIGNMENT,
                "%s: pools, q and out need 16-byte alignment and strides of whole 16-byte "
                "vectors", fn);
  const int64_t rows_total = n_blocks * n_kv_heads * block_size;
  if (rows_total >= (int64_t(1) << 31))
    return fail(MZ_ERR_UNSUPPORTED, "%s: pool has >= 2^31 rows", fn);

  const bool bf16 = dtype == MZ_DTYPE_BF16;
  CUtensorMap tk, tv;
  const auto type = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int sub_log2 = 4;  // rows per copy box: gcd(block_size, 128)
  while (sub_log2 < 7 && block_size % (1 << (sub_log2 + 1)) == 0) ++sub_log2;
  if (int rc = make_group_map(&tk, k_pool, rows_total, head_dim, type, 1 << sub_log2)) return rc;
  if (int rc = make_group_map(&tv, v_pool, rows_total, head_dim, type, 1 << sub_log2)) return rc;

  PParams p;
  p.out = out;
  p.o_st = out_tok_stride;
  p.o_sh = out_head_stride;
  p.out_f32 = out_dtype == MZ_DTYPE_F32;
  p.q = q;
  p.q_st = q_tok_stride;
  p.q_sh = q_head_stride;
  p.n_rows = n_rows;
  p.q_start = q_start;
  p.q_len = q_len;
  p.ctx = ctx_lens;
  p.tables = block_tables;
  p.max_blocks = max_blocks_per_seq;
  p.Hkv = n_kv_heads;
  p.G = G;
  p.bs = block_size;
  p.n_blocks = n_blocks;
  p.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
  p.sub_log2 = sub_log2;
  p.err = dev_err;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_seqs > 65535 || n_kv_heads > 65535)
    return fail(MZ_ERR_UNSUPPORTED, "%s: grid too large", fn);
  const int tpc = tcp::kM / G;
  // The persistent form (one CTA per SM over all query blocks) by default;
  // MLXZ_B200_PREFILL_PERSIST=0 launches one CTA per query block instead
  if (decode::env_int("MLXZ_B200_PREFILL_PERSIST", 1, 0, 1) == 1) {
    p.n_seqs = n_seqs;
    p.qblocks = (max_q_len + tpc - 1) / tpc;
    const int64_t items = (int64_t)n_seqs * n_kv_heads * p.qblocks;
    if (items >= (int64_t(1) << 31)) return fail(MZ_ERR_UNSUPPORTED, "%s: too many query blocks", fn);
    const int sms = sm_count(current_device());
    if (sms <= 0) return fail(MZ_ERR_CUDA, "%s: cannot query the SM count", fn);
    const dim3 grid_ps(static_cast<unsigned>(std::min<int64_t>(items, sms)));
#define MZ_PSLAUNCH(D_, BF_)                                                                     \
  do {                                                                                           \
    if (int rc = smem_attr_ps<D_, BF_>()) return rc;                                             \
    paged_prefill_ps_kernel<D_, BF_>                                                             \
        <<<grid_ps, tcp::kThreads, tcp::TCfg<D_>::kSmemBytes, s>>>(tk, tv, p);                   \
  } while (0)
    if (head_dim == 128) {
      if (bf16) MZ_PSLAUNCH(128, true); else MZ_PSLAUNCH(128, false);
    } else {
      if (bf16) MZ_PSLAUNCH(64, true); else MZ_PSLAUNCH(64, false);
    }
#undef MZ_PSLAUNCH
    MZ_CHECK_LAUNCH(fn);
    return MZ_OK;
  }
  const dim3 grid((max_q_len + tpc - 1) / tpc, n_kv_heads, n_seqs);
#define MZ_TCLAUNCH(D_, BF_)                                                                     \
  do {                                                                                           \
    if (int rc = smem_attr_tc<D_, BF_>()) return rc;                                             \
    paged_prefill_tc_kernel<D_, BF_>                                                             \
        <<<grid, tcp::kThreads, tcp::TCfg<D_>::kSmemBytes, s>>>(tk, tv, p);                      \
  } while (0)
  if (head_dim == 128) {
    if (bf16) MZ_TCLAUNCH(128, true); else MZ_TCLAUNCH(128, false);
  } else {
    if (bf16) MZ_TCLAUNCH(64, true); else MZ_TCLAUNCH(64, false);
  }
#undef MZ_TCLAUNCH
  MZ_CHECK_LAUNCH(fn);
  return MZ_OK;
}
