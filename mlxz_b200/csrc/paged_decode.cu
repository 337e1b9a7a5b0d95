// Fused GQA paged decode attention for sm_100a.
//
// Work decomposition.  The KV of every (sequence b, kv head h) is a list of
// 16-token tiles (a block of block_size tokens is block_size/16 tiles).  All
// tiles of all (b, h) pairs, in (b, h, t) order, form one flat sequence of T
// tiles.  The grid is a persistent set of W warps; warp w owns the contiguous
// share [w*per, (w+1)*per) with per = ceil(T / W), so every warp streams the
// same number of tiles whatever the context lengths are (no tail from ragged
// sequences).  A (b, h) pair that lies inside one warp's share is finished by
// that warp.  A pair cut by share boundaries leaves one partial (running max
// m, running sum l, unnormalised O) per piece in the workspace; the warp that
// finishes the last piece (per-pair arrival counter) merges them.
//
// Per warp, a STAGES-deep ring of shared-memory stages is filled by 2-D bulk
// tensor copies (cp.async.bulk.tensor, 128-byte swizzle, no multicast) that
// complete on per-stage mbarriers; lane 0 issues, all lanes consume.  The
// grouped query rows (n_q * G <= 16) form the M=16 side of mma.sync m16n8k16:
// S = Q.K^T over the tile (2 n-tiles of 8 tokens), an fp32 online softmax in
// the exp2 domain, then O += P.V (D/8 n-tiles).  For bf16, P is split into
// hi + lo bf16 parts so P.V carries ~16 mantissa bits of P.
//
// Roofline: each tile moves 2 * 16 * D * 2 bytes (K and V) and needs
// 4 * rows * 16 * D flops; with rows = 4 (GQA group 4) that is 2 flop/byte,
// so the kernel is HBM-bound and the bulk-copy pipeline depth is what matters.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <mutex>

#include "common.cuh"

namespace mz {
namespace decode {

constexpr int kWarps = 4;
constexpr int kTileTok = 16;
constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s bound on any single wait

template <int D>
struct Cfg {
  static constexpr int kStages = (D == 64) ? 6 : 3;
  static constexpr int kTileBytes = kTileTok * D * 2;        // one of K or V
  static constexpr int kStageBytes = 2 * kTileBytes;         // K + V
  static constexpr int kSmemTiles = kWarps * kStages * kStageBytes;
  static constexpr int kSmemBytes = kSmemTiles + kWarps * kStages * 8 + 1024;  // + barriers + align
};

struct Params {
  void *out;
  int64_t o_sb, o_st, o_sh;
  int out_f32;
  const void *q;
  int64_t q_sb, q_st, q_sh;
  int n_q, G, rows;
  const int32_t *tables;
  int max_blocks;
  const int32_t *ctx;
  int B, Hkv;
  int bs, tpb;  // block size, tiles per block
  int64_t n_blocks;
  float scale_log2;
  int32_t *counters;  // [B * Hkv]
  float *ml;          // [slots][rows][2]
  float *part;        // [slots][rows][D]
  int32_t *err;
};

struct Cursor {
  int b, h, t, n, ctx;
  int64_t pos;
};

__device__ __forceinline__ int ntiles_of(int ctx) { return (ctx + kTileTok - 1) / kTileTok; }

__device__ __forceinline__ int clamped_ctx(const Params &p, int b) {
  int c = p.ctx[b];
  const int cap = p.max_blocks * p.bs;
  if (c < 0 || c > cap) {
    dev_error(p.err, MZ_DEVERR_CONTEXT);
    c = c < 0 ? 0 : cap;
  }
  return c;
}

__device__ __forceinline__ void advance(Cursor &c, const Params &p) {
  ++c.pos;
  if (++c.t == c.n) {
    c.t = 0;
    if (++c.h == p.Hkv) {
      c.h = 0;
      for (;;) {
        if (++c.b >= p.B) {
          c.n = 0;
          break;
        }
        c.ctx = clamped_ctx(p, c.b);
        c.n = ntiles_of(c.ctx);
        if (c.n > 0) break;
      }
    }
  }
}

// Address of output (or q) element row r of pair (b, h), dim 0.
__device__ __forceinline__ int64_t row_offset(int64_t sb, int64_t st, int64_t sh, int b, int h,
                                              int r, int G) {
  const int i = r / G, g = r - (r / G) * G;
  return (int64_t)b * sb + (int64_t)i * st + (int64_t)(h * G + g) * sh;
}

__device__ __forceinline__ void store_pair(const Params &p, int64_t off, float x, float y,
                                           bool bf16) {
  if (p.out_f32) {
    *reinterpret_cast<float2 *>(static_cast<float *>(p.out) + off) = make_float2(x, y);
  } else if (bf16) {
    *reinterpret_cast<__nv_bfloat162 *>(static_cast<__nv_bfloat16 *>(p.out) + off) =
        __floats2bfloat162_rn(x, y);
  } else {
    *reinterpret_cast<__half2 *>(static_cast<__half *>(p.out) + off) = __floats2half2_rn(x, y);
  }
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kWarps * 32, 2)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const Params p) {
  using C = Cfg<D>;
  constexpr int S = C::kStages;
  constexpr int KS = D / 16;  // k-steps of Q.K^T, also n-tile pairs of P.V
  constexpr int NT = D / 8;   // n-tiles of P.V

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int W = gridDim.x * kWarps;
  const int wid = blockIdx.x * kWarps + warp;

  uint8_t *stages = smem + warp * S * C::kStageBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kSmemTiles) + warp * S;
  const uint32_t bar0 = smem_u32(bars);
  const uint32_t stage0 = smem_u32(stages);

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(bar0 + 8 * s, 1);
    fence_mbar_init();
  }
  __syncwarp();

  // Sequences with no context produce zeros.
  for (int b = wid; b < p.B; b += W) {
    if (clamped_ctx(p, b) != 0) continue;
    for (int h = 0; h < p.Hkv; ++h)
      for (int r = 0; r < p.rows; ++r) {
        const int64_t o = row_offset(p.o_sb, p.o_st, p.o_sh, b, h, r, p.G);
        for (int d = 2 * lane; d < D; d += 64) store_pair(p, o + d, 0.f, 0.f, BF16);
      }
  }

  // Total tiles T and this warp's share.
  int64_t tot = 0;
  for (int b = lane; b < p.B; b += 32) tot += ntiles_of(clamped_ctx(p, b));
#pragma unroll
  for (int o = 16; o; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
  tot *= p.Hkv;
  if (tot == 0) return;
  const int64_t per = (tot + W - 1) / W;
  const int64_t p0 = (int64_t)wid * per;
  if (p0 >= tot) return;
  const int my_n = static_cast<int>(min(per, tot - p0));

  // Locate tile p0: find b with prefix(b) <= p0 < prefix(b+1), prefix in tiles*Hkv.
  Cursor start;
  {
    int64_t base = 0;
    int bf = 0;
    for (int b0 = 0; b0 < p.B; b0 += 32) {
      const int b = b0 + lane;
      const int64_t c = (b < p.B) ? (int64_t)ntiles_of(clamped_ctx(p, b)) * p.Hkv : 0;
      int64_t incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const unsigned m = __ballot_sync(0xffffffffu, base + incl > p0);
      if (m) {
        const int L = __ffs(m) - 1;
        base += __shfl_sync(0xffffffffu, incl - c, L);
        bf = b0 + L;
        break;
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    start.b = bf;
    start.ctx = clamped_ctx(p, bf);
    start.n = ntiles_of(start.ctx);
    const int64_t r = p0 - base;
    start.h = static_cast<int>(r / start.n);
    start.t = static_cast<int>(r - (int64_t)start.h * start.n);
    start.pos = p0;
  }

  const uint64_t pol = l2_policy_evict_first();
  auto issue = [&](int s, const Cursor &c) {
    if (lane == 0) {
      int32_t blk = p.tables[(int64_t)c.b * p.max_blocks + c.t / p.tpb];
      if (blk < 0 || blk >= p.n_blocks) {
        dev_error(p.err, MZ_DEVERR_BLOCK_ID);
        blk = 0;
      }
      const int y = static_cast<int>(((int64_t)blk * p.Hkv + c.h) * p.bs + (c.t % p.tpb) * kTileTok);
      const uint32_t bar = bar0 + 8 * s;
      const uint32_t dk = stage0 + s * C::kStageBytes;
      mbar_arrive_expect_tx(bar, C::kStageBytes);
#pragma unroll
      for (int c2 = 0; c2 < D / 64; ++c2) {
        tma_load_2d(dk + c2 * 2048, &tmK, c2 * 64, y, bar, pol);
        tma_load_2d(dk + C::kTileBytes + c2 * 2048, &tmV, c2 * 64, y, bar, pol);
      }
    }
  };

  // Per-lane ldmatrix geometry (see the swizzle note at smem_off).
  const int mi = lane >> 3, r8 = lane & 7;
  const int tokK = r8 + 8 * (mi >> 1), subK = mi & 1;  // K: m0,m1 tok 0-7; m2,m3 tok 8-15
  const int tokV = r8 + 8 * (mi & 1), subV = mi >> 1;  // V: m0,m2 tok 0-7; m1,m3 tok 8-15
  // 128-byte swizzle of a [16 tok][64 dim] 2-KiB box: 16-byte unit u of line
  // `tok` lives at unit u ^ (tok & 7).  D = 128 uses two boxes (dims 0-63, 64-127).
  auto smem_off = [](int tok, int d) -> uint32_t {
    const int box = d >> 6, u = (d & 63) >> 3;
    return box * 2048 + tok * 128 + ((u ^ (tok & 7)) << 4);
  };

  const int g = lane >> 2, cq = lane & 3;  // mma fragment row / column-pair

  Cursor pc = start, cc = start;
  int issued = 0;
  {
    const int pro = my_n < S ? my_n : S;
    for (; issued < pro; ++issued) {
      issue(issued, pc);
      advance(pc, p);
    }
  }

  uint32_t qa[KS][4];
  float oacc[NT][4];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  int seg_t0 = 0;
  const bool two_groups = p.rows > 8;

  for (int i = 0; i < my_n; ++i) {
    const int s = i % S;
    const uint32_t ph = (i / S) & 1;

    if (i == 0 || cc.t == 0) {
      // New (b, h) segment: load the grouped query rows as A fragments.
      seg_t0 = cc.t;
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
#pragma unroll
      for (int n = 0; n < NT; ++n) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.f;
      const auto *q16 = static_cast<const uint16_t *>(p.q);
      const int64_t qo0 = (g < p.rows) ? row_offset(p.q_sb, p.q_st, p.q_sh, cc.b, cc.h, g, p.G) : -1;
      const int64_t qo1 =
          (g + 8 < p.rows) ? row_offset(p.q_sb, p.q_st, p.q_sh, cc.b, cc.h, g + 8, p.G) : -1;
#pragma unroll
      for (int j = 0; j < KS; ++j) {
        const int d = 16 * j + 2 * cq;
        qa[j][0] = qo0 >= 0 ? *reinterpret_cast<const uint32_t *>(q16 + qo0 + d) : 0u;
        qa[j][1] = qo1 >= 0 ? *reinterpret_cast<const uint32_t *>(q16 + qo1 + d) : 0u;
        qa[j][2] = qo0 >= 0 ? *reinterpret_cast<const uint32_t *>(q16 + qo0 + d + 8) : 0u;
        qa[j][3] = qo1 >= 0 ? *reinterpret_cast<const uint32_t *>(q16 + qo1 + d + 8) : 0u;
      }
    }

    if (!mbar_wait_bounded(bar0 + 8 * s, ph, kTimeoutNs)) {
      // Give up: record it, let this warp's copies in flight land (bounded), return.
      if (lane == 0) dev_error(p.err, MZ_DEVERR_TIMEOUT);
      for (int k = i; k < issued; ++k)
        (void)mbar_wait_bounded(bar0 + 8 * (k % S), (k / S) & 1, kTimeoutNs);
      return;
    }

    const uint32_t kb = stage0 + s * C::kStageBytes;
    const uint32_t vb = kb + C::kTileBytes;
    const int nvalid = min(kTileTok, cc.ctx - cc.t * kTileTok);
    if (nvalid < kTileTok) {
      // Rows past the context may hold stale data; make them exact zeros so
      // that 0 * V stays 0 in P.V.
      uint8_t *vt = stages + s * C::kStageBytes + C::kTileBytes;
      for (int e = lane; e < (kTileTok - nvalid) * (D / 8); e += 32) {
        const int tok = nvalid + e / (D / 8), d = (e % (D / 8)) * 8;
        *reinterpret_cast<uint4 *>(vt + smem_off(tok, d)) = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }

    // S = Q . K^T : rows x 16 tokens.
    float sacc[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.f;
#pragma unroll
    for (int j = 0; j < KS; ++j) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(kb + smem_off(tokK, 16 * j + 8 * subK), b0, b1, b2, b3);
      mma_16816<BF16>(sacc[0], qa[j], b0, b1);
      mma_16816<BF16>(sacc[1], qa[j], b2, b3);
    }

    // Online softmax (exp2 domain), rows g (regs 0,1) and g+8 (regs 2,3).
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = n * 8 + 2 * cq + (e & 1);
        float x = sacc[n][e] * p.scale_log2;
        if (tok >= nvalid) x = -INFINITY;
        sacc[n][e] = x;
        if (e < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    const float mn0 = fmaxf(m0, mx0);
    const float a0 = fast_exp2(m0 - mn0);
    m0 = mn0;
    float a1 = 1.f;
    if (two_groups) {
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn1 = fmaxf(m1, mx1);
      a1 = fast_exp2(m1 - mn1);
      m1 = mn1;
    }
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      sacc[n][0] = fast_exp2(sacc[n][0] - m0);
      sacc[n][1] = fast_exp2(sacc[n][1] - m0);
      rs0 += sacc[n][0] + sacc[n][1];
      if (two_groups) {
        sacc[n][2] = fast_exp2(sacc[n][2] - m1);
        sacc[n][3] = fast_exp2(sacc[n][3] - m1);
        rs1 += sacc[n][2] + sacc[n][3];
      } else {
        sacc[n][2] = sacc[n][3] = 0.f;
      }
    }
    l0 = l0 * a0 + rs0;
    l1 = l1 * a1 + rs1;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      oacc[n][0] *= a0;
      oacc[n][1] *= a0;
      oacc[n][2] *= a1;
      oacc[n][3] *= a1;
    }

    // P as A fragments (hi, and lo for bf16).
    uint32_t ph_[4], pl_[4];
    {
      float hi[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) hi[n][e] = round16<BF16>(sacc[n][e]);
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

    // O += P . V
#pragma unroll
    for (int j = 0; j < KS; ++j) {
      uint32_t v0, v1, v2, v3;
      ldsm_x4_trans(vb + smem_off(tokV, 16 * j + 8 * subV), v0, v1, v2, v3);
      mma_16816<BF16>(oacc[2 * j], ph_, v0, v1);
      mma_16816<BF16>(oacc[2 * j + 1], ph_, v2, v3);
      if constexpr (BF16) {
        mma_16816<BF16>(oacc[2 * j], pl_, v0, v1);
        mma_16816<BF16>(oacc[2 * j + 1], pl_, v2, v3);
      }
    }

    // Segment end: last tile of the pair, or last tile of this warp's share.
    if (cc.t == cc.n - 1 || i == my_n - 1) {
      float L0 = l0, L1 = l1;
      L0 += __shfl_xor_sync(0xffffffffu, L0, 1);
      L0 += __shfl_xor_sync(0xffffffffu, L0, 2);
      L1 += __shfl_xor_sync(0xffffffffu, L1, 1);
      L1 += __shfl_xor_sync(0xffffffffu, L1, 2);
      const int bh = cc.b * p.Hkv + cc.h;
      if (seg_t0 == 0 && cc.t == cc.n - 1) {
        const float i0 = 1.f / L0, i1 = two_groups ? 1.f / L1 : 0.f;
        if (g < p.rows) {
          const int64_t o = row_offset(p.o_sb, p.o_st, p.o_sh, cc.b, cc.h, g, p.G);
#pragma unroll
          for (int n = 0; n < NT; ++n)
            store_pair(p, o + n * 8 + 2 * cq, oacc[n][0] * i0, oacc[n][1] * i0, BF16);
        }
        if (g + 8 < p.rows) {
          const int64_t o = row_offset(p.o_sb, p.o_st, p.o_sh, cc.b, cc.h, g + 8, p.G);
#pragma unroll
          for (int n = 0; n < NT; ++n)
            store_pair(p, o + n * 8 + 2 * cq, oacc[n][2] * i1, oacc[n][3] * i1, BF16);
        }
      } else {
        const int64_t slot = (int64_t)wid + bh;
        float *pr = p.part + slot * p.rows * D;
        float *mlr = p.ml + slot * p.rows * 2;
        if (g < p.rows) {
#pragma unroll
          for (int n = 0; n < NT; ++n)
            *reinterpret_cast<float2 *>(pr + g * D + n * 8 + 2 * cq) =
                make_float2(oacc[n][0], oacc[n][1]);
          if (cq == 0) *reinterpret_cast<float2 *>(mlr + 2 * g) = make_float2(m0, L0);
        }
        if (g + 8 < p.rows) {
#pragma unroll
          for (int n = 0; n < NT; ++n)
            *reinterpret_cast<float2 *>(pr + (g + 8) * D + n * 8 + 2 * cq) =
                make_float2(oacc[n][2], oacc[n][3]);
          if (cq == 0) *reinterpret_cast<float2 *>(mlr + 2 * (g + 8)) = make_float2(m1, L1);
        }
        __threadfence();
        __syncwarp();
        int old = 0;
        if (lane == 0) old = atomicAdd(p.counters + bh, 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        const int64_t pbh = cc.pos - cc.t;  // flat index of tile 0 of this pair
        const int64_t wf = pbh / per, wl = (pbh + cc.n - 1) / per;
        const int nparts = static_cast<int>(wl - wf + 1);
        if (old == nparts - 1) {
          // Last piece: merge every piece's (m, l, O) and write the output.
          __threadfence();
          const int E = p.rows * D;
          for (int e = 4 * lane; e < E; e += 128) {
            const int r = e / D, d = e - (e / D) * D;
            float M = -INFINITY, Ls = 0.f;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int k = 0; k < nparts; ++k) {
              const int64_t sl = wf + k + bh;
              const float2 mlk = __ldcg(reinterpret_cast<const float2 *>(p.ml + (sl * p.rows + r) * 2));
              const float4 ok = __ldcg(reinterpret_cast<const float4 *>(p.part + (sl * p.rows + r) * D + d));
              const float Mn = fmaxf(M, mlk.x);
              const float sa = fast_exp2(M - Mn), sb = fast_exp2(mlk.x - Mn);
              Ls = Ls * sa + mlk.y * sb;
              acc.x = acc.x * sa + ok.x * sb;
              acc.y = acc.y * sa + ok.y * sb;
              acc.z = acc.z * sa + ok.z * sb;
              acc.w = acc.w * sa + ok.w * sb;
              M = Mn;
            }
            const float inv = 1.f / Ls;
            const int64_t o = row_offset(p.o_sb, p.o_st, p.o_sh, cc.b, cc.h, r, p.G) + d;
            store_pair(p, o, acc.x * inv, acc.y * inv, BF16);
            store_pair(p, o + 2, acc.z * inv, acc.w * inv, BF16);
          }
          if (lane == 0) p.counters[bh] = 0;
        }
      }
    }

    __syncwarp();
    if (issued < my_n) {
      if (lane == 0) fence_proxy_async_smem();
      issue(s, pc);
      advance(pc, p);
      ++issued;
    }
    advance(cc, p);
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Tensor map over a pool seen as rows of `D` 16-bit elements, box 64 x 16.
int make_pool_map(CUtensorMap *m, const void *pool, int64_t rows, int D, bool bf16) {
  auto fn = encode_fn();
  if (!fn) return fail(MZ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(D) * 2};
  cuuint32_t box[2] = {64, kTileTok};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void *>(pool), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MZ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MZ_OK;
}

template <int D, bool BF16>
int kernel_ctas_per_sm(int *out) {
  static int cached = -1;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, []() {
    auto k = paged_decode_kernel<D, BF16>;
    err = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<D>::kSmemBytes);
    if (err != cudaSuccess) return;
    int n = 0;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kWarps * 32, Cfg<D>::kSmemBytes);
    cached = n;
  });
  if (err != cudaSuccess) return cuda_fail(err, "paged_decode: occupancy query");
  *out = cached;
  return MZ_OK;
}

int ctas_per_sm(int D, bool bf16, int *out) {
  if (D == 128) return bf16 ? kernel_ctas_per_sm<128, true>(out) : kernel_ctas_per_sm<128, false>(out);
  return bf16 ? kernel_ctas_per_sm<64, true>(out) : kernel_ctas_per_sm<64, false>(out);
}

struct WsLayout {
  size_t counters, ml, part, total;
};

inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

WsLayout ws_layout(int64_t n_pairs, int64_t warps, int rows, int D) {
  WsLayout w;
  const int64_t slots = warps + n_pairs;
  w.counters = 0;
  w.ml = align256(n_pairs * sizeof(int32_t));
  w.part = w.ml + align256(slots * rows * 2 * sizeof(float));
  w.total = w.part + align256(slots * rows * D * sizeof(float));
  return w;
}

int resolve_warps(int D, bool bf16, int num_warps, int device, int64_t *warps) {
  if (num_warps < 0) return fail(MZ_ERR_INVALID_ARG, "num_warps < 0");
  if (num_warps > 0) {
    *warps = (num_warps + kWarps - 1) / kWarps * kWarps;
    return MZ_OK;
  }
  // The workspace is sized from this count, so use the larger occupancy of
  // the two element types: then one size fits both.
  int per_sm = 0, per_sm_other = 0;
  if (int rc = ctas_per_sm(D, bf16, &per_sm)) return rc;
  if (int rc = ctas_per_sm(D, !bf16, &per_sm_other)) return rc;
  if (per_sm_other > per_sm) per_sm = per_sm_other;
  if (per_sm < 1) return fail(MZ_ERR_CUDA, "paged_decode kernel cannot be resident on an SM");
  const int sms = sm_count(device);
  if (sms <= 0) return fail(MZ_ERR_CUDA, "cannot query SM count of device %d", device);
  *warps = (int64_t)sms * per_sm * kWarps;
  return MZ_OK;
}

}  // namespace decode
}  // namespace mz

using namespace mz;
using namespace mz::decode;

extern "C" int mz_paged_decode_workspace_size(int32_t n_seqs, int32_t n_kv_heads,
                                              int32_t rows_per_kv_head, int32_t head_dim,
                                              int32_t num_warps, int32_t device, size_t *bytes) {
  if (!bytes) return fail(MZ_ERR_INVALID_ARG, "bytes is null");
  if (n_seqs < 0 || n_kv_heads <= 0 || rows_per_kv_head <= 0 || rows_per_kv_head > 16)
    return fail(MZ_ERR_INVALID_ARG, "workspace_size: bad sizes");
  if (head_dim != 64 && head_dim != 128)
    return fail(MZ_ERR_UNSUPPORTED, "head_dim %d (supported: 64, 128)", head_dim);
  int64_t warps = 0;
  if (device < 0) device = current_device();
  // Occupancy is the same for bf16 and fp16 instantiations.
  if (int rc = resolve_warps(head_dim, true, num_warps, device, &warps)) return rc;
  *bytes = ws_layout((int64_t)n_seqs * n_kv_heads, warps, rows_per_kv_head, head_dim).total;
  return MZ_OK;
}

extern "C" int mz_paged_decode(void *out, int32_t out_dtype, int64_t out_seq_stride,
                               int64_t out_tok_stride, int64_t out_head_stride, const void *q,
                               int64_t q_seq_stride, int64_t q_tok_stride, int64_t q_head_stride,
                               int32_t n_q_tokens, const void *k_pool, const void *v_pool,
                               const int32_t *block_tables, int32_t max_blocks_per_seq,
                               const int32_t *ctx_lens, int32_t n_seqs, int32_t n_heads,
                               int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
                               int64_t n_blocks, float scale, int32_t dtype, int32_t num_warps,
                               void *workspace, size_t workspace_bytes, int32_t *dev_err,
                               mz_stream_t stream) {
  if (dtype != MZ_DTYPE_F16 && dtype != MZ_DTYPE_BF16)
    return fail(MZ_ERR_UNSUPPORTED, "mz_paged_decode: dtype must be F16 or BF16");
  if (out_dtype != dtype && out_dtype != MZ_DTYPE_F32)
    return fail(MZ_ERR_UNSUPPORTED, "mz_paged_decode: out_dtype must equal dtype or be F32");
  if (head_dim != 64 && head_dim != 128)
    return fail(MZ_ERR_UNSUPPORTED, "mz_paged_decode: head_dim %d (supported: 64, 128)", head_dim);
  if (block_size <= 0 || block_size % kTileTok)
    return fail(MZ_ERR_UNSUPPORTED, "mz_paged_decode: block_size %d is not a multiple of 16",
                block_size);
  if (n_seqs < 0 || n_kv_heads <= 0 || n_heads <= 0 || n_heads % n_kv_heads || n_q_tokens <= 0 ||
      max_blocks_per_seq <= 0 || n_blocks <= 0)
    return fail(MZ_ERR_INVALID_ARG, "mz_paged_decode: bad sizes");
  const int G = n_heads / n_kv_heads;
  const int rows = n_q_tokens * G;
  if (rows > 16)
    return fail(MZ_ERR_UNSUPPORTED,
                "mz_paged_decode: n_q_tokens * (n_heads / n_kv_heads) = %d exceeds 16", rows);
  if (!std::isfinite(scale)) return fail(MZ_ERR_INVALID_ARG, "mz_paged_decode: scale not finite");
  if (n_seqs == 0) return MZ_OK;
  if (!out || !q || !k_pool || !v_pool || !block_tables || !ctx_lens || !workspace)
    return fail(workspace ? MZ_ERR_INVALID_ARG : MZ_ERR_WORKSPACE, "mz_paged_decode: null pointer");
  if (!aligned(k_pool, 16) || !aligned(v_pool, 16) || !aligned(q, 4) || (q_seq_stride & 1) ||
      (q_tok_stride & 1) || (q_head_stride & 1))
    return fail(MZ_ERR_ALIGNMENT,
                "mz_paged_decode: pools need 16-byte alignment, q 4-byte alignment and even strides");
  const int ob = out_dtype == MZ_DTYPE_F32 ? 8 : 4;
  if (!aligned(out, ob) || (out_seq_stride & 1) || (out_tok_stride & 1) || (out_head_stride & 1))
    return fail(MZ_ERR_ALIGNMENT, "mz_paged_decode: out needs %d-byte alignment and even strides",
                ob);
  const int64_t rows_total = n_blocks * n_kv_heads * block_size;
  if (rows_total >= (int64_t(1) << 31))
    return fail(MZ_ERR_UNSUPPORTED, "mz_paged_decode: pool has >= 2^31 rows");
  const bool bf16 = dtype == MZ_DTYPE_BF16;
  const int device = current_device();
  int64_t warps = 0;
  if (int rc = resolve_warps(head_dim, bf16, num_warps, device, &warps)) return rc;
  const WsLayout ws = ws_layout((int64_t)n_seqs * n_kv_heads, warps, rows, head_dim);
  if (workspace_bytes < ws.total)
    return fail(MZ_ERR_WORKSPACE, "mz_paged_decode: workspace %zu bytes < required %zu",
                workspace_bytes, ws.total);
  if (!aligned(workspace, 256)) return fail(MZ_ERR_ALIGNMENT, "workspace must be 256-byte aligned");

  CUtensorMap tk, tv;
  if (int rc = make_pool_map(&tk, k_pool, rows_total, head_dim, bf16)) return rc;
  if (int rc = make_pool_map(&tv, v_pool, rows_total, head_dim, bf16)) return rc;

  Params p;
  p.out = out;
  p.o_sb = out_seq_stride;
  p.o_st = out_tok_stride;
  p.o_sh = out_head_stride;
  p.out_f32 = out_dtype == MZ_DTYPE_F32;
  p.q = q;
  p.q_sb = q_seq_stride;
  p.q_st = q_tok_stride;
  p.q_sh = q_head_stride;
  p.n_q = n_q_tokens;
  p.G = G;
  p.rows = rows;
  p.tables = block_tables;
  p.max_blocks = max_blocks_per_seq;
  p.ctx = ctx_lens;
  p.B = n_seqs;
  p.Hkv = n_kv_heads;
  p.bs = block_size;
  p.tpb = block_size / kTileTok;
  p.n_blocks = n_blocks;
  p.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
  auto *w8 = static_cast<uint8_t *>(workspace);
  p.counters = reinterpret_cast<int32_t *>(w8 + ws.counters);
  p.ml = reinterpret_cast<float *>(w8 + ws.ml);
  p.part = reinterpret_cast<float *>(w8 + ws.part);
  p.err = dev_err;

  // Make sure the instantiation's smem attribute is set (cached per kernel).
  int per_sm = 0;
  if (int rc = ctas_per_sm(head_dim, bf16, &per_sm)) return rc;
  const unsigned grid = static_cast<unsigned>(warps / kWarps);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define MZ_LAUNCH(D_, BF_)                                                               \
  paged_decode_kernel<D_, BF_><<<grid, kWarps * 32, Cfg<D_>::kSmemBytes, s>>>(tk, tv, p)
  if (head_dim == 128) {
    if (bf16) MZ_LAUNCH(128, true); else MZ_LAUNCH(128, false);
  } else {
    if (bf16) MZ_LAUNCH(64, true); else MZ_LAUNCH(64, false);
  }
#undef MZ_LAUNCH
  MZ_CHECK_LAUNCH("mz_paged_decode");
  return MZ_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant: the same kernel, with its scratch (split-piece
// partials and per-pair arrival counters) in a fixed array built into the
// library instead of a caller-supplied workspace.  For callers that cannot
// allocate device memory when they call in: a host whose own pool already
// owns the GPU's memory, an FFI binding with no device allocator of its own,
// or a latency-bound path where cudaMalloc's implicit device synchronisation
// is not allowed.  The array is loaded with the library's device code, so
// every GPU that runs this code holds it until the process exits.
// ---------------------------------------------------------------------------
namespace mz {
namespace decode {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;  // 16 MiB per device
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

struct StaticScratchSlot {
  std::once_flag once;
  void *ptr = nullptr;
  cudaError_t err = cudaSuccess;
};
constexpr int kMaxStaticDevices = 64;
StaticScratchSlot g_static_slots[kMaxStaticDevices];

// Device address of g_static_scratch on `device`, which must be the current
// device.  Host code cannot use the symbol's name as a device pointer, so the
// address is looked up once per device with cudaGetSymbolAddress.
int static_scratch_ptr(int device, void **ptr) {
  if (device < 0 || device >= kMaxStaticDevices)
    return fail(MZ_ERR_CUDA, "no usable current device (%d)", device);
  StaticScratchSlot &s = g_static_slots[device];
  std::call_once(s.once, [&s]() { s.err = cudaGetSymbolAddress(&s.ptr, g_static_scratch); });
  if (s.err != cudaSuccess) return cuda_fail(s.err, "cudaGetSymbolAddress(decode scratch)");
  if (!s.ptr) return fail(MZ_ERR_CUDA, "decode scratch has no device address");
  *ptr = s.ptr;
  return MZ_OK;
}

}  // namespace decode
}  // namespace mz

extern "C" int mz_paged_decode_noalloc(void *out, int32_t out_dtype, int64_t out_seq_stride,
                                       int64_t out_tok_stride, int64_t out_head_stride,
                                       const void *q, int64_t q_seq_stride, int64_t q_tok_stride,
                                       int64_t q_head_stride, int32_t n_q_tokens,
                                       const void *k_pool, const void *v_pool,
                                       const int32_t *block_tables, int32_t max_blocks_per_seq,
                                       const int32_t *ctx_lens, int32_t n_seqs, int32_t n_heads,
                                       int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
                                       int64_t n_blocks, float scale, int32_t dtype,
                                       int32_t num_warps, int32_t *dev_err, mz_stream_t stream) {
  if (dtype != MZ_DTYPE_F16 && dtype != MZ_DTYPE_BF16)
    return fail(MZ_ERR_UNSUPPORTED, "mz_paged_decode_noalloc: dtype must be F16 or BF16");
  if (out_dtype != dtype && out_dtype != MZ_DTYPE_F32)
    return fail(MZ_ERR_UNSUPPORTED, "mz_paged_decode_noalloc: out_dtype must equal dtype or be F32");
  if (head_dim != 64 && head_dim != 128)
    return fail(MZ_ERR_UNSUPPORTED, "mz_paged_decode_noalloc: head_dim %d (supported: 64, 128)",
                head_dim);
  if (block_size <= 0 || block_size % kTileTok)
    return fail(MZ_ERR_UNSUPPORTED,
                "mz_paged_decode_noalloc: block_size %d is not a multiple of 16", block_size);
  if (n_seqs < 0 || n_kv_heads <= 0 || n_heads <= 0 || n_heads % n_kv_heads || n_q_tokens <= 0 ||
      max_blocks_per_seq <= 0 || n_blocks <= 0)
    return fail(MZ_ERR_INVALID_ARG, "mz_paged_decode_noalloc: bad sizes");
  const int G = n_heads / n_kv_heads;
  const int rows = n_q_tokens * G;
  if (rows > 16)
    return fail(MZ_ERR_UNSUPPORTED,
                "mz_paged_decode_noalloc: n_q_tokens * (n_heads / n_kv_heads) = %d exceeds 16", rows);
  if (!std::isfinite(scale))
    return fail(MZ_ERR_INVALID_ARG, "mz_paged_decode_noalloc: scale not finite");
  if (n_seqs == 0) return MZ_OK;
  if (!out || !q || !k_pool || !v_pool || !block_tables || !ctx_lens)
    return fail(MZ_ERR_INVALID_ARG, "mz_paged_decode_noalloc: null pointer");
  if (!aligned(k_pool, 16) || !aligned(v_pool, 16) || !aligned(q, 4) || (q_seq_stride & 1) ||
      (q_tok_stride & 1) || (q_head_stride & 1))
    return fail(MZ_ERR_ALIGNMENT,
                "mz_paged_decode_noalloc: pools need 16-byte alignment, q 4-byte alignment and "
                "even strides");
  const int ob = out_dtype == MZ_DTYPE_F32 ? 8 : 4;
  if (!aligned(out, ob) || (out_seq_stride & 1) || (out_tok_stride & 1) || (out_head_stride & 1))
    return fail(MZ_ERR_ALIGNMENT,
                "mz_paged_decode_noalloc: out needs %d-byte alignment and even strides", ob);
  const int64_t rows_total = n_blocks * n_kv_heads * block_size;
  if (rows_total >= (int64_t(1) << 31))
    return fail(MZ_ERR_UNSUPPORTED, "mz_paged_decode_noalloc: pool has >= 2^31 rows");
  const bool bf16 = dtype == MZ_DTYPE_BF16;
  const int device = current_device();
  int64_t warps = 0;
  if (int rc = resolve_warps(head_dim, bf16, num_warps, device, &warps)) return rc;
  const int64_t n_pairs = (int64_t)n_seqs * n_kv_heads;
  const WsLayout ws = ws_layout(n_pairs, warps, rows, head_dim);
  if (ws.total > kStaticScratchBytes)
    return fail(MZ_ERR_TOO_LARGE,
                "mz_paged_decode_noalloc: these sizes need %zu bytes of scratch but the built-in "
                "area holds %zu; lower n_seqs * n_kv_heads, rows or num_warps, or call "
                "mz_paged_decode with a workspace",
                ws.total, kStaticScratchBytes);
  void *scratch = nullptr;
  if (int rc = static_scratch_ptr(device, &scratch)) return rc;

  CUtensorMap tk, tv;
  if (int rc = make_pool_map(&tk, k_pool, rows_total, head_dim, bf16)) return rc;
  if (int rc = make_pool_map(&tv, v_pool, rows_total, head_dim, bf16)) return rc;

  Params p;
  p.out = out;
  p.o_sb = out_seq_stride;
  p.o_st = out_tok_stride;
  p.o_sh = out_head_stride;
  p.out_f32 = out_dtype == MZ_DTYPE_F32;
  p.q = q;
  p.q_sb = q_seq_stride;
  p.q_st = q_tok_stride;
  p.q_sh = q_head_stride;
  p.n_q = n_q_tokens;
  p.G = G;
  p.rows = rows;
  p.tables = block_tables;
  p.max_blocks = max_blocks_per_seq;
  p.ctx = ctx_lens;
  p.B = n_seqs;
  p.Hkv = n_kv_heads;
  p.bs = block_size;
  p.tpb = block_size / kTileTok;
  p.n_blocks = n_blocks;
  p.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
  auto *w8 = static_cast<uint8_t *>(scratch);
  p.counters = reinterpret_cast<int32_t *>(w8 + ws.counters);
  p.ml = reinterpret_cast<float *>(w8 + ws.ml);
  p.part = reinterpret_cast<float *>(w8 + ws.part);
  p.err = dev_err;

  int per_sm = 0;
  if (int rc = ctas_per_sm(head_dim, bf16, &per_sm)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The area keeps whatever the previous call left; the arrival counters
  // must start at zero, so clear them on this stream first.
  cudaError_t e = cudaMemsetAsync(p.counters, 0, n_pairs * sizeof(int32_t), s);
  if (e != cudaSuccess) return cuda_fail(e, "mz_paged_decode_noalloc: clearing counters");
  const unsigned grid = static_cast<unsigned>(warps / kWarps);
#define MZ_LAUNCH(D_, BF_)                                                               \
  paged_decode_kernel<D_, BF_><<<grid, kWarps * 32, Cfg<D_>::kSmemBytes, s>>>(tk, tv, p)
  if (head_dim == 128) {
    if (bf16) MZ_LAUNCH(128, true); else MZ_LAUNCH(128, false);
  } else {
    if (bf16) MZ_LAUNCH(64, true); else MZ_LAUNCH(64, false);
  }
#undef MZ_LAUNCH
  MZ_CHECK_LAUNCH("mz_paged_decode_noalloc");
  return MZ_OK;
}
