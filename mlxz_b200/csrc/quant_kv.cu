// 4/8-bit affine group quantised KV: quantise-on-append and dequant-fused
// paged decode attention (sm_100a).
//
// Format (per layer, per K and V), the paged form of mlx_lm's quantised cache
// state ((data, scales, biases), src/mlxz/prefix_cache/base.py:18):
//   codes  [n_blocks][H][bs][D * bits / 32] uint32, element i of a row at word
//          i / (32 / bits), bits (i % (32 / bits)) * bits up (LSB first);
//   scales [n_blocks][H][bs][D / 64] fp16, biases likewise (group size 64).
// Quantisation of one 64-value group, all in IEEE fp32 round-to-nearest-even:
//   scale = (max - min) / (2^bits - 1); s16 = fp16(scale); b16 = fp16(min);
//   q = clamp(rint((w - b16) / s16), 0, 2^bits - 1), q = 0 when s16 == 0;
//   dequantised w' = s16 * q + b16.
//
// Decode never materialises dequantised K/V.  The integer codes 0..255 are
// exact in fp16, so they enter mma.sync directly, and the affine map is applied
// around the products:
//   S[r][t] = sum_g s_k[t][g] * (Q_g . q_k[t]_g) + b_k[t][g] * sum(Q_g[r])
//   O[r][d] = sum_t (p[r][t] * s_v[t][g(d)]) * q_v[t][d] + sum_t p[r][t] * b_v[t][g(d)]
// with Q converted to fp16 once per piece.  The dot products run over a
// permutation of the head dimension chosen so that each lane's codes are
// contiguous bytes (Q is loaded with the same permutation; V's output columns
// are un-permuted when written).  Tiles arrive by 1-D bulk copies (codes,
// scales and biases of K and V: six copies per 16-token tile) into a per-warp
// ring, with the same persistent-warp scheduler as the bf16 kernel.
//
// Roofline: a tile moves 2 * 16 * (D * bits / 8 + 4 * D / 64) bytes; with
// D = 128 that is 4352 B (8-bit) or 2304 B (4-bit), against 8192 B at bf16.
#include "decode_common.cuh"

namespace mz {
namespace decode {

// ---------------------------------------------------------------------------
// Quantise-on-append.
// ---------------------------------------------------------------------------

struct QAppendParams {
  uint32_t *kq, *vq;
  __half *ks, *kb, *vs, *vb;
  const uint16_t *kn, *vn;
  int64_t n_tok_stride, n_head_stride;  // elements
  int qbf16;
  // slot source: slots != nullptr, else tables + positions
  const int64_t *slots;
  const int32_t *tables;
  int max_blocks;
  const int32_t *positions;
  int64_t n_tokens;
  int H, bs;
  int64_t n_blocks;
  int32_t *err;
};

// One warp per (token, head, K or V) row of D values; lane l holds elements
// [l * E, (l + 1) * E), E = D / 32; a 64-value group is 64 / E lanes.
template <int D, int BITS>
__global__ void __launch_bounds__(256) quant_append_kernel(const QAppendParams p) {
  constexpr int E = D / 32;
  constexpr int LG = 64 / E;           // lanes per group
  constexpr int NG = D / 64;
  constexpr int W32 = D * BITS / 32;   // words per row
  constexpr int LBITS = E * BITS;      // bits per lane
  constexpr int LW = 32 / LBITS;       // lanes per word (1, 2 or 4)
  constexpr float NB = float((1 << BITS) - 1);
  const int lane = threadIdx.x & 31;
  const int64_t wglobal = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t total = p.n_tokens * p.H * 2;
  if (wglobal >= total) return;
  const int kv = static_cast<int>(wglobal & 1);
  const int64_t r = wglobal >> 1;
  const int h = static_cast<int>(r % p.H);
  const int64_t i = r / p.H;

  int64_t slot;
  if (p.slots) {
    slot = p.slots[i];
    if (slot < 0) return;
    if (slot >= p.n_blocks * p.bs) {
      if (lane == 0 && h == 0 && kv == 0) dev_error(p.err, MZ_DEVERR_SLOT);
      return;
    }
  } else {
    const int pos = p.positions[i];
    if (pos < 0) return;
    if (pos >= p.max_blocks * p.bs) {
      if (lane == 0 && h == 0 && kv == 0) dev_error(p.err, MZ_DEVERR_CONTEXT);
      return;
    }
    const int32_t blk = p.tables[i * p.max_blocks + pos / p.bs];
    if (blk < 0 || blk >= p.n_blocks) {
      if (lane == 0 && h == 0 && kv == 0) dev_error(p.err, MZ_DEVERR_BLOCK_ID);
      return;
    }
    slot = (int64_t)blk * p.bs + pos % p.bs;
  }
  const int64_t row = ((slot / p.bs) * p.H + h) * p.bs + slot % p.bs;

  const uint16_t *src = (kv ? p.vn : p.kn) + i * p.n_tok_stride + (int64_t)h * p.n_head_stride +
                        lane * E;
  float x[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const uint16_t b = src[e];
    x[e] = p.qbf16 ? __uint_as_float(static_cast<uint32_t>(b) << 16)
                   : __half2float(__ushort_as_half(b));
  }
  float mn = x[0], mx = x[0];
#pragma unroll
  for (int e = 1; e < E; ++e) {
    mn = fminf(mn, x[e]);
    mx = fmaxf(mx, x[e]);
  }
#pragma unroll
  for (int o = LG / 2; o; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const __half s16 = __float2half_rn(__fdiv_rn(__fsub_rn(mx, mn), NB));
  const __half b16 = __float2half_rn(mn);
  const float sf = __half2float(s16), bf = __half2float(b16);
  uint32_t bitsv = 0;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    float qf = 0.f;
    if (sf != 0.f) qf = fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(x[e], bf), sf)), 0.f), NB);
    bitsv |= static_cast<uint32_t>(qf) << (BITS * e);
  }
  uint32_t word = bitsv << (LBITS * (lane % LW));
#pragma unroll
  for (int o = 1; o < LW; o <<= 1) word |= __shfl_xor_sync(0xffffffffu, word, o);
  uint32_t *qrow = (kv ? p.vq : p.kq) + row * W32;
  if (lane % LW == 0) qrow[lane / LW] = word;
  if (lane % LG == 0) {
    const int g = lane / LG;
    (kv ? p.vs : p.ks)[row * NG + g] = s16;
    (kv ? p.vb : p.kb)[row * NG + g] = b16;
  }
}

int quant_append(const QAppendParams &qp, int D, int bits, cudaStream_t s) {
  const int64_t warps = qp.n_tokens * qp.H * 2;
  if (warps == 0) return MZ_OK;
  const int64_t threads = warps * 32;
  const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
#define MZ_QA(D_, B_) quant_append_kernel<D_, B_><<<grid, 256, 0, s>>>(qp)
  if (D == 128) {
    if (bits == 8) MZ_QA(128, 8); else MZ_QA(128, 4);
  } else {
    if (bits == 8) MZ_QA(64, 8); else MZ_QA(64, 4);
  }
#undef MZ_QA
  MZ_CHECK_LAUNCH("mz_kv_quant_append");
  return MZ_OK;
}

// ---------------------------------------------------------------------------
// Dequant-fused paged decode.
// ---------------------------------------------------------------------------

template <int D, int BITS>
struct QCfg {
  static constexpr int RB = D * BITS / 8;   // code bytes per token row
  static constexpr int NG = D / 64;         // groups per row
  static constexpr int TD = kTileTok * RB;  // code bytes per tile (K or V)
  static constexpr int TS = kTileTok * NG * 2;  // scale (or bias) bytes per tile
  static constexpr int kTx = 2 * TD + 4 * TS;
  static constexpr int kStageBytes = (kTx + 127) / 128 * 128;
  static constexpr int kStagesFit = (96 * 1024) / (kWarps * kStageBytes);
  static constexpr int kStages = kStagesFit > 8 ? 8 : (kStagesFit < 3 ? 3 : kStagesFit);
  static constexpr int kSmemTiles = kWarps * kStages * kStageBytes;
  static constexpr int kSmemBars = kWarps * kStages * 8;
  static constexpr int kSmemUnits = kWarps * kUnitQ * 32;
  static constexpr int kSmemBytes = kSmemTiles + kSmemBars + kSmemUnits + 128;
  // P' = p * s_v is stored in fp16 scaled by this power of two (keeps small
  // weights out of fp16 subnormals; removed exactly at the end).
  static constexpr float kPScale = BITS == 8 ? 256.f : 16.f;
};

__device__ __forceinline__ uint32_t h2_sub1024(uint32_t x) {
  __half2 h = *reinterpret_cast<__half2 *>(&x);
  h = __hsub2(h, __floats2half2_rn(1024.f, 1024.f));
  return *reinterpret_cast<uint32_t *>(&h);
}
// two bytes at positions 0 and 2 of x (after masking) -> half2 of their values
__device__ __forceinline__ uint32_t u8pair_to_h2(uint32_t x) {
  return h2_sub1024((x & 0x00FF00FFu) | 0x64006400u);
}
// two nibbles at bit 0 and bit 16 of x -> half2 of their values
__device__ __forceinline__ uint32_t u4pair_to_h2(uint32_t x) {
  return h2_sub1024((x & 0x000F000Fu) | 0x64006400u);
}

__device__ __forceinline__ float load_q16(const uint16_t *q, int64_t off, bool bf16) {
  const uint16_t b = q[off];
  return bf16 ? __uint_as_float(static_cast<uint32_t>(b) << 16) : __half2float(__ushort_as_half(b));
}

template <int D, int BITS>
__global__ void __launch_bounds__(kWarps * 32, 2) paged_decode_q_kernel(const Params p) {
  using C = QCfg<D, BITS>;
  constexpr int S = C::kStages;
  constexpr int NG = C::NG;
  constexpr int KS = D / 16;   // k-steps of Q.K (4 per group)
  constexpr int NT = D / 8;    // n-tiles of P.V (8 per group)

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                              ~static_cast<uintptr_t>(127));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int W = gridDim.x * kWarps;
  const int wid = blockIdx.x * kWarps + warp;

  uint8_t *stages = smem + warp * S * C::kStageBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kSmemTiles) + warp * S;
  Unit *uq = reinterpret_cast<Unit *>(smem + C::kSmemTiles + C::kSmemBars) + warp * kUnitQ;
  const uint32_t bar0 = smem_u32(bars);
  const uint32_t stage0 = smem_u32(stages);

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(bar0 + 8 * s, 1);
    fence_mbar_init();
  }
  __syncwarp();

  zero_empty_outputs<D>(p, wid, W, lane);
  Sched sch;
  if (!sch.init(p, lane, wid, W, uq)) return;

  const uint64_t pol = l2_policy_evict_first();
  auto issue = [&](int s, const Cursor &c) {
    if (lane == 0) {
      int32_t blk = p.tables[(int64_t)c.b * p.max_blocks + c.t / p.tpb];
      if (blk < 0 || blk >= p.n_blocks) {
        dev_error(p.err, MZ_DEVERR_BLOCK_ID);
        blk = 0;
      }
      const int64_t row0 = ((int64_t)blk * p.Hkv + c.h) * p.bs + (c.t % p.tpb) * kTileTok;
      const uint32_t bar = bar0 + 8 * s;
      const uint32_t st = stage0 + s * C::kStageBytes;
      mbar_arrive_expect_tx(bar, C::kTx);
      bulk_load(st, p.kq + row0 * C::RB, C::TD, bar, pol);
      bulk_load(st + C::TD, p.vq + row0 * C::RB, C::TD, bar, pol);
      bulk_load(st + 2 * C::TD, p.k_scales + row0 * NG, C::TS, bar, pol);
      bulk_load(st + 2 * C::TD + C::TS, p.k_biases + row0 * NG, C::TS, bar, pol);
      bulk_load(st + 2 * C::TD + 2 * C::TS, p.v_scales + row0 * NG, C::TS, bar, pol);
      bulk_load(st + 2 * C::TD + 3 * C::TS, p.v_biases + row0 * NG, C::TS, bar, pol);
    }
  };

  const int g = lane >> 2, cq = lane & 3;
  const bool two_groups = p.rows > 8;

  uint32_t qa[KS][4];     // Q (fp16) A fragments over the permuted head dim
  float qsum[2][NG];      // sum of Q over each group, rows g and g+8
  float oacc[NT][4];      // 256/16-scaled P'.q_v accumulators
  float rb[2][NG];        // sum_t p * b_v per row and group (lane partial)
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  UnitReader ur;
  bool seg_first = true;

  sch.refill<S>(p, 0, issue);
  for (int i = 0; i < sch.issued; ++i) {
    const int s = i % S;
    if (ur.need_pop()) {
      ur.pop(uq);
      seg_first = true;
    }
    const Cursor &cc = ur.cc;

    if (seg_first || cc.t == 0) {
      seg_first = false;
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
#pragma unroll
      for (int n = 0; n < NT; ++n) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.f;
#pragma unroll
      for (int gg = 0; gg < NG; ++gg) rb[0][gg] = rb[1][gg] = qsum[0][gg] = qsum[1][gg] = 0.f;
      const auto *q16 = static_cast<const uint16_t *>(p.q);
      const bool qb = p.q_bf16;
#pragma unroll
      for (int rs = 0; rs < 2; ++rs) {
        const int row = g + 8 * rs;
        const bool live = row < p.rows;
        const int64_t qo = live ? row_offset(p.q_sb, p.q_st, p.q_sh, cc.b, cc.h, row, p.G) : 0;
#pragma unroll
        for (int j = 0; j < KS; ++j) {
          const int G = j / 4, w = j % 4;
          int e0, e1, e2, e3;  // head-dim indices of k-slots 2c, 2c+1, 2c+8, 2c+9
          if constexpr (BITS == 8) {
            const int d0 = 64 * G + 16 * cq + 4 * w;
            e0 = d0; e1 = d0 + 1; e2 = d0 + 2; e3 = d0 + 3;
          } else {
            const int base = 64 * G + 16 * cq + 8 * (w >> 1), j0 = 2 * (w & 1);
            e0 = base + j0; e1 = base + j0 + 4; e2 = base + j0 + 1; e3 = base + j0 + 5;
          }
          float f0 = 0.f, f1 = 0.f, f2 = 0.f, f3 = 0.f;
          if (live) {
            f0 = __half2float(__float2half_rn(load_q16(q16, qo + e0, qb)));
            f1 = __half2float(__float2half_rn(load_q16(q16, qo + e1, qb)));
            f2 = __half2float(__float2half_rn(load_q16(q16, qo + e2, qb)));
            f3 = __half2float(__float2half_rn(load_q16(q16, qo + e3, qb)));
          }
          qa[j][rs] = pack2<false>(f0, f1);
          qa[j][2 + rs] = pack2<false>(f2, f3);
          qsum[rs][G] += (f0 + f1) + (f2 + f3);
        }
      }
#pragma unroll
      for (int rs = 0; rs < 2; ++rs)
#pragma unroll
        for (int gg = 0; gg < NG; ++gg) {
          float v = qsum[rs][gg];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          qsum[rs][gg] = v;
        }
    }

    if (!wait_stage<S>(p, bar0, i, sch.issued, lane)) return;

    const uint8_t *st = stages + s * C::kStageBytes;
    const uint8_t *kd = st, *vd = st + C::TD;
    const __half *ksc = reinterpret_cast<const __half *>(st + 2 * C::TD);
    const __half *kbi = reinterpret_cast<const __half *>(st + 2 * C::TD + C::TS);
    const __half *vsc = reinterpret_cast<const __half *>(st + 2 * C::TD + 2 * C::TS);
    const __half *vbi = reinterpret_cast<const __half *>(st + 2 * C::TD + 3 * C::TS);
    const int nvalid = min(kTileTok, cc.ctx - cc.t * kTileTok);
    const bool last_tile = (cc.t == cc.n - 1);

    // ---- S = Q . K^T with K = s_k * q_k + b_k ----
    float sacc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float acc[NG][4];
#pragma unroll
      for (int gg = 0; gg < NG; ++gg) acc[gg][0] = acc[gg][1] = acc[gg][2] = acc[gg][3] = 0.f;
      const int tk = nt * 8 + g;
#pragma unroll
      for (int G = 0; G < NG; ++G) {
        if constexpr (BITS == 8) {
          const uint4 kw = *reinterpret_cast<const uint4 *>(kd + tk * C::RB + 64 * G + 16 * cq);
          const uint32_t wv[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const uint32_t b0 = u8pair_to_h2(__byte_perm(wv[w], 0, 0x4140));
            const uint32_t b1 = u8pair_to_h2(__byte_perm(wv[w], 0, 0x4342));
            mma_16816<false>(acc[G], qa[4 * G + w], b0, b1);
          }
        } else {
          const uint2 kw = *reinterpret_cast<const uint2 *>(kd + tk * C::RB + 32 * G + 8 * cq);
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const uint32_t wx = (w >> 1) ? kw.y : kw.x;
            const int j0 = 2 * (w & 1);
            const uint32_t b0 = u4pair_to_h2(wx >> (4 * j0));
            const uint32_t b1 = u4pair_to_h2(wx >> (4 * (j0 + 1)));
            mma_16816<false>(acc[G], qa[4 * G + w], b0, b1);
          }
        }
      }
      // tokens nt*8 + 2c and +1 (C-fragment columns)
      const int t0 = nt * 8 + 2 * cq;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = t0 + (e & 1), rs = e >> 1;
        float x = 0.f;
#pragma unroll
        for (int G = 0; G < NG; ++G)
          x += __half2float(ksc[tok * NG + G]) * acc[G][e] +
               __half2float(kbi[tok * NG + G]) * qsum[rs][G];
        x *= p.scale_log2;
        if (tok >= nvalid) x = -INFINITY;
        sacc[nt][e] = x;
      }
    }

    // ---- online softmax (rows g: regs 0,1; g+8: regs 2,3) ----
    float mx0 = fmaxf(fmaxf(sacc[0][0], sacc[0][1]), fmaxf(sacc[1][0], sacc[1][1]));
    float mx1 = fmaxf(fmaxf(sacc[0][2], sacc[0][3]), fmaxf(sacc[1][2], sacc[1][3]));
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
    for (int nt = 0; nt < 2; ++nt) {
      sacc[nt][0] = fast_exp2(sacc[nt][0] - m0);
      sacc[nt][1] = fast_exp2(sacc[nt][1] - m0);
      rs0 += sacc[nt][0] + sacc[nt][1];
      if (two_groups) {
        sacc[nt][2] = fast_exp2(sacc[nt][2] - m1);
        sacc[nt][3] = fast_exp2(sacc[nt][3] - m1);
        rs1 += sacc[nt][2] + sacc[nt][3];
      } else {
        sacc[nt][2] = sacc[nt][3] = 0.f;
      }
    }
    l0 = l0 * a0 + rs0;
    l1 = l1 * a1 + rs1;
    if (__any_sync(0xffffffffu, a0 != 1.f || a1 != 1.f)) {
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        oacc[n][0] *= a0;
        oacc[n][1] *= a0;
        oacc[n][2] *= a1;
        oacc[n][3] *= a1;
      }
#pragma unroll
      for (int gg = 0; gg < NG; ++gg) {
        rb[0][gg] *= a0;
        rb[1][gg] *= a1;
      }
    }

    // ---- O += (p * s_v) . q_v ;  rb += p * b_v ----
    // this lane's tokens in the P fragments: 2c, 2c+1 (regs 0,1) and 8+2c, 9+2c (regs 2,3)
    const int ta = 2 * cq, tb = 8 + 2 * cq;
    float sv[4][NG], bv[4][NG];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int tok = (k < 2 ? ta : tb) + (k & 1);
      const bool ok = tok < nvalid;
#pragma unroll
      for (int G = 0; G < NG; ++G) {
        sv[k][G] = ok ? __half2float(vsc[tok * NG + G]) * C::kPScale : 0.f;
        bv[k][G] = ok ? __half2float(vbi[tok * NG + G]) : 0.f;
      }
    }
    // P values by (row set, token slot k)
    const float pv[2][4] = {{sacc[0][0], sacc[0][1], sacc[1][0], sacc[1][1]},
                            {sacc[0][2], sacc[0][3], sacc[1][2], sacc[1][3]}};
#pragma unroll
    for (int G = 0; G < NG; ++G) {
      uint32_t pa[4];
      pa[0] = pack2<false>(pv[0][0] * sv[0][G], pv[0][1] * sv[1][G]);
      pa[1] = pack2<false>(pv[1][0] * sv[0][G], pv[1][1] * sv[1][G]);
      pa[2] = pack2<false>(pv[0][2] * sv[2][G], pv[0][3] * sv[3][G]);
      pa[3] = pack2<false>(pv[1][2] * sv[2][G], pv[1][3] * sv[3][G]);
#pragma unroll
      for (int rs = 0; rs < 2; ++rs)
        rb[rs][G] += pv[rs][0] * bv[0][G] + pv[rs][1] * bv[1][G] + pv[rs][2] * bv[2][G] +
                     pv[rs][3] * bv[3][G];
      // V codes of tokens ta, ta+1, tb, tb+1 for head dims 64G + 8g + [0, 8)
      if constexpr (BITS == 8) {
        const uint2 va0 = *reinterpret_cast<const uint2 *>(vd + (ta)*C::RB + 64 * G + 8 * g);
        const uint2 va1 = *reinterpret_cast<const uint2 *>(vd + (ta + 1) * C::RB + 64 * G + 8 * g);
        const uint2 vb0 = *reinterpret_cast<const uint2 *>(vd + (tb)*C::RB + 64 * G + 8 * g);
        const uint2 vb1 = *reinterpret_cast<const uint2 *>(vd + (tb + 1) * C::RB + 64 * G + 8 * g);
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const uint32_t sel = static_cast<uint32_t>((m & 3) | ((4 + (m & 3)) << 8));
          const uint32_t wa0 = m < 4 ? va0.x : va0.y, wa1 = m < 4 ? va1.x : va1.y;
          const uint32_t wb0 = m < 4 ? vb0.x : vb0.y, wb1 = m < 4 ? vb1.x : vb1.y;
          const uint32_t b0 = u8pair_to_h2(__byte_perm(wa0, wa1, sel));
          const uint32_t b1 = u8pair_to_h2(__byte_perm(wb0, wb1, sel));
          mma_16816<false>(oacc[8 * G + m], pa, b0, b1);
        }
      } else {
        const uint32_t va0 = *reinterpret_cast<const uint32_t *>(vd + (ta)*C::RB + 32 * G + 4 * g);
        const uint32_t va1 = *reinterpret_cast<const uint32_t *>(vd + (ta + 1) * C::RB + 32 * G + 4 * g);
        const uint32_t vb0 = *reinterpret_cast<const uint32_t *>(vd + (tb)*C::RB + 32 * G + 4 * g);
        const uint32_t vb1 = *reinterpret_cast<const uint32_t *>(vd + (tb + 1) * C::RB + 32 * G + 4 * g);
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const uint32_t sel = static_cast<uint32_t>((m >> 1) | ((4 + (m >> 1)) << 8));
          const int sh = 4 * (m & 1);
          const uint32_t b0 = u4pair_to_h2(__byte_perm(va0, va1, sel) >> sh);
          const uint32_t b1 = u4pair_to_h2(__byte_perm(vb0, vb1, sel) >> sh);
          mma_16816<false>(oacc[8 * G + m], pa, b0, b1);
        }
      }
    }

    // ---- piece end ----
    if (last_tile || ur.left == 1) {
      float L0 = l0, L1 = l1;
      L0 += __shfl_xor_sync(0xffffffffu, L0, 1);
      L0 += __shfl_xor_sync(0xffffffffu, L0, 2);
      L1 += __shfl_xor_sync(0xffffffffu, L1, 1);
      L1 += __shfl_xor_sync(0xffffffffu, L1, 2);
      float R[2][NG];
#pragma unroll
      for (int rs = 0; rs < 2; ++rs)
#pragma unroll
        for (int gg = 0; gg < NG; ++gg) {
          float v = rb[rs][gg];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          R[rs][gg] = v;
        }
      // value of C-fragment (n-tile 8G + m, reg e): row g + 8*(e >> 1),
      // head dim 64G + 16c + 8*(e & 1) + m
      constexpr float kInvP = 1.f / C::kPScale;
      const int bh = cc.b * p.Hkv + cc.h;
      const int pbh = cc.pos - cc.t;
      const int uf = sch.unit_of(pbh), ul = sch.unit_of(pbh + cc.n - 1);
      const bool full = uf == ul;
      const int64_t slot = (int64_t)ur.unit + bh;
#pragma unroll
      for (int rs = 0; rs < 2; ++rs) {
        const int row = g + 8 * rs;
        if (row >= p.rows) continue;
        const float inv = full ? 1.f / (rs ? L1 : L0) : 1.f;
        const int64_t o = full ? row_offset(p.o_sb, p.o_st, p.o_sh, cc.b, cc.h, row, p.G) : 0;
        float *pr = p.part + (slot * p.rows + row) * D;
#pragma unroll
        for (int G = 0; G < NG; ++G)
#pragma unroll
          for (int half = 0; half < 2; ++half)
#pragma unroll
            for (int m = 0; m < 8; m += 2) {
              const int e = 2 * rs + half;
              const int d = 64 * G + 16 * cq + 8 * half + m;
              const float x = (oacc[8 * G + m][e] * kInvP + R[rs][G]) * inv;
              const float y = (oacc[8 * G + m + 1][e] * kInvP + R[rs][G]) * inv;
              if (full)
                store_pair(p, o + d, x, y);
              else
                *reinterpret_cast<float2 *>(pr + d) = make_float2(x, y);
            }
        if (!full && cq == 0)
          *reinterpret_cast<float2 *>(p.ml + (slot * p.rows + row) * 2) =
              make_float2(rs ? m1 : m0, rs ? L1 : L0);
      }
      if (!full) arrive_and_merge<D>(p, cc, bh, uf, ul - uf + 1, lane);
      seg_first = true;
    }

    __syncwarp();
    --ur.left;
    advance(ur.cc, p);
    sch.refill<S>(p, i + 1, issue);
  }
}

template <int D, int BITS>
int q_kernel_ctas_per_sm(int *out) {
  static int cached = -1;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  return kernel_occupancy(paged_decode_q_kernel<D, BITS>, QCfg<D, BITS>::kSmemBytes, &cached,
                          &once, &err, out);
}

int q_ctas_per_sm(int D, int bits, int *out) {
  if (D == 128) return bits == 8 ? q_kernel_ctas_per_sm<128, 8>(out) : q_kernel_ctas_per_sm<128, 4>(out);
  return bits == 8 ? q_kernel_ctas_per_sm<64, 8>(out) : q_kernel_ctas_per_sm<64, 4>(out);
}

int q_resolve_warps(int D, int bits, int num_warps, int device, int64_t *warps) {
  if (num_warps < 0) return fail(MZ_ERR_INVALID_ARG, "num_warps < 0");
  if (num_warps > 0) {
    *warps = (num_warps + kWarps - 1) / kWarps * kWarps;
    return MZ_OK;
  }
  int per_sm = 0;
  if (int rc = q_ctas_per_sm(D, bits, &per_sm)) return rc;
  if (per_sm < 1) return fail(MZ_ERR_CUDA, "quantised decode kernel cannot be resident on an SM");
  const int sms = sm_count(device);
  if (sms <= 0) return fail(MZ_ERR_CUDA, "cannot query SM count of device %d", device);
  *warps = (int64_t)sms * per_sm * kWarps;
  return MZ_OK;
}

int check_q_shape(int D, int bits, int group, const char *fn) {
  if (D != 64 && D != 128) return fail(MZ_ERR_UNSUPPORTED, "%s: head_dim %d (supported: 64, 128)", fn, D);
  if (bits != 4 && bits != 8) return fail(MZ_ERR_UNSUPPORTED, "%s: bits %d (supported: 4, 8)", fn, bits);
  if (group != 64) return fail(MZ_ERR_UNSUPPORTED, "%s: group_size %d (supported: 64)", fn, group);
  return MZ_OK;
}

}  // namespace decode
}  // namespace mz

using namespace mz;
using namespace mz::decode;

namespace {
int quant_append_common(QAppendParams &qp, void *k_codes, void *k_scales, void *k_biases,
                        void *v_codes, void *v_scales, void *v_biases, const void *k_new,
                        const void *v_new, int32_t n_kv_heads, int32_t head_dim,
                        int32_t block_size, int64_t n_blocks, int32_t bits, int32_t group_size,
                        int32_t dtype, int32_t *dev_err, mz_stream_t stream, const char *fn) {
  if (int rc = check_q_shape(head_dim, bits, group_size, fn)) return rc;
  if (dtype != MZ_DTYPE_F16 && dtype != MZ_DTYPE_BF16)
    return fail(MZ_ERR_UNSUPPORTED, "%s: dtype must be F16 or BF16", fn);
  if (n_kv_heads <= 0 || block_size <= 0 || n_blocks <= 0)
    return fail(MZ_ERR_INVALID_ARG, "%s: bad sizes", fn);
  if (qp.n_tokens == 0) return MZ_OK;
  if (!k_codes || !k_scales || !k_biases || !v_codes || !v_scales || !v_biases || !k_new || !v_new)
    return fail(MZ_ERR_INVALID_ARG, "%s: null pointer", fn);
  if (!aligned(k_codes, 4) || !aligned(v_codes, 4) || !aligned(k_scales, 2) ||
      !aligned(k_biases, 2) || !aligned(v_scales, 2) || !aligned(v_biases, 2) ||
      !aligned(k_new, 2) || !aligned(v_new, 2))
    return fail(MZ_ERR_ALIGNMENT, "%s: misaligned pointer", fn);
  qp.kq = static_cast<uint32_t *>(k_codes);
  qp.vq = static_cast<uint32_t *>(v_codes);
  qp.ks = static_cast<__half *>(k_scales);
  qp.kb = static_cast<__half *>(k_biases);
  qp.vs = static_cast<__half *>(v_scales);
  qp.vb = static_cast<__half *>(v_biases);
  qp.kn = static_cast<const uint16_t *>(k_new);
  qp.vn = static_cast<const uint16_t *>(v_new);
  qp.qbf16 = dtype == MZ_DTYPE_BF16;
  qp.H = n_kv_heads;
  qp.bs = block_size;
  qp.n_blocks = n_blocks;
  qp.err = dev_err;
  return quant_append(qp, head_dim, bits, static_cast<cudaStream_t>(stream));
}
}  // namespace

extern "C" int mz_kv_quant_append(void *k_codes, void *k_scales, void *k_biases, void *v_codes,
                                  void *v_scales, void *v_biases, const void *k_new,
                                  const void *v_new, int64_t new_tok_stride,
                                  int64_t new_head_stride, const int64_t *slot_mapping,
                                  int64_t n_tokens, int32_t n_kv_heads, int32_t head_dim,
                                  int32_t block_size, int64_t n_blocks, int32_t bits,
                                  int32_t group_size, int32_t dtype, int32_t *dev_err,
                                  mz_stream_t stream) {
  if (n_tokens < 0) return fail(MZ_ERR_INVALID_ARG, "mz_kv_quant_append: n_tokens < 0");
  if (n_tokens > 0 && !slot_mapping)
    return fail(MZ_ERR_INVALID_ARG, "mz_kv_quant_append: null slot_mapping");
  QAppendParams qp{};
  qp.n_tok_stride = new_tok_stride;
  qp.n_head_stride = new_head_stride;
  qp.slots = slot_mapping;
  qp.n_tokens = n_tokens;
  return quant_append_common(qp, k_codes, k_scales, k_biases, v_codes, v_scales, v_biases, k_new,
                             v_new, n_kv_heads, head_dim, block_size, n_blocks, bits, group_size,
                             dtype, dev_err, stream, "mz_kv_quant_append");
}

extern "C" int mz_kv_quant_append_paged(void *k_codes, void *k_scales, void *k_biases,
                                        void *v_codes, void *v_scales, void *v_biases,
                                        const void *k_new, const void *v_new,
                                        int64_t new_seq_stride, int64_t new_head_stride,
                                        const int32_t *block_tables, int32_t max_blocks_per_seq,
                                        const int32_t *positions, int32_t n_seqs,
                                        int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
                                        int64_t n_blocks, int32_t bits, int32_t group_size,
                                        int32_t dtype, int32_t *dev_err, mz_stream_t stream) {
  if (n_seqs < 0 || max_blocks_per_seq <= 0)
    return fail(MZ_ERR_INVALID_ARG, "mz_kv_quant_append_paged: bad n_seqs / max_blocks_per_seq");
  if (n_seqs > 0 && (!block_tables || !positions))
    return fail(MZ_ERR_INVALID_ARG, "mz_kv_quant_append_paged: null tables / positions");
  QAppendParams qp{};
  qp.n_tok_stride = new_seq_stride;
  qp.n_head_stride = new_head_stride;
  qp.tables = block_tables;
  qp.max_blocks = max_blocks_per_seq;
  qp.positions = positions;
  qp.n_tokens = n_seqs;
  return quant_append_common(qp, k_codes, k_scales, k_biases, v_codes, v_scales, v_biases, k_new,
                             v_new, n_kv_heads, head_dim, block_size, n_blocks, bits, group_size,
                             dtype, dev_err, stream, "mz_kv_quant_append_paged");
}

extern "C" int mz_paged_decode_q_workspace_size(int32_t n_seqs, int32_t n_kv_heads,
                                                int32_t rows_per_kv_head, int32_t head_dim,
                                                int32_t bits, int32_t num_warps, int32_t device,
                                                size_t *bytes) {
  if (!bytes) return fail(MZ_ERR_INVALID_ARG, "bytes is null");
  if (n_seqs < 0 || n_kv_heads <= 0 || rows_per_kv_head <= 0 || rows_per_kv_head > 16)
    return fail(MZ_ERR_INVALID_ARG, "workspace_size: bad sizes");
  if (int rc = check_q_shape(head_dim, bits, 64, "mz_paged_decode_q_workspace_size")) return rc;
  if (device < 0) device = current_device();
  int64_t warps = 0;
  if (int rc = q_resolve_warps(head_dim, bits, num_warps, device, &warps)) return rc;
  *bytes = ws_layout((int64_t)n_seqs * n_kv_heads, warps, rows_per_kv_head, head_dim).total;
  return MZ_OK;
}

extern "C" int mz_paged_decode_q(void *out, int32_t out_dtype, int64_t out_seq_stride,
                                 int64_t out_tok_stride, int64_t out_head_stride, const void *q,
                                 int64_t q_seq_stride, int64_t q_tok_stride, int64_t q_head_stride,
                                 int32_t n_q_tokens, const void *k_codes, const void *k_scales,
                                 const void *k_biases, const void *v_codes, const void *v_scales,
                                 const void *v_biases, const int32_t *block_tables,
                                 int32_t max_blocks_per_seq, const int32_t *ctx_lens,
                                 int32_t n_seqs, int32_t n_heads, int32_t n_kv_heads,
                                 int32_t head_dim, int32_t block_size, int64_t n_blocks,
                                 int32_t bits, int32_t group_size, float scale, int32_t dtype,
                                 int32_t num_warps, void *workspace, size_t workspace_bytes,
                                 int32_t *dev_err, mz_stream_t stream) {
  const char *fn = "mz_paged_decode_q";
  if (int rc = check_q_shape(head_dim, bits, group_size, fn)) return rc;
  if (dtype != MZ_DTYPE_F16 && dtype != MZ_DTYPE_BF16)
    return fail(MZ_ERR_UNSUPPORTED, "%s: dtype (of q) must be F16 or BF16", fn);
  if (out_dtype != dtype && out_dtype != MZ_DTYPE_F32)
    return fail(MZ_ERR_UNSUPPORTED, "%s: out_dtype must equal dtype or be F32", fn);
  if (block_size <= 0 || block_size % kTileTok)
    return fail(MZ_ERR_UNSUPPORTED, "%s: block_size %d is not a multiple of 16", fn, block_size);
  if (n_seqs < 0 || n_kv_heads <= 0 || n_heads <= 0 || n_heads % n_kv_heads || n_q_tokens <= 0 ||
      max_blocks_per_seq <= 0 || n_blocks <= 0)
    return fail(MZ_ERR_INVALID_ARG, "%s: bad sizes", fn);
  const int rows = n_q_tokens * (n_heads / n_kv_heads);
  if (rows > 16) return fail(MZ_ERR_UNSUPPORTED, "%s: %d query rows per KV head exceed 16", fn, rows);
  if (!std::isfinite(scale)) return fail(MZ_ERR_INVALID_ARG, "%s: scale not finite", fn);
  if (n_seqs == 0) return MZ_OK;
  if (!out || !q || !k_codes || !k_scales || !k_biases || !v_codes || !v_scales || !v_biases ||
      !block_tables || !ctx_lens)
    return fail(MZ_ERR_INVALID_ARG, "%s: null pointer", fn);
  if (!workspace) return fail(MZ_ERR_WORKSPACE, "%s: workspace is null", fn);
  if (!aligned(k_codes, 16) || !aligned(v_codes, 16) || !aligned(k_scales, 16) ||
      !aligned(k_biases, 16) || !aligned(v_scales, 16) || !aligned(v_biases, 16) ||
      !aligned(q, 2))
    return fail(MZ_ERR_ALIGNMENT, "%s: code/scale pools need 16-byte alignment", fn);
  const int ob = out_dtype == MZ_DTYPE_F32 ? 8 : 4;
  if (!aligned(out, ob) || (out_seq_stride & 1) || (out_tok_stride & 1) || (out_head_stride & 1))
    return fail(MZ_ERR_ALIGNMENT, "%s: out needs %d-byte alignment and even strides", fn, ob);
  if ((int64_t)n_seqs * n_kv_heads * max_blocks_per_seq * (block_size / kTileTok) >= (int64_t(1) << 30))
    return fail(MZ_ERR_UNSUPPORTED, "%s: more than 2^30 tiles of context", fn);
  const int device = current_device();
  int64_t warps = 0;
  if (int rc = q_resolve_warps(head_dim, bits, num_warps, device, &warps)) return rc;
  const WsLayout ws = ws_layout((int64_t)n_seqs * n_kv_heads, warps, rows, head_dim);
  if (workspace_bytes < ws.total)
    return fail(MZ_ERR_WORKSPACE, "%s: workspace %zu bytes < required %zu", fn, workspace_bytes,
                ws.total);
  if (!aligned(workspace, 256)) return fail(MZ_ERR_ALIGNMENT, "%s: workspace must be 256-byte aligned", fn);

  Params p{};
  p.out = out;
  p.o_sb = out_seq_stride;
  p.o_st = out_tok_stride;
  p.o_sh = out_head_stride;
  p.out_f32 = out_dtype == MZ_DTYPE_F32;
  p.q = q;
  p.q_sb = q_seq_stride;
  p.q_st = q_tok_stride;
  p.q_sh = q_head_stride;
  p.q_bf16 = dtype == MZ_DTYPE_BF16;
  p.n_q = n_q_tokens;
  p.G = n_heads / n_kv_heads;
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
  p.kq = static_cast<const uint8_t *>(k_codes);
  p.vq = static_cast<const uint8_t *>(v_codes);
  p.k_scales = static_cast<const __half *>(k_scales);
  p.k_biases = static_cast<const __half *>(k_biases);
  p.v_scales = static_cast<const __half *>(v_scales);
  p.v_biases = static_cast<const __half *>(v_biases);
  auto *w8 = static_cast<uint8_t *>(workspace);
  p.counters = reinterpret_cast<int32_t *>(w8 + ws.counters);
  p.ml = reinterpret_cast<float *>(w8 + ws.ml);
  p.part = reinterpret_cast<float *>(w8 + ws.part);
  set_schedule(p, ws);
  p.err = dev_err;

  int per_sm = 0;
  if (int rc = q_ctas_per_sm(head_dim, bits, &per_sm)) return rc;
  const unsigned grid = static_cast<unsigned>(warps / kWarps);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define MZ_LQ(D_, B_)                                                                        \
  paged_decode_q_kernel<D_, B_><<<grid, kWarps * 32, QCfg<D_, B_>::kSmemBytes, s>>>(p)
  if (head_dim == 128) {
    if (bits == 8) MZ_LQ(128, 8); else MZ_LQ(128, 4);
  } else {
    if (bits == 8) MZ_LQ(64, 8); else MZ_LQ(64, 4);
  }
#undef MZ_LQ
  MZ_CHECK_LAUNCH(fn);
  return MZ_OK;
}
