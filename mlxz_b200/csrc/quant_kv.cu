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
// Decode never materialises dequantised K/V; the affine map is applied around
// the products:
//   S[r][t] = sum_g s_k[t][g] * (Q_g . q_k[t]_g) + b_k[t][g] * sum(Q_g[r])
//   O[r][d] = sum_t (p[r][t] * s_v[t][g(d)]) * q_v[t][d] + sum_t p[r][t] * b_v[t][g(d)]
// Q_g . q_k runs on the integer tensor cores (K codes as stored, u8; Q in
// 16-bit fixed point per row and group, split into signed bytes); P.V on the
// fp16 tensor cores (V codes exact in fp16, P' as an fp16 hi + lo pair).  The
// dot products run over a permutation of the head dimension chosen so that
// each lane's codes are contiguous bytes (Q is packed with the same
// permutation; V's output columns are un-permuted when written).  A tile's
// codes arrive by bulk (tensor) copies and its scales and biases by cp.async
// into a per-warp ring, with the same persistent-warp scheduler as the bf16
// kernel; the warp takes two tiles of a pair per step.
//
// Roofline: a tile moves 2 * 16 * (D * bits / 8 + 4 * D / 64) bytes; with
// D = 128 that is 4352 B (8-bit) or 2304 B (4-bit), against 8192 B at bf16.
#include <algorithm>

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

template <int D, int BITS, int NQ>
struct QCfg {
  static constexpr int RB = D * BITS / 8;   // code bytes per token row
  static constexpr int NG = D / 64;         // groups per row
  static constexpr int TD = kTileTok * RB;  // code bytes per tile (K or V)
  static constexpr int TS = kTileTok * NG * 2;  // scale (or bias) bytes per tile
  // 128-byte code rows (8-bit, D = 128) arrive by 2-D bulk tensor copies with
  // the 128-byte swizzle (conflict-free fragment reads with tok_of below);
  // other rows by 1-D bulk copies.  (For the 64-byte rows of 4-bit codes the
  // 64-byte swizzle with tok_of(m) = m ^ (((m >> 1) & 1) * 5) removes the bank
  // conflicts too, but measured slower: that kernel is bound by its ALU work,
  // and the swizzled addresses add to it.)
  static constexpr int kSwz = (RB == 128) ? 128 : 0;
  static constexpr bool kSwizzled = kSwz != 0;
  static constexpr int kTx = 2 * TD;  // bytes the code copies bring (scales come by cp.async)
  static constexpr int kCodeStage = 2 * TD;          // K + V codes (1024-aligned)
  static constexpr int kScaleStage = 4 * TS;         // K/V scales and biases
  static constexpr int kStageBytes = kCodeStage + kScaleStage;
  static constexpr int kCtas = NQ <= 2 ? 3 : 2;  // CTAs per SM the shared memory is sized for
  static constexpr int kStagesFit = (210 * 1024 / kCtas) / (kWarps * kStageBytes);
  static constexpr int kStages = kStagesFit > 8 ? 8 : (kStagesFit < 3 ? 3 : kStagesFit);
  static constexpr int kSmemCodes = kWarps * kStages * kCodeStage;
  static constexpr int kSmemScales = kWarps * kStages * kScaleStage;
  static constexpr int kSmemBars = kWarps * kStages * 8;
  static constexpr int kSmemUnits = kWarps * kUnitQ * static_cast<int>(sizeof(Unit));
  static constexpr int kSmemDefer = kWarps * kMaxDeferred * static_cast<int>(sizeof(Deferred));
  static constexpr int kSmemBytes =
      kSmemCodes + kSmemScales + kSmemBars + kSmemUnits + kSmemDefer + 1024;
  // P' = p * s_v is stored in fp16 scaled by this power of two (keeps small
  // weights out of fp16 subnormals; removed exactly at the end).
  static constexpr float kPScale = BITS == 8 ? 256.f : 16.f;
};

// Byte offset of (row, byte) in a code tile: the 128-byte swizzle (16-byte
// unit u of row r at u ^ (r & 7)), or plain rows.
template <class C>
__device__ __forceinline__ uint32_t code_off(int row, int byte) {
  if constexpr (C::kSwz == 128) {
    return swz128(row, byte);
  } else {
    return row * C::RB + byte;
  }
}

// Token of the tile held in mma row (or k index) m, chosen so that the K reads
// (rows m, m+1 in one quarter-warp phase) and the V reads (rows 2c or 2c+1,
// c = 0..3, in one half-warp phase) fall in distinct bank groups under the
// 128-byte swizzle (checked against a model of the shared-memory banks: the
// minimum number of wavefronts for every read): odd rows are exchanged with
// the row four away (m ^ 4).  Scores, masks, scales and V rows all go through
// this map, so the order of the tokens inside a tile is immaterial.
template <class C>
__device__ __forceinline__ int tok_of(int m) {
  if constexpr (C::kSwz == 128) {
    return m ^ ((m & 1) << 2);
  } else {
    return m;
  }
}

constexpr uint32_t kMagic = 0x64646464u;  // fp16 0x64xx = 1024 + xx

// Codes enter the P.V products centred on the middle of their range (code -
// 128 for 8-bit, code - 8 for 4-bit; exact in fp16): with the 1024 of the
// magic bias left in, a whole context's P.V sums would carry 1024 * sum P' and
// lose the result to cancellation once that is removed.
template <int BITS>
constexpr float kCodeCentre = BITS == 8 ? 128.f : 8.f;
template <int BITS>
constexpr uint32_t kCentreBits = BITS == 8 ? 0x64806480u : 0x64086408u;  // half2 of 1024 + centre
template <int BITS>
__device__ __forceinline__ uint32_t centred(uint32_t biased) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(biased), "r"(kCentreBits<BITS>));
  return r;
}
// half2 of (1024 + 16 n) -> half2 of n - 8 (x / 16 - 72, exact in fp16)
__device__ __forceinline__ uint32_t centred_hi_nibble(uint32_t biased16) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(biased16), "r"(0x2C002C00u), "r"(0xD480D480u));
  return r;
}

__device__ __forceinline__ float load_q16(const uint16_t *q, int64_t off, bool bf16) {
  const uint16_t b = q[off];
  return bf16 ? __uint_as_float(static_cast<uint32_t>(b) << 16) : __half2float(__ushort_as_half(b));
}

// D(16x8 s32) += A(16x32 u8, row-major) * B(32x8 s8, column-major)
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// x as an fp16 pair (hi, lo) with hi + lo = x to ~22 bits: the two columns of
// one query in the P.V products.
__device__ __forceinline__ uint32_t split_hilo(float x) {
  const __half h = __float2half_rn(x);
  const __half l = __float2half_rn(x - __half2float(h));
  return static_cast<uint32_t>(__half_as_ushort(h)) |
         (static_cast<uint32_t>(__half_as_ushort(l)) << 16);
}

// The query rows of a KV head go in groups of four (NQ groups, rows <= 4 NQ);
// lane (g, c) = (lane / 4, lane % 4) carries query row 4 nq + c of every group.
//
// QK on integer tensor cores (mma.m16n8k32, u8 x s8 -> s32), exact:
//   A[tok][k]  = the K codes as stored (8-bit) or split into bytes (4-bit:
//                x & 0x0F0F0F0F and (x >> 4) & 0x0F0F0F0F), tokens the M side;
//   B[k][col]  = Q in 16-bit fixed point per (row, group of 64 dims),
//                q16 = rint(q * 32639 / max|q|) = 256 hi + lo (hi, lo signed
//                bytes), column 2 i the hi bytes of row i, 2 i + 1 the lo bytes;
//   S[tok][i]  = sum_g s_k[tok][g] * sq[i][g] * (256 D[tok][2i] + D[tok][2i+1])
//                + b_k[tok][g] * sum(q~[i]_g),   q~ = q16 * sq (sq = max|q| / 32639)
// over a permutation of the head dimension within each group (the k slots of
// lane c in a k-step come from its own contiguous code words: 8 bytes at
// 8-bit, one word's low and high nibbles at 4-bit; Q is packed with the same
// permutation).
// PV on fp16 tensor cores (mma.m16n8k16): O^T[d][col] = sum_t A[d][t] B[t][col],
// A = V codes - centre (half2 of two tokens of one dim), B = P'^T by movmatrix,
// where P' = p * s_v * kPScale goes in as an fp16 pair (hi in column 2 i, lo in
// 2 i + 1), so the two columns of a row add up to P'.V at ~22 bits of P'.
// The centre comes back through sum P', the bias through sum p * b_v.
template <int D, int BITS, int NQ>
__global__ void __launch_bounds__(kWarps * 32, QCfg<D, BITS, NQ>::kCtas)
    paged_decode_q_kernel(const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const Params p) {
  using C = QCfg<D, BITS, NQ>;
  constexpr int S = C::kStages;
  constexpr int NG = C::NG;
  constexpr int MT = D / 16;  // m-tiles of P.V (4 per group)

  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base, derived from the shared array by pointer
  // arithmetic so that the compiler keeps every access in the shared window
  // (a round trip through an integer would turn them into generic accesses)
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int W = gridDim.x * kWarps;
  const int wid = blockIdx.x * kWarps + warp;

  uint8_t *codes = smem + warp * S * C::kCodeStage;
  uint8_t *scales = smem + C::kSmemCodes + warp * S * C::kScaleStage;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kSmemCodes + C::kSmemScales) + warp * S;
  Unit *uq = reinterpret_cast<Unit *>(smem + C::kSmemCodes + C::kSmemScales + C::kSmemBars) +
             warp * kUnitQ;
  Deferred *dq = reinterpret_cast<Deferred *>(smem + C::kSmemCodes + C::kSmemScales +
                                              C::kSmemBars + C::kSmemUnits) +
                 warp * kMaxDeferred;
  int nd = 0;  // merges this warp owns, run after its tile loop
  const uint32_t bar0 = smem_u32(bars);
  const uint32_t code0 = smem_u32(codes);
  const uint32_t scale0 = smem_u32(scales);

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(bar0 + 8 * s, 1);
    fence_mbar_init();
  }
  __syncwarp();

  zero_empty_outputs<D>(p, wid, W, lane);
  Sched sch;
  if (!sch.init(p, lane, wid, W, uq)) return;

  const uint64_t pol = l2_policy_evict_first();
  // Copies go out for up to two tiles at a time, tile A from lanes 0..15 and
  // tile B from lanes 16..31.  A tile's K and V codes arrive by two bulk
  // (tensor) copies, which take warp-uniform operands, so lane 0 issues them
  // for both tiles; its scales and biases (4 x 64 bytes at D = 128) arrive
  // as 16-byte cp.async pieces from the lanes of its half, each piece tracked
  // by the stage barrier (cp.async.mbarrier.arrive raises the pending count,
  // then arrives when the piece lands), so the barrier completes when all of
  // the tile is in shared memory.  Small bulk copies cost the copy engine as
  // much as large ones; as cp.async pieces the 64-byte arrays leave it two
  // copies per tile.  When a half issues a tile it also loads the table entry
  // of the tile two on, which it issues next, so no table load sits on the
  // issue path.
  const int half = lane >> 4, hl = lane & 15;
  int32_t pf_blk = 0;
  int pf_key = -1;  // table index of pf_blk, -1: none
  // this lane's 16-byte piece of its tile's four scale / bias arrays (hl < kPieces)
  constexpr int kPer = C::TS / 16, kPieces = 4 * kPer;
  static_assert(kPieces <= 16, "scale pieces exceed a half warp");
  const int pc_arr = min(hl / kPer, 3);
  const uint32_t pc_off = static_cast<uint32_t>(hl - pc_arr * kPer) * 16u;
  const uint32_t pc_dst = pc_arr * C::TS + pc_off;
  const uint8_t *pc_src =
      reinterpret_cast<const uint8_t *>(pc_arr == 0 ? p.k_scales : pc_arr == 1 ? p.k_biases
                                        : pc_arr == 2 ? p.v_scales : p.v_biases) + pc_off;
  auto issue2 = [&](bool two, int sa, const Cursor &ca, int sb, const Cursor &cb) {
    int64_t row0 = 0;
    if (half == 0 || two) {
      const Cursor &c = half ? cb : ca;
      const int s = half ? sb : sa;
      const int tb = p.tpb == 1 ? c.t : c.t / p.tpb;
      const int key = c.b * p.max_blocks + tb;
      int32_t blk = key == pf_key ? pf_blk : __ldg(p.tables + key);
      if (c.t + 2 < c.n) {
        pf_key = c.b * p.max_blocks + (p.tpb == 1 ? c.t + 2 : (c.t + 2) / p.tpb);
        pf_blk = __ldg(p.tables + pf_key);
      } else {
        pf_key = -1;
      }
      if (blk < 0 || blk >= p.n_blocks) {
        if (hl == 0) dev_error(p.err, MZ_DEVERR_BLOCK_ID);
        blk = 0;
      }
      const int sub = p.tpb == 1 ? 0 : c.t - tb * p.tpb;
      row0 = ((int64_t)blk * p.Hkv + c.h) * p.bs + sub * kTileTok;
      if (hl < kPieces) {
        cp_async16(scale0 + s * C::kScaleStage + pc_dst, pc_src + row0 * (NG * 2));
        asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(bar0 + 8 * s) : "memory");
      }
    }
    __syncwarp();  // every piece's pending count is raised before its barrier can complete
    const int64_t row_b = __shfl_sync(0xffffffffu, row0, 16);
    if (lane == 0) {
      fence_proxy_async_smem();
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (u == 1 && !two) break;
        const int st = u ? sb : sa;
        const int64_t r = u ? row_b : row0;
        const uint32_t bar = bar0 + 8 * st;
        const uint32_t dst = code0 + st * C::kCodeStage;
        mbar_arrive_expect_tx(bar, C::kTx);
        if constexpr (C::kSwizzled) {
          tma_load_2d(dst, &tmK, 0, static_cast<int>(r), bar, pol);
          tma_load_2d(dst + C::TD, &tmV, 0, static_cast<int>(r), bar, pol);
        } else {
          bulk_load(dst, p.kq + r * C::RB, C::TD, bar, pol);
          bulk_load(dst + C::TD, p.vq + r * C::RB, C::TD, bar, pol);
        }
      }
    }
  };
  // keep S tiles in flight, two per round where two stages are free and the
  // unit has two tiles left
  auto refill = [&](int consumed) {
    while (!sch.p_done && sch.issued - consumed < S) {
      if (sch.p_left == 0 && !sch.next_unit(p)) {
        sch.p_done = true;
        break;
      }
      const bool two = sch.p_left >= 2 && sch.issued - consumed <= S - 2;
      const Cursor ca = sch.pc;
      const int sa = sch.istage;
      advance(sch.pc, p);
      --sch.p_left;
      ++sch.issued;
      if (++sch.istage == S) sch.istage = 0;
      Cursor cb = ca;
      int sb = sa;
      if (two) {
        cb = sch.pc;
        sb = sch.istage;
        advance(sch.pc, p);
        --sch.p_left;
        ++sch.issued;
        if (++sch.istage == S) sch.istage = 0;
      }
      issue2(two, sa, ca, sb, cb);
    }
  };

  const int g = lane >> 2, cq = lane & 3;

  uint32_t qb[NQ][NG][2][2];  // Q bytes (B fragments), column g of group nq, k-step j of group G
  float qsc[NQ][NG];          // sq * log2(e) * scale of row 4 nq + cq, group G
  float qsm[NQ][NG];          // sum(q~) * log2(e) * scale, same row and group
  float oacc[NQ][MT][4];      // O^T (less centre * sum P'), P-scaled; cols (hi, lo) of one row
  float rb[NQ][NG];           // sum_t p * b_v (lane partial over its tokens g, g+8)
  float cp[NQ][NG];           // sum_t P' (lane partial) -- restores the centre
  float mrow[NQ], lrow[NQ];

  UnitReader ur;
  bool seg_first = true;

  refill(0);
  bool ring_idle = true;
  int s = 0;           // stage of tile i
  uint32_t phase = 0;  // its barrier phase
  for (int i = 0; i < sch.issued;) {
    if (ur.need_pop()) {
      ur.pop(uq);
      seg_first = true;
    }
    const Cursor &cc = ur.cc;

    if (seg_first || cc.t == 0) {
      seg_first = false;
      const auto *q16 = static_cast<const uint16_t *>(p.q);
      const bool qbf = p.q_bf16;
#pragma unroll
      for (int nq = 0; nq < NQ; ++nq) {
        // B column g holds the hi (g even) or lo (g odd) bytes of row 4 nq + g / 2
        const int row = 4 * nq + (g >> 1);
        const bool live = row < p.rows;
        const int64_t qo = live ? row_offset(p.q_sb, p.q_st, p.q_sh, cc.b, cc.h, row, p.G) : 0;
#pragma unroll
        for (int G = 0; G < NG; ++G) {
          float f[16];  // head dims 64 G + 16 cq + e
          float mx = 0.f;
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            f[e] = live ? load_q16(q16, qo + 64 * G + 16 * cq + e, qbf) : 0.f;
            mx = fmaxf(mx, fabsf(f[e]));
          }
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
          const float qf = mx > 0.f ? 32639.f / mx : 0.f;
          int qi[16];
          int sum = 0;
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            int v = __float2int_rn(f[e] * qf);
            v = max(-32639, min(32639, v));
            qi[e] = v;
            sum += v;
          }
          sum += __shfl_xor_sync(0xffffffffu, sum, 1);
          sum += __shfl_xor_sync(0xffffffffu, sum, 2);
          uint32_t by[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int hi = (qi[e] + 128) >> 8;  // q16 = 256 hi + lo, lo in [-128, 127]
            by[e] = static_cast<uint32_t>((g & 1) ? qi[e] - (hi << 8) : hi) & 0xFFu;
          }
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            if constexpr (BITS == 8) {
              // k slots 4c..4c+3 <-> dims 16c + 8j + 0..3, slots 16+4c.. <-> + 4..7
              qb[nq][G][j][0] = by[8 * j] | by[8 * j + 1] << 8 | by[8 * j + 2] << 16 | by[8 * j + 3] << 24;
              qb[nq][G][j][1] = by[8 * j + 4] | by[8 * j + 5] << 8 | by[8 * j + 6] << 16 | by[8 * j + 7] << 24;
            } else {
              // k slots 4c..4c+3 <-> dims 16c + 8j + {0,2,4,6}, slots 16+4c.. <-> {1,3,5,7}
              qb[nq][G][j][0] = by[8 * j] | by[8 * j + 2] << 8 | by[8 * j + 4] << 16 | by[8 * j + 6] << 24;
              qb[nq][G][j][1] = by[8 * j + 1] | by[8 * j + 3] << 8 | by[8 * j + 5] << 16 | by[8 * j + 7] << 24;
            }
          }
          const float sq = mx * (1.f / 32639.f);
          const float cs = sq * p.scale_log2, cb = static_cast<float>(sum) * sq * p.scale_log2;
          // row 4 nq + cq (this lane's scores) was packed by lane 8 cq
          qsc[nq][G] = __shfl_sync(0xffffffffu, cs, 8 * cq);
          qsm[nq][G] = __shfl_sync(0xffffffffu, cb, 8 * cq);
          rb[nq][G] = cp[nq][G] = 0.f;
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) oacc[nq][m][0] = oacc[nq][m][1] = oacc[nq][m][2] = oacc[nq][m][3] = 0.f;
        mrow[nq] = -INFINITY;
        lrow[nq] = 0.f;
      }
    }

    // Two tiles of the pair per step when the piece has them (u = 0, 1); a
    // step of one tile runs the same code with tile 1 masked out.
    const bool has2 = ur.left >= 2 && cc.t + 1 < cc.n && i + 1 < sch.issued;
    const int nt = has2 ? 2 : 1;
    const int s1 = s + 1 == S ? 0 : s + 1;
    const uint32_t phase1 = s + 1 == S ? phase ^ 1u : phase;
    bool ready = mbar_wait_bounded(bar0 + 8 * s, phase, kTimeoutNs);
    if (has2) ready = ready && mbar_wait_bounded(bar0 + 8 * s1, phase1, kTimeoutNs);
    if (!__all_sync(0xffffffffu, ready)) {
      (void)wait_stage<S>(p, bar0, i, sch.issued, lane);  // records the timeout, drains the copies
      ring_idle = false;
      break;
    }

    const int su[2] = {s, has2 ? s1 : s};
    int nval[2];  // valid tokens of each tile (0: no tile)
    nval[0] = min(kTileTok, cc.ctx - cc.t * kTileTok);
    nval[1] = has2 ? min(kTileTok, cc.ctx - (cc.t + 1) * kTileTok) : 0;

    // ---- S = K . Q^T per group, integer (tokens g, g+8; row 4 nq + cq) ----
    int acc[2][NQ][NG][4];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint8_t *kd = codes + su[u] * C::kCodeStage;
#pragma unroll
      for (int G = 0; G < NG; ++G) {
#pragma unroll
        for (int nq = 0; nq < NQ; ++nq)
          acc[u][nq][G][0] = acc[u][nq][G][1] = acc[u][nq][G][2] = acc[u][nq][G][3] = 0;
        if constexpr (BITS == 8) {
          const uint4 k0 = *reinterpret_cast<const uint4 *>(kd + code_off<C>(tok_of<C>(g), 64 * G + 16 * cq));
          const uint4 k1 = *reinterpret_cast<const uint4 *>(kd + code_off<C>(tok_of<C>(g + 8), 64 * G + 16 * cq));
#pragma unroll
          for (int nq = 0; nq < NQ; ++nq) {
            mma_u8s8(acc[u][nq][G], k0.x, k1.x, k0.y, k1.y, qb[nq][G][0][0], qb[nq][G][0][1]);
            mma_u8s8(acc[u][nq][G], k0.z, k1.z, k0.w, k1.w, qb[nq][G][1][0], qb[nq][G][1][1]);
          }
        } else {
          const uint2 k0 = *reinterpret_cast<const uint2 *>(kd + code_off<C>(tok_of<C>(g), 32 * G + 8 * cq));
          const uint2 k1 = *reinterpret_cast<const uint2 *>(kd + code_off<C>(tok_of<C>(g + 8), 32 * G + 8 * cq));
          const uint32_t l0 = k0.x & 0x0F0F0F0Fu, h0 = (k0.x >> 4) & 0x0F0F0F0Fu;
          const uint32_t l1 = k1.x & 0x0F0F0F0Fu, h1 = (k1.x >> 4) & 0x0F0F0F0Fu;
          const uint32_t l2 = k0.y & 0x0F0F0F0Fu, h2 = (k0.y >> 4) & 0x0F0F0F0Fu;
          const uint32_t l3 = k1.y & 0x0F0F0F0Fu, h3 = (k1.y >> 4) & 0x0F0F0F0Fu;
#pragma unroll
          for (int nq = 0; nq < NQ; ++nq) {
            mma_u8s8(acc[u][nq][G], l0, l1, h0, h1, qb[nq][G][0][0], qb[nq][G][0][1]);
            mma_u8s8(acc[u][nq][G], l2, l3, h2, h3, qb[nq][G][1][0], qb[nq][G][1][1]);
          }
        }
      }
    }
    // scores: sc[nq][2 u + ts] <-> (token tok_of(g + 8 ts) of tile u, row 4 nq + cq), log2 units
    float sc[NQ][4];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint8_t *ss = scales + su[u] * C::kScaleStage;
      const __half *ksc = reinterpret_cast<const __half *>(ss);
      const __half *kbi = reinterpret_cast<const __half *>(ss + C::TS);
      float skv[2][NG], bkv[2][NG];
#pragma unroll
      for (int ts = 0; ts < 2; ++ts) {
        if constexpr (NG == 2) {
          const float2 sk = __half22float2(*reinterpret_cast<const __half2 *>(ksc + tok_of<C>(g + 8 * ts) * 2));
          const float2 bk = __half22float2(*reinterpret_cast<const __half2 *>(kbi + tok_of<C>(g + 8 * ts) * 2));
          skv[ts][0] = sk.x;
          skv[ts][1] = sk.y;
          bkv[ts][0] = bk.x;
          bkv[ts][1] = bk.y;
        } else {
#pragma unroll
          for (int G = 0; G < NG; ++G) {
            skv[ts][G] = __half2float(ksc[tok_of<C>(g + 8 * ts) * NG + G]);
            bkv[ts][G] = __half2float(kbi[tok_of<C>(g + 8 * ts) * NG + G]);
          }
        }
      }
#pragma unroll
      for (int nq = 0; nq < NQ; ++nq)
#pragma unroll
        for (int ts = 0; ts < 2; ++ts) {
          float x = 0.f;
#pragma unroll
          for (int G = 0; G < NG; ++G) {
            const int si = acc[u][nq][G][2 * ts] * 256 + acc[u][nq][G][2 * ts + 1];
            x = fmaf(static_cast<float>(si), skv[ts][G] * qsc[nq][G], fmaf(bkv[ts][G], qsm[nq][G], x));
          }
          if (tok_of<C>(g + 8 * ts) >= nval[u]) x = -INFINITY;
          sc[nq][2 * u + ts] = x;
        }
    }

    // ---- online softmax per query row, over the step's 32 tokens ----
    float alpha[NQ];
    bool moved = false;
#pragma unroll
    for (int nq = 0; nq < NQ; ++nq) {
      float mx = fmaxf(fmaxf(sc[nq][0], sc[nq][1]), fmaxf(sc[nq][2], sc[nq][3]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float mn = fmaxf(mrow[nq], mx);
      alpha[nq] = fast_exp2(mrow[nq] - mn);
      moved |= alpha[nq] != 1.f;
      mrow[nq] = mn;
#pragma unroll
      for (int k = 0; k < 4; ++k) sc[nq][k] = fast_exp2(sc[nq][k] - mn);
      lrow[nq] = lrow[nq] * alpha[nq] + ((sc[nq][0] + sc[nq][1]) + (sc[nq][2] + sc[nq][3]));
    }
    if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
      for (int nq = 0; nq < NQ; ++nq) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          oacc[nq][m][0] *= alpha[nq];
          oacc[nq][m][1] *= alpha[nq];
          oacc[nq][m][2] *= alpha[nq];
          oacc[nq][m][3] *= alpha[nq];
        }
#pragma unroll
        for (int G = 0; G < NG; ++G) {
          rb[nq][G] *= alpha[nq];
          cp[nq][G] *= alpha[nq];
        }
      }
    }

    // ---- O^T += (V codes - centre) . P'^T ; rb += p * b_v ; cp += P' ----
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint8_t *vd = codes + su[u] * C::kCodeStage + C::TD;
      const uint8_t *ss = scales + su[u] * C::kScaleStage;
      const __half *vsc = reinterpret_cast<const __half *>(ss + 2 * C::TS);
      const __half *vbi = reinterpret_cast<const __half *>(ss + 3 * C::TS);
      // V scales (times the P' scale) and biases of this lane's tokens g,
      // g+8 for every group; 0 past the context (and for a missing tile)
      float svg[2][NG], bvg[2][NG];
#pragma unroll
      for (int ts = 0; ts < 2; ++ts) {
        const int tok = tok_of<C>(g + 8 * ts);
        const bool ok = tok < nval[u];
        if constexpr (NG == 2) {
          const float2 sv2 = __half22float2(*reinterpret_cast<const __half2 *>(vsc + tok * 2));
          const float2 bv2 = __half22float2(*reinterpret_cast<const __half2 *>(vbi + tok * 2));
          svg[ts][0] = ok ? sv2.x * C::kPScale : 0.f;
          svg[ts][1] = ok ? sv2.y * C::kPScale : 0.f;
          bvg[ts][0] = ok ? bv2.x : 0.f;
          bvg[ts][1] = ok ? bv2.y : 0.f;
        } else {
#pragma unroll
          for (int G = 0; G < NG; ++G) {
            svg[ts][G] = ok ? __half2float(vsc[tok * NG + G]) * C::kPScale : 0.f;
            bvg[ts][G] = ok ? __half2float(vbi[tok * NG + G]) : 0.f;
          }
        }
      }
#pragma unroll
      for (int G = 0; G < NG; ++G) {
        uint32_t pb[NQ][2];
#pragma unroll
        for (int nq = 0; nq < NQ; ++nq) {
          const float x0 = sc[nq][2 * u] * svg[0][G], x1 = sc[nq][2 * u + 1] * svg[1][G];
          cp[nq][G] += x0 + x1;
          rb[nq][G] = fmaf(sc[nq][2 * u], bvg[0][G], fmaf(sc[nq][2 * u + 1], bvg[1][G], rb[nq][G]));
          pb[nq][0] = movmatrix_trans(split_hilo(x0));  // k slots 2c, 2c+1 (tokens of rows 0..7)
          pb[nq][1] = movmatrix_trans(split_hilo(x1));  // k slots 2c+8, 2c+9
        }
        if constexpr (BITS == 8) {
          // V codes of k slots 2c, 2c+1, 2c+8, 2c+9 (tokens tok_of(.)), head dims 64G + 8g + [0, 8)
          const uint2 v0 = *reinterpret_cast<const uint2 *>(vd + code_off<C>(tok_of<C>(2 * cq), 64 * G + 8 * g));
          const uint2 v1 = *reinterpret_cast<const uint2 *>(vd + code_off<C>(tok_of<C>(2 * cq + 1), 64 * G + 8 * g));
          const uint2 v2 = *reinterpret_cast<const uint2 *>(vd + code_off<C>(tok_of<C>(2 * cq + 8), 64 * G + 8 * g));
          const uint2 v3 = *reinterpret_cast<const uint2 *>(vd + code_off<C>(tok_of<C>(2 * cq + 9), 64 * G + 8 * g));
          // byte interleaves: [ra.bk, rb.bk, ra.bk+1, rb.bk+1]
          const uint32_t lo01a = __byte_perm(v0.x, v1.x, 0x5140), lo23a = __byte_perm(v0.x, v1.x, 0x7362);
          const uint32_t hi01a = __byte_perm(v0.y, v1.y, 0x5140), hi23a = __byte_perm(v0.y, v1.y, 0x7362);
          const uint32_t lo01b = __byte_perm(v2.x, v3.x, 0x5140), lo23b = __byte_perm(v2.x, v3.x, 0x7362);
          const uint32_t hi01b = __byte_perm(v2.y, v3.y, 0x5140), hi23b = __byte_perm(v2.y, v3.y, 0x7362);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            // m-tile 4G + v: row g <-> dim 64G + 8g + v, row g + 8 <-> dim 64G + 8g + 4 + v
            const uint32_t sel = (v & 1) ? 0x4342u : 0x4140u;
            uint32_t a[4];
            a[0] = centred<8>(__byte_perm((v < 2) ? lo01a : lo23a, kMagic, sel));
            a[1] = centred<8>(__byte_perm((v < 2) ? hi01a : hi23a, kMagic, sel));
            a[2] = centred<8>(__byte_perm((v < 2) ? lo01b : lo23b, kMagic, sel));
            a[3] = centred<8>(__byte_perm((v < 2) ? hi01b : hi23b, kMagic, sel));
#pragma unroll
            for (int nq = 0; nq < NQ; ++nq) mma_16816<false>(oacc[nq][4 * G + v], a, pb[nq][0], pb[nq][1]);
          }
        } else {
          // 4-bit: one word per token holds head dims 64G + 8g + [0, 8)
          const uint32_t v0 = *reinterpret_cast<const uint32_t *>(vd + code_off<C>(tok_of<C>(2 * cq), 32 * G + 4 * g));
          const uint32_t v1 = *reinterpret_cast<const uint32_t *>(vd + code_off<C>(tok_of<C>(2 * cq + 1), 32 * G + 4 * g));
          const uint32_t v2 = *reinterpret_cast<const uint32_t *>(vd + code_off<C>(tok_of<C>(2 * cq + 8), 32 * G + 4 * g));
          const uint32_t v3 = *reinterpret_cast<const uint32_t *>(vd + code_off<C>(tok_of<C>(2 * cq + 9), 32 * G + 4 * g));
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            // m-tile 4G + v: row g <-> dim 64G + 8g + 2v (low nibble of byte v),
            // row g + 8 <-> dim 64G + 8g + 2v + 1 (high nibble)
            const uint32_t sel = static_cast<uint32_t>(v | (v << 4) | ((4 + v) << 8) | ((4 + v) << 12));
            const uint32_t z01 = __byte_perm(v0, v1, sel), z23 = __byte_perm(v2, v3, sel);
            uint32_t a[4];
            a[0] = centred<4>((z01 & 0x000F000Fu) | 0x64006400u);
            a[1] = centred_hi_nibble((z01 & 0x00F000F0u) | 0x64006400u);
            a[2] = centred<4>((z23 & 0x000F000Fu) | 0x64006400u);
            a[3] = centred_hi_nibble((z23 & 0x00F000F0u) | 0x64006400u);
#pragma unroll
            for (int nq = 0; nq < NQ; ++nq) mma_16816<false>(oacc[nq][4 * G + v], a, pb[nq][0], pb[nq][1]);
          }
        }
      }
    }

    // ---- piece end ----
    if (cc.t + nt == cc.n || ur.left == nt) {
      const int bh = cc.b * p.Hkv + cc.h;
      const int pbh = cc.pos - cc.t;
      const int uf = sch.unit_of(pbh), ul = sch.unit_of(pbh + cc.n - 1);
      const bool full = uf == ul;
      const int64_t slot = (int64_t)ur.unit + bh;
      constexpr float kInvP = 1.f / C::kPScale;
#pragma unroll
      for (int nq = 0; nq < NQ; ++nq) {
        float L = lrow[nq];
        L += __shfl_xor_sync(0xffffffffu, L, 4);
        L += __shfl_xor_sync(0xffffffffu, L, 8);
        L += __shfl_xor_sync(0xffffffffu, L, 16);
        float Rg[NG], Cg[NG];
#pragma unroll
        for (int G = 0; G < NG; ++G) {
          float r = rb[nq][G], c = cp[nq][G];
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {
            r += __shfl_xor_sync(0xffffffffu, r, o);
            c += __shfl_xor_sync(0xffffffffu, c, o);
          }
          Rg[G] = r;
          Cg[G] = c * kCodeCentre<BITS>;  // the V codes entered centred
        }
        const int row = 4 * nq + cq;
        if (row >= p.rows) continue;
        const float inv = full ? 1.f / L : 1.f;
        const int64_t o = full ? row_offset(p.o_sb, p.o_st, p.o_sh, cc.b, cc.h, row, p.G) : 0;
        float *pr = p.part + (slot * p.rows + row) * D;
#pragma unroll
        for (int G = 0; G < NG; ++G) {
          float val[8];  // head dims 64G + 8g + j, j = 0..7
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const float x0 = ((oacc[nq][4 * G + v][0] + oacc[nq][4 * G + v][1] + Cg[G]) * kInvP + Rg[G]) * inv;
            const float x1 = ((oacc[nq][4 * G + v][2] + oacc[nq][4 * G + v][3] + Cg[G]) * kInvP + Rg[G]) * inv;
            if constexpr (BITS == 8) {
              val[v] = x0;
              val[4 + v] = x1;
            } else {
              val[2 * v] = x0;
              val[2 * v + 1] = x1;
            }
          }
          const int d0 = 64 * G + 8 * g;
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            if (full)
              store_pair(p, o + d0 + j, val[j], val[j + 1]);
            else
              *reinterpret_cast<float2 *>(pr + d0 + j) = make_float2(val[j], val[j + 1]);
          }
        }
        if (!full && g == 0)
          *reinterpret_cast<float2 *>(p.ml + (slot * p.rows + row) * 2) = make_float2(mrow[nq], L);
      }
      if (!full) arrive_or_defer<D>(p, cc, bh, uf, ul - uf + 1, lane, dq, nd);
      seg_first = true;
    }

    __syncwarp();
    for (int k = 0; k < nt; ++k) {
      --ur.left;
      advance(ur.cc, p);
      if (++s == S) {
        s = 0;
        phase ^= 1u;
      }
    }
    i += nt;
    refill(i);
  }
  run_deferred<D>(p, dq, nd, codes, S * C::kCodeStage, ring_idle, lane);
}

template <int D, int BITS, int NQ>
int q_kernel_ctas_per_sm(int *out) {
  static DeviceOnce once;
  return kernel_occupancy(paged_decode_q_kernel<D, BITS, NQ>, QCfg<D, BITS, NQ>::kSmemBytes, once,
                          out);
}

template <int NQ>
int q_ctas_per_sm_nq(int D, int bits, int *out) {
  if (D == 128)
    return bits == 8 ? q_kernel_ctas_per_sm<128, 8, NQ>(out) : q_kernel_ctas_per_sm<128, 4, NQ>(out);
  return bits == 8 ? q_kernel_ctas_per_sm<64, 8, NQ>(out) : q_kernel_ctas_per_sm<64, 4, NQ>(out);
}

// Occupancy used to size grids and workspaces: the largest of the query-row
// instantiations, so one workspace size fits all of them.
int q_ctas_per_sm(int D, int bits, int *out) {
  int a = 0, b = 0, c = 0;
  if (int rc = q_ctas_per_sm_nq<1>(D, bits, &a)) return rc;
  if (int rc = q_ctas_per_sm_nq<2>(D, bits, &b)) return rc;
  if (int rc = q_ctas_per_sm_nq<4>(D, bits, &c)) return rc;
  *out = std::max(a, std::max(b, c));
  return MZ_OK;
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

namespace mz {
namespace decode {
// tcgen05 (kind::i8) form, quant_decode_tc.cu
bool qtc_supports(int head_dim, int rows);
int launch_decode_q_tc(const Params &p, int bits, int64_t rows_total, int grid, cudaStream_t s);
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

  const int64_t rows_total = n_blocks * n_kv_heads * block_size;
  // The mma.sync kernel (the default for both widths: integer Q.K^T on the
  // tensor cores, two tiles per step, and faster than the tcgen05 form at the
  // 8B shape) or, with MLXZ_B200_QDECODE_TC=1, the tcgen05 form (head_dim
  // 128; 1, 2, 4, 8 or 16 query rows per KV head).  The tcgen05 grid is one
  // CTA per SM, or fewer when num_warps caps the launch (its partials then
  // fit the workspace sized for num_warps).
  const int tc_mode = env_int("MLXZ_B200_QDECODE_TC", -1, -1, 1);
  const bool use_tc = qtc_supports(head_dim, rows) && tc_mode == 1;
  if (use_tc) {
    const int sms = sm_count(device);
    if (sms <= 0) return fail(MZ_ERR_CUDA, "%s: cannot query SM count of device %d", fn, device);
    int grid = sms;
    if (num_warps > 0) grid = static_cast<int>(std::min<int64_t>(sms, std::max<int64_t>(1, warps / kWarps)));
    return launch_decode_q_tc(p, bits, rows_total, grid, static_cast<cudaStream_t>(stream));
  }
  // 2-D maps over the code pools (rows of D * bits / 8 bytes), used by the
  // swizzled instantiations (128-byte rows); others take 1-D bulk copies.
  CUtensorMap tk{}, tv{};
  const int rb = head_dim * bits / 8;
  if (rb == 128) {
    if (rows_total >= (int64_t(1) << 31))
      return fail(MZ_ERR_UNSUPPORTED, "%s: pool has >= 2^31 rows", fn);
    if (int rc = make_row_map(&tk, k_codes, rows_total, rb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 128)) return rc;
    if (int rc = make_row_map(&tv, v_codes, rows_total, rb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 128)) return rc;
  }
  int per_sm = 0;  // also sets the kernels' shared-memory attributes (once)
  if (int rc = q_ctas_per_sm(head_dim, bits, &per_sm)) return rc;
  const unsigned grid = static_cast<unsigned>(warps / kWarps);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define MZ_LQ(D_, B_, NQ_)                                                                    \
  paged_decode_q_kernel<D_, B_, NQ_><<<grid, kWarps * 32, QCfg<D_, B_, NQ_>::kSmemBytes, s>>>(tk, tv, p)
#define MZ_LQ_NQ(NQ_)                                                \
  do {                                                               \
    if (head_dim == 128) {                                           \
      if (bits == 8) MZ_LQ(128, 8, NQ_); else MZ_LQ(128, 4, NQ_);    \
    } else {                                                         \
      if (bits == 8) MZ_LQ(64, 8, NQ_); else MZ_LQ(64, 4, NQ_);      \
    }                                                                \
  } while (0)
  // query rows per KV head in groups of four
  if (rows <= 4)
    MZ_LQ_NQ(1);
  else if (rows <= 8)
    MZ_LQ_NQ(2);
  else
    MZ_LQ_NQ(4);
#undef MZ_LQ_NQ
#undef MZ_LQ
  MZ_CHECK_LAUNCH(fn);
  return MZ_OK;
}
