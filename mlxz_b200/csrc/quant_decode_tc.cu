// Dequant-fused paged decode of 4/8-bit affine group-64 KV on the tcgen05
// tensor cores (kind::i8), head_dim 128, sm_100a.
//
// Why integer MMAs: the codes 0..255 (0..15 for 4-bit) are exact unsigned
// 8-bit integers, so they go into the tensor core as they lie in shared
// memory, with no per-element conversion.  The other operand is turned into
// 16-bit fixed point split into two unsigned bytes, and the affine map and the
// offsets are applied once per (token, query row) or (head dim, query row):
//
//   QK (per 128-token tile, per group g of 64 head dims), transposed so the
//   tokens are the M = 128 side:
//     S_g[t][n] = sum_{d in g} c_K[t][d] * B_Q[d][n],    B_Q columns:
//       n = r          hi byte of u_r[d] = q_r[d] + 32768,
//       n = rows + r   lo byte of u_r[d],
//       n = 2 rows     1 (gives sum_d c_K[t][d]),
//     with q_r = rint(Q_r / s_r) in [-32767, 32767], s_r = max_d |Q_r[d]| / 32767;
//     sum_{d in g} c q_r = 256 S[hi] + S[lo] - 32768 S[ones] (exact in int32), and
//     score[t][r] = s_r * sum_g s_K[t][g] * that + sum_g b_K[t][g] * sum_{d in g} s_r q_r[d].
//   PV (per tile, per group g), transposed so the head dims are the M side:
//     O_g[d][n] = sum_t c_V[t][d] * B_P[t][n],   B_P like B_Q with
//       u = rint(p_r[t] s_V[t][g] / sP_gr) + 32768, sP_gr = max_t |p_r[t] s_V[t][g]| / 32767
//       (the maximum found as 2^(max_t (x_r[t] + log2 |s_V[t][g]|) - m_r) in the same
//       exchange as the row maxima),
//     and out[r][d] = sum_tiles sP_gr (256 O[hi] + O[lo] - 32768 O[ones])
//                     + sum_t p_r[t] b_V[t][g(d)], normalised by sum_t p_r[t].
//   p_r[t] = 2^(score - m_r) with m_r the running maximum (exact per tile, so
//   p <= 1 and the 16-bit P' keeps 15 bits for the tile's largest weight).
//
// One CTA per SM, persistent; the flat list of 128-token tiles of all
// (sequence, KV head) pairs is cut into equal contiguous shares, and a pair
// cut by share boundaries leaves (m, l, O) partials that the last CTA to
// finish a piece of it merges (per-pair arrival counters in the workspace).
// Warps:
//   warp 0     copies: codes by one 2-D bulk tensor copy of K and of V per
//              16-token sub-tile (8-bit: 128-byte rows, 128-byte swizzle, the
//              layout the MMA reads; 4-bit: 64-byte rows, 64-byte swizzle; no
//              multicast), every tile's scales and biases by 16-byte cp.async
//              (a small bulk copy costs about as much issue time as a 2 KiB
//              one), all counted on the stage's mbarrier; block ids loaded
//              four tiles ahead
//   warp 1     TMEM allocation and the MMAs (one elected lane), each QK / PV
//              issued as soon as its inputs are in
//   token groups (one or two warpgroups; two take alternate tiles, each with
//              its own online-softmax state for the piece): thread = token of
//              the tile (TMEM lane): scores, exchange of tile maxima, P'
//   dim role (one warpgroup): thread = head dim (TMEM lane): the Q operand of
//              each piece, reads PV, accumulates O per token group, combines
//              the groups' states at a piece's end, writes outputs /
//              partials, merges; 4-bit: widens the next tile's codes to bytes
// Every wait is bounded (a wait that gives up sets MZ_DEVERR_TIMEOUT and an
// abort flag; the roles leave their loops together, the copy warp waits for
// its copies in flight, the MMA warp drains, warp 1 frees the TMEM).
//
// Widened 4-bit rows: word w of a row (dims 8w..8w+7, one nibble each) becomes
// bytes 8w..8w+7 = dims 8w + {0, 2, 4, 6, 1, 3, 5, 7} (low nibbles, then high
// nibbles, two instructions per word).  The head dims are permuted inside
// each 8-dim group; Q is loaded with the same permutation and outputs are
// stored through it, so the permutation never shows.
#include "decode_common.cuh"
#include "tcgen05.cuh"

namespace mz {
namespace decode {
namespace qtc {

constexpr int kT = 128;  // tokens per tile
constexpr int kD = 128;  // head dim
constexpr int kProdWarp = 0, kMmaWarp = 1, kTokWarp0 = 2;

template <int BITS, int ROWS>
struct Cfg {
  // token groups: two (alternate tiles, each with its own online-softmax
  // state) when the registers allow it, else one
  static constexpr int TGN = ROWS <= 4 ? 2 : 1;
  // softmax units per tile (each with its own max, P' scale and PV): one
  // warp of 32 tokens for up to 4 query rows, two warps for 8, four for 16
  // (the O columns of the units fill the TMEM)
  static constexpr int U = ROWS <= 4 ? 4 : (ROWS <= 8 ? 2 : 1);
  static constexpr int WPU = 4 / U;  // warps per unit
  static constexpr int kThreads = 64 + 128 * TGN + 128 + 32;
  static constexpr int kDimWarp0 = kTokWarp0 + 4 * TGN;
  static constexpr int kProdWarp2 = kDimWarp0 + 4;  // second copy warp (odd tiles)
  static constexpr int kBarDim = 2 + TGN * U;  // named barrier of the dim role (unit barriers below it)
  static constexpr int kBarProd = kBarDim + 1;  // named barrier of the two copy warps
  static constexpr int NB = ((2 * ROWS + 1 + 15) / 16) * 16;  // B operand columns
  static constexpr int kUnits = NB / 16;                      // 16-byte units per B row
  static constexpr int RB = kD * BITS / 8;                    // code bytes per token row
  static constexpr int kCodeTile = kT * 128;  // widened codes, 128 rows x 128 bytes
  static constexpr int kRawTile = kT * RB;    // 4-bit rows as stored
  static constexpr int kSub = 16;             // tokens per copy
  // A stage holds one tile as copied: 8-bit K and V codes in the layout the
  // MMAs read, or 4-bit codes as stored; then the scales and biases
  // [4 arrays][128 tok][2] fp16.  4-bit codes are widened to bytes, and the
  // scales copied, into one of W separate slots, so a stage is free again
  // once it is widened, while the slot waits for the tile's PV.
  static constexpr int kKr = 0, kVr = kRawTile;  // codes within a stage
  static constexpr int kSc = 2 * kRawTile;
  static constexpr int kScBytes = 4 * kT * 4;
  static constexpr int kStage = kSc + kScBytes;
  static constexpr int W = BITS == 4 ? 3 : 0;     // widened slots
  static constexpr int kKc = 0, kVc = kCodeTile;  // codes within a widened slot (8-bit: the stage)
  static constexpr int kWSc = 2 * kCodeTile;      // scales within a widened slot
  static constexpr int kWide = kWSc + kScBytes;
  static constexpr int kBop = kT * NB;  // one B operand
  static constexpr int NX4 = (3 * ROWS + 3) / 4;  // int4 words of one exchange slot
  // misc area (offsets from kMisc)
  static constexpr int kBars = 0;                                  // barriers
  static constexpr int kWords = 512;                               // tmem slot, abort, merge word, stops
  static constexpr int kXch = 576;                                 // [TGN][2][4 warps][NX4] int4
  static constexpr int kQx = kXch + TGN * 2 * 4 * NX4 * 16;        // [4 warps][ROWS]
  static constexpr int kQp = kQx + 4 * ROWS * 4;                   // [2][ROWS] s_q
  static constexpr int kQs = kQp + 2 * ROWS * 4;                   // [2][2 groups][ROWS]
  static constexpr int kTp = kQs + 2 * 2 * ROWS * 4;               // [2][U][3 ROWS]
  static constexpr int kPe = kTp + 2 * U * 3 * ROWS * 4;           // [2][TGN][U][4 ROWS]
  static constexpr int kLx = kPe + 2 * TGN * U * 4 * ROWS * 4;     // [TGN][4 warps][3 ROWS]
  static constexpr int kIds = kLx + TGN * 4 * 3 * ROWS * 4;  // [2 warps][4 tiles][8 sub-tiles] block ids
  static constexpr int kMiscBytes = kIds + 2 * 4 * 8 * 4;
  // as many stages as the shared memory holds (up to 8): the copies of
  // several tiles must be in flight to cover the memory latency under load
  static constexpr int kFixed = W * kWide + 6 * kBop + kMiscBytes + 1024;
  static constexpr int kStagesFit = (227 * 1024 - kFixed) / kStage;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kWidenAhead = W - 1;  // 4-bit: tiles widened ahead of the dim role's tile
  static constexpr int kWideBase = kStages * kStage;  // widened slots [W]
  static constexpr int kQb = kWideBase + W * kWide;   // Q operands [2]
  static constexpr int kPb = kQb + 2 * kBop;    // P' operands [2 bufs][2 groups]
  static constexpr int kMisc = kPb + 4 * kBop;
  static constexpr int kSmemBytes = kMisc + kMiscBytes + 1024;
  static_assert(kStages >= 3, "at least three stages");
  static_assert(BITS == 8 || kWidenAhead + 2 <= kStages, "4-bit widening stays behind the copies");
  static_assert(W <= 4, "widened-slot barriers");
  static constexpr int kCols = (4 + 4 * U) * NB;  // S [2][2][NB], O [2][U][2][NB]
  static constexpr uint32_t kTmemCols = kCols <= 128 ? 128 : (kCols <= 256 ? 256 : 512);
  static_assert(kCols <= 512, "TMEM columns");
  static_assert(kStage % 1024 == 0 && kWide % 1024 == 0, "1024-byte alignment of the swizzled tiles");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

// barrier slots
// (kFull, kEmpty: per stage; kKx, kVx, kWEmpty: per widened slot; kDrainT:
// per unit)
constexpr int kFull = 0, kKx = 8, kVx = 16, kEmpty = 24, kSFull = 32, kSEmpty = 34, kQFull = 36,
              kTpB = 38, kOFull = 40, kOEmpty = 42, kPeB = 44, kPeEmpty = 46, kDrain = 48,
              kDrainT = 49, kWEmpty = 57, kNumBars = 61;
static_assert(8 * kNumBars <= 512, "barrier area");

struct TCur {
  int b, h, t, n, ctx;
};

__device__ __forceinline__ int ntl(int ctx) { return (ctx + kT - 1) / kT; }

// Tiles of the whole problem (warp-uniform).
__device__ __forceinline__ int total_tiles(const Params &p, int lane) {
  int t = 0;
  for (int b = lane; b < p.B; b += 32) t += ntl(clamped_ctx(p, b));
#pragma unroll
  for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t * p.Hkv;
}

// Cursor at flat tile x (0 <= x < T), found with a warp scan over sequences.
__device__ __forceinline__ TCur locate_tc(const Params &p, int x, int lane) {
  int base = 0, bf = 0;
  for (int b0 = 0; b0 < p.B; b0 += 32) {
    const int b = b0 + lane;
    const int c = (b < p.B) ? ntl(clamped_ctx(p, b)) * p.Hkv : 0;
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const unsigned m = __ballot_sync(0xffffffffu, base + incl > x);
    if (m) {
      const int L = __ffs(m) - 1;
      base += __shfl_sync(0xffffffffu, incl - c, L);
      bf = b0 + L;
      break;
    }
    base += __shfl_sync(0xffffffffu, incl, 31);
  }
  TCur c;
  c.b = bf;
  c.ctx = clamped_ctx(p, bf);
  c.n = ntl(c.ctx);
  const int r = x - base;
  c.h = r / c.n;
  c.t = r - c.h * c.n;
  return c;
}

// Next tile in flat order (pairs with no context are skipped).
__device__ __forceinline__ void adv(TCur &c, const Params &p) {
  if (++c.t < c.n) return;
  c.t = 0;
  if (++c.h < p.Hkv) return;
  c.h = 0;
  for (;;) {
    if (++c.b >= p.B) {
      c.n = 0;
      return;
    }
    c.ctx = clamped_ctx(p, c.b);
    c.n = ntl(c.ctx);
    if (c.n > 0) return;
  }
}

// The first tile of the pair after c's.
__device__ __forceinline__ TCur next_pair(TCur c, const Params &p) {
  c.t = c.n - 1;
  adv(c, p);
  return c;
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_group3() {
  asm volatile("cp.async.wait_group 3;" ::: "memory");
}
__device__ __forceinline__ void cp_async16_hint(uint32_t dst, const void *src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "l"(pol)
               : "memory");
}
// The mbarrier gets one arrival (counted in its expected count) once every
// cp.async this thread issued before has landed.
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
// Non-blocking test of an mbarrier phase.
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(phase)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void mbar_arrive1(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void bar_sync_n(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// Named barrier over n threads that also ORs a predicate across them.
__device__ __forceinline__ bool bar_or(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 q, %2, 0;\n\t"
      "barrier.cta.red.or.pred p, %1, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(static_cast<int>(v)), "r"(n)
      : "memory");
  return r != 0;
}

// Order-preserving map of floats to signed ints (and back).
__device__ __forceinline__ int f2ord(float f) {
  const int i = __float_as_int(f);
  return i ^ ((i >> 31) & 0x7FFFFFFF);
}
__device__ __forceinline__ float ord2f(int i) { return __int_as_float(i ^ ((i >> 31) & 0x7FFFFFFF)); }

// Head dim held in byte position q of a widened code row (4-bit) or q itself.
template <int BITS>
__device__ __forceinline__ int dim_of(int q) {
  if constexpr (BITS == 4) {
    const int j = q & 7;
    return (q & ~7) + (j < 4 ? 2 * j : 2 * j - 7);
  } else {
    return q;
  }
}

__device__ __forceinline__ float ld_q(const void *q, int64_t off, bool bf16) {
  const uint16_t b = static_cast<const uint16_t *>(q)[off];
  return bf16 ? __uint_as_float(static_cast<uint32_t>(b) << 16) : __half2float(__ushort_as_half(b));
}

__device__ __forceinline__ void store_one(const Params &p, int64_t off, float v) {
  if (p.out_f32) {
    static_cast<float *>(p.out)[off] = v;
  } else if (p.q_bf16) {
    static_cast<__nv_bfloat16 *>(p.out)[off] = __float2bfloat16_rn(v);
  } else {
    static_cast<__half *>(p.out)[off] = __float2half_rn(v);
  }
}

// Row r of a B operand: bytes [hi_0..hi_{R-1}, lo_0..lo_{R-1}, 1, 0...] of the
// 16-bit values u_r, written as kUnits 16-byte stores (16-byte rows,
// MN-major without swizzle: unit j of row k at j * 2048 + k * 16).
template <int ROWS, int UNITS>
__device__ __forceinline__ void store_brow(uint8_t *base, int k, const uint32_t (&u)[ROWS]) {
  uint32_t w[UNITS * 4];
#pragma unroll
  for (int i = 0; i < UNITS * 4; ++i) w[i] = 0;
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    w[r >> 2] |= (u[r] >> 8) << (8 * (r & 3));
    w[(ROWS + r) >> 2] |= (u[r] & 0xFFu) << (8 * ((ROWS + r) & 3));
  }
  w[(2 * ROWS) >> 2] |= 1u << (8 * ((2 * ROWS) & 3));
#pragma unroll
  for (int j = 0; j < UNITS; ++j)
    *reinterpret_cast<uint4 *>(base + j * 2048 + k * 16) =
        make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}

// 4-bit: widen row `row` of a raw tile (64-byte rows, 64-byte swizzle) into the
// 128-byte-swizzled byte tile.
__device__ __forceinline__ void widen_row(const uint8_t *raw, uint8_t *dst, int row) {
  const int sw = (row >> 1) & 3;
  uint8_t *d = dst + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint4 x = *reinterpret_cast<const uint4 *>(raw + row * 64 + ((k ^ sw) << 4));
    const uint32_t wv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t a = wv[2 * h], b = wv[2 * h + 1];
      const uint4 y = make_uint4(a & 0x0F0F0F0Fu, (a >> 4) & 0x0F0F0F0Fu, b & 0x0F0F0F0Fu,
                                 (b >> 4) & 0x0F0F0F0Fu);
      const int u = 2 * k + h;  // 16-byte unit of the widened row
      *reinterpret_cast<uint4 *>(d + ((u ^ (row & 7)) << 4)) = y;
    }
  }
}

template <int BITS, int ROWS>
__global__ void __launch_bounds__(Cfg<BITS, ROWS>::kThreads, 1)
    paged_decode_qtc_kernel(const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const Params p) {
  using C = Cfg<BITS, ROWS>;
  constexpr int S = C::kStages;
  constexpr int NB = C::NB;
  constexpr int TGN = C::TGN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  uint8_t *misc = smem + C::kMisc;
  const uint32_t bars = sbase + C::kMisc + C::kBars;
  auto bar = [&](int i) { return bars + 8 * i; };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(misc + C::kWords);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(misc + C::kWords + 4);
  volatile int *merge_word = reinterpret_cast<volatile int *>(misc + C::kWords + 8);
  auto stage = [&](int s) { return smem + s * C::kStage; };
  auto stage_u = [&](int s) { return sbase + s * C::kStage; };
  auto wide = [&](int w) { return smem + C::kWideBase + w * C::kWide; };
  auto wide_u = [&](int w) { return sbase + C::kWideBase + w * C::kWide; };
  // the codes the MMAs of tile i read (8-bit: its stage; 4-bit: its widened slot)
  auto codes_u = [&](int i) { return BITS == 8 ? stage_u(i % S) : wide_u(i % C::W); };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (warp == kProdWarp && lane == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(bar(kFull + s), 33);  // lane 0 (+ bulk tensor bytes) and 32 cp.async arrivals
      // 8-bit: the units' PV commits; 4-bit: the dim role's widening
      mbar_init(bar(kEmpty + s), BITS == 8 ? C::U : 128);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(bar(kSFull + j), 1);
      mbar_init(bar(kSEmpty + j), 128);
      mbar_init(bar(kQFull + j), 128);
      mbar_init(bar(kTpB + j), C::U);
      mbar_init(bar(kOFull + j), C::U);
      mbar_init(bar(kOEmpty + j), 128);
      mbar_init(bar(kPeB + j), TGN * C::U);
      mbar_init(bar(kPeEmpty + j), 128);
    }
    mbar_init(bar(kDrain), 1);
    for (int w = 0; w < C::W; ++w) {
      mbar_init(bar(kKx + w), 128);
      mbar_init(bar(kVx + w), 128);
      mbar_init(bar(kWEmpty + w), C::U);  // the units' PV commits
    }
    for (int j = 0; j < TGN * C::U; ++j) mbar_init(bar(kDrainT + j), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tc::tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const uint32_t kS0 = 0, kO0 = 4 * NB;  // TMEM columns: S[buf][group], O[buf][unit][group]

  auto give_up = [&]() {
    dev_error(p.err, MZ_DEVERR_TIMEOUT);
    *abort_flag = 1;
  };
  auto wait_b = [&](int i, uint32_t parity) { return mbar_wait_bounded(bar(i), parity, kTimeoutNs); };

  const int T = total_tiles(p, lane);
  const int per = (T + gridDim.x - 1) / gridDim.x;
  const int x0 = static_cast<int>(blockIdx.x) * per;
  const int cnt = max(0, min(per, T - x0));

  if (warp == kProdWarp || warp == C::kProdWarp2) {
    // ---------------- copies ----------------
    // Two warps issue the copies, warp kProdWarp the even tiles of the share
    // and kProdWarp2 the odd ones: one warp's serial issue of a tile (block
    // ids, sixteen bulk tensor copies, the scales) takes longer than the
    // period the memory system sustains.
    const int pw = warp == kProdWarp ? 0 : 1;
    const uint64_t pol = l2_policy_evict_first();
    int stop = cnt;  // first tile of this warp not issued (cnt when all were)
    if (pw < cnt) {
      TCur c = locate_tc(p, x0, lane);
      if (pw) adv(c, p);
      // block ids are copied four own tiles ahead of their use into a ring in
      // shared memory (cp.async, one group per tile: a table load under full
      // HBM traffic takes about as long as issuing a tile's copies)
      int32_t *idring = reinterpret_cast<int32_t *>(misc + C::kIds) + pw * 32;
      const uint32_t idring_u = sbase + C::kMisc + C::kIds + pw * 128;
      TCur ca = c;  // cursor of the tile whose ids load next
      auto load_ids = [&](int slot) {
        const int tok0 = ca.t * kT + lane * C::kSub;
        if (lane < kT / C::kSub && tok0 < ca.ctx)
          cp_async4(idring_u + (slot * 8 + lane) * 4,
                    p.tables + (int64_t)ca.b * p.max_blocks + tok0 / p.bs);
        cp_async_commit();
      };
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        if (pw + 2 * a < cnt) {
          load_ids(a);
          adv(ca, p);
          adv(ca, p);
        } else {
          cp_async_commit();
        }
      }
      for (int i = pw, j = 0; i < cnt; i += 2, ++j) {
        if (__any_sync(0xffffffffu, *abort_flag != 0)) {
          stop = i;
          break;
        }
        cp_async_wait_group3();  // this tile's ids (groups of later tiles may be pending)
        const int32_t id_cur = lane < 8 ? idring[(j & 3) * 8 + lane] : 0;
        const int s = i % S;
        if (i >= S && !__all_sync(0xffffffffu, wait_b(kEmpty + s, ((i - S) / S) & 1))) {
          if (lane == 0) give_up();
          stop = i;
          break;
        }
        const int nv = min(kT, c.ctx - c.t * kT);
        const int nsub = (nv + C::kSub - 1) / C::kSub;
        const uint32_t sb = stage_u(s), fb = bar(kFull + s);
        // pool row of sub-tile `lane` (lanes < nsub)
        int64_t row0 = 0;
        if (lane < nsub) {
          int32_t blk = id_cur;
          if (blk < 0 || blk >= p.n_blocks) {
            dev_error(p.err, MZ_DEVERR_BLOCK_ID);
            blk = 0;
          }
          row0 = ((int64_t)blk * p.Hkv + c.h) * p.bs + (c.t * kT + lane * C::kSub) % p.bs;
        }
        // codes: one 2-D bulk tensor copy of K and of V per sub-tile (8-bit:
        // 128-byte rows, 128-byte swizzle, the layout the MMA reads; 4-bit:
        // 64-byte rows, 64-byte swizzle, widened later); the stage's full
        // barrier counts their bytes (lane 0) and one cp.async arrival of
        // every lane (the scales)
        if (lane == 0) mbar_arrive_expect_tx(fb, static_cast<uint32_t>(nsub * 2 * C::kSub * C::RB));
        __syncwarp();
        if (lane < nsub) {
          tma_load_2d(sb + C::kKr + lane * C::kSub * C::RB, &tmK, 0,
                      static_cast<int>(row0), fb, pol);
          tma_load_2d(sb + C::kVr + lane * C::kSub * C::RB, &tmV, 0,
                      static_cast<int>(row0), fb, pol);
        }
        {
          // scales and biases: 4 arrays x 16 tokens x 4 bytes per sub-tile =
          // 16 chunks of 16 bytes; lane l copies chunk (l & 3) of sub-tile l / 4
          // of every array
          const int j = lane >> 2, part = lane & 3;
          const int64_t rj = __shfl_sync(0xffffffffu, row0, j);
          if (j < nsub) {
            const __half *arr[4] = {p.k_scales, p.k_biases, p.v_scales, p.v_biases};
#pragma unroll
            for (int a = 0; a < 4; ++a)
              cp_async16_hint(sb + C::kSc + a * (kT * 4) + j * (C::kSub * 4) + part * 16,
                              arr[a] + rj * 2 + part * 8, pol);
          }
        }
        cp_async_arrive_noinc(fb);
        // the ids of own tile j + 4 into the slot just read
        if (i + 8 < cnt) {
          load_ids(j & 3);
          adv(ca, p);
          adv(ca, p);
        } else {
          cp_async_commit();
        }
        adv(c, p);
        adv(c, p);
      }
    }
    // copies still in flight land before the CTA leaves: the last tile
    // issued into each stage (a later phase of a stage needs the earlier
    // one complete first)
    int *stops = reinterpret_cast<int *>(misc + C::kWords + 16);
    if (lane == 0) stops[pw] = stop;
    bar_sync_n(C::kBarProd, 64);
    if (pw == 0 && lane == 0) {
      const int st0 = stops[0], st1 = stops[1];
      int found = 0;
      for (int j = cnt - 1; j >= 0 && found < S; --j) {
        if (j >= ((j & 1) ? st1 : st0)) continue;
        if (j + S < cnt && j + S < (((j + S) & 1) ? st1 : st0)) continue;  // stage reused later
        (void)wait_b(kFull + j % S, (j / S) & 1);
        ++found;
      }
    }
    __syncwarp();
  }
  else if (warp == kMmaWarp) {
    // ---------------- QK MMAs ----------------
    // QK(j) in tile order, once its codes are in (4-bit: widened), its S
    // buffer is free (S(j - 2) read) and, for a piece's first tile, the
    // piece's Q operand is written.  PV(j) is issued by the token group that
    // wrote P'(j).
    constexpr uint32_t idQK = tc::idesc_u8(kT, NB, false, true);
    bool ok = true;
    if (cnt > 0) {
      TCur cq = locate_tc(p, x0, lane);
      int kq = -1;  // piece of the last QK
      for (int nq = 0; nq < cnt; ++nq) {
        const bool newp = (nq == 0) || (cq.t == 0);
        const int kk = newp ? kq + 1 : kq;
        bool r = true;
        if (lane == 0)
          r = (BITS == 8 ? wait_b(kFull + nq % S, (nq / S) & 1)
                         : wait_b(kKx + nq % C::W, (nq / C::W) & 1)) &&
              (nq < 2 || wait_b(kSEmpty + (nq & 1), ((nq - 2) >> 1) & 1)) &&
              (!newp || wait_b(kQFull + (kk & 1), (kk >> 1) & 1)) && *abort_flag == 0;
        if (!__shfl_sync(0xffffffffu, r, 0)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const int s = nq % S, buf = nq & 1;
        const uint32_t qb = sbase + C::kQb + (kk & 1) * C::kBop;
        const uint32_t kc = codes_u(nq) + C::kKc;
#pragma unroll
        for (int g = 0; g < 2; ++g)
#pragma unroll
          for (int k = 0; k < 2; ++k)
            tc::mma_i8_elect(tmem + kS0 + buf * 2 * NB + g * NB,
                             tc::smem_desc_sw128(kc + 64 * g + 32 * k, 16, 1024),
                             tc::smem_desc_none(qb + 1024 * g + 512 * k, 128, 2048), idQK, k > 0);
        tc::commit_elect(bar(kSFull + buf));
        kq = kk;
        adv(cq, p);
      }
    }
    if (!ok && lane == 0) give_up();
    // every MMA issued has completed before the TMEM is freed
    tc::commit_elect(bar(kDrain));
    (void)wait_b(kDrain, 0);
    __syncwarp();
  }
  else if (warp < C::kDimWarp0) {
    // ---------------- token groups ----------------
    // Group tg takes the tiles i with i % TGN == tg; thread = token of the
    // tile (TMEM lane).  The group's tokens form U units (one warp each for
    // up to 4 query rows, two warps for 8, four for 16), and each unit keeps
    // its own online-softmax state for the piece, its own P' scale per tile
    // and issues its own PV: no exchange between the warps of a group on the
    // way from S to PV.  Units publish their state at the piece's end; the
    // dim role combines them.
    const int tg = (warp - kTokWarp0) >> 2;
    const int wq = warp & 3;                       // warp within the group
    const int u = wq / C::WPU;                     // unit within the group
    const int ubar = 2 + tg * C::U + u;            // the unit's named barrier (WPU > 1)
    const int uslot = tg * C::U + u;               // the unit's slot among all units
    const bool issuer = (wq % C::WPU) == 0;        // the unit's first warp issues its PV
    const int tok = 32 * wq + lane;
    const uint32_t tl = tmem + (static_cast<uint32_t>(wq * 32) << 16);
    int4 *xch = reinterpret_cast<int4 *>(misc + C::kXch) + tg * 2 * 4 * C::NX4;
    const float *qp = reinterpret_cast<const float *>(misc + C::kQp);
    const float *qs = reinterpret_cast<const float *>(misc + C::kQs);
    float *tp = reinterpret_cast<float *>(misc + C::kTp);
    float *pe = reinterpret_cast<float *>(misc + C::kPe);
    float *lx = reinterpret_cast<float *>(misc + C::kLx) + tg * 4 * 3 * ROWS;
    constexpr int NX = 3 * ROWS, NX4 = C::NX4, WPU = C::WPU, U = C::U;
    constexpr uint32_t idPV = tc::idesc_u8(kD, NB, true, true);
    // named barrier over the unit's warps (a warp barrier for one-warp units)
    // that also ORs a failure flag across them
    auto unit_or = [&](bool v) -> bool {
      if constexpr (WPU == 1) return __any_sync(0xffffffffu, v);
      else return bar_or(ubar, 32 * WPU, v);
    };
    bool bad = false, pv_issued = false;
    if (cnt > 0) {
      TCur c = locate_tc(p, x0, lane);
      float m[ROWS], l[ROWS], rb[2][ROWS], sq[ROWS], qsum[2][ROWS];
      int k = -1, kq = -1;
      for (int i = 0; i < cnt; ++i) {
        const bool first = (i == 0) || (c.t == 0);
        const bool last = (i == cnt - 1) || (c.t == c.n - 1);
        if (first) {
          ++k;
#pragma unroll
          for (int r = 0; r < ROWS; ++r) {
            m[r] = -INFINITY;
            l[r] = 0.f;
            rb[0][r] = rb[1][r] = 0.f;
          }
        }
        if (i % TGN == tg) {
          const int s = i % S, buf = i & 1;
          if (kq != k) {
            // the piece's Q quantities, published with its Q operand
            if (!bad && !wait_b(kQFull + (k & 1), (k >> 1) & 1)) bad = true;
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
              sq[r] = qp[(k & 1) * ROWS + r];
              qsum[0][r] = qs[((k & 1) * 2 + 0) * ROWS + r];
              qsum[1][r] = qs[((k & 1) * 2 + 1) * ROWS + r];
            }
            kq = k;
          }
          // scores of this tile
          uint32_t sr[2 * NB];
          if (!bad && !wait_b(kSFull + buf, (i >> 1) & 1)) bad = true;
          tc::fence_after_sync();
#pragma unroll
          for (int j = 0; j < 2 * NB; j += 32) {
            uint32_t r32[32];
            tc::ld32(tl + kS0 + buf * 2 * NB + j, r32);
            tc::wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (j + e < 2 * NB) sr[j + e] = r32[e];
          }
          tc::fence_before_sync();
          mbar_arrive1(bar(kSEmpty + buf));
          // the tile's scales: in its stage (8-bit) or its widened slot
          if constexpr (BITS == 8) {
            if (!bad && !wait_b(kFull + s, (i / S) & 1)) bad = true;
          } else {
            if (!bad && !wait_b(kKx + i % C::W, (i / C::W) & 1)) bad = true;
          }
          const uint8_t *sc = BITS == 8 ? stage(s) + C::kSc : wide(i % C::W) + C::kWSc;
          const float2 sk = __half22float2(*reinterpret_cast<const __half2 *>(sc + 0 * kT * 4 + tok * 4));
          const float2 bk = __half22float2(*reinterpret_cast<const __half2 *>(sc + 1 * kT * 4 + tok * 4));
          const float2 sv = __half22float2(*reinterpret_cast<const __half2 *>(sc + 2 * kT * 4 + tok * 4));
          const float2 bv = __half22float2(*reinterpret_cast<const __half2 *>(sc + 3 * kT * 4 + tok * 4));
          const int nv = min(kT, c.ctx - c.t * kT);
          const bool valid = tok < nv;
          float x[ROWS];
#pragma unroll
          for (int r = 0; r < ROWS; ++r) {
            const int d0 = static_cast<int>(sr[r] * 256u + sr[ROWS + r] - (sr[2 * ROWS] << 15));
            const int d1 = static_cast<int>(sr[NB + r] * 256u + sr[NB + ROWS + r] - (sr[NB + 2 * ROWS] << 15));
            float v = sq[r] * fmaf(sk.x, static_cast<float>(d0), sk.y * static_cast<float>(d1));
            v = fmaf(bk.x, qsum[0][r], fmaf(bk.y, qsum[1][r], v));
            x[r] = valid ? v * p.scale_log2 : -INFINITY;
          }
          // the unit's tile maxima: per row of the score, and per (group of
          // dims, row) of score + log2 |s_V| (the largest |p s_V| once the
          // new row maximum is known)
          int mx[NX4 * 4];
          {
            const float l2v0 = valid ? __log2f(fabsf(sv.x)) : -INFINITY;
            const float l2v1 = valid ? __log2f(fabsf(sv.y)) : -INFINITY;
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
              mx[r] = __reduce_max_sync(0xffffffffu, f2ord(x[r]));
              mx[ROWS + r] = __reduce_max_sync(0xffffffffu, f2ord(x[r] + l2v0));
              mx[2 * ROWS + r] = __reduce_max_sync(0xffffffffu, f2ord(x[r] + l2v1));
            }
#pragma unroll
            for (int e = NX; e < NX4 * 4; ++e) mx[e] = 0;
          }
          if constexpr (WPU > 1) {
            const int par = (i / TGN) & 1;
            if (lane == 0)
#pragma unroll
              for (int e = 0; e < NX4; ++e)
                xch[(par * 4 + wq) * NX4 + e] = make_int4(mx[4 * e], mx[4 * e + 1], mx[4 * e + 2], mx[4 * e + 3]);
            if (unit_or(bad || *abort_flag != 0)) {
              bad = true;
              break;
            }
#pragma unroll
            for (int e = 0; e < NX4; ++e) {
              int4 a = xch[(par * 4 + u * WPU) * NX4 + e];
#pragma unroll
              for (int w = 1; w < WPU; ++w) {
                const int4 b = xch[(par * 4 + u * WPU + w) * NX4 + e];
                a = make_int4(max(a.x, b.x), max(a.y, b.y), max(a.z, b.z), max(a.w, b.w));
              }
              mx[4 * e] = a.x;
              mx[4 * e + 1] = a.y;
              mx[4 * e + 2] = a.z;
              mx[4 * e + 3] = a.w;
            }
          }
          float mnew[ROWS], alpha[ROWS], inv_sp[2][ROWS], sp[2][ROWS];
#pragma unroll
          for (int r = 0; r < ROWS; ++r) {
            mnew[r] = fmaxf(m[r], ord2f(mx[r]));
            // a unit with no token of the piece yet keeps m = -inf: factor 1
            alpha[r] = mnew[r] > -INFINITY ? fast_exp2(m[r] - mnew[r]) : 1.f;
            m[r] = mnew[r];
#pragma unroll
            for (int g = 0; g < 2; ++g) {
              // largest |p s_V| of the unit's tile = 2^(ymax - mnew), taken
              // with a little headroom for the approximate log / exp:
              // sP = that / 32767
              const float e = ord2f(mx[(1 + g) * ROWS + r]) - mnew[r];
              const bool any = e > -INFINITY;
              sp[g][r] = any ? fast_exp2(e) * (1.000244140625f / 32767.f) : 0.f;
              inv_sp[g][r] = any ? fast_exp2(-e) * (32767.f / 1.000244140625f) : 0.f;
            }
          }
          // weights, the running sums, the P' operand of both groups of dims
          uint32_t u0[ROWS], u1[ROWS];
#pragma unroll
          for (int r = 0; r < ROWS; ++r) {
            const float pr = valid ? fast_exp2(x[r] - mnew[r]) : 0.f;
            l[r] = fmaf(l[r], alpha[r], pr);
            rb[0][r] = fmaf(rb[0][r], alpha[r], valid ? pr * bv.x : 0.f);
            rb[1][r] = fmaf(rb[1][r], alpha[r], valid ? pr * bv.y : 0.f);
            const int q0 = valid ? __float2int_rn(pr * sv.x * inv_sp[0][r]) : 0;
            const int q1 = valid ? __float2int_rn(pr * sv.y * inv_sp[1][r]) : 0;
            u0[r] = static_cast<uint32_t>(max(-32767, min(32767, q0)) + 32768);
            u1[r] = static_cast<uint32_t>(max(-32767, min(32767, q1)) + 32768);
          }
          // P'[buf] was read by PV(i - 2)
          if (i >= 2 && !bad && !wait_b(kOFull + buf, ((i - 2) >> 1) & 1)) bad = true;
          store_brow<ROWS, C::kUnits>(smem + C::kPb + (buf * 2 + 0) * C::kBop, tok, u0);
          store_brow<ROWS, C::kUnits>(smem + C::kPb + (buf * 2 + 1) * C::kBop, tok, u1);
          fence_proxy_async_smem();
          // the unit's P' is complete: its first warp issues the unit's PV
          if (unit_or(bad || *abort_flag != 0)) {
            bad = true;
            break;
          }
          if (issuer) {
            // O columns free (O(i - 2) read by the dim role), 4-bit V widened
            bool r = true;
            if (lane == 0)
              r = (i < 2 || wait_b(kOEmpty + buf, ((i - 2) >> 1) & 1)) &&
                  (BITS == 8 || wait_b(kVx + i % C::W, (i / C::W) & 1));
            if (__shfl_sync(0xffffffffu, r, 0)) {
              tc::fence_after_sync();
              const uint32_t vc = codes_u(i) + C::kVc;
#pragma unroll
              for (int g = 0; g < 2; ++g) {
                const uint32_t pb = sbase + C::kPb + (buf * 2 + g) * C::kBop;
#pragma unroll
                for (int kk = 0; kk < WPU; ++kk) {
                  const int ks = u * WPU + kk;  // 32-token step of the tile
                  tc::mma_i8_elect(tmem + kO0 + ((buf * U + u) * 2 + g) * NB,
                                   tc::smem_desc_sw128(vc + 4096 * ks, 16384, 1024),
                                   tc::smem_desc_none(pb + 512 * ks, 128, 2048), idPV, kk > 0);
                }
              }
              tc::commit_elect(bar(kOFull + buf));
              tc::commit_elect(bar(BITS == 8 ? kEmpty + s : kWEmpty + i % C::W));
              pv_issued = true;
            } else {
              bad = true;
              if (lane == 0) give_up();  // the group stops at its next barrier
            }
            if (lane == 0) {
              // the dim role's factors for this tile and unit (tp[buf] was
              // read for tile i - 2)
              float *t = tp + (buf * U + u) * 3 * ROWS;
#pragma unroll
              for (int r = 0; r < ROWS; ++r) {
                t[r] = alpha[r];
                t[ROWS + r] = sp[0][r];
                t[2 * ROWS + r] = sp[1][r];
              }
              mbar_arrive1(bar(kTpB + buf));
            }
          }
        }
        if (last) {
          // the unit's row sums and bias sums of the piece over its tokens
          // (zero, with m = -inf, when it had no token of the piece)
          float v[3 * ROWS];
#pragma unroll
          for (int r = 0; r < ROWS; ++r) {
            v[r] = l[r];
            v[ROWS + r] = rb[0][r];
            v[2 * ROWS + r] = rb[1][r];
          }
#pragma unroll
          for (int e = 0; e < 3 * ROWS; ++e)
#pragma unroll
            for (int o = 16; o; o >>= 1) v[e] += __shfl_xor_sync(0xffffffffu, v[e], o);
          if constexpr (WPU > 1) {
            if (lane == 0)
#pragma unroll
              for (int e = 0; e < 3 * ROWS; ++e) lx[wq * 3 * ROWS + e] = v[e];
          }
          if (unit_or(bad || *abort_flag != 0)) {
            bad = true;
            break;
          }
          if (issuer && lane == 0) {
            if (k >= 2 && !bad && !wait_b(kPeEmpty + (k & 1), ((k - 2) >> 1) & 1)) bad = true;
            float *pk = pe + ((k & 1) * TGN * U + uslot) * 4 * ROWS;
#pragma unroll
            for (int e = 0; e < 3 * ROWS; ++e) {
              float sum = v[e];
#pragma unroll
              for (int w = 1; w < WPU; ++w) sum += lx[(wq + w) * 3 * ROWS + e];
              pk[ROWS + e] = sum;
            }
#pragma unroll
            for (int r = 0; r < ROWS; ++r) pk[r] = m[r];
            mbar_arrive1(bar(kPeB + (k & 1)));
          }
          if constexpr (WPU > 1) bar_sync_n(ubar, 32 * WPU);  // lx read before the next piece writes it
        }
        adv(c, p);
      }
    }
    // this warp's PVs complete before the TMEM is freed
    if (pv_issued) {
      tc::commit_elect(bar(kDrainT + uslot));
      (void)wait_b(kDrainT + uslot, 0);
    }
    if (bad && lane == 0) give_up();
  }
  else {
    // ---------------- dim role ----------------
    const int q = 32 * (warp & 3) + lane;  // operand row = TMEM lane
    const int dim = dim_of<BITS>(q);
    const int g = q >> 6;
    const int wq = warp & 3;  // quadrants 0, 1 hold dims of group 0, quadrants 2, 3 group 1
    const uint32_t tl = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const float *tp = reinterpret_cast<const float *>(misc + C::kTp);
    const float *pe = reinterpret_cast<const float *>(misc + C::kPe);
    int *qx = reinterpret_cast<int *>(misc + C::kQx);
    float *qp = reinterpret_cast<float *>(misc + C::kQp);
    float *qs = reinterpret_cast<float *>(misc + C::kQs);

    // Q operand of a piece (pair c) into buffer kk & 1, with its scale and
    // per-group sums for the token groups; thread = operand row (head dim
    // dim_of(q)).  Plain named barriers: no waits inside.
    auto write_q = [&](int kk, const TCur &c) {
      float qv[ROWS];
      uint32_t am[ROWS];
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        qv[r] = ld_q(p.q, row_offset(p.q_sb, p.q_st, p.q_sh, c.b, c.h, r, p.G) + dim, p.q_bf16);
        am[r] = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(qv[r])));
      }
      if (lane == 0)
#pragma unroll
        for (int r = 0; r < ROWS; ++r) qx[wq * ROWS + r] = static_cast<int>(am[r]);
      bar_sync_n(C::kBarDim, 128);
      float inv[ROWS], sq[ROWS];
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        uint32_t mxv = 0;
#pragma unroll
        for (int w = 0; w < 4; ++w) mxv = max(mxv, static_cast<uint32_t>(qx[w * ROWS + r]));
        const float amax = __uint_as_float(mxv);
        sq[r] = amax / 32767.f;
        inv[r] = amax > 0.f ? 32767.f / amax : 0.f;
      }
      bar_sync_n(C::kBarDim, 128);  // every thread has read qx
      uint32_t u[ROWS];
      int isum[ROWS];
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        const int qi = max(-32767, min(32767, __float2int_rn(qv[r] * inv[r])));
        u[r] = static_cast<uint32_t>(qi + 32768);
        isum[r] = __reduce_add_sync(0xffffffffu, qi);
      }
      if (lane == 0)
#pragma unroll
        for (int r = 0; r < ROWS; ++r) qx[wq * ROWS + r] = isum[r];
      store_brow<ROWS, C::kUnits>(smem + C::kQb + (kk & 1) * C::kBop, q, u);
      fence_proxy_async_smem();
      bar_sync_n(C::kBarDim, 128);
      if (q == 0) {
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
          qp[(kk & 1) * ROWS + r] = sq[r];
          qs[((kk & 1) * 2 + 0) * ROWS + r] = sq[r] * static_cast<float>(qx[0 * ROWS + r] + qx[1 * ROWS + r]);
          qs[((kk & 1) * 2 + 1) * ROWS + r] = sq[r] * static_cast<float>(qx[2 * ROWS + r] + qx[3 * ROWS + r]);
        }
      }
      bar_sync_n(C::kBarDim, 128);  // qp / qs written, qx free again
      mbar_arrive1(bar(kQFull + (kk & 1)));
    };

    // sequences without context: zero outputs (CTA b mod grid)
    for (int b = blockIdx.x; b < p.B; b += gridDim.x) {
      if (clamped_ctx(p, b) != 0) continue;
      for (int h = 0; h < p.Hkv; ++h)
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
          store_one(p, row_offset(p.o_sb, p.o_st, p.o_sh, b, h, r, p.G) + dim, 0.f);
    }
    bool bad = false;
    if (cnt > 0) {
      TCur c = locate_tc(p, x0, lane);
      write_q(0, c);
      // the second piece's Q, if the share reaches past the first pair
      if (x0 + (c.n - c.t) < x0 + cnt) write_q(1, next_pair(c, p));
      constexpr int U = C::U;
      float o[TGN * U][ROWS];  // per unit (token group t, unit u at t * U + u)
#pragma unroll
      for (int t = 0; t < TGN * U; ++t)
#pragma unroll
        for (int r = 0; r < ROWS; ++r) o[t][r] = 0.f;
      // 4-bit: tile j's codes are widened into slot j % W kWidenAhead tiles
      // before the dim role reaches tile j (the slot's previous tile, j - W,
      // had its O read already); the stage is released to the copies
      auto widen = [&](int j) {
        const int sj = j % S, wj = j % C::W;
        if (!bad && !wait_b(kFull + sj, (j / S) & 1)) bad = true;
        if (j >= C::W && !bad && !wait_b(kWEmpty + wj, ((j - C::W) / C::W) & 1)) bad = true;
        widen_row(stage(sj) + C::kKr, wide(wj) + C::kKc, q);
        widen_row(stage(sj) + C::kVr, wide(wj) + C::kVc, q);
        static_assert(C::kScBytes == 128 * 16, "one 16-byte piece of the scales per thread");
        *reinterpret_cast<uint4 *>(wide(wj) + C::kWSc + 16 * q) =
            *reinterpret_cast<const uint4 *>(stage(sj) + C::kSc + 16 * q);
        fence_proxy_async_smem();
        mbar_arrive1(bar(kKx + wj));
        mbar_arrive1(bar(kVx + wj));
        mbar_arrive1(bar(kEmpty + sj));
      };
      if constexpr (BITS == 4)
        for (int j = 0; j < C::kWidenAhead && j < cnt; ++j) widen(j);
      int k = -1;
      for (int i = 0; i < cnt; ++i) {
        const int buf = i & 1;
        const bool first = (i == 0) || (c.t == 0);
        const bool last = (i == cnt - 1) || (c.t == c.n - 1);
        if (first) {
          ++k;
          // the next piece's Q: every QK of the piece before this one is
          // complete (O of the tile before has been read)
          if (k >= 1 && x0 + i + (c.n - c.t) < x0 + cnt) write_q(k + 1, next_pair(c, p));
        }
        if constexpr (BITS == 4) {
          if (i + C::kWidenAhead < cnt) widen(i + C::kWidenAhead);
        }
        if (!bad && !(wait_b(kOFull + buf, (i >> 1) & 1) && wait_b(kTpB + buf, (i >> 1) & 1)))
          bad = true;
        if (__any_sync(0xffffffffu, bad)) bad = true;
        tc::fence_after_sync();
        const int gi = i % TGN;
#pragma unroll
        for (int uu = 0; uu < U; ++uu) {
          uint32_t orr[NB];
#pragma unroll
          for (int j = 0; j < NB; j += 16) {
            uint32_t r16[16];
            tc::ld16(tl + kO0 + ((buf * U + uu) * 2 + g) * NB + j, r16);
#pragma unroll
            for (int e = 0; e < 16; ++e) orr[j + e] = r16[e];
          }
          tc::wait_ld();
          const float *t = tp + (buf * U + uu) * 3 * ROWS;
#pragma unroll
          for (int tt = 0; tt < TGN; ++tt) {
            if (tt != gi) continue;
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
              const int v = static_cast<int>(orr[r] * 256u + orr[ROWS + r] - (orr[2 * ROWS] << 15));
              o[tt * U + uu][r] = fmaf(o[tt * U + uu][r], t[r], t[(1 + g) * ROWS + r] * static_cast<float>(v));
            }
          }
        }
        tc::fence_before_sync();
        mbar_arrive1(bar(kOEmpty + buf));
        if (last) {
          // combine the units' states: weights 2^(m_u - M)
          if (!bad && !wait_b(kPeB + (k & 1), (k >> 1) & 1)) bad = true;
          float mr[ROWS], lr[ROWS], num[ROWS];
#pragma unroll
          for (int r = 0; r < ROWS; ++r) {
            float M = -INFINITY;
#pragma unroll
            for (int t = 0; t < TGN * U; ++t) M = fmaxf(M, pe[((k & 1) * TGN * U + t) * 4 * ROWS + r]);
            float L = 0.f, n = 0.f;
#pragma unroll
            for (int t = 0; t < TGN * U; ++t) {
              const float *pk = pe + ((k & 1) * TGN * U + t) * 4 * ROWS;
              const float w = pk[r] > -INFINITY ? fast_exp2(pk[r] - M) : 0.f;
              L = fmaf(w, pk[ROWS + r], L);
              n = fmaf(w, o[t][r] + pk[(2 + g) * ROWS + r], n);
            }
            mr[r] = M;
            lr[r] = L;
            num[r] = n;
          }
          mbar_arrive1(bar(kPeEmpty + (k & 1)));
          const int bh = c.b * p.Hkv + c.h;
          const int pbh = x0 + i - c.t;  // flat index of the pair's first tile
          const int uf = pbh / per, ul = (pbh + c.n - 1) / per;
          if (uf == ul) {
#pragma unroll
            for (int r = 0; r < ROWS; ++r)
              store_one(p, row_offset(p.o_sb, p.o_st, p.o_sh, c.b, c.h, r, p.G) + dim,
                        num[r] / lr[r]);
          } else {
            // partial of this piece; the last piece to arrive merges them all
            const int64_t slot = (int64_t)blockIdx.x + bh;
#pragma unroll
            for (int r = 0; r < ROWS; ++r) p.part[(slot * ROWS + r) * kD + dim] = num[r];
            if (q == 0)
#pragma unroll
              for (int r = 0; r < ROWS; ++r)
                *reinterpret_cast<float2 *>(p.ml + (slot * ROWS + r) * 2) = make_float2(mr[r], lr[r]);
            __threadfence();
            if (bar_or(C::kBarDim, 128, bad || *abort_flag != 0)) {
              bad = true;
              break;
            }
            const int nparts = ul - uf + 1;
            if (q == 0) *merge_word = atomicAdd(p.counters + bh, 1);
            bar_sync_n(C::kBarDim, 128);
            const int old = *merge_word;
            bar_sync_n(C::kBarDim, 128);  // merge_word read before it is written again
            if (old == nparts - 1) {
              __threadfence();
#pragma unroll
              for (int r = 0; r < ROWS; ++r) {
                float M = -INFINITY;
                for (int u = 0; u < nparts; ++u)
                  M = fmaxf(M, __ldcg(p.ml + (((int64_t)uf + u + bh) * ROWS + r) * 2));
                float nm = 0.f, den = 0.f;
                for (int u = 0; u < nparts; ++u) {
                  const int64_t sl = (int64_t)uf + u + bh;
                  const float2 ml = __ldcg(reinterpret_cast<const float2 *>(p.ml + (sl * ROWS + r) * 2));
                  const float w = fast_exp2(ml.x - M);
                  nm = fmaf(__ldcg(p.part + (sl * ROWS + r) * kD + dim), w, nm);
                  den = fmaf(ml.y, w, den);
                }
                store_one(p, row_offset(p.o_sb, p.o_st, p.o_sh, c.b, c.h, r, p.G) + dim, nm / den);
              }
              if (q == 0) p.counters[bh] = 0;
            }
          }
#pragma unroll
          for (int t = 0; t < TGN * U; ++t)
#pragma unroll
            for (int r = 0; r < ROWS; ++r) o[t][r] = 0.f;
        }
        adv(c, p);
      }
    }
    if (bad && lane == 0) give_up();
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, C::kTmemCols);
  }
}

// 2-D map over a code pool seen as rows of `rb` bytes, box rb x 16 rows,
// swizzle matching the row width (128 or 64 bytes).
int make_code_map(CUtensorMap *m, const void *base, int64_t rows, int rb) {
  auto fn = encode_fn();
  if (!fn) return fail(MZ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(rb), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(rb)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(rb), 16};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  rb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MZ_ERR_CUDA, "cuTensorMapEncodeTiled (codes) failed (%d)", (int)r);
  return MZ_OK;
}

template <int BITS, int ROWS>
int launch_one(const Params &p, const CUtensorMap &tk, const CUtensorMap &tv, int grid,
               cudaStream_t s) {
  static DeviceOnce once;
  if (int rc = smem_optin(paged_decode_qtc_kernel<BITS, ROWS>, Cfg<BITS, ROWS>::kSmemBytes, once,
                          "quantised decode (tcgen05): shared memory attribute"))
    return rc;
  paged_decode_qtc_kernel<BITS, ROWS><<<grid, Cfg<BITS, ROWS>::kThreads, Cfg<BITS, ROWS>::kSmemBytes, s>>>(tk, tv, p);
  MZ_CHECK_LAUNCH("mz_paged_decode_q (tcgen05)");
  return MZ_OK;
}

}  // namespace qtc

bool qtc_supports(int head_dim, int rows) {
  return head_dim == qtc::kD && (rows == 1 || rows == 2 || rows == 4 || rows == 8 || rows == 16);
}

// Grid of the tcgen05 kernel: one CTA per SM.
int qtc_grid(int device) { return sm_count(device); }

int launch_decode_q_tc(const Params &p, int bits, int64_t rows_total, int grid, cudaStream_t s) {
  if (rows_total >= (int64_t(1) << 31)) return fail(MZ_ERR_UNSUPPORTED, "mz_paged_decode_q: pool has >= 2^31 rows");
  CUtensorMap tk{}, tv{};
  const int rb = qtc::kD * bits / 8;
  if (int rc = qtc::make_code_map(&tk, p.kq, rows_total, rb)) return rc;
  if (int rc = qtc::make_code_map(&tv, p.vq, rows_total, rb)) return rc;
#define MZ_QTC(B_, R_) return qtc::launch_one<B_, R_>(p, tk, tv, grid, s)
  if (bits == 8) {
    switch (p.rows) {
      case 1: MZ_QTC(8, 1);
      case 2: MZ_QTC(8, 2);
      case 4: MZ_QTC(8, 4);
      case 8: MZ_QTC(8, 8);
      case 16: MZ_QTC(8, 16);
    }
  } else {
    switch (p.rows) {
      case 1: MZ_QTC(4, 1);
      case 2: MZ_QTC(4, 2);
      case 4: MZ_QTC(4, 4);
      case 8: MZ_QTC(4, 8);
      case 16: MZ_QTC(4, 16);
    }
  }
#undef MZ_QTC
  return fail(MZ_ERR_UNSUPPORTED, "mz_paged_decode_q (tcgen05): %d rows", p.rows);
}

}  // namespace decode
}  // namespace mz
