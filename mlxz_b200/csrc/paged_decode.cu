// Fused GQA paged decode attention for sm_100a, bf16 / fp16 K/V.
//
// Scheduling (persistent warps, flat tile list, static shares + optional
// dynamic chunks, merge of split pairs by the last-arriving piece) lives in
// decode_common.cuh.  Per warp, a STAGES-deep ring of shared-memory stages is
// filled by 2-D bulk tensor copies (cp.async.bulk.tensor, 128-byte swizzle, no
// multicast) that complete on per-stage mbarriers; lane 0 issues, all lanes
// consume.  The grouped query rows (n_q * G <= 16) form the M=16 side of
// mma.sync m16n8k16: S = Q.K^T over the tile (2 n-tiles of 8 tokens), an fp32
// online softmax in the exp2 domain, then O += P.V (D/8 n-tiles).  For bf16, P
// is split into hi + lo bf16 parts so P.V carries ~16 mantissa bits of P.
//
// Optional fused append (decode step): the new token of each sequence, the
// last one attended, is written into its pool slot and patched into the staged
// tile before use, so no separate append launch is needed.
//
// Roofline: each tile moves 2 * 16 * D * 2 bytes (K and V) and needs
// 4 * rows * 16 * D flops; with rows = 4 (GQA group 4) that is 2 flop/byte,
// so the kernel is HBM-bound and the bulk-copy pipeline depth is what matters.
// Measured on B200, per-warp streaming rates differ by 5-10 %, which leaves a
// tail, but dynamic chunks cost more than they save (8B shape, batch 64: 196
// us static, 237 us with 15 % in 9-tile chunks: every chunk adds a piece to
// merge), so the default hands out everything statically; merges of split
// pairs are deferred to the end of each warp's loop.
#include "decode_common.cuh"

#ifndef MZ_DECODE_STAGES_D128
#define MZ_DECODE_STAGES_D128 3
#endif

namespace mz {
namespace decode {

template <int D>
struct Cfg {
  static constexpr int kStages = (D == 64) ? 6 : MZ_DECODE_STAGES_D128;
  static constexpr int kTileBytes = kTileTok * D * 2;        // one of K or V
  static constexpr int kStageBytes = 2 * kTileBytes;         // K + V
  static constexpr int kSmemTiles = kWarps * kStages * kStageBytes;
  static constexpr int kSmemBars = kWarps * kStages * 8;
  static constexpr int kSmemUnits = kWarps * kUnitQ * static_cast<int>(sizeof(Unit));
  static constexpr int kSmemDefer = kWarps * kMaxDeferred * static_cast<int>(sizeof(Deferred));
  static constexpr int kSmemBytes = kSmemTiles + kSmemBars + kSmemUnits + kSmemDefer + 1024;
};

template <int D, bool BF16, bool GATHER>
__device__ __forceinline__ void decode_tiles(const CUtensorMap &tmK, const CUtensorMap &tmV,
                                             const Params &p) {
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
  Unit *uq = reinterpret_cast<Unit *>(smem + C::kSmemTiles + C::kSmemBars) + warp * kUnitQ;
  Deferred *dq = reinterpret_cast<Deferred *>(smem + C::kSmemTiles + C::kSmemBars + C::kSmemUnits) +
                 warp * kMaxDeferred;
  int nd = 0;  // merges this warp owns, run after its tile loop
  const uint32_t bar0 = smem_u32(bars);
  const uint32_t stage0 = smem_u32(stages);

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(bar0 + 8 * s, 1);
    fence_mbar_init();
  }
  __syncwarp();

  Sched sch;
  const bool any_work = sch.init(p, lane, wid, W, uq);  // T == 0: no counter is touched

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

  // Per-lane ldmatrix geometry.
  const int mi = lane >> 3, r8 = lane & 7;
  const int tokK = r8 + 8 * (mi >> 1), subK = mi & 1;  // K: m0,m1 tok 0-7; m2,m3 tok 8-15
  const int tokV = r8 + 8 * (mi & 1), subV = mi >> 1;  // V: m0,m2 tok 0-7; m1,m3 tok 8-15
  const int g = lane >> 2, cq = lane & 3;              // mma fragment row / column-pair

  uint32_t qa[KS][4];
  float oacc[NT][4];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const bool two_groups = p.rows > 8;

  UnitReader ur;
  bool seg_first = true;

  // Until the launch ahead has completed (programmatic dependent launch) only
  // ctx, the tables and the pools are read: the first tiles of the static
  // share are already on their way when the wait returns.
  if (any_work) sch.prefetch_static<S>(p, issue);
  wait_for_previous_grid();
  if constexpr (GATHER) wait_peers_previous(p);
  zero_empty_outputs<D, GATHER>(p, wid, W, lane);
  if (!any_work) return;

  sch.refill<S>(p, 0, issue);
  bool ring_idle = true;
  for (int i = 0; i < sch.issued; ++i) {
    const int s = i % S;
    if (ur.need_pop()) {
      ur.pop(uq);
      seg_first = true;
    }
    const Cursor &cc = ur.cc;

    if (seg_first || cc.t == 0) {
      // New piece: load the grouped query rows as A fragments.
      seg_first = false;
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

    if (!wait_stage<S>(p, bar0, i, sch.issued, lane)) {
      ring_idle = false;
      break;
    }

    uint8_t *kt = stages + s * C::kStageBytes;
    uint8_t *vt = kt + C::kTileBytes;
    const uint32_t kb = stage0 + s * C::kStageBytes;
    const uint32_t vb = kb + C::kTileBytes;
    const int nvalid = min(kTileTok, cc.ctx - cc.t * kTileTok);
    const bool last_tile = (cc.t == cc.n - 1);
    if (p.kn != nullptr && last_tile) {
      // Fused append: the sequence's new token is its last attended one.  Write
      // it to its pool slot and into the staged tile (which may predate it).
      const int pos = cc.ctx - 1;
      const int row = pos & (kTileTok - 1);
      constexpr int U = D / 8;  // 16-byte units per row
      if (lane < 2 * U) {
        const bool is_v = lane >= U;
        const int d = (lane - (is_v ? U : 0)) * 8;
        const uint16_t *src =
            (is_v ? p.vn : p.kn) + (int64_t)cc.b * p.kn_sb + (int64_t)cc.h * p.kn_sh + d;
        const uint4 val = *reinterpret_cast<const uint4 *>(src);
        *reinterpret_cast<uint4 *>((is_v ? vt : kt) + swz128(row, 2 * d)) = val;
        const int32_t blk = p.tables[(int64_t)cc.b * p.max_blocks + pos / p.bs];
        if (blk >= 0 && blk < p.n_blocks) {
          uint16_t *dst = (is_v ? p.v_pool : p.k_pool) +
                          ((((int64_t)blk * p.Hkv + cc.h) * p.bs + pos % p.bs) * D + d);
          *reinterpret_cast<uint4 *>(dst) = val;
        }
      }
      __syncwarp();
    }
    if (nvalid < kTileTok) {
      // Rows past the context may hold stale data; make them exact zeros so
      // that 0 * V stays 0 in P.V.
      for (int e = lane; e < (kTileTok - nvalid) * (D / 8); e += 32) {
        const int tok = nvalid + e / (D / 8), d = (e % (D / 8)) * 8;
        *reinterpret_cast<uint4 *>(vt + swz128(tok, 2 * d)) = make_uint4(0, 0, 0, 0);
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
      ldsm_x4(kb + swz128(tokK, 2 * (16 * j + 8 * subK)), b0, b1, b2, b3);
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
    if (__any_sync(0xffffffffu, a0 != 1.f || a1 != 1.f)) {
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        oacc[n][0] *= a0;
        oacc[n][1] *= a0;
        oacc[n][2] *= a1;
        oacc[n][3] *= a1;
      }
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
      ldsm_x4_trans(vb + swz128(tokV, 2 * (16 * j + 8 * subV)), v0, v1, v2, v3);
      mma_16816<BF16>(oacc[2 * j], ph_, v0, v1);
      mma_16816<BF16>(oacc[2 * j + 1], ph_, v2, v3);
      if constexpr (BF16) {
        mma_16816<BF16>(oacc[2 * j], pl_, v0, v1);
        mma_16816<BF16>(oacc[2 * j + 1], pl_, v2, v3);
      }
    }

    // Piece end: last tile of the pair, or last tile of the unit.
    if (last_tile || ur.left == 1) {
      float L0 = l0, L1 = l1;
      L0 += __shfl_xor_sync(0xffffffffu, L0, 1);
      L0 += __shfl_xor_sync(0xffffffffu, L0, 2);
      L1 += __shfl_xor_sync(0xffffffffu, L1, 1);
      L1 += __shfl_xor_sync(0xffffffffu, L1, 2);
      const int bh = cc.b * p.Hkv + cc.h;
      const int pbh = cc.pos - cc.t;  // flat index of tile 0 of this pair
      // units holding the pair's first and last piece (batch-invariant: the
      // pair's pieces are the consecutive units W + fp ...)
      const int uf = p.batch_invariant ? sch.W + ur.fp : sch.unit_of(pbh);
      const int ul = p.batch_invariant ? uf + ur.np - 1 : sch.unit_of(pbh + cc.n - 1);
      if (uf == ul) {
        const float i0 = 1.f / L0, i1 = two_groups ? 1.f / L1 : 0.f;
        if (g < p.rows) {
          const int64_t o = row_offset(p.o_sb, p.o_st, p.o_sh, cc.b, cc.h, g, p.G);
#pragma unroll
          for (int n = 0; n < NT; ++n)
            store_pair(p, o + n * 8 + 2 * cq, oacc[n][0] * i0, oacc[n][1] * i0);
        }
        if (g + 8 < p.rows) {
          const int64_t o = row_offset(p.o_sb, p.o_st, p.o_sh, cc.b, cc.h, g + 8, p.G);
#pragma unroll
          for (int n = 0; n < NT; ++n)
            store_pair(p, o + n * 8 + 2 * cq, oacc[n][2] * i1, oacc[n][3] * i1);
        }
        if constexpr (GATHER) forward_rows<D>(p, cc.b, cc.h, lane);
      } else {
        const int64_t slot = (int64_t)ur.unit + bh;
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
        arrive_or_defer<D, GATHER>(p, cc, bh, uf, ul - uf + 1, lane, dq, nd);
      }
      seg_first = true;  // the next tile starts a new piece
    }

    __syncwarp();
    --ur.left;
    advance(ur.cc, p);
    sch.refill<S>(p, i + 1, issue);
  }
  run_deferred<D, GATHER>(p, dq, nd, stages, S * C::kStageBytes, ring_idle, lane);
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kWarps * 32, 2)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const Params p) {
  launch_dependents();
  decode_tiles<D, BF16, false>(tmK, tmV, p);
}

// The all-gather instantiation: every output store also goes to the peers'
// buffers, and the grid's last block signals them.
template <int D, bool BF16>
__global__ void __launch_bounds__(kWarps * 32, 2)
    paged_decode_gather_kernel(const __grid_constant__ CUtensorMap tmK,
                               const __grid_constant__ CUtensorMap tmV, const Params p) {
  launch_dependents();
  decode_tiles<D, BF16, true>(tmK, tmV, p);
  gather_arrive(p);
}


// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------

// Tensor map over a pool seen as rows of `D` 16-bit elements, box 64 x 16.
int make_pool_map(CUtensorMap *m, const void *pool, int64_t rows, int D, bool bf16) {
  return make_row_map(m, pool, rows, D,
                      bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                      64);
}

template <int D, bool BF16>
int kernel_ctas_per_sm(int *out) {
  static DeviceOnce once;
  return kernel_occupancy(paged_decode_kernel<D, BF16>, Cfg<D>::kSmemBytes, once, out);
}

// Dynamic shared-memory opt-in for the all-gather instantiation (once per device).
template <int D, bool BF16>
int gather_smem_attr() {
  static DeviceOnce once;
  return smem_optin(paged_decode_gather_kernel<D, BF16>, Cfg<D>::kSmemBytes, once,
                    "setting the all-gather kernel's shared memory");
}

int ctas_per_sm(int D, bool bf16, int *out) {
  if (D == 128) return bf16 ? kernel_ctas_per_sm<128, true>(out) : kernel_ctas_per_sm<128, false>(out);
  return bf16 ? kernel_ctas_per_sm<64, true>(out) : kernel_ctas_per_sm<64, false>(out);
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

// Everything a decode launch needs besides its scratch.
struct DecodeArgs {
  void *out;
  int32_t out_dtype;
  int64_t o_sb, o_st, o_sh;
  const void *q;
  int64_t q_sb, q_st, q_sh;
  int32_t n_q;
  const void *k_pool, *v_pool;
  const int32_t *tables;
  int32_t max_blocks;
  const int32_t *ctx;
  int32_t B, Hq, Hkv, D, bs;
  int64_t n_blocks;
  float scale;
  int32_t dtype, num_warps;
  const void *kn, *vn;
  int64_t kn_sb, kn_sh;
  int32_t *err;
  cudaStream_t stream;
  const mz_peer_outputs *peers = nullptr;  // all-gather over peer memory, or none
  uint32_t flags = 0;                      // MZ_LAUNCH_*
};

// The most pieces a batch-invariant launch cuts: every pair at full capacity.
inline int64_t bi_max_pieces(int64_t B, int64_t Hkv, int64_t max_blocks, int bs) {
  const int64_t tiles = max_blocks * (bs / kTileTok);
  return B * Hkv * ((tiles + kBiPieceTiles - 1) / kBiPieceTiles);
}

// Host-side checks shared by the entry points; fills the resolved warp count
// and workspace layout.
int validate(const DecodeArgs &a, const char *fn, int64_t *warps, WsLayout *ws) {
  if (a.dtype != MZ_DTYPE_F16 && a.dtype != MZ_DTYPE_BF16)
    return fail(MZ_ERR_UNSUPPORTED, "%s: dtype must be F16 or BF16", fn);
  if (a.out_dtype != a.dtype && a.out_dtype != MZ_DTYPE_F32)
    return fail(MZ_ERR_UNSUPPORTED, "%s: out_dtype must equal dtype or be F32", fn);
  if (a.D != 64 && a.D != 128)
    return fail(MZ_ERR_UNSUPPORTED, "%s: head_dim %d (supported: 64, 128)", fn, a.D);
  if (a.bs <= 0 || a.bs % kTileTok)
    return fail(MZ_ERR_UNSUPPORTED, "%s: block_size %d is not a multiple of 16", fn, a.bs);
  if (a.B < 0 || a.Hkv <= 0 || a.Hq <= 0 || a.Hq % a.Hkv || a.n_q <= 0 || a.max_blocks <= 0 ||
      a.n_blocks <= 0)
    return fail(MZ_ERR_INVALID_ARG, "%s: bad sizes", fn);
  const int rows = a.n_q * (a.Hq / a.Hkv);
  if (rows > 16)
    return fail(MZ_ERR_UNSUPPORTED, "%s: n_q_tokens * (n_heads / n_kv_heads) = %d exceeds 16", fn,
                rows);
  if (!std::isfinite(a.scale)) return fail(MZ_ERR_INVALID_ARG, "%s: scale not finite", fn);
  if (a.B == 0) return MZ_OK;
  if (!a.out || !a.q || !a.k_pool || !a.v_pool || !a.tables || !a.ctx)
    return fail(MZ_ERR_INVALID_ARG, "%s: null pointer", fn);
  if (!aligned(a.k_pool, 16) || !aligned(a.v_pool, 16) || !aligned(a.q, 4) || (a.q_sb & 1) ||
      (a.q_st & 1) || (a.q_sh & 1))
    return fail(MZ_ERR_ALIGNMENT,
                "%s: pools need 16-byte alignment, q 4-byte alignment and even strides", fn);
  const int ob = a.out_dtype == MZ_DTYPE_F32 ? 8 : 4;
  if (!aligned(a.out, ob) || (a.o_sb & 1) || (a.o_st & 1) || (a.o_sh & 1))
    return fail(MZ_ERR_ALIGNMENT, "%s: out needs %d-byte alignment and even strides", fn, ob);
  if (a.kn || a.vn) {
    if (!a.kn || !a.vn || !aligned(a.kn, 16) || !aligned(a.vn, 16) || (a.kn_sb % 8) ||
        (a.kn_sh % 8))
      return fail(MZ_ERR_ALIGNMENT,
                  "%s: k_new/v_new need 16-byte alignment and strides that are multiples of 8", fn);
    if (a.n_q != 1) return fail(MZ_ERR_UNSUPPORTED, "%s: fused append needs n_q_tokens == 1", fn);
  }
  if (a.peers) {
    const mz_peer_outputs &pe = *a.peers;
    if (pe.n_ranks < 1 || pe.n_ranks > MZ_MAX_RANKS || pe.rank < 0 || pe.rank >= pe.n_ranks)
      return fail(MZ_ERR_INVALID_ARG, "%s: n_ranks %d / rank %d out of range (1..%d ranks)", fn,
                  pe.n_ranks, pe.rank, MZ_MAX_RANKS);
    if (pe.epoch == 0) return fail(MZ_ERR_INVALID_ARG, "%s: epoch must be nonzero", fn);
    if (a.o_sh != a.D || (a.o_sb * (ob / 2)) % 16 != 0)
      return fail(MZ_ERR_INVALID_ARG,
                  "%s: the gathered buffer needs dense rows (out_head_stride == head_dim) and "
                  "16-byte aligned sequence rows", fn);
    if (!pe.arrivals || !aligned(pe.arrivals, 4))
      return fail(MZ_ERR_INVALID_ARG, "%s: arrivals must be a 4-byte aligned device word", fn);
    for (int r = 0; r < pe.n_ranks; ++r) {
      if (!pe.out[r] || !aligned(pe.out[r], 16))
        return fail(MZ_ERR_ALIGNMENT, "%s: out[%d] is null or not 16-byte aligned", fn, r);
      if (r != pe.rank && (!pe.signal[r] || !aligned(pe.signal[r], 4)))
        return fail(MZ_ERR_INVALID_ARG, "%s: signal[%d] is null or misaligned", fn, r);
    }
  }
  const int64_t rows_total = a.n_blocks * a.Hkv * a.bs;
  if (rows_total >= (int64_t(1) << 31))
    return fail(MZ_ERR_UNSUPPORTED, "%s: pool has >= 2^31 rows", fn);
  if ((int64_t)a.B * a.Hkv * a.max_blocks * (a.bs / kTileTok) >= (int64_t(1) << 30))
    return fail(MZ_ERR_UNSUPPORTED, "%s: more than 2^30 tiles of context", fn);
  const int device = current_device();
  if (int rc = resolve_warps(a.D, a.dtype == MZ_DTYPE_BF16, a.num_warps, device, warps)) return rc;
  *ws = ws_layout((int64_t)a.B * a.Hkv, *warps, rows, a.D,
                  (a.flags & MZ_DECODE_BATCH_INVARIANT) ? bi_max_pieces(a.B, a.Hkv, a.max_blocks, a.bs) : 0);
  return MZ_OK;
}

// Launch with scratch at `scratch`; `clear_counters` zeroes the counter words
// on the stream first (for scratch that does not start zeroed).
int launch(const DecodeArgs &a, int64_t warps, const WsLayout &ws, void *scratch,
           bool clear_counters, const char *fn) {
  if (!aligned(scratch, 256)) return fail(MZ_ERR_ALIGNMENT, "%s: workspace must be 256-byte aligned", fn);
  const bool bf16 = a.dtype == MZ_DTYPE_BF16;
  const int64_t rows_total = a.n_blocks * a.Hkv * a.bs;
  CUtensorMap tk, tv;
  if (int rc = make_pool_map(&tk, a.k_pool, rows_total, a.D, bf16)) return rc;
  if (int rc = make_pool_map(&tv, a.v_pool, rows_total, a.D, bf16)) return rc;

  Params p;
  p.out = a.out;
  p.o_sb = a.o_sb;
  p.o_st = a.o_st;
  p.o_sh = a.o_sh;
  p.out_f32 = a.out_dtype == MZ_DTYPE_F32;
  p.q = a.q;
  p.q_sb = a.q_sb;
  p.q_st = a.q_st;
  p.q_sh = a.q_sh;
  p.n_q = a.n_q;
  p.G = a.Hq / a.Hkv;
  p.rows = a.n_q * p.G;
  p.tables = a.tables;
  p.max_blocks = a.max_blocks;
  p.ctx = a.ctx;
  p.B = a.B;
  p.Hkv = a.Hkv;
  p.bs = a.bs;
  p.tpb = a.bs / kTileTok;
  p.n_blocks = a.n_blocks;
  p.scale_log2 = static_cast<float>(static_cast<double>(a.scale) * 1.4426950408889634);
  p.kn = static_cast<const uint16_t *>(a.kn);
  p.vn = static_cast<const uint16_t *>(a.vn);
  p.kn_sb = a.kn_sb;
  p.kn_sh = a.kn_sh;
  p.k_pool = static_cast<uint16_t *>(const_cast<void *>(a.k_pool));
  p.v_pool = static_cast<uint16_t *>(const_cast<void *>(a.v_pool));
  auto *w8 = static_cast<uint8_t *>(scratch);
  p.counters = reinterpret_cast<int32_t *>(w8 + ws.counters);
  p.ml = reinterpret_cast<float *>(w8 + ws.ml);
  p.part = reinterpret_cast<float *>(w8 + ws.part);
  set_schedule(p, ws);
  p.q_bf16 = bf16;
  p.kq = p.vq = nullptr;
  p.k_scales = p.k_biases = p.v_scales = p.v_biases = nullptr;
  p.err = a.err;
  p.batch_invariant = (a.flags & MZ_DECODE_BATCH_INVARIANT) ? 1 : 0;
  if (a.peers) {
    const mz_peer_outputs &pe = *a.peers;
    p.out = pe.out[pe.rank];
    int j = 0;
    for (int r = 0; r < pe.n_ranks; ++r) {
      if (r == pe.rank) continue;
      p.peer_out[j] = pe.out[r];
      p.peer_sig[j] = reinterpret_cast<uint32_t *>(pe.signal[r]) + pe.rank;
      ++j;
    }
    p.n_peer = j;
    p.epoch = pe.epoch;
    p.arrivals = pe.arrivals;
    if (a.flags & MZ_LAUNCH_WAIT_PREVIOUS) {
      p.own_sig = reinterpret_cast<const uint32_t *>(pe.signal[pe.rank]);
      p.own_rank = pe.rank;
      p.n_ranks = pe.n_ranks;
      p.wait_epoch = pe.epoch == 1u ? 0xFFFFFFFFu : pe.epoch - 1u;  // epochs skip 0
    }
  }

  int per_sm = 0;  // also sets the kernel's shared-memory attribute (once)
  if (int rc = ctas_per_sm(a.D, bf16, &per_sm)) return rc;
  if (clear_counters) {
    cudaError_t e = cudaMemsetAsync(p.counters, 0, ws.counter_words * sizeof(int32_t), a.stream);
    if (e != cudaSuccess) return cuda_fail(e, "clearing decode counters");
  }
  const unsigned grid = static_cast<unsigned>(warps / kWarps);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (a.flags & MZ_LAUNCH_OVERLAP_PREVIOUS) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t le = cudaSuccess;
#define MZ_LAUNCH(D_, BF_)                                                          \
  do {                                                                              \
    cfg.dynamicSmemBytes = Cfg<D_>::kSmemBytes;                                     \
    if (a.peers) {                                                                  \
      if (int rc = gather_smem_attr<D_, BF_>()) return rc;                          \
      le = cudaLaunchKernelEx(&cfg, paged_decode_gather_kernel<D_, BF_>, tk, tv, p); \
    } else {                                                                        \
      le = cudaLaunchKernelEx(&cfg, paged_decode_kernel<D_, BF_>, tk, tv, p);       \
    }                                                                               \
  } while (0)
  if (a.D == 128) {
    if (bf16) MZ_LAUNCH(128, true); else MZ_LAUNCH(128, false);
  } else {
    if (bf16) MZ_LAUNCH(64, true); else MZ_LAUNCH(64, false);
  }
#undef MZ_LAUNCH
  if (le != cudaSuccess) return cuda_fail(le, fn);
  MZ_CHECK_LAUNCH(fn);
  return MZ_OK;
}

DecodeArgs make_args(void *out, int32_t out_dtype, int64_t out_seq_stride, int64_t out_tok_stride,
                     int64_t out_head_stride, const void *q, int64_t q_seq_stride,
                     int64_t q_tok_stride, int64_t q_head_stride, int32_t n_q_tokens,
                     const void *k_pool, const void *v_pool, const int32_t *block_tables,
                     int32_t max_blocks_per_seq, const int32_t *ctx_lens, int32_t n_seqs,
                     int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
                     int64_t n_blocks, float scale, int32_t dtype, int32_t num_warps,
                     int32_t *dev_err, mz_stream_t stream) {
  DecodeArgs a;
  a.out = out;
  a.out_dtype = out_dtype;
  a.o_sb = out_seq_stride;
  a.o_st = out_tok_stride;
  a.o_sh = out_head_stride;
  a.q = q;
  a.q_sb = q_seq_stride;
  a.q_st = q_tok_stride;
  a.q_sh = q_head_stride;
  a.n_q = n_q_tokens;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.tables = block_tables;
  a.max_blocks = max_blocks_per_seq;
  a.ctx = ctx_lens;
  a.B = n_seqs;
  a.Hq = n_heads;
  a.Hkv = n_kv_heads;
  a.D = head_dim;
  a.bs = block_size;
  a.n_blocks = n_blocks;
  a.scale = scale;
  a.dtype = dtype;
  a.num_warps = num_warps;
  a.kn = a.vn = nullptr;
  a.kn_sb = a.kn_sh = 0;
  a.err = dev_err;
  a.stream = static_cast<cudaStream_t>(stream);
  return a;
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
  if (int rc = resolve_warps(head_dim, true, num_warps, device, &warps)) return rc;
  *bytes = ws_layout((int64_t)n_seqs * n_kv_heads, warps, rows_per_kv_head, head_dim).total;
  return MZ_OK;
}

extern "C" int mz_paged_decode_workspace_size_ex(int32_t n_seqs, int32_t n_kv_heads,
                                                 int32_t rows_per_kv_head, int32_t head_dim,
                                                 int32_t num_warps, int32_t max_blocks_per_seq,
                                                 int32_t block_size, uint32_t flags,
                                                 int32_t device, size_t *bytes) {
  if (!bytes) return fail(MZ_ERR_INVALID_ARG, "bytes is null");
  if (n_seqs < 0 || n_kv_heads <= 0 || rows_per_kv_head <= 0 || rows_per_kv_head > 16 ||
      max_blocks_per_seq <= 0 || block_size <= 0 || block_size % kTileTok)
    return fail(MZ_ERR_INVALID_ARG, "workspace_size_ex: bad sizes");
  if (head_dim != 64 && head_dim != 128)
    return fail(MZ_ERR_UNSUPPORTED, "head_dim %d (supported: 64, 128)", head_dim);
  if (flags & ~(MZ_LAUNCH_OVERLAP_PREVIOUS | MZ_DECODE_BATCH_INVARIANT | MZ_LAUNCH_WAIT_PREVIOUS))
    return fail(MZ_ERR_INVALID_ARG, "workspace_size_ex: unknown flags");
  int64_t warps = 0;
  if (device < 0) device = current_device();
  if (int rc = resolve_warps(head_dim, true, num_warps, device, &warps)) return rc;
  const int64_t pieces = (flags & MZ_DECODE_BATCH_INVARIANT)
                             ? bi_max_pieces(n_seqs, n_kv_heads, max_blocks_per_seq, block_size)
                             : 0;
  *bytes = ws_layout((int64_t)n_seqs * n_kv_heads, warps, rows_per_kv_head, head_dim, pieces).total;
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
  const DecodeArgs a = make_args(out, out_dtype, out_seq_stride, out_tok_stride, out_head_stride,
                                 q, q_seq_stride, q_tok_stride, q_head_stride, n_q_tokens, k_pool,
                                 v_pool, block_tables, max_blocks_per_seq, ctx_lens, n_seqs,
                                 n_heads, n_kv_heads, head_dim, block_size, n_blocks, scale,
                                 dtype, num_warps, dev_err, stream);
  int64_t warps = 0;
  WsLayout ws;
  if (int rc = validate(a, "mz_paged_decode", &warps, &ws)) return rc;
  if (n_seqs == 0) return MZ_OK;
  if (!workspace) return fail(MZ_ERR_WORKSPACE, "mz_paged_decode: workspace is null");
  if (workspace_bytes < ws.total)
    return fail(MZ_ERR_WORKSPACE, "mz_paged_decode: workspace %zu bytes < required %zu",
                workspace_bytes, ws.total);
  return launch(a, warps, ws, workspace, false, "mz_paged_decode");
}

static int append_decode(void *out, int32_t out_dtype, int64_t out_seq_stride,
                         int64_t out_head_stride, const void *q, int64_t q_seq_stride,
                         int64_t q_head_stride, void *k_pool, void *v_pool, const void *k_new,
                         const void *v_new, int64_t new_seq_stride, int64_t new_head_stride,
                         const int32_t *block_tables, int32_t max_blocks_per_seq,
                         const int32_t *ctx_lens, int32_t n_seqs, int32_t n_heads,
                         int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
                         int64_t n_blocks, float scale, int32_t dtype, int32_t num_warps,
                         uint32_t flags, void *workspace, size_t workspace_bytes,
                         int32_t *dev_err, mz_stream_t stream, const char *fn) {
  DecodeArgs a = make_args(out, out_dtype, out_seq_stride, 0, out_head_stride, q, q_seq_stride, 0,
                           q_head_stride, 1, k_pool, v_pool, block_tables, max_blocks_per_seq,
                           ctx_lens, n_seqs, n_heads, n_kv_heads, head_dim, block_size, n_blocks,
                           scale, dtype, num_warps, dev_err, stream);
  a.kn = k_new;
  a.vn = v_new;
  a.kn_sb = new_seq_stride;
  a.kn_sh = new_head_stride;
  if (flags & ~(MZ_LAUNCH_OVERLAP_PREVIOUS | MZ_DECODE_BATCH_INVARIANT))
    return fail(MZ_ERR_INVALID_ARG, "%s: unknown flags", fn);
  a.flags = flags;
  if (!k_new || !v_new) return fail(MZ_ERR_INVALID_ARG, "%s: null k_new / v_new", fn);
  int64_t warps = 0;
  WsLayout ws;
  if (int rc = validate(a, fn, &warps, &ws)) return rc;
  if (n_seqs == 0) return MZ_OK;
  if (!workspace) return fail(MZ_ERR_WORKSPACE, "%s: workspace is null", fn);
  if (workspace_bytes < ws.total)
    return fail(MZ_ERR_WORKSPACE, "%s: workspace %zu bytes < required %zu", fn, workspace_bytes,
                ws.total);
  return launch(a, warps, ws, workspace, false, fn);
}

extern "C" int mz_paged_append_decode(
    void *out, int32_t out_dtype, int64_t out_seq_stride, int64_t out_head_stride, const void *q,
    int64_t q_seq_stride, int64_t q_head_stride, void *k_pool, void *v_pool, const void *k_new,
    const void *v_new, int64_t new_seq_stride, int64_t new_head_stride,
    const int32_t *block_tables, int32_t max_blocks_per_seq, const int32_t *ctx_lens,
    int32_t n_seqs, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
    int64_t n_blocks, float scale, int32_t dtype, int32_t num_warps, void *workspace,
    size_t workspace_bytes, int32_t *dev_err, mz_stream_t stream) {
  return append_decode(out, out_dtype, out_seq_stride, out_head_stride, q, q_seq_stride,
                       q_head_stride, k_pool, v_pool, k_new, v_new, new_seq_stride,
                       new_head_stride, block_tables, max_blocks_per_seq, ctx_lens, n_seqs,
                       n_heads, n_kv_heads, head_dim, block_size, n_blocks, scale, dtype,
                       num_warps, 0u, workspace, workspace_bytes, dev_err, stream,
                       "mz_paged_append_decode");
}

extern "C" int mz_paged_append_decode_ex(
    void *out, int32_t out_dtype, int64_t out_seq_stride, int64_t out_head_stride, const void *q,
    int64_t q_seq_stride, int64_t q_head_stride, void *k_pool, void *v_pool, const void *k_new,
    const void *v_new, int64_t new_seq_stride, int64_t new_head_stride,
    const int32_t *block_tables, int32_t max_blocks_per_seq, const int32_t *ctx_lens,
    int32_t n_seqs, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
    int64_t n_blocks, float scale, int32_t dtype, int32_t num_warps, uint32_t flags,
    void *workspace, size_t workspace_bytes, int32_t *dev_err, mz_stream_t stream) {
  return append_decode(out, out_dtype, out_seq_stride, out_head_stride, q, q_seq_stride,
                       q_head_stride, k_pool, v_pool, k_new, v_new, new_seq_stride,
                       new_head_stride, block_tables, max_blocks_per_seq, ctx_lens, n_seqs,
                       n_heads, n_kv_heads, head_dim, block_size, n_blocks, scale, dtype,
                       num_warps, flags, workspace, workspace_bytes, dev_err, stream,
                       "mz_paged_append_decode_ex");
}

extern "C" int mz_paged_append_decode_allgather(
    const mz_peer_outputs *peers, int32_t out_dtype, int64_t out_seq_stride,
    int64_t out_head_stride, const void *q, int64_t q_seq_stride, int64_t q_head_stride,
    void *k_pool, void *v_pool, const void *k_new, const void *v_new, int64_t new_seq_stride,
    int64_t new_head_stride, const int32_t *block_tables, int32_t max_blocks_per_seq,
    const int32_t *ctx_lens, int32_t n_seqs, int32_t n_heads, int32_t n_kv_heads,
    int32_t head_dim, int32_t block_size, int64_t n_blocks, float scale, int32_t dtype,
    int32_t num_warps, uint32_t flags, void *workspace, size_t workspace_bytes,
    int32_t *dev_err, mz_stream_t stream) {
  const char *fn = "mz_paged_append_decode_allgather";
  if (flags & ~(MZ_LAUNCH_OVERLAP_PREVIOUS | MZ_DECODE_BATCH_INVARIANT | MZ_LAUNCH_WAIT_PREVIOUS))
    return fail(MZ_ERR_INVALID_ARG, "%s: unknown flags", fn);
  if (!peers) return fail(MZ_ERR_INVALID_ARG, "%s: peers is null", fn);
  if (peers->rank < 0 || peers->rank >= MZ_MAX_RANKS)
    return fail(MZ_ERR_INVALID_ARG, "%s: rank %d out of range", fn, peers->rank);
  if ((flags & MZ_LAUNCH_WAIT_PREVIOUS) &&
      (!peers->signal[peers->rank] || !aligned(peers->signal[peers->rank], 4)))
    return fail(MZ_ERR_INVALID_ARG,
                "%s: MZ_LAUNCH_WAIT_PREVIOUS needs signal[rank] (this rank's own words)", fn);
  DecodeArgs a = make_args(peers->out[peers->rank], out_dtype, out_seq_stride, 0, out_head_stride,
                           q, q_seq_stride, 0, q_head_stride, 1, k_pool, v_pool, block_tables,
                           max_blocks_per_seq, ctx_lens, n_seqs, n_heads, n_kv_heads, head_dim,
                           block_size, n_blocks, scale, dtype, num_warps, dev_err, stream);
  a.kn = k_new;
  a.vn = v_new;
  a.kn_sb = new_seq_stride;
  a.kn_sh = new_head_stride;
  a.peers = peers;
  a.flags = flags;
  if (!k_new || !v_new) return fail(MZ_ERR_INVALID_ARG, "%s: null k_new / v_new", fn);
  if (n_seqs <= 0)
    return fail(MZ_ERR_INVALID_ARG, "%s: n_seqs must be positive (the peers wait for a signal)",
                fn);
  int64_t warps = 0;
  WsLayout ws;
  if (int rc = validate(a, fn, &warps, &ws)) return rc;
  if (!workspace) return fail(MZ_ERR_WORKSPACE, "%s: workspace is null", fn);
  if (workspace_bytes < ws.total)
    return fail(MZ_ERR_WORKSPACE, "%s: workspace %zu bytes < required %zu", fn, workspace_bytes,
                ws.total);
  return launch(a, warps, ws, workspace, false, fn);
}

// ---------------------------------------------------------------------------
// Allocation-free variant: the same kernel, with its scratch (split-piece
// partials, per-pair arrival counters and the chunk ticket) in a fixed array
// built into the library instead of a caller-supplied workspace.  For callers
// that cannot allocate device memory when they call in: a host whose own pool
// already owns the GPU's memory, an FFI binding with no device allocator of
// its own, or a latency-bound path where cudaMalloc's implicit device
// synchronisation is not allowed.  The array is loaded with the library's
// device code, so every GPU that runs this code holds it until the process
// exits.
// ---------------------------------------------------------------------------
namespace mz {
namespace decode {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;  // 16 MiB per device
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

constexpr int kMaxStaticDevices = 64;
std::mutex g_static_mu;
void *g_static_ptr[kMaxStaticDevices] = {};

// Device address of g_static_scratch on `device`, which must be the current
// device.  Host code cannot use the symbol's name as a device pointer, so the
// address is looked up with cudaGetSymbolAddress and kept once it succeeded.
// A failed lookup (for example one made while the stream is being captured)
// is not remembered: its error is cleared from the runtime's sticky slot and
// the next call looks the address up again.
int static_scratch_ptr(int device, void **ptr) {
  if (device < 0 || device >= kMaxStaticDevices)
    return fail(MZ_ERR_CUDA, "no usable current device (%d)", device);
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_ptr[device]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();  // later launch checks must not see this error
      return cuda_fail(e, "cudaGetSymbolAddress(decode scratch)");
    }
    if (!p) return fail(MZ_ERR_CUDA, "decode scratch has no device address");
    g_static_ptr[device] = p;
  }
  *ptr = g_static_ptr[device];
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
  const DecodeArgs a = make_args(out, out_dtype, out_seq_stride, out_tok_stride, out_head_stride,
                                 q, q_seq_stride, q_tok_stride, q_head_stride, n_q_tokens, k_pool,
                                 v_pool, block_tables, max_blocks_per_seq, ctx_lens, n_seqs,
                                 n_heads, n_kv_heads, head_dim, block_size, n_blocks, scale,
                                 dtype, num_warps, dev_err, stream);
  int64_t warps = 0;
  WsLayout ws;
  if (int rc = validate(a, "mz_paged_decode_noalloc", &warps, &ws)) return rc;
  if (n_seqs == 0) return MZ_OK;
  if (ws.total > kStaticScratchBytes)
    return fail(MZ_ERR_TOO_LARGE,
                "mz_paged_decode_noalloc: these sizes need %zu bytes of scratch but the built-in "
                "area holds %zu; lower n_seqs * n_kv_heads, rows or num_warps, or call "
                "mz_paged_decode with a workspace",
                ws.total, kStaticScratchBytes);
  void *scratch = nullptr;
  if (int rc = static_scratch_ptr(current_device(), &scratch)) return rc;
  // The area keeps whatever the previous call left; the counters must start
  // at zero, so launch() clears them on this stream first.
  return launch(a, warps, ws, scratch, true, "mz_paged_decode_noalloc");
}
