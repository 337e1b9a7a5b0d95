// Pieces shared by the paged decode kernels (bf16/fp16 K/V and quantised K/V):
// launch parameters, the flat tile cursor, the per-warp unit scheduler and
// the merge of split pieces.
//
// Work decomposition.  The KV of every (sequence b, kv head h) -- a "pair" --
// is a list of 16-token tiles (a block of block_size tokens is block_size/16
// tiles).  All tiles of all pairs, in (b, h, t) order, form one flat sequence
// of T tiles, cut into units:
//   * static units: the first T_s tiles (MLXZ_B200_DECODE_STATIC_PCT percent
//     of T, all of it by default), one contiguous share of per_s = ceil(T_s / W)
//     tiles per warp (W persistent warps);
//   * dynamic units: the rest, if any, in chunks of C tiles that warps claim
//     with an atomic ticket once their static share is done.  C is at least
//     1/64 of the longest pair; when that is more than a quarter of a warp's
//     fair share (few, long pairs) the split is all static.
// A pair that lies inside one unit is finished by the warp that runs the unit.
// A pair cut by unit boundaries leaves one partial (running max m, running sum
// l, unnormalised O) per piece in the workspace at slot (unit + pair); the
// warp that finishes the pair's last piece (per-pair arrival counter) merges
// them.  Counters clean themselves up, so a zeroed workspace stays reusable.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace mz {
namespace decode {

constexpr int kWarps = 4;           // warps per CTA, each an independent tile stream
constexpr int kTileTok = 16;        // tokens per tile
constexpr int kUnitQ = 8;           // per-warp ring of unit descriptors
constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s bound on any single wait
constexpr int kMaxDynPieces = 64;  // dynamic chunks cut a pair into at most this many pieces
// Batch-invariant schedule: every pair is cut at the same pair-relative tile
// boundaries, one piece per kBiPieceTiles tiles (512 tokens), whatever else is
// in the batch; pieces go out by ticket and a pair's partials are merged in
// piece order, so its bytes depend only on its own data.
constexpr int kBiPieceTiles = 32;

struct Params {
  void *out;
  int64_t o_sb, o_st, o_sh;
  int out_f32;
  const void *q;
  int64_t q_sb, q_st, q_sh;
  int q_bf16;  // element type of q (and of out unless out_f32)
  int n_q, G, rows;
  const int32_t *tables;
  int max_blocks;
  const int32_t *ctx;
  int B, Hkv;
  int bs, tpb;  // block size, tiles per block
  int64_t n_blocks;
  float scale_log2;
  // fused append (kn == nullptr: none) -- bf16/fp16 pools only
  const uint16_t *kn, *vn;
  int64_t kn_sb, kn_sh;
  uint16_t *k_pool, *v_pool;
  // quantised pools: packed codes and per-token group scales and biases (fp16)
  const uint8_t *kq, *vq;
  const __half *k_scales, *k_biases, *v_scales, *v_biases;
  // workspace
  int32_t *counters;  // [n_pairs] arrival counters, then [2] = ticket, exited
  float *ml;          // [slots][rows][2]
  float *part;        // [slots][rows][D]
  int max_chunks;
  int static_pct;  // share of tiles handed out statically (1..100)
  int min_chunk;   // smallest dynamic chunk (tiles)
  int32_t *err;
  // all-gather over peer memory (n_peer > 0): every output store also goes to
  // peer_out[r] (the same rows in rank r's gathered buffer, mapped into this
  // GPU's address space); once all blocks have stored, the last one publishes
  // `epoch` into each peer_sig[r] (rank r's signal word for this rank).
  int overlap_prev = 0;  // launched as a programmatic dependent of the kernel ahead
  int batch_invariant = 0;  // fixed pair-relative pieces: a pair's bytes do not depend on the batch
  int n_peer = 0;
  void *peer_out[MZ_MAX_RANKS - 1] = {};
  uint32_t *peer_sig[MZ_MAX_RANKS - 1] = {};
  uint32_t epoch = 0;
  int32_t *arrivals = nullptr;  // grid arrival counter, zero between launches
  // Wait folded into this launch (MZ_LAUNCH_WAIT_PREVIOUS): before anything is
  // read from q or stored, every peer's word in own_sig (this GPU's signal
  // words, one per rank; own_rank's is not used) must reach wait_epoch.
  const uint32_t *own_sig = nullptr;
  int own_rank = 0, n_ranks = 1;
  uint32_t wait_epoch = 0;  // 0: no folded wait
};

struct Cursor {
  int b, h, t, n, ctx;
  int pos;
};

// A unit descriptor, passed from the producer to the consumer.  fp / np: the
// pair's first piece and piece count (batch-invariant schedule only).
struct Unit {
  int start, end, u, b, h, t, n, ctx, fp, np;
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

// Cursor at flat tile x (0 <= x < T), found with a warp scan over sequences.
__device__ __forceinline__ Cursor locate(const Params &p, int x, int lane) {
  int base = 0, bf = 0;
  for (int b0 = 0; b0 < p.B; b0 += 32) {
    const int b = b0 + lane;
    const int c = (b < p.B) ? ntiles_of(clamped_ctx(p, b)) * p.Hkv : 0;
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
  Cursor cur;
  cur.b = bf;
  cur.ctx = clamped_ctx(p, bf);
  cur.n = ntiles_of(cur.ctx);
  const int r = x - base;
  cur.h = r / cur.n;
  cur.t = r - cur.h * cur.n;
  cur.pos = x;
  return cur;
}

// Element offset of query/output row r (query token r / G, head h*G + r % G)
// of pair (b, h), dim 0.
__device__ __forceinline__ int64_t row_offset(int64_t sb, int64_t st, int64_t sh, int b, int h,
                                              int r, int G) {
  const int i = r / G, g = r - (r / G) * G;
  return (int64_t)b * sb + (int64_t)i * st + (int64_t)(h * G + g) * sh;
}

__device__ __forceinline__ void store_pair(const Params &p, int64_t off, float x, float y) {
  if (p.out_f32) {
    *reinterpret_cast<float2 *>(static_cast<float *>(p.out) + off) = make_float2(x, y);
  } else if (p.q_bf16) {
    *reinterpret_cast<__nv_bfloat162 *>(static_cast<__nv_bfloat16 *>(p.out) + off) =
        __floats2bfloat162_rn(x, y);
  } else {
    *reinterpret_cast<__half2 *>(static_cast<__half *>(p.out) + off) = __floats2half2_rn(x, y);
  }
}

// All-gather instantiation: once a warp has stored pair (b, h)'s rows in this
// GPU's buffer, it copies them -- rows * D contiguous elements, since the
// gathered buffer has dense rows and one query token -- to the same place in
// every peer's buffer, 16 bytes per lane, 512 contiguous bytes per warp store.
template <int D>
__device__ __forceinline__ void forward_rows(const Params &p, int b, int h, int lane) {
  __syncwarp();
  const int eb = p.out_f32 ? 4 : 2;
  const int64_t off = row_offset(p.o_sb, p.o_st, p.o_sh, b, h, 0, p.G) * eb;
  const int bytes = p.rows * D * eb;
  const uint8_t *src = static_cast<const uint8_t *>(p.out) + off;
  for (int x = 16 * lane; x < bytes; x += 512) {
    const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(src + x));
    for (int r = 0; r < p.n_peer; ++r)
      *reinterpret_cast<uint4 *>(static_cast<uint8_t *>(p.peer_out[r]) + off + x) = v;
  }
}

// Programmatic dependent launch: let the next launch on the stream begin its
// prologue, and wait for the launch ahead to complete (both no-ops when the
// launches were not made with programmatic stream serialization).
__device__ __forceinline__ void launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void wait_for_previous_grid() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void st_release_sys(uint32_t *addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t *addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// The peer wait folded into a launch: thread s of each block polls signal word
// s (s != own rank; the peers store it with a system-scope release once their
// previous launch's rows are all in this GPU's buffer) until it reaches
// wait_epoch (wrap-safe), bounded by kTimeoutNs; the block barrier then orders
// every thread's later reads and stores after those acquires.  A word that
// does not arrive in time sets MZ_DEVERR_TIMEOUT and the launch carries on.
// Every thread of the block must call it.
__device__ __forceinline__ void wait_peers_previous(const Params &p) {
  if (p.wait_epoch == 0) return;
  const int s = threadIdx.x;
  if (s < p.n_ranks && s != p.own_rank) {
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
      if (static_cast<int32_t>(ld_acquire_sys_u32(p.own_sig + s) - p.wait_epoch) >= 0) break;
      if ((it & 63u) == 63u) {
        const uint64_t now = global_timer_ns();
        if (t0 == 0) {
          t0 = now;
        } else if (now - t0 > kTimeoutNs) {
          dev_error(p.err, MZ_DEVERR_TIMEOUT);
          break;
        }
        __nanosleep(128);
      }
    }
  }
  __syncthreads();
}

// Called by every thread of the grid after its last output store (every exit
// path leads here, so the block barrier is reached by all).  The block's
// stores are gathered by the barrier; one thread per block fences them at
// system scope and counts the block in; the block that completes the count
// re-zeroes the counter and publishes the launch's epoch to every peer.
// Barrier -> fence -> counter -> fence -> release store orders every block's
// peer stores before the signal a peer acquires.
__device__ __forceinline__ void gather_arrive(const Params &p) {
  if (p.n_peer == 0) return;
  __syncthreads();
  if (threadIdx.x != 0) return;
  __threadfence_system();
  if (atomicAdd(p.arrivals, 1) != static_cast<int>(gridDim.x) - 1) return;
  *p.arrivals = 0;  // every block has arrived; the next launch starts from zero
  __threadfence_system();
  for (int r = 0; r < p.n_peer; ++r) st_release_sys(p.peer_sig[r], p.epoch);
}

// 128-byte swizzle of a [16 rows][128 bytes] box (what a bulk tensor copy with
// CU_TENSOR_MAP_SWIZZLE_128B writes): 16-byte unit u of row r lives at unit
// u ^ (r & 7).  Rows wider than 128 bytes are split into 2-KiB boxes.
__device__ __forceinline__ uint32_t swz128(int row, int byte) {
  const int box = byte >> 7, u = (byte & 127) >> 4;
  return box * 2048 + row * 128 + ((u ^ (row & 7)) << 4) + (byte & 15);
}

// Sequences with no context produce zeros (every warp takes b = wid mod W).
template <int D, bool GATHER = false>
__device__ __forceinline__ void zero_empty_outputs(const Params &p, int wid, int W, int lane) {
  for (int b = wid; b < p.B; b += W) {
    if (clamped_ctx(p, b) != 0) continue;
    for (int h = 0; h < p.Hkv; ++h) {
      for (int r = 0; r < p.rows; ++r) {
        const int64_t o = row_offset(p.o_sb, p.o_st, p.o_sh, b, h, r, p.G);
        for (int d = 2 * lane; d < D; d += 64) store_pair(p, o + d, 0.f, 0.f);
      }
      if constexpr (GATHER) forward_rows<D>(p, b, h, lane);
    }
  }
}

// Per-warp scheduler: static share first, then dynamic chunks by ticket.  All
// lanes run it in lockstep (the values are warp-uniform); lane 0 does the
// atomics and writes the unit ring, which the consumer reads after a
// __syncwarp.
struct Sched {
  int lane, wid, W;
  int tot, per_s, t_s, chunk, n_chunks;
  int32_t *ticket;
  Unit *uq;
  Cursor pc;
  int p_left, pushed, issued;
  int istage;  // issued % S, kept incrementally
  bool p_done, static_taken;

  // Returns false (nothing to do, no counter touched) when T == 0.
  __device__ bool init(const Params &p, int lane_, int wid_, int W_, Unit *uq_) {
    lane = lane_;
    wid = wid_;
    W = W_;
    uq = uq_;
    int t = 0, longest = 0;
    for (int b = lane; b < p.B; b += 32) {
      const int n = ntiles_of(clamped_ctx(p, b));
      t += n;
      longest = max(longest, n);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      t += __shfl_xor_sync(0xffffffffu, t, o);
      longest = max(longest, __shfl_xor_sync(0xffffffffu, longest, o));
    }
    tot = t * p.Hkv;
    if (tot == 0) return false;
    ticket = p.counters + (int64_t)p.B * p.Hkv;
    p_left = pushed = issued = istage = 0;
    p_done = static_taken = false;
    if (p.batch_invariant) {
      // every (sequence, KV head) pair is cut into pieces of kBiPieceTiles
      // tiles at fixed pair-relative boundaries, taken by ticket in pair and
      // piece order; the arithmetic of a pair is the same whatever else is in
      // the batch
      int pc = 0;
      for (int b = lane; b < p.B; b += 32)
        pc += (ntiles_of(clamped_ctx(p, b)) + kBiPieceTiles - 1) / kBiPieceTiles;
#pragma unroll
      for (int o = 16; o; o >>= 1) pc += __shfl_xor_sync(0xffffffffu, pc, o);
      per_s = 0;
      t_s = 0;
      chunk = 1 << 30;
      n_chunks = pc * p.Hkv;
      return true;
    }
    // static share: ceil(T * pct / 100 / W) tiles per warp (the last shares
    // may be short or empty), so with pct = 100 warps differ by <= one tile
    const int64_t target = (int64_t)tot * p.static_pct / 100;
    per_s = static_cast<int>((target + W - 1) / W);
    t_s = static_cast<int>(min((int64_t)per_s * W, (int64_t)tot));
    int dyn = tot - t_s;
    chunk = (dyn + p.max_chunks - 1) / p.max_chunks;
    if (chunk < p.min_chunk) chunk = p.min_chunk;
    // The dynamic chunks cut a pair into at most kMaxDynPieces pieces (a merge
    // of many pieces is the owner's tail).  When that needs chunks longer than
    // a quarter of a warp's fair share they would no longer even out the
    // finish times, so the split is all static.
    const int need = (longest + kMaxDynPieces - 1) / kMaxDynPieces;
    if (chunk < need) chunk = need;
    const int fair = static_cast<int>((tot + W - 1) / W);
    if (dyn > 0 && 4 * chunk > fair) {
      per_s = fair;
      t_s = tot;
      dyn = 0;
    }
    n_chunks = (dyn + chunk - 1) / chunk;
    return true;
  }

  __device__ __forceinline__ int unit_of(int x) const {
    return x < t_s ? x / per_s : W + (x - t_s) / chunk;
  }

  __device__ bool next_unit(const Params &p) {
    int start = 0, end = 0, u = 0, fp = 0, np = 1;
    bool ok = false;
    if (!static_taken) {
      static_taken = true;
      if (per_s > 0 && (int64_t)wid * per_s < t_s) {
        start = wid * per_s;
        end = min(start + per_s, t_s);
        u = wid;
        ok = true;
      }
    }
    while (!ok) {
      int tk = 0;
      if (lane == 0) tk = atomicAdd(ticket, 1);
      tk = __shfl_sync(0xffffffffu, tk, 0);
      if (tk >= n_chunks) {
        // Out of work.  The last warp out resets the ticket for the next call.
        if (lane == 0) {
          const int out_n = atomicAdd(ticket + 1, 1);
          if (out_n == W - 1) {
            ticket[0] = 0;
            ticket[1] = 0;
          }
        }
        return false;
      }
      if (p.batch_invariant) {
        // piece tk: sequence b found by a scan over the sequences' piece
        // counts (Hkv * ceil(n_b / C) each; empty sequences have none), then
        // head h and piece j of pair (b, h), whose tiles start at flat index
        // Hkv * (tiles of the sequences before b) + h * n_b
        int pbase = 0, tbase = 0, bf = 0;
        for (int b0 = 0; b0 < p.B; b0 += 32) {
          const int b = b0 + lane;
          const int n = (b < p.B) ? ntiles_of(clamped_ctx(p, b)) : 0;
          const int pc = p.Hkv * ((n + kBiPieceTiles - 1) / kBiPieceTiles);
          int ip = pc, it = n;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, ip, o);
            const int z = __shfl_up_sync(0xffffffffu, it, o);
            if (lane >= o) {
              ip += y;
              it += z;
            }
          }
          const unsigned m = __ballot_sync(0xffffffffu, pbase + ip > tk);
          if (m) {
            const int L = __ffs(m) - 1;
            pbase += __shfl_sync(0xffffffffu, ip - pc, L);
            tbase += __shfl_sync(0xffffffffu, it - n, L);
            bf = b0 + L;
            break;
          }
          pbase += __shfl_sync(0xffffffffu, ip, 31);
          tbase += __shfl_sync(0xffffffffu, it, 31);
        }
        const int n = ntiles_of(clamped_ctx(p, bf));
        np = (n + kBiPieceTiles - 1) / kBiPieceTiles;
        const int r = tk - pbase;
        const int h = r / np, j = r - (r / np) * np;
        const int first = tbase * p.Hkv + h * n;
        start = first + j * kBiPieceTiles;
        end = min(start + kBiPieceTiles, first + n);
        fp = pbase + h * np;
      } else {
        start = t_s + tk * chunk;
        end = min(start + chunk, tot);
      }
      u = W + tk;
      ok = true;
    }
    push_unit(p, start, end, u, fp, np);
    return true;
  }

  // Cursor at the unit's first tile; the unit descriptor goes to the ring.
  __device__ __forceinline__ void push_unit(const Params &p, int start, int end, int u,
                                            int fp = 0, int np = 1) {
    pc = locate(p, start, lane);
    if (lane == 0) {
      Unit un;
      un.start = start;
      un.end = end;
      un.u = u;
      un.b = pc.b;
      un.h = pc.h;
      un.t = pc.t;
      un.n = pc.n;
      un.ctx = pc.ctx;
      un.fp = fp;
      un.np = np;
      uq[pushed % kUnitQ] = un;
    }
    ++pushed;
    p_left = end - start;
  }

  // Before the launch waits for the kernel ahead of it (programmatic dependent
  // launch): start the copies of the first (up to S) tiles of this warp's
  // static share.  Reads only ctx, the block tables and the pools (through
  // locate and issue); no ticket, no workspace word.
  template <int S, class IssueFn>
  __device__ __forceinline__ void prefetch_static(const Params &p, IssueFn &&issue) {
    if (static_taken) return;
    static_taken = true;
    if (!(per_s > 0 && (int64_t)wid * per_s < t_s)) return;
    const int start = wid * per_s;
    push_unit(p, start, min(start + per_s, t_s), wid);
    while (p_left > 0 && issued < S) {
      issue(istage, pc);
      advance(pc, p);
      --p_left;
      ++issued;
      if (++istage == S) istage = 0;
    }
  }

  // Keep S tiles in flight; issue(stage, cursor) starts one tile's copies.
  template <int S, class IssueFn>
  __device__ __forceinline__ void refill(const Params &p, int consumed, IssueFn &&issue) {
    while (!p_done && issued - consumed < S) {
      if (p_left == 0 && !next_unit(p)) {
        p_done = true;
        break;
      }
      if (lane == 0 && issued >= S) fence_proxy_async_smem();
      issue(istage, pc);
      advance(pc, p);
      --p_left;
      ++issued;
      if (++istage == S) istage = 0;
    }
  }
};

// Consumer side of the unit ring.
struct UnitReader {
  Cursor cc;
  int left = 0, unit = 0, popped = 0, fp = 0, np = 1;

  __device__ __forceinline__ bool need_pop() const { return left == 0; }
  __device__ __forceinline__ void pop(const Unit *uq) {
    __syncwarp();
    const Unit un = uq[popped % kUnitQ];
    ++popped;
    cc.b = un.b;
    cc.h = un.h;
    cc.t = un.t;
    cc.n = un.n;
    cc.ctx = un.ctx;
    cc.pos = un.start;
    left = un.end - un.start;
    unit = un.u;
    fp = un.fp;
    np = un.np;
  }
};

// ---------------------------------------------------------------------------
// Merge of split pairs.  After a warp has written its piece of pair bh to its
// slot it counts its arrival; the warp that brings the count to nparts owns
// the merge of every piece's (m, l, O) (slots uf + bh .. uf + nparts - 1 + bh,
// consecutive) into the output, and resets the counter.
//
// Most pieces end where their warp's unit ends, so merges cluster at the end
// of the kernel and their latency would be its tail.  The owner therefore
// records the merge in a per-warp list in shared memory and carries on
// streaming; when its tile loop is over (its stage ring idle) it runs the list,
// staging each pair's partials into the ring with cp.async -- one round trip
// for all of them -- and combining them from shared memory.  A list that is
// full falls back to merging at once from global memory.
// ---------------------------------------------------------------------------
constexpr int kMaxDeferred = 8;  // deferred merges per warp

struct Deferred {
  int b, h, uf, nparts;
};

// Counts this warp's arrival for pair bh; true for the warp that owns the merge.
__device__ __forceinline__ bool arrive(const Params &p, int bh, int nparts, int lane) {
  __threadfence();
  __syncwarp();
  int old = 0;
  if (lane == 0) old = atomicAdd(p.counters + bh, 1);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old != nparts - 1) return false;
  __threadfence();
  return true;
}

// Combine of one piece (m, l, O-slice) into the running (M, Ls, acc): the
// online-softmax merge, pieces taken in slot order.
__device__ __forceinline__ void merge_piece(float &M, float &Ls, float4 &acc, float2 ml, float4 o) {
  const float Mn = fmaxf(M, ml.x);
  const float sa = fast_exp2(M - Mn), sb = fast_exp2(ml.x - Mn);
  Ls = Ls * sa + ml.y * sb;
  acc.x = acc.x * sa + o.x * sb;
  acc.y = acc.y * sa + o.y * sb;
  acc.z = acc.z * sa + o.z * sb;
  acc.w = acc.w * sa + o.w * sb;
  M = Mn;
}

// Merge straight from global memory: the pieces are read four at a time, all
// four loads in flight before the combine that needs them.
template <int D, bool GATHER>
__device__ __forceinline__ void merge_global(const Params &p, int b, int h, int uf, int nparts,
                                             int lane) {
  const int bh = b * p.Hkv + h;
  const int E = p.rows * D;
  for (int e = 4 * lane; e < E; e += 128) {
    const int r = e / D, d = e - (e / D) * D;
    float M = -INFINITY, Ls = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k0 = 0; k0 < nparts; k0 += 4) {
      float2 mlk[4];
      float4 ok[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        mlk[j] = make_float2(-INFINITY, 0.f);
        ok[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (k0 + j < nparts) {
          const int64_t sl = (int64_t)uf + k0 + j + bh;
          mlk[j] = __ldcg(reinterpret_cast<const float2 *>(p.ml + (sl * p.rows + r) * 2));
          ok[j] = __ldcg(reinterpret_cast<const float4 *>(p.part + (sl * p.rows + r) * D + d));
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (k0 + j < nparts) merge_piece(M, Ls, acc, mlk[j], ok[j]);
    }
    const float inv = 1.f / Ls;
    const int64_t o = row_offset(p.o_sb, p.o_st, p.o_sh, b, h, r, p.G) + d;
    store_pair(p, o, acc.x * inv, acc.y * inv);
    store_pair(p, o + 2, acc.z * inv, acc.w * inv);
  }
  if constexpr (GATHER) forward_rows<D>(p, b, h, lane);
  if (lane == 0) p.counters[bh] = 0;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Merge with the pieces staged in shared memory `buf` (buf_bytes, 16-byte
// aligned, idle), as many pieces per round trip as fit.
template <int D, bool GATHER>
__device__ __forceinline__ void merge_staged(const Params &p, int b, int h, int uf, int nparts,
                                             uint8_t *buf, int buf_bytes, int lane) {
  const int bh = b * p.Hkv + h;
  const int part_bytes = p.rows * D * 4;
  const int per = buf_bytes / (part_bytes + p.rows * 8);
  if (per < 1) {
    merge_global<D, GATHER>(p, b, h, uf, nparts, lane);
    return;
  }
  constexpr int kIt = 16 * D / 128;  // 4-element steps per lane for up to 16 rows
  const int E = p.rows * D;
  float M[kIt], Ls[kIt];
  float4 acc[kIt];
#pragma unroll
  for (int it = 0; it < kIt; ++it) {
    M[it] = -INFINITY;
    Ls[it] = 0.f;
    acc[it] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const uint32_t buf_s = smem_u32(buf);
  const float *part_s = reinterpret_cast<const float *>(buf);
  for (int k0 = 0; k0 < nparts; k0 += per) {
    const int cnt = min(per, nparts - k0);
    const int64_t slot = (int64_t)uf + k0 + bh;
    const uint8_t *src = reinterpret_cast<const uint8_t *>(p.part + slot * p.rows * D);
    const int pb = cnt * part_bytes;
    __syncwarp();  // the previous round's reads of buf are done
    for (int x = 16 * lane; x < pb; x += 512) cp_async16(buf_s + x, src + x);
    const float *mls = p.ml + slot * p.rows * 2;
    for (int x = lane; x < cnt * p.rows; x += 32) cp_async8(buf_s + pb + 8 * x, mls + 2 * x);
    cp_async_wait_all();
    __syncwarp();
    const float2 *ml_s = reinterpret_cast<const float2 *>(buf + pb);
    for (int k = 0; k < cnt; ++k) {
#pragma unroll
      for (int it = 0; it < kIt; ++it) {
        const int e = 4 * lane + 128 * it;
        if (e < E) {
          const float2 ml = ml_s[k * p.rows + e / D];
          const float4 o = *reinterpret_cast<const float4 *>(part_s + k * (p.rows * D) + e);
          merge_piece(M[it], Ls[it], acc[it], ml, o);
        }
      }
    }
  }
#pragma unroll
  for (int it = 0; it < kIt; ++it) {
    const int e = 4 * lane + 128 * it;
    if (e < E) {
      const int r = e / D, d = e - r * D;
      const float inv = 1.f / Ls[it];
      const int64_t o = row_offset(p.o_sb, p.o_st, p.o_sh, b, h, r, p.G) + d;
      store_pair(p, o, acc[it].x * inv, acc[it].y * inv);
      store_pair(p, o + 2, acc[it].z * inv, acc[it].w * inv);
    }
  }
  if constexpr (GATHER) forward_rows<D>(p, b, h, lane);
  if (lane == 0) p.counters[bh] = 0;
}

// In the tile loop, after this warp's piece of the pair has been written.
// Small merges (rows * pieces <= kMergeNow) run at once; larger ones are
// deferred while the list has room.
constexpr int kMergeNow = 16;

template <int D, bool GATHER = false>
__device__ __forceinline__ void arrive_or_defer(const Params &p, const Cursor &cc, int bh, int uf,
                                                int nparts, int lane, Deferred *dq, int &nd) {
  if (!arrive(p, bh, nparts, lane)) return;
  if (p.rows * nparts > kMergeNow && nd < kMaxDeferred) {
    if (lane == 0) dq[nd] = Deferred{cc.b, cc.h, uf, nparts};
    ++nd;
  } else {
    merge_global<D, GATHER>(p, cc.b, cc.h, uf, nparts, lane);
  }
}

// After the tile loop: run the deferred merges with the idle stage ring `buf`.
// `ring_idle` false (a wait gave up with copies maybe still landing): leave
// the outputs and only reset the pairs' counters.
template <int D, bool GATHER = false>
__device__ __forceinline__ void run_deferred(const Params &p, const Deferred *dq, int nd,
                                             uint8_t *buf, int buf_bytes, bool ring_idle,
                                             int lane) {
  __syncwarp();
  for (int j = 0; j < nd; ++j) {
    const Deferred d = dq[j];
    if (ring_idle) {
      merge_staged<D, GATHER>(p, d.b, d.h, d.uf, d.nparts, buf, buf_bytes, lane);
    } else if (lane == 0) {
      p.counters[d.b * p.Hkv + d.h] = 0;
    }
  }
}

// Bounded wait on a stage; on timeout, record it and let this warp's copies
// in flight (tiles first..issued-1) land, bounded, before the caller returns.
template <int S>
__device__ __forceinline__ bool wait_stage(const Params &p, uint32_t bar0, int i, int issued,
                                           int lane) {
  // warp-uniform outcome: a lane that saw the phase complete waits for the rest
  if (__all_sync(0xffffffffu, mbar_wait_bounded(bar0 + 8 * (i % S), (i / S) & 1, kTimeoutNs)))
    return true;
  if (lane == 0) dev_error(p.err, MZ_DEVERR_TIMEOUT);
  for (int k = i; k < issued; ++k) (void)mbar_wait_bounded(bar0 + 8 * (k % S), (k / S) & 1, kTimeoutNs);
  return false;
}

// ---------------------------------------------------------------------------
// Host-side helpers.
// ---------------------------------------------------------------------------

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 2-D tensor map over `rows` rows of `row_elems` elements, box = box_elems x
// box_rows rows, 128-byte swizzle.
inline int make_row_map(CUtensorMap *m, const void *base, int64_t rows, int row_elems,
                        CUtensorMapDataType type, int elem_bytes, int box_elems,
                        int box_rows = kTileTok) {
  auto fn = encode_fn();
  if (!fn) return fail(MZ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_elems), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_elems) * elem_bytes};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_elems), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, type, 2, const_cast<void *>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MZ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MZ_OK;
}

struct WsLayout {
  size_t counters, ml, part, total;
  int64_t counter_words;
  int max_chunks;
};

inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Workspace for W warps: per-pair counters + 2 scheduler words, then (m, l)
// and O partials for W static units + max_chunks dynamic units + one extra
// slot per pair (slot = unit + pair).  max_pieces: the most pieces a
// batch-invariant launch can cut (0 for the default schedule).
inline WsLayout ws_layout(int64_t n_pairs, int64_t warps, int rows, int D,
                          int64_t max_pieces = 0) {
  WsLayout w;
  w.max_chunks = static_cast<int>(2 * warps > max_pieces ? 2 * warps : max_pieces);
  const int64_t slots = warps + w.max_chunks + n_pairs;
  w.counter_words = n_pairs + 2;
  w.counters = 0;
  w.ml = align256(w.counter_words * sizeof(int32_t));
  w.part = w.ml + align256(slots * rows * 2 * sizeof(float));
  w.total = w.part + align256(slots * rows * D * sizeof(float));
  return w;
}

// Scheduler tuning knob from the environment (read at each launch), clamped.
inline int env_int(const char *name, int dflt, int lo, int hi) {
  const char *v = getenv(name);
  if (!v || !*v) return dflt;
  long x = strtol(v, nullptr, 10);
  return static_cast<int>(x < lo ? lo : (x > hi ? hi : x));
}

inline void set_schedule(Params &p, const WsLayout &ws) {
  p.max_chunks = ws.max_chunks;
  p.static_pct = env_int("MLXZ_B200_DECODE_STATIC_PCT", 100, 1, 100);
  p.min_chunk = env_int("MLXZ_B200_DECODE_MIN_CHUNK", 16, 1, 1 << 20);
}

// Occupancy of a decode kernel instantiation (cached; also sets its shared
// memory attribute once).
template <class KernelPtr>
int kernel_occupancy(KernelPtr k, int smem_bytes, DeviceOnce &once, int *out) {
  return device_once(
      once,
      [&](int *n) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
        if (e != cudaSuccess) return e;
        return cudaOccupancyMaxActiveBlocksPerMultiprocessor(n, k, kWarps * 32, smem_bytes);
      },
      out, "paged decode: occupancy query");
}

}  // namespace decode
}  // namespace mz
