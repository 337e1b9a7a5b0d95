// Byte-exact KV movement kernels: slot append, decode-step append, block-table
// gather, block copy (copy-on-write), and block pack/unpack for the host tier.
//
// All of these are HBM-bound copies.  Each thread moves VEC-byte words, where
// VEC is the widest of 16/8/4/2 bytes that divides every base address, stride
// and row size involved, so 16-byte rows move as single 128-bit accesses.
#include "common.cuh"

namespace mz {
namespace {

template <int VEC>
struct VecT;
template <>
struct VecT<16> {
  using T = uint4;
};
template <>
struct VecT<8> {
  using T = uint2;
};
template <>
struct VecT<4> {
  using T = uint32_t;
};
template <>
struct VecT<2> {
  using T = uint16_t;
};

int pick_vec(std::initializer_list<uint64_t> quantities) {
  uint64_t acc = 0;
  for (uint64_t q : quantities) acc |= q;
  if ((acc & 15) == 0) return 16;
  if ((acc & 7) == 0) return 8;
  if ((acc & 3) == 0) return 4;
  if ((acc & 1) == 0) return 2;
  return 0;
}

unsigned grid_for(int64_t units, int threads) {
  int64_t g = (units + threads - 1) / threads;
  const int64_t cap = 148LL * 64;  // enough waves; kernels grid-stride beyond it
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<unsigned>(g);
}

// ---------------------------------------------------------------------------
// Slot append (PagedKVCache.append_kv): token i's head-h row -> slot_mapping[i].
// ---------------------------------------------------------------------------
template <int VEC>
__global__ void append_slots_kernel(uint8_t *__restrict__ kp, uint8_t *__restrict__ vp,
                                    const uint8_t *__restrict__ kn, const uint8_t *__restrict__ vn,
                                    int64_t tok_stride, int64_t head_stride,
                                    const int64_t *__restrict__ slots, int64_t n_tokens, int H,
                                    int row_bytes, int bs, int64_t n_slots, int32_t *err) {
  using V = typename VecT<VEC>::T;
  const int vecs = row_bytes / VEC;
  const int64_t total = n_tokens * H * vecs;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int v = static_cast<int>(u % vecs);
    const int64_t r = u / vecs;
    const int h = static_cast<int>(r % H);
    const int64_t i = r / H;
    const int64_t slot = slots[i];
    if (slot < 0) continue;
    if (slot >= n_slots) {
      if (h == 0 && v == 0) dev_error(err, MZ_DEVERR_SLOT);
      continue;
    }
    const int64_t blk = slot / bs;
    const int pos = static_cast<int>(slot - blk * bs);
    const int64_t dst = ((blk * H + h) * bs + pos) * row_bytes + (int64_t)v * VEC;
    const int64_t src = i * tok_stride + h * head_stride + (int64_t)v * VEC;
    *reinterpret_cast<V *>(kp + dst) = *reinterpret_cast<const V *>(kn + src);
    *reinterpret_cast<V *>(vp + dst) = *reinterpret_cast<const V *>(vn + src);
  }
}

// ---------------------------------------------------------------------------
// Decode-step append: sequence b's new token goes to position positions[b].
// ---------------------------------------------------------------------------
template <int VEC>
__global__ void append_paged_kernel(uint8_t *__restrict__ kp, uint8_t *__restrict__ vp,
                                    const uint8_t *__restrict__ kn, const uint8_t *__restrict__ vn,
                                    int64_t seq_stride, int64_t head_stride,
                                    const int32_t *__restrict__ tables, int max_blocks,
                                    const int32_t *__restrict__ positions, int n_seqs, int H,
                                    int row_bytes, int bs, int64_t n_blocks, int32_t *err) {
  using V = typename VecT<VEC>::T;
  const int vecs = row_bytes / VEC;
  const int64_t total = (int64_t)n_seqs * H * vecs;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int v = static_cast<int>(u % vecs);
    const int64_t r = u / vecs;
    const int h = static_cast<int>(r % H);
    const int b = static_cast<int>(r / H);
    const int pos = positions[b];
    if (pos < 0) continue;
    const bool first = (h == 0 && v == 0);
    if (pos >= max_blocks * bs) {
      if (first) dev_error(err, MZ_DEVERR_CONTEXT);
      continue;
    }
    const int32_t blk = tables[(int64_t)b * max_blocks + pos / bs];
    if (blk < 0 || blk >= n_blocks) {
      if (first) dev_error(err, MZ_DEVERR_BLOCK_ID);
      continue;
    }
    const int64_t dst = (((int64_t)blk * H + h) * bs + pos % bs) * row_bytes + (int64_t)v * VEC;
    const int64_t src = (int64_t)b * seq_stride + h * head_stride + (int64_t)v * VEC;
    *reinterpret_cast<V *>(kp + dst) = *reinterpret_cast<const V *>(kn + src);
    *reinterpret_cast<V *>(vp + dst) = *reinterpret_cast<const V *>(vn + src);
  }
}

// ---------------------------------------------------------------------------
// Gather (PagedKVCache.get_kv): grid.z = sequence, grid.y = kv head.
// ---------------------------------------------------------------------------
template <int VEC>
__global__ void gather_kernel(uint8_t *__restrict__ ok, uint8_t *__restrict__ ov,
                              const uint8_t *__restrict__ kp, const uint8_t *__restrict__ vp,
                              const int32_t *__restrict__ tables, int max_blocks,
                              const int32_t *__restrict__ ctx_lens,
                              const int64_t *__restrict__ out_off, int64_t max_ctx, int H,
                              int row_bytes, int bs, int64_t n_blocks, int32_t *err) {
  using V = typename VecT<VEC>::T;
  const int b = blockIdx.z;
  const int h = blockIdx.y;
  int64_t ctx = ctx_lens[b];
  if (ctx < 0 || ctx > (int64_t)max_blocks * bs || ctx > max_ctx) {
    if (h == 0 && blockIdx.x == 0 && threadIdx.x == 0) dev_error(err, MZ_DEVERR_CONTEXT);
    return;
  }
  const int vecs = row_bytes / VEC;
  const int64_t total = ctx * vecs;
  const int64_t out_base = (out_off[b] * H + (int64_t)h * ctx) * row_bytes;
  const int32_t *tab = tables + (int64_t)b * max_blocks;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int v = static_cast<int>(u % vecs);
    const int64_t t = u / vecs;
    const int32_t blk = tab[t / bs];
    if (blk < 0 || blk >= n_blocks) {
      if (v == 0) dev_error(err, MZ_DEVERR_BLOCK_ID);
      continue;
    }
    const int64_t src = (((int64_t)blk * H + h) * bs + t % bs) * row_bytes + (int64_t)v * VEC;
    const int64_t dst = out_base + t * row_bytes + (int64_t)v * VEC;
    *reinterpret_cast<V *>(ok + dst) = *reinterpret_cast<const V *>(kp + src);
    *reinterpret_cast<V *>(ov + dst) = *reinterpret_cast<const V *>(vp + src);
  }
}

// ---------------------------------------------------------------------------
// Whole-block movers.  grid.x = copy index, grid.y = pool.  mode 0: pool ->
// pool (src_ids -> dst_ids); mode 1: pool -> staging (pack); mode 2:
// staging -> pool (unpack).  16-byte words, four loads in flight per thread.
// ---------------------------------------------------------------------------
constexpr int kBlockThreads = 256;

template <int MODE>
__global__ void __launch_bounds__(kBlockThreads)
    block_move_kernel(uint8_t *__restrict__ pool, int64_t pool_stride, int n_pools,
                      int64_t block_bytes, const int32_t *__restrict__ ids_a,
                      const int32_t *__restrict__ ids_b, uint8_t *__restrict__ staging,
                      int64_t n_blocks, int32_t *err) {
  const int64_t i = blockIdx.x;
  const int p = blockIdx.y;
  const int32_t a = ids_a[i];
  if (a < 0 || a >= n_blocks) {
    if (threadIdx.x == 0 && p == 0) dev_error(err, MZ_DEVERR_BLOCK_ID);
    return;
  }
  const uint8_t *src;
  uint8_t *dst;
  uint8_t *pool_p = pool + (int64_t)p * pool_stride;
  if constexpr (MODE == 0) {
    const int32_t bdst = ids_b[i];
    if (bdst < 0 || bdst >= n_blocks) {
      if (threadIdx.x == 0 && p == 0) dev_error(err, MZ_DEVERR_BLOCK_ID);
      return;
    }
    if (bdst == a) return;
    src = pool_p + (int64_t)a * block_bytes;
    dst = pool_p + (int64_t)bdst * block_bytes;
  } else if constexpr (MODE == 1) {
    src = pool_p + (int64_t)a * block_bytes;
    dst = staging + (i * n_pools + p) * block_bytes;
  } else {
    src = staging + (i * n_pools + p) * block_bytes;
    dst = pool_p + (int64_t)a * block_bytes;
  }
  const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
  uint4 *d4 = reinterpret_cast<uint4 *>(dst);
  const int64_t n4 = block_bytes / 16;
  constexpr int U = 4;
  int64_t k = threadIdx.x;
  for (; k + (U - 1) * kBlockThreads < n4; k += U * kBlockThreads) {
    uint4 r[U];
#pragma unroll
    for (int j = 0; j < U; ++j) r[j] = s4[k + j * kBlockThreads];
#pragma unroll
    for (int j = 0; j < U; ++j) d4[k + j * kBlockThreads] = r[j];
  }
  for (; k < n4; k += kBlockThreads) d4[k] = s4[k];
}

int check_common(int32_t H, int32_t D, int32_t bs, int64_t n_blocks, int eb) {
  if (eb == 0) return fail(MZ_ERR_INVALID_ARG, "unknown dtype");
  if (H <= 0 || D <= 0 || bs <= 0 || n_blocks <= 0)
    return fail(MZ_ERR_INVALID_ARG, "n_kv_heads, head_dim, block_size and n_blocks must be > 0");
  return MZ_OK;
}

int block_move(int mode, void *pool, int64_t pool_stride, int32_t n_pools, int64_t block_bytes,
               const int32_t *ids_a, const int32_t *ids_b, void *staging, int32_t n,
               int64_t n_blocks, int32_t *err, mz_stream_t stream, const char *what) {
  if (n < 0 || n_pools <= 0 || n_pools > 65535 || block_bytes <= 0 || n_blocks <= 0)
    return fail(MZ_ERR_INVALID_ARG, "%s: bad sizes (n=%d n_pools=%d block_bytes=%lld)", what, n,
                n_pools, (long long)block_bytes);
  if (n == 0) return MZ_OK;
  if (!pool || !ids_a || (mode == 0 && !ids_b) || (mode != 0 && !staging))
    return fail(MZ_ERR_INVALID_ARG, "%s: null pointer", what);
  if ((block_bytes % 16) || (pool_stride % 16) || !aligned(pool, 16) ||
      (staging && !aligned(staging, 16)))
    return fail(MZ_ERR_ALIGNMENT, "%s: block_bytes, pool stride and bases must be 16-byte aligned",
                what);
  if (n_pools > 1 && pool_stride < n_blocks * block_bytes)
    return fail(MZ_ERR_INVALID_ARG, "%s: pool_stride_bytes smaller than one pool", what);
  dim3 grid(static_cast<unsigned>(n), static_cast<unsigned>(n_pools));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t *p8 = static_cast<uint8_t *>(pool);
  uint8_t *st8 = static_cast<uint8_t *>(staging);
  if (mode == 0)
    block_move_kernel<0><<<grid, kBlockThreads, 0, s>>>(p8, pool_stride, n_pools, block_bytes,
                                                        ids_a, ids_b, st8, n_blocks, err);
  else if (mode == 1)
    block_move_kernel<1><<<grid, kBlockThreads, 0, s>>>(p8, pool_stride, n_pools, block_bytes,
                                                        ids_a, ids_b, st8, n_blocks, err);
  else
    block_move_kernel<2><<<grid, kBlockThreads, 0, s>>>(p8, pool_stride, n_pools, block_bytes,
                                                        ids_a, ids_b, st8, n_blocks, err);
  MZ_CHECK_LAUNCH(what);
  return MZ_OK;
}

}  // namespace
}  // namespace mz

using namespace mz;

extern "C" int mz_kv_append(void *k_pool, void *v_pool, const void *k_new, const void *v_new,
                            int64_t new_tok_stride, int64_t new_head_stride,
                            const int64_t *slot_mapping, int64_t n_tokens, int32_t n_kv_heads,
                            int32_t head_dim, int32_t block_size, int64_t n_blocks, int32_t dtype,
                            int32_t *dev_err, mz_stream_t stream) {
  const int eb = dtype_bytes(dtype);
  if (int rc = check_common(n_kv_heads, head_dim, block_size, n_blocks, eb)) return rc;
  if (n_tokens < 0) return fail(MZ_ERR_INVALID_ARG, "mz_kv_append: n_tokens < 0");
  if (n_tokens == 0) return MZ_OK;
  if (!k_pool || !v_pool || !k_new || !v_new || !slot_mapping)
    return fail(MZ_ERR_INVALID_ARG, "mz_kv_append: null pointer");
  const int row = head_dim * eb;
  const int64_t ts = new_tok_stride * eb, hs = new_head_stride * eb;
  const int vec = pick_vec({(uint64_t)row, (uint64_t)ts, (uint64_t)hs, (uint64_t)(uintptr_t)k_pool,
                            (uint64_t)(uintptr_t)v_pool, (uint64_t)(uintptr_t)k_new,
                            (uint64_t)(uintptr_t)v_new});
  if (vec == 0) return fail(MZ_ERR_ALIGNMENT, "mz_kv_append: pointers must be 2-byte aligned");
  const int64_t units = n_tokens * n_kv_heads * (row / vec);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned g = grid_for(units, 256);
  auto *kp = static_cast<uint8_t *>(k_pool);
  auto *vp = static_cast<uint8_t *>(v_pool);
  auto *kn = static_cast<const uint8_t *>(k_new);
  auto *vn = static_cast<const uint8_t *>(v_new);
  const int64_t n_slots = n_blocks * block_size;
#define MZ_APPEND(V)                                                                            \
  append_slots_kernel<V><<<g, 256, 0, s>>>(kp, vp, kn, vn, ts, hs, slot_mapping, n_tokens,      \
                                           n_kv_heads, row, block_size, n_slots, dev_err)
  switch (vec) {
    case 16: MZ_APPEND(16); break;
    case 8: MZ_APPEND(8); break;
    case 4: MZ_APPEND(4); break;
    default: MZ_APPEND(2); break;
  }
#undef MZ_APPEND
  MZ_CHECK_LAUNCH("mz_kv_append");
  return MZ_OK;
}

extern "C" int mz_kv_append_paged(void *k_pool, void *v_pool, const void *k_new,
                                  const void *v_new, int64_t new_seq_stride,
                                  int64_t new_head_stride, const int32_t *block_tables,
                                  int32_t max_blocks_per_seq, const int32_t *positions,
                                  int32_t n_seqs, int32_t n_kv_heads, int32_t head_dim,
                                  int32_t block_size, int64_t n_blocks, int32_t dtype,
                                  int32_t *dev_err, mz_stream_t stream) {
  const int eb = dtype_bytes(dtype);
  if (int rc = check_common(n_kv_heads, head_dim, block_size, n_blocks, eb)) return rc;
  if (n_seqs < 0 || max_blocks_per_seq <= 0)
    return fail(MZ_ERR_INVALID_ARG, "mz_kv_append_paged: bad n_seqs / max_blocks_per_seq");
  if (n_seqs == 0) return MZ_OK;
  if (!k_pool || !v_pool || !k_new || !v_new || !block_tables || !positions)
    return fail(MZ_ERR_INVALID_ARG, "mz_kv_append_paged: null pointer");
  const int row = head_dim * eb;
  const int64_t ss = new_seq_stride * eb, hs = new_head_stride * eb;
  const int vec = pick_vec({(uint64_t)row, (uint64_t)ss, (uint64_t)hs, (uint64_t)(uintptr_t)k_pool,
                            (uint64_t)(uintptr_t)v_pool, (uint64_t)(uintptr_t)k_new,
                            (uint64_t)(uintptr_t)v_new});
  if (vec == 0) return fail(MZ_ERR_ALIGNMENT, "mz_kv_append_paged: pointers must be 2-byte aligned");
  const int64_t units = (int64_t)n_seqs * n_kv_heads * (row / vec);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned g = grid_for(units, 256);
  auto *kp = static_cast<uint8_t *>(k_pool);
  auto *vp = static_cast<uint8_t *>(v_pool);
  auto *kn = static_cast<const uint8_t *>(k_new);
  auto *vn = static_cast<const uint8_t *>(v_new);
#define MZ_APPEND(V)                                                                          \
  append_paged_kernel<V><<<g, 256, 0, s>>>(kp, vp, kn, vn, ss, hs, block_tables,              \
                                           max_blocks_per_seq, positions, n_seqs, n_kv_heads, \
                                           row, block_size, n_blocks, dev_err)
  switch (vec) {
    case 16: MZ_APPEND(16); break;
    case 8: MZ_APPEND(8); break;
    case 4: MZ_APPEND(4); break;
    default: MZ_APPEND(2); break;
  }
#undef MZ_APPEND
  MZ_CHECK_LAUNCH("mz_kv_append_paged");
  return MZ_OK;
}

extern "C" int mz_kv_gather(void *out_k, void *out_v, const void *k_pool, const void *v_pool,
                            const int32_t *block_tables, int32_t max_blocks_per_seq,
                            const int32_t *ctx_lens, const int64_t *out_token_offsets,
                            int32_t n_seqs, int64_t max_ctx, int32_t n_kv_heads,
                            int32_t head_dim, int32_t block_size, int64_t n_blocks, int32_t dtype,
                            int32_t *dev_err, mz_stream_t stream) {
  const int eb = dtype_bytes(dtype);
  if (int rc = check_common(n_kv_heads, head_dim, block_size, n_blocks, eb)) return rc;
  if (n_seqs < 0 || n_seqs > 65535 || max_ctx < 0 || max_blocks_per_seq <= 0 ||
      n_kv_heads > 65535)
    return fail(MZ_ERR_INVALID_ARG, "mz_kv_gather: bad n_seqs / max_ctx / max_blocks_per_seq");
  if (n_seqs == 0 || max_ctx == 0) return MZ_OK;
  if (!out_k || !out_v || !k_pool || !v_pool || !block_tables || !ctx_lens || !out_token_offsets)
    return fail(MZ_ERR_INVALID_ARG, "mz_kv_gather: null pointer");
  const int row = head_dim * eb;
  const int vec = pick_vec({(uint64_t)row, (uint64_t)(uintptr_t)k_pool, (uint64_t)(uintptr_t)v_pool,
                            (uint64_t)(uintptr_t)out_k, (uint64_t)(uintptr_t)out_v});
  if (vec == 0) return fail(MZ_ERR_ALIGNMENT, "mz_kv_gather: pointers must be 2-byte aligned");
  const int64_t per_head = max_ctx * (row / vec);
  int64_t gx = (per_head + 255) / 256;
  if (gx > 1024) gx = 1024;
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(n_kv_heads),
            static_cast<unsigned>(n_seqs));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto *ok = static_cast<uint8_t *>(out_k);
  auto *ov = static_cast<uint8_t *>(out_v);
  auto *kp = static_cast<const uint8_t *>(k_pool);
  auto *vp = static_cast<const uint8_t *>(v_pool);
#define MZ_GATHER(V)                                                                       \
  gather_kernel<V><<<grid, 256, 0, s>>>(ok, ov, kp, vp, block_tables, max_blocks_per_seq,  \
                                        ctx_lens, out_token_offsets, max_ctx, n_kv_heads, \
                                        row, block_size, n_blocks, dev_err)
  switch (vec) {
    case 16: MZ_GATHER(16); break;
    case 8: MZ_GATHER(8); break;
    case 4: MZ_GATHER(4); break;
    default: MZ_GATHER(2); break;
  }
#undef MZ_GATHER
  MZ_CHECK_LAUNCH("mz_kv_gather");
  return MZ_OK;
}

extern "C" int mz_block_copy(void *pool_base, int64_t pool_stride_bytes, int32_t n_pools,
                             int64_t block_bytes, const int32_t *src_ids, const int32_t *dst_ids,
                             int32_t n_copies, int64_t n_blocks, int32_t *dev_err,
                             mz_stream_t stream) {
  return block_move(0, pool_base, pool_stride_bytes, n_pools, block_bytes, src_ids, dst_ids,
                    nullptr, n_copies, n_blocks, dev_err, stream, "mz_block_copy");
}

extern "C" int mz_block_pack(void *staging, const void *pool_base, int64_t pool_stride_bytes,
                             int32_t n_pools, int64_t block_bytes, const int32_t *ids,
                             int32_t n_ids, int64_t n_blocks, int32_t *dev_err,
                             mz_stream_t stream) {
  return block_move(1, const_cast<void *>(pool_base), pool_stride_bytes, n_pools, block_bytes, ids,
                    nullptr, staging, n_ids, n_blocks, dev_err, stream, "mz_block_pack");
}

extern "C" int mz_block_unpack(void *pool_base, int64_t pool_stride_bytes, int32_t n_pools,
                               int64_t block_bytes, const void *staging, const int32_t *ids,
                               int32_t n_ids, int64_t n_blocks, int32_t *dev_err,
                               mz_stream_t stream) {
  return block_move(2, pool_base, pool_stride_bytes, n_pools, block_bytes, ids, nullptr,
                    const_cast<void *>(staging), n_ids, n_blocks, dev_err, stream,
                    "mz_block_unpack");
}
