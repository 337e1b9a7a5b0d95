/*
 * mlxz_b200.h -- C ABI of the B200 (sm_100a) KV-cache kernels.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream.
 * Nothing here allocates, frees or synchronises: launches are asynchronous on
 * the given stream and the caller owns every buffer for the duration of the
 * launch.  Functions return MZ_OK (0) or a negative MZ_ERR_* code; the text
 * of the most recent error on the calling thread is read with mz_last_error.
 *
 * Data layout shared by all kernels (same as the reference's pool,
 * src/mlxz/paged_attention/paged_kv.py:33-44):
 *   K pool, V pool : [n_blocks][n_kv_heads][block_size][head_dim], row-major,
 *                    element type `dtype` (MZ_DTYPE_*).
 *   block tables   : int32 [n_seqs][max_blocks_per_seq]; entry j of sequence b
 *                    is the physical block holding tokens [j*bs, (j+1)*bs).
 *   slot           : block_id * block_size + position_in_block.
 *
 * Device error word: every kernel takes an optional `int32_t *dev_err`
 * (device memory, may be NULL).  Instead of trapping, a kernel that meets an
 * out-of-range block id, slot or context length skips that access and ORs an
 * MZ_DEVERR_* bit into the word.  A bounded wait that gives up sets
 * MZ_DEVERR_TIMEOUT.  The caller clears the word and reads it back when it
 * wants to check.
 */
#ifndef MLXZ_B200_H
#define MLXZ_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MZ_API __attribute__((visibility("default")))
#else
#define MZ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* A cudaStream_t (CUstream).  NULL selects the legacy default stream. */
typedef void *mz_stream_t;

/* Largest group of ranks an all-gather over peer memory spans (GPUs of one
 * NVLink domain), and the size of an exported memory handle. */
#define MZ_MAX_RANKS 8
#define MZ_IPC_HANDLE_BYTES 64

enum mz_status {
  MZ_OK = 0,
  MZ_ERR_INVALID_ARG = -1, /* a size, stride or pointer argument is invalid  */
  MZ_ERR_UNSUPPORTED = -2, /* valid, but outside what the kernels implement  */
  MZ_ERR_ALIGNMENT = -3,   /* a pointer or stride breaks a stated alignment  */
  MZ_ERR_CUDA = -4,        /* a CUDA runtime or driver call failed           */
  MZ_ERR_WORKSPACE = -5,   /* workspace missing or smaller than required     */
  MZ_ERR_TOO_LARGE = -6    /* problem larger than a fixed-capacity variant   */
};

enum mz_dtype { MZ_DTYPE_F16 = 0, MZ_DTYPE_BF16 = 1, MZ_DTYPE_F32 = 2 };

enum mz_device_error {
  MZ_DEVERR_BLOCK_ID = 1, /* block-table entry outside [0, n_blocks)          */
  MZ_DEVERR_SLOT = 2,     /* slot outside [0, n_blocks * block_size)          */
  MZ_DEVERR_CONTEXT = 4,  /* context length < 0 or > table capacity           */
  MZ_DEVERR_TIMEOUT = 8,  /* a bounded wait on an mbarrier or flag gave up    */
  MZ_DEVERR_ROWS = 16     /* a sequence's query rows outside [0, n_rows)      */
};

/* ABI version of this header (bumped on any signature change). */
MZ_API int mz_abi_version(void);

/* Copies the calling thread's last error message into buf (NUL-terminated,
 * truncated to len).  Returns the status code that produced it. */
MZ_API int mz_last_error(char *buf, size_t len);

/* ------------------------------------------------------------------------ */
/* KV append.                                                                */
/* ------------------------------------------------------------------------ */

/* Scatter n_tokens new K/V rows into the pools by slot.
 * Replaces PagedKVCache.append_kv, src/mlxz/paged_attention/paged_kv.py:63-93
 * (the per-token write `pool[blocks[pos // bs], :, pos % bs, :] = k[0, :, i, :]`
 * at :85-91; block-table growth stays on the host).
 * k_new/v_new element (token i, head h, dim d) sits at
 *   base + i * new_tok_stride + h * new_head_stride + d        (elements).
 * slot_mapping: int64 [n_tokens] device array; a negative slot skips the row.
 * Bit-exact copy. */
MZ_API int mz_kv_append(void *k_pool, void *v_pool, const void *k_new, const void *v_new,
                 int64_t new_tok_stride, int64_t new_head_stride,
                 const int64_t *slot_mapping, int64_t n_tokens, int32_t n_kv_heads,
                 int32_t head_dim, int32_t block_size, int64_t n_blocks, int32_t dtype,
                 int32_t *dev_err, mz_stream_t stream);

/* Decode-step append: one new token per sequence, written at position
 * positions[b] of sequence b through its block table (negative position skips).
 * Replaces the per-request cache update inside the batched decode of
 * ContinuousBatchingEngine._process_decodes, src/mlxz/engine/continuous.py:625-633,
 * with one launch over ragged sequences.
 * k_new/v_new element (seq b, head h, dim d) at base + b*new_seq_stride +
 * h*new_head_stride + d.  Bit-exact copy. */
MZ_API int mz_kv_append_paged(void *k_pool, void *v_pool, const void *k_new, const void *v_new,
                       int64_t new_seq_stride, int64_t new_head_stride,
                       const int32_t *block_tables, int32_t max_blocks_per_seq,
                       const int32_t *positions, int32_t n_seqs, int32_t n_kv_heads,
                       int32_t head_dim, int32_t block_size, int64_t n_blocks, int32_t dtype,
                       int32_t *dev_err, mz_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Block-table gather.                                                       */
/* ------------------------------------------------------------------------ */

/* Materialise contiguous K/V for n_seqs sequences.
 * Replaces PagedKVCache.get_kv, src/mlxz/paged_attention/paged_kv.py:95-137.
 * Sequence b is written as [n_kv_heads][ctx_lens[b]][head_dim] starting at
 * element out_token_offsets[b] * n_kv_heads * head_dim of out_k / out_v
 * (so one sequence gives the reference's (1, H, T, D) layout).
 * max_ctx must be >= every ctx_lens[b] (it sizes the grid).  Bit-exact. */
MZ_API int mz_kv_gather(void *out_k, void *out_v, const void *k_pool, const void *v_pool,
                 const int32_t *block_tables, int32_t max_blocks_per_seq,
                 const int32_t *ctx_lens, const int64_t *out_token_offsets, int32_t n_seqs,
                 int64_t max_ctx, int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
                 int64_t n_blocks, int32_t dtype, int32_t *dev_err, mz_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Fused GQA paged decode attention.                                         */
/* ------------------------------------------------------------------------ */

/* Bytes of workspace mz_paged_decode needs for these sizes on `device`
 * (num_warps as passed to mz_paged_decode; 0 = the default grid).
 * rows_per_kv_head = n_q_tokens * (n_heads / n_kv_heads), at most 16. */
MZ_API int mz_paged_decode_workspace_size(int32_t n_seqs, int32_t n_kv_heads, int32_t rows_per_kv_head,
                                   int32_t head_dim, int32_t num_warps, int32_t device,
                                   size_t *bytes);

/* out = softmax(q . K^T * scale) . V over each sequence's first ctx_lens[b]
 * tokens, with query head hq reading KV head hq / (n_heads / n_kv_heads) and
 * no mask, as in paged_attention_forward, src/mlxz/paged_attention/attention.py:9-49
 * (get_kv + mx.repeat + mx.fast.scaled_dot_product_attention, :23-42), fused:
 * no gather, no repeat.  Online softmax, fp32 accumulation.
 * q element (seq b, query token i, head h, dim d) at
 *   q + b*q_seq_stride + i*q_tok_stride + h*q_head_stride + d   (elements, dtype),
 * out likewise with out_* strides and element type out_dtype (dtype or F32).
 * Supported: dtype F16/BF16, head_dim 64 or 128, block_size a multiple of 16,
 * n_q_tokens * (n_heads / n_kv_heads) <= 16.  K/V pools need 16-byte
 * alignment, q and out 4-byte (8-byte for F32 out) alignment and even strides.
 * A sequence with ctx_lens[b] == 0 gets zeros.
 * workspace: >= mz_paged_decode_workspace_size bytes, zero-filled before its
 * first use; every successful call leaves its counter region -- the first
 * 4 * (n_seqs * n_kv_heads + 2) bytes -- zeroed again.  Where that region
 * ends depends on the sizes, so a workspace reused by a call with other
 * n_seqs, n_kv_heads, rows or head_dim must be zero-filled again first (its
 * partials may lie where the new counters go).  After a call that set a
 * dev_err bit, zero the workspace before reuse.
 * num_warps: persistent warps to launch (0 = one full wave of the device). */
MZ_API int mz_paged_decode(void *out, int32_t out_dtype, int64_t out_seq_stride, int64_t out_tok_stride,
                    int64_t out_head_stride, const void *q, int64_t q_seq_stride,
                    int64_t q_tok_stride, int64_t q_head_stride, int32_t n_q_tokens,
                    const void *k_pool, const void *v_pool, const int32_t *block_tables,
                    int32_t max_blocks_per_seq, const int32_t *ctx_lens, int32_t n_seqs,
                    int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
                    int64_t n_blocks, float scale, int32_t dtype, int32_t num_warps,
                    void *workspace, size_t workspace_bytes, int32_t *dev_err,
                    mz_stream_t stream);

/* Fused decode step: append one new token per sequence, then attend.
 * The new token of sequence b is the last attended one (position
 * ctx_lens[b] - 1): its K/V rows, k_new/v_new element (b, h, d) at
 * base + b*new_seq_stride + h*new_head_stride + d, are written to that slot of
 * the pools through the block table (bit-exact, as mz_kv_append_paged) and used
 * by the attention in the same launch.  Replaces the per-layer pair
 * cache.update_and_fetch + SDPA of the reference's batched decode
 * (src/mlxz/engine/continuous.py:625-633) for one layer.  q/out are
 * [n_seqs][n_heads][head_dim] with the given strides (one query token).
 * k_new/v_new need 16-byte alignment and strides that are multiples of 8.
 * Workspace and the other rules as mz_paged_decode. */
MZ_API int mz_paged_append_decode(void *out, int32_t out_dtype, int64_t out_seq_stride,
                                  int64_t out_head_stride, const void *q, int64_t q_seq_stride,
                                  int64_t q_head_stride, void *k_pool, void *v_pool,
                                  const void *k_new, const void *v_new, int64_t new_seq_stride,
                                  int64_t new_head_stride, const int32_t *block_tables,
                                  int32_t max_blocks_per_seq, const int32_t *ctx_lens,
                                  int32_t n_seqs, int32_t n_heads, int32_t n_kv_heads,
                                  int32_t head_dim, int32_t block_size, int64_t n_blocks,
                                  float scale, int32_t dtype, int32_t num_warps, void *workspace,
                                  size_t workspace_bytes, int32_t *dev_err, mz_stream_t stream);

/* Chunked prefill attention over paged KV.  Sequence b's n_b = q_len[b]
 * query tokens are rows q_start[b] .. q_start[b] + n_b - 1 of the n_rows rows
 * of q and out (rows outside [0, n_rows): MZ_DEVERR_ROWS, sequence skipped)
 * (element (row t, head hq, dim d) at base + t*tok_stride + hq*head_stride + d,
 * of dtype; out of out_dtype = dtype or F32) at positions
 * [ctx_lens[b] - n_b, ctx_lens[b]) of the sequence, their K/V already in the
 * pools (mz_kv_append).  Token i attends to the sequence's first
 * ctx_lens[b] - n_b + i + 1 tokens (causal), query head hq reading KV head
 * hq / (n_heads / n_kv_heads); softmax(q.K^T*scale).V with fp32 accumulation.
 * max_q_len >= every q_len[b] sizes the grid.
 * Replaces the prompt pass over a request cache that follows
 * ChunkedPrefillScheduler.get_next_chunk (src/mlxz/scheduler/chunker.py:53-76):
 * mlx_lm's causal scaled_dot_product_attention of a prompt chunk at a cache
 * offset, here over paged KV.  Supported: F16 / BF16, head_dim 64 or 128,
 * block_size a multiple of 16, n_heads / n_kv_heads dividing 128, scale > 0;
 * q and out 16-byte aligned with strides of whole 16-byte vectors. */
MZ_API int mz_paged_prefill(void *out, int32_t out_dtype, int64_t out_tok_stride,
                            int64_t out_head_stride, const void *q, int64_t q_tok_stride,
                            int64_t q_head_stride, int32_t n_rows, const int32_t *q_start,
                            const int32_t *q_len,
                            int32_t max_q_len, const void *k_pool, const void *v_pool,
                            const int32_t *block_tables, int32_t max_blocks_per_seq,
                            const int32_t *ctx_lens, int32_t n_seqs, int32_t n_heads,
                            int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
                            int64_t n_blocks, float scale, int32_t dtype, int32_t *dev_err,
                            mz_stream_t stream);

/* Launch flags of the _ex / allgather entry points.
 * MZ_LAUNCH_OVERLAP_PREVIOUS: the launch may begin while the kernel ahead of it
 * on the stream is still running (programmatic dependent launch): its blocks
 * take SMs as that kernel's blocks finish, schedule their work and start the
 * copies of their first K/V tiles, then wait for that kernel to complete before
 * they read q / k_new / v_new or write anything.  Valid only when the kernel
 * ahead writes none of this launch's pools, block tables or ctx_lens (e.g. it
 * is the previous layer's decode). */
#define MZ_LAUNCH_OVERLAP_PREVIOUS 1u
/* MZ_DECODE_BATCH_INVARIANT: every (sequence, KV head) pair is cut into
 * pieces at fixed pair-relative boundaries (512 tokens), the pieces are
 * handed out by ticket, and a pair's pieces are merged in piece order, so a
 * sequence's output bytes do not depend on its position in the batch or on
 * the other sequences.  The batch-position determinism gate of the
 * reference's plan (MLXZ_IMPLEMENTATION_PLAN.md:1058-1059: prefix-cache drift
 * < 1e-4, batch-position determinism bytewise).  Its workspace depends on the
 * table width: size it with mz_paged_decode_workspace_size_ex. */
#define MZ_DECODE_BATCH_INVARIANT 2u
/* MZ_LAUNCH_WAIT_PREVIOUS (mz_paged_append_decode_allgather only): the launch
 * itself first waits, bounded like mz_peer_wait, until every peer's signal
 * word in signal[rank] (this rank's own words) holds epoch - 1, i.e. until the
 * peers' rows of this rank's previous launch are in its gathered buffer; only
 * then does it read q / k_new / v_new or store anything.  It replaces the
 * mz_peer_wait launch between two layers, so with MZ_LAUNCH_OVERLAP_PREVIOUS
 * the next layer's first K/V copies still start while the previous layer
 * drains.  Work queued after the launch then sees the previous launch's
 * gathered buffer complete. */
#define MZ_LAUNCH_WAIT_PREVIOUS 4u

/* Workspace bytes of a decode launch with these flags (MZ_LAUNCH_*,
 * MZ_DECODE_BATCH_INVARIANT): mz_paged_decode_workspace_size, plus, for a
 * batch-invariant launch, room for the partials of every piece the widest
 * tables (max_blocks_per_seq blocks of block_size tokens) can cut.  No
 * counterpart in the reference (MLX manages its own scratch). */
MZ_API int mz_paged_decode_workspace_size_ex(int32_t n_seqs, int32_t n_kv_heads,
                                             int32_t rows_per_kv_head, int32_t head_dim,
                                             int32_t num_warps, int32_t max_blocks_per_seq,
                                             int32_t block_size, uint32_t flags, int32_t device,
                                             size_t *bytes);

/* mz_paged_append_decode with launch flags (MZ_LAUNCH_*).  Same reference
 * counterpart and rules as mz_paged_append_decode. */
MZ_API int mz_paged_append_decode_ex(void *out, int32_t out_dtype, int64_t out_seq_stride,
                                     int64_t out_head_stride, const void *q,
                                     int64_t q_seq_stride, int64_t q_head_stride, void *k_pool,
                                     void *v_pool, const void *k_new, const void *v_new,
                                     int64_t new_seq_stride, int64_t new_head_stride,
                                     const int32_t *block_tables, int32_t max_blocks_per_seq,
                                     const int32_t *ctx_lens, int32_t n_seqs, int32_t n_heads,
                                     int32_t n_kv_heads, int32_t head_dim, int32_t block_size,
                                     int64_t n_blocks, float scale, int32_t dtype,
                                     int32_t num_warps, uint32_t flags, void *workspace,
                                     size_t workspace_bytes, int32_t *dev_err,
                                     mz_stream_t stream);

/* Destinations of one rank's decode output in a head-sharded group of
 * n_ranks GPUs (one process each, KV heads split evenly; rank r holds query
 * heads [r*n_heads, (r+1)*n_heads) of the n_ranks*n_heads in the gathered
 * [n_seqs][n_ranks*n_heads][head_dim] buffer every rank keeps).
 *   out[r]:    in rank r's gathered buffer, the first element of THIS rank's
 *              head block (base + rank*n_heads*head_dim), as an address this
 *              GPU can store to (out[rank] local; the others mapped with
 *              mz_ipc_open);
 *   signal[r]: rank r's n_ranks signal words (zero before the first launch),
 *              mapped likewise (signal[rank], this rank's own words, is read
 *              only by launches with MZ_LAUNCH_WAIT_PREVIOUS);
 *   arrivals:  one int32 in this GPU's memory, zero before the first launch
 *              (each launch leaves it zero);
 *   epoch:     nonzero, one more per launch, the same on every rank. */
typedef struct mz_peer_outputs {
  int32_t n_ranks;
  int32_t rank;
  void *out[MZ_MAX_RANKS];
  int32_t *signal[MZ_MAX_RANKS];
  int32_t *arrivals;
  uint32_t epoch;
} mz_peer_outputs;

/* mz_paged_append_decode whose output rows are stored into every rank's
 * gathered buffer (this GPU's own and, over NVLink, each peer's) as they are
 * finished, instead of a separate all-gather after the launch; the launch's
 * last block then publishes `epoch` into signal word `rank` of every peer.
 * Each rank follows the launch with mz_peer_wait, or with its next launch
 * made with MZ_LAUNCH_WAIT_PREVIOUS, before it reads the gathered buffer.
 * out_seq_stride / out_head_stride are those of the gathered buffer
 * (n_ranks*n_heads*head_dim and head_dim for a dense one).
 * No counterpart in the reference (one device only); it replaces the
 * all-gather of head-sharded attention outputs that a multi-GPU step runs
 * after mz_paged_append_decode.  Peers write a gathered buffer for the next
 * time as soon as this rank's launch before that one has completed, so this
 * rank's readers of a buffer must be ordered before that preceding launch.
 * n_seqs must be positive.  flags: MZ_LAUNCH_*.  Other
 * arguments and rules as mz_paged_append_decode. */
MZ_API int mz_paged_append_decode_allgather(
    const mz_peer_outputs *peers, int32_t out_dtype, int64_t out_seq_stride,
    int64_t out_head_stride, const void *q, int64_t q_seq_stride, int64_t q_head_stride,
    void *k_pool, void *v_pool, const void *k_new, const void *v_new, int64_t new_seq_stride,
    int64_t new_head_stride, const int32_t *block_tables, int32_t max_blocks_per_seq,
    const int32_t *ctx_lens, int32_t n_seqs, int32_t n_heads, int32_t n_kv_heads,
    int32_t head_dim, int32_t block_size, int64_t n_blocks, float scale, int32_t dtype,
    int32_t num_warps, uint32_t flags, void *workspace, size_t workspace_bytes,
    int32_t *dev_err, mz_stream_t stream);

/* Enqueue on `stream` a wait until signal[s] (this rank's words, s != rank)
 * has reached `epoch` for every peer s, with acquire semantics at system
 * scope, so work queued after it sees the peers' stored rows.  Gives up after
 * timeout_ns (at most 60 s) and sets MZ_DEVERR_TIMEOUT in *dev_err.  No
 * counterpart in the reference (one device only). */
MZ_API int mz_peer_wait(const int32_t *signal, int32_t n_ranks, int32_t rank, uint32_t epoch,
                        uint64_t timeout_ns, int32_t *dev_err, mz_stream_t stream);

/* CUDA IPC for the gathered buffers and signal words: export writes an
 * MZ_IPC_HANDLE_BYTES handle of the allocation that holds `ptr` and ptr's
 * byte offset in it; open (in another process of the node, with its device
 * current) maps it and returns the mapping's base (for close) and base +
 * offset.  No counterpart in the reference (one device only). */
MZ_API int mz_ipc_export(const void *ptr, void *handle, uint64_t *offset);
MZ_API int mz_ipc_open(const void *handle, uint64_t offset, void **base, void **ptr);
MZ_API int mz_ipc_close(void *base);

/* mz_paged_decode without a workspace argument: it allocates nothing.
 * No counterpart in the reference (which has no device memory management);
 * it exists for callers that cannot allocate device memory when they call in,
 * e.g. a host whose own memory pool already owns the GPU, an FFI binding with
 * no device allocator of its own, or a latency-bound path where cudaMalloc's
 * implicit synchronisation is not allowed.
 * Scratch: a fixed 16 MiB array built into the library (a file-scope
 * __device__ array), held by every GPU that loads the library until the
 * process exits.  Sizes whose scratch would exceed it (see
 * mz_paged_decode_workspace_size) return MZ_ERR_TOO_LARGE; for the 8B-shape
 * batch of 64 sequences it needs about 8.5 MiB.
 * The first call on each device looks the array's address up with
 * cudaGetSymbolAddress (with that device current); make that first call before
 * any stream capture.  Each call clears the array's counters on `stream`
 * before its kernel.  All calls on a device share the one array, so calls that
 * overlap on the GPU (other streams, other host threads) race: serialise them.
 * Arguments and results are otherwise those of mz_paged_decode. */
MZ_API int mz_paged_decode_noalloc(void *out, int32_t out_dtype, int64_t out_seq_stride,
                                   int64_t out_tok_stride, int64_t out_head_stride, const void *q,
                                   int64_t q_seq_stride, int64_t q_tok_stride,
                                   int64_t q_head_stride, int32_t n_q_tokens, const void *k_pool,
                                   const void *v_pool, const int32_t *block_tables,
                                   int32_t max_blocks_per_seq, const int32_t *ctx_lens,
                                   int32_t n_seqs, int32_t n_heads, int32_t n_kv_heads,
                                   int32_t head_dim, int32_t block_size, int64_t n_blocks,
                                   float scale, int32_t dtype, int32_t num_warps,
                                   int32_t *dev_err, mz_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Prefix-cache block movement.                                              */
/* ------------------------------------------------------------------------ */

/* Copy whole blocks src_ids[i] -> dst_ids[i] in each of n_pools pools; pool p
 * starts at pool_base + p * pool_stride_bytes and holds n_blocks blocks of
 * block_bytes.  The data half of copy-on-write: BlockManager.copy_on_write,
 * src/mlxz/paged_attention/block_manager.py:111-134, leaves the copy to the
 * caller (:118).  It also replaces the prefix deep copies of
 * src/mlxz/prefix_cache/memory.py:19-35 when a shared partial block is
 * written.  dst ids must be distinct and must not appear in src_ids.
 * block_bytes and pool_stride_bytes must be multiples of 16 and pool_base
 * 16-byte aligned.  Bit-exact. */
MZ_API int mz_block_copy(void *pool_base, int64_t pool_stride_bytes, int32_t n_pools, int64_t block_bytes,
                  const int32_t *src_ids, const int32_t *dst_ids, int32_t n_copies,
                  int64_t n_blocks, int32_t *dev_err, mz_stream_t stream);

/* Gather blocks ids[0..n_ids) of every pool into a contiguous staging buffer
 * laid out [n_ids][n_pools][block_bytes] (the device side of eviction to the
 * pinned host tier; the caller then copies staging to host on a side stream).
 * Replaces the eviction path of PrefixCacheMemory._evict_until_room,
 * src/mlxz/prefix_cache/memory.py:181-192, which dropped entries instead of
 * moving them to a slower tier.  Same alignment rules as mz_block_copy. */
MZ_API int mz_block_pack(void *staging, const void *pool_base, int64_t pool_stride_bytes, int32_t n_pools,
                  int64_t block_bytes, const int32_t *ids, int32_t n_ids, int64_t n_blocks,
                  int32_t *dev_err, mz_stream_t stream);

/* Inverse of mz_block_pack: scatter staging [n_ids][n_pools][block_bytes] into
 * blocks ids[i] (the reload half: restore of an evicted prefix,
 * src/mlxz/engine/continuous.py:258-259). */
MZ_API int mz_block_unpack(void *pool_base, int64_t pool_stride_bytes, int32_t n_pools,
                    int64_t block_bytes, const void *staging, const int32_t *ids, int32_t n_ids,
                    int64_t n_blocks, int32_t *dev_err, mz_stream_t stream);

/* ------------------------------------------------------------------------ */
/* 4/8-bit affine group quantised KV.                                        */
/* ------------------------------------------------------------------------ */

/* Quantised pools, per layer and per K / V (the paged form of mlx_lm's
 * quantised cache state ((data, scales, biases), used by the reference at
 * src/mlxz/engine/cache_utils.py:12-92 and src/mlxz/prefix_cache/base.py:18)):
 *   codes  uint32 [n_blocks][n_kv_heads][block_size][head_dim * bits / 32],
 *          element i of a row at word i / (32/bits), bits (i % (32/bits))*bits
 *          upward (least significant first);
 *   scales fp16 [n_blocks][n_kv_heads][block_size][head_dim / 64], biases alike.
 * Per 64-value group, in IEEE fp32 round-to-nearest-even:
 *   scale = (max - min) / (2^bits - 1), s16 = fp16(scale), b16 = fp16(min),
 *   q = clamp(rint((w - b16) / s16), 0, 2^bits - 1), q = 0 when s16 == 0;
 *   dequantised value s16 * q + b16.  Inputs finite, |w| <= 65504.
 * Supported: bits 4 or 8, group_size 64, head_dim 64 or 128. */

/* Quantise-on-append by slot (the quantised form of mz_kv_append; replaces the
 * quantisation inside QuantizedKVCache.update_and_fetch that the reference
 * reaches through cache_utils.py:54-92).  k_new/v_new element (token i, head
 * h, dim d) at base + i*new_tok_stride + h*new_head_stride + d (dtype F16 or
 * BF16).  Negative slots skip.  Bit-exact to the rule above. */
MZ_API int mz_kv_quant_append(void *k_codes, void *k_scales, void *k_biases, void *v_codes,
                              void *v_scales, void *v_biases, const void *k_new, const void *v_new,
                              int64_t new_tok_stride, int64_t new_head_stride,
                              const int64_t *slot_mapping, int64_t n_tokens, int32_t n_kv_heads,
                              int32_t head_dim, int32_t block_size, int64_t n_blocks, int32_t bits,
                              int32_t group_size, int32_t dtype, int32_t *dev_err,
                              mz_stream_t stream);

/* Decode-step form: one token per sequence at positions[b] through the block
 * table (the quantised form of mz_kv_append_paged). */
MZ_API int mz_kv_quant_append_paged(void *k_codes, void *k_scales, void *k_biases, void *v_codes,
                                    void *v_scales, void *v_biases, const void *k_new,
                                    const void *v_new, int64_t new_seq_stride,
                                    int64_t new_head_stride, const int32_t *block_tables,
                                    int32_t max_blocks_per_seq, const int32_t *positions,
                                    int32_t n_seqs, int32_t n_kv_heads, int32_t head_dim,
                                    int32_t block_size, int64_t n_blocks, int32_t bits,
                                    int32_t group_size, int32_t dtype, int32_t *dev_err,
                                    mz_stream_t stream);

/* Dequantise whole quantised blocks into a 16-bit staging pool: block
 * block_ids[i] of the quantised K and V pools (layout of mz_kv_quant_append)
 * becomes block i of k_out / v_out, [n_ids][n_kv_heads][block_size][head_dim]
 * of out_dtype (F16 or BF16), value = f32(scale) * q + f32(bias) rounded to
 * out_dtype.  Ids outside [0, n_blocks): MZ_DEVERR_BLOCK_ID, block skipped.
 * Used for the prompt pass over a quantised cache: mlx_lm's QuantizedKVCache
 * (src/mlxz/engine/cache_utils.py:54-92) attends a prompt chunk over the
 * quantised keys and values; here the chunk's blocks are dequantised once per
 * layer and mz_paged_prefill runs on them. */
MZ_API int mz_kv_dequant_blocks(void *k_out, void *v_out, int32_t out_dtype, const void *k_codes,
                                const void *k_scales, const void *k_biases, const void *v_codes,
                                const void *v_scales, const void *v_biases,
                                const int32_t *block_ids, int32_t n_ids, int32_t n_kv_heads,
                                int32_t head_dim, int32_t block_size, int64_t n_blocks,
                                int32_t bits, int32_t *dev_err, mz_stream_t stream);

/* Workspace bytes for mz_paged_decode_q (same layout rules as
 * mz_paged_decode_workspace_size). */
MZ_API int mz_paged_decode_q_workspace_size(int32_t n_seqs, int32_t n_kv_heads,
                                            int32_t rows_per_kv_head, int32_t head_dim,
                                            int32_t bits, int32_t num_warps, int32_t device,
                                            size_t *bytes);

/* Paged decode attention over quantised K/V with the dequantisation fused in
 * (attention over the dequantised values s16 * q + b16; the reference attends
 * over mlx_lm's quantised cache through mx.quantized_matmul).  Arguments as
 * mz_paged_decode, with the six quantised pools in place of the K/V pools; q
 * (and out unless F32) of element type `dtype`, converted to fp16 for the
 * products (exact for bf16 values with fp16-representable magnitude).
 * Pools need 16-byte alignment. */
MZ_API int mz_paged_decode_q(void *out, int32_t out_dtype, int64_t out_seq_stride,
                             int64_t out_tok_stride, int64_t out_head_stride, const void *q,
                             int64_t q_seq_stride, int64_t q_tok_stride, int64_t q_head_stride,
                             int32_t n_q_tokens, const void *k_codes, const void *k_scales,
                             const void *k_biases, const void *v_codes, const void *v_scales,
                             const void *v_biases, const int32_t *block_tables,
                             int32_t max_blocks_per_seq, const int32_t *ctx_lens, int32_t n_seqs,
                             int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                             int32_t block_size, int64_t n_blocks, int32_t bits,
                             int32_t group_size, float scale, int32_t dtype, int32_t num_warps,
                             void *workspace, size_t workspace_bytes, int32_t *dev_err,
                             mz_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MLXZ_B200_H */
