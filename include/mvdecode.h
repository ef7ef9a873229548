/*
 * mvdecode -- B200 (sm_100a) paged GQA decode attention and paged KV append.
 *
 * C ABI of libmvdecode.so. Every entry point takes plain device pointers,
 * element strides and sizes, enqueues work on the caller's CUDA stream and
 * returns an MV_* status code; on failure mv_last_error() names the problem
 * (thread-local). Nothing here synchronises the device or reads device
 * memory from the host. Call with the device that owns the pointers current.
 *
 * Layouts (the reference's own, so a micro-vllm cache drops in unchanged):
 *   q, out        [batch, num_q_heads, head_dim]   head_dim stride 1, outer strides given
 *   K/V pages     [num_blocks, num_kv_heads, block_size, head_dim]  contiguous
 *   block_table   [batch, >= blocks_per_seq]       row stride given, int32 or int64
 *   context_lens  [batch]                          tokens to attend, incl. this step's
 * Query head j uses KV head j / (num_q_heads / num_kv_heads).
 */
#ifndef MVDECODE_H_
#define MVDECODE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define MV_API __attribute__((visibility("default")))
#else
#define MV_API
#endif

#define MV_ABI_VERSION 1

/* Element type of q, pages and outputs. */
#define MV_DTYPE_F32 0
#define MV_DTYPE_F16 1
#define MV_DTYPE_BF16 2

/* Integer type of block tables, context lengths and positions. */
#define MV_INDEX_I32 0
#define MV_INDEX_I64 1

/* Meaning of a per-sequence position array given to mv_write_paged_kv. */
#define MV_POSITIONS_START 0 /* logical slot of the first new token */
#define MV_POSITIONS_END 1   /* length after the append; first slot = end - num_tokens */

/* Flags for mv_paged_decode / mv_paged_decode_workspace_size. */
#define MV_FLAG_FORCE_SIMT 1u /* use the CUDA-core kernel even where the tensor-core one applies */
#define MV_FLAG_PERSISTENT 2u /* tensor-core kernel on the persistent schedule instead of the split grid */
#define MV_FLAG_FUSED_MERGE 4u /* split grid: the last split CTA of each sequence/head merges it */
#define MV_FLAG_CLUSTER 8u /* tensor-core cluster kernel (contexts up to 8192 tokens), no merge pass */
#define MV_FLAG_WIDE 16u /* split grid in the wide shape (8 warps, deeper rings; head_dim 64/128) */
#define MV_FLAG_CHUNK_ROWS 32u /* mv_paged_chunk_attention: one query row per token, not query tiles */
#define MV_FLAG_CHUNK_MMA_SYNC 64u /* mv_paged_chunk_attention: 64-row mma.sync tiles, not tcgen05 tiles */
#define MV_FLAG_CUDA_CORE_MATH 128u /* split grid (default shape, GQA group <= 8, head_dim 64/128): the same TMA
                                      pipeline with fp32 FMA math instead of the tensor-core tile (for comparison) */
#define MV_FLAG_STREAM 256u /* tensor-core kernel on the per-warp stream schedule wherever its shape allows
                              (bf16/fp16, page 16, head_dim 64/128, GQA group <= 8, at most 1024 sequences,
                              pages_per_split <= 64 or 0 for automatic); MV_ERR_UNSUPPORTED elsewhere */
#define MV_FLAG_SPLIT_GRID 512u /* never pick the stream schedule automatically (keep the split grid) */

/* Status codes. */
#define MV_OK 0
#define MV_ERR_INVALID_ARGUMENT 1
#define MV_ERR_UNSUPPORTED 2
#define MV_ERR_WORKSPACE_TOO_SMALL 3
#define MV_ERR_CUDA 4

/* Device status bits (sticky, per device; see mv_device_status). */
#define MV_DEVICE_STATUS_WAIT_TIMEOUT 1u
#define MV_DEVICE_STATUS_BAD_PAGE_ID 2u /* a used block-table entry was outside [0, num_blocks): its rows are NaN, its write skipped */

/* Kernel paths reported by mv_paged_decode_plan. */
#define MV_PATH_SIMT 0            /* CUDA cores, one CTA per (split, KV head, sequence) */
#define MV_PATH_TMA_MMA 1         /* TMA + tensor cores, one CTA per (split, KV head, sequence) */
#define MV_PATH_TMA_MMA_PERSISTENT 2 /* TMA + tensor cores, persistent, equal page ranges per warp */
#define MV_PATH_TMA_MMA_CLUSTER 3 /* TMA + tensor cores, one CTA cluster per (sequence, KV head) */
#define MV_PATH_TMA_MMA_STREAM 4  /* TMA + tensor cores, one CTA per SM, every warp an independent page stream over
                                     a queue of (sequence, KV head, run of pages) items; the split merge after */

MV_API int mv_abi_version(void);

/* Message for the last non-MV_OK status returned on this thread. */
MV_API const char* mv_last_error(void);

/*
 * Workspace bytes mv_paged_decode needs for this geometry on the current
 * device (0 when no split-KV pass is needed). max_context_len bounds every
 * context length; pages_per_split 0 lets the library choose.
 * Replaces no reference call: the reference kernel allocates an output-sized
 * running buffer itself (src/micro_vllm/csrc/online_attention.cuh:154-156).
 */
MV_API int mv_paged_decode_workspace_size(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                   int32_t head_dim, int32_t block_size, int64_t max_context_len,
                                   int32_t pages_per_split, uint32_t flags, int32_t dtype,
                                   size_t* bytes);

/*
 * Which kernel mv_paged_decode would run, and its split-KV shape. k_cache and
 * v_cache are only inspected for alignment. With pages_per_split == 0 the
 * default tensor-core split grid may give each sequence's first split up to
 * twice chosen_pages_per_split pages (at most 128); max_splits counts that.
 */
MV_API int mv_paged_decode_plan(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                         int32_t head_dim, int32_t block_size, int64_t max_context_len,
                         int32_t pages_per_split, uint32_t flags, int32_t dtype,
                         const void* k_cache, const void* v_cache,
                         int32_t* path, int32_t* chosen_pages_per_split, int32_t* max_splits);

/*
 * Paged GQA decode attention: for every sequence b and query head j,
 *   out[b, j] = softmax(scale * K_b q[b, j]) V_b
 * over the first context_lens[b] tokens of the pages block_table[b, :].
 *
 * Replaces the reference's _decode_attention_paged(query, key_pages,
 * value_pages, table, length) (src/micro_vllm/csrc/decode_attention.cpp:147-152,
 * launched at decode_attention_paged.cu:51-57): that call is batch 1, with
 * context_lens == NULL, max_context_len == length, an int64 table and
 * scale == head_dim ** -0.5.
 *
 * context_lens may be NULL: every sequence then attends max_context_len tokens.
 * Device-side contract (the host cannot see device lengths or table contents):
 *   - a used page whose ID is outside [0, num_blocks) makes that sequence's
 *     whole GQA group NaN, with no out-of-bounds read (as the reference);
 *   - a length of 0 gives zeros; a negative length, or one above
 *     max_context_len or blocks_per_seq * block_size, gives NaN.
 * workspace: mv_paged_decode_workspace_size bytes of device scratch (may be
 * NULL when that size is 0). Its first 256 KiB hold split arrival counters:
 * zero-fill the buffer before its first use; every completed call leaves those
 * counters at zero again (nothing else is written there), so a buffer is
 * zeroed once and reused by later calls of any shape. Calls that share a
 * workspace must not overlap on the GPU (order them on one stream).
 * dtype: MV_DTYPE_* of q, pages and out; accumulation is fp32.
 */
MV_API int mv_paged_decode(const void* q, int64_t q_stride_seq, int64_t q_stride_head,
                    const void* k_cache, const void* v_cache, int64_t num_blocks,
                    int32_t num_kv_heads, int32_t block_size, int32_t head_dim,
                    const void* block_table, int32_t block_table_type,
                    int64_t block_table_stride, int64_t blocks_per_seq,
                    const void* context_lens, int32_t context_lens_type,
                    int64_t max_context_len, int32_t batch, int32_t num_q_heads, float scale,
                    void* out, int64_t out_stride_seq, int64_t out_stride_head,
                    void* workspace, size_t workspace_bytes, int32_t pages_per_split,
                    uint32_t flags, int32_t dtype, void* stream);

/*
 * Attention of a chunk of num_tokens new tokens per sequence over its pages:
 * query token t of sequence b (q[b, t], [batch, num_tokens, num_q_heads,
 * head_dim] with the given element strides) attends the first
 * context_lens[b] - (num_tokens - 1 - t) tokens -- its causal prefix, the
 * chunk's own earlier tokens included; context_lens counts the tokens after
 * the chunk, whose K/V must already be in the pages (mv_write_paged_kv).
 *
 * Replaces the reference's cached multi-token path, which gathers the pages
 * into contiguous K/V and runs causal attention
 * (src/micro_vllm/model.py:178-182, paged_kv_cache.py:178-193,
 * attention.py:57-94). fp16/bf16 with head_dim 64 or 128, 16-token pages,
 * at least 16 (token x query head) rows per (sequence, KV head) and a 4-byte
 * aligned query run as query tiles on tensor cores that share one stream of
 * the pages: 128 rows per CTA on tcgen05 (TMEM accumulators) from 64 rows up
 * with a 16-byte aligned query, else 64 rows per CTA on mma.sync
 * (MV_FLAG_CHUNK_MMA_SYNC forces these). Otherwise -- or with MV_FLAG_CHUNK_ROWS --
 * the split grid or the CUDA-core kernel run one decode query row per
 * (sequence, token), each reading its own prefix. Workspace:
 * mv_paged_chunk_workspace_size. Flags PERSISTENT, CLUSTER, WIDE and
 * FUSED_MERGE are ignored. Other contracts as mv_paged_decode.
 */
/*
 * Workspace bytes mv_paged_chunk_attention needs for this geometry (the same
 * arguments, num_tokens per sequence). No reference counterpart: the
 * reference's chunk path allocates its gathered K/V itself.
 */
MV_API int mv_paged_chunk_workspace_size(int32_t batch, int32_t num_tokens, int32_t num_q_heads,
                                         int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                         int64_t max_context_len, int32_t pages_per_split, uint32_t flags,
                                         int32_t dtype, size_t* bytes);

MV_API int mv_paged_chunk_attention(const void* q, int64_t q_stride_seq, int64_t q_stride_token,
                                    int64_t q_stride_head, const void* k_cache, const void* v_cache,
                                    int64_t num_blocks, int32_t num_kv_heads, int32_t block_size,
                                    int32_t head_dim, const void* block_table,
                                    int32_t block_table_type, int64_t block_table_stride,
                                    int64_t blocks_per_seq, const void* context_lens,
                                    int32_t context_lens_type, int64_t max_context_len,
                                    int32_t batch, int32_t num_tokens, int32_t num_q_heads,
                                    float scale, void* out, int64_t out_stride_seq,
                                    int64_t out_stride_token, int64_t out_stride_head,
                                    void* workspace, size_t workspace_bytes, int32_t pages_per_split,
                                    uint32_t flags, int32_t dtype, void* stream);

/*
 * GQA decode over contiguous caches: for every sequence b and query head j,
 *   out[b, j] = softmax(scale * K_b q[b, j]) V_b
 * over the first context_lens[b] tokens (all sequences: max_context_len when
 * context_lens is NULL) of K_b = k_cache[b, j / G, 0:len, :], which holds
 * cache_len tokens. Element strides per sequence, KV head and token (feature
 * stride 1; zero strides broadcast), for K and V separately.
 *
 * Replaces the reference's decode_attention_gqa(query, key, value)
 * (src/micro_vllm/csrc/decode_attention.cpp:138-142, kernel
 * decode_attention_online.cu:47-52): that call is batch 1, context_lens NULL,
 * max_context_len == cache_len == key.size(2), scale == head_dim ** -0.5.
 * Caches whose base and strides in use are 16-byte multiples run the
 * tensor-core split grid (fp16/bf16, head_dim 64/128/256, GQA group <= 16),
 * every other case the CUDA-core kernel; the workspace contract is
 * mv_paged_decode's, sized by mv_contiguous_decode_plan. Lengths above the
 * bound give NaN rows, as in mv_paged_decode.
 */
MV_API int mv_contiguous_decode_plan(const void* k_cache, int64_t k_stride_seq, int64_t k_stride_head,
                                     int64_t k_stride_token, const void* v_cache,
                                     int64_t v_stride_seq, int64_t v_stride_head,
                                     int64_t v_stride_token, int64_t cache_len,
                                     int32_t num_kv_heads, int32_t head_dim,
                                     int64_t max_context_len, int32_t batch, int32_t num_q_heads,
                                     int32_t pages_per_split, uint32_t flags, int32_t dtype,
                                     int32_t* path, int32_t* chosen_pages_per_split,
                                     int32_t* max_splits, size_t* workspace_bytes);
MV_API int mv_contiguous_decode(const void* q, int64_t q_stride_seq, int64_t q_stride_head,
                                const void* k_cache, int64_t k_stride_seq, int64_t k_stride_head,
                                int64_t k_stride_token, const void* v_cache, int64_t v_stride_seq,
                                int64_t v_stride_head, int64_t v_stride_token, int64_t cache_len,
                                int32_t num_kv_heads, int32_t head_dim, const void* context_lens,
                                int32_t context_lens_type, int64_t max_context_len, int32_t batch,
                                int32_t num_q_heads, float scale, void* out, int64_t out_stride_seq,
                                int64_t out_stride_head, void* workspace, size_t workspace_bytes,
                                int32_t pages_per_split, uint32_t flags, int32_t dtype, void* stream);

/*
 * Paged KV append (reshape-and-cache): token t of sequence b goes to logical
 * position start_b + t, i.e. page block_table[b, pos / block_size], slot
 * pos % block_size. Copies are bit-exact (no conversion).
 *
 * Replaces the reference's write_paged_kv(key, value, key_pages, value_pages,
 * page_table, start) (src/micro_vllm/csrc/paged_kv_cache.cpp:96-107, kernel
 * paged_kv_cache.cu:44-62): that call is batch 1, positions == NULL and start
 * the host-side start.
 *
 * key/value: [batch, num_kv_heads, num_tokens, head_dim] with the given element
 * strides (feature stride 1; zero strides broadcast). positions: NULL (every
 * sequence starts at `start`) or a device array read per positions_kind.
 * A token whose position is negative, beyond blocks_per_seq pages, or whose
 * physical page ID is outside [0, num_blocks) is skipped, never written out of
 * bounds (as the reference kernel skips bad IDs).
 */
MV_API int mv_write_paged_kv(const void* key, int64_t key_stride_seq, int64_t key_stride_head,
                      int64_t key_stride_token, const void* value, int64_t value_stride_seq,
                      int64_t value_stride_head, int64_t value_stride_token, void* k_cache,
                      void* v_cache, int64_t num_blocks, int32_t num_kv_heads,
                      int32_t block_size, int32_t head_dim, const void* block_table,
                      int32_t block_table_type, int64_t block_table_stride,
                      int64_t blocks_per_seq, const void* positions, int32_t positions_type,
                      int32_t positions_kind, int64_t start, int32_t batch, int32_t num_tokens,
                      int32_t dtype, void* stream);

/*
 * One decode step's append and attention in one call: the same result, in the
 * pool and in out, as mv_write_paged_kv(key, value, ..., positions =
 * context_lens, MV_POSITIONS_END, num_tokens = 1) followed by
 * mv_paged_decode(...) on the same stream. With context_lens NULL the row goes
 * to position max_context_len - 1 of every sequence.
 *
 * Replaces the pair of reference calls the decode layer makes per step:
 * PagedKVCache.append -> _write_paged_kv (src/micro_vllm/paged_kv_cache.py:163-172)
 * and then decode_attention_paged (src/micro_vllm/model.py:215-216, 177).
 *
 * key/value: [batch, num_kv_heads] rows of head_dim elements, feature stride 1,
 * element strides per sequence and per head. Where the split-grid tensor-core
 * kernel runs (mv_paged_decode_plan path MV_PATH_TMA_MMA) with 16-byte aligned
 * rows, or the CUDA-core kernel (MV_PATH_SIMT), the CTA that attends a
 * sequence's last page writes the row into the pool and into its staged copy
 * of that page: no separate append launch. Otherwise the append kernel runs
 * first (two launches). The page that
 * receives a sequence's new row must not be read by another sequence in the
 * same call (as with any in-place append); the other arguments and contracts
 * are those of mv_paged_decode.
 *
 * rope_cos/rope_sin (both or NULL): [rope_rows, head_dim] tables of the element
 * type (row p = the reference's rope_cos_sin at position p,
 * src/micro_vllm/model.py:79-98). When given, q and key arrive unrotated and
 * are rotated at position context_lens[b] - 1 inside the decode kernel, as
 * apply_rope does before the append (model.py:110-123, 214-215); the pool
 * receives the rotated key. A position without a table row gives a NaN group
 * and no write. Needs the fused path (an even head_dim; on MV_PATH_TMA_MMA
 * 16-byte aligned rows and tables): otherwise MV_ERR_UNSUPPORTED -- rotate
 * with mv_apply_rope first and pass NULL tables.
 */
MV_API int mv_paged_decode_append(const void* q, int64_t q_stride_seq, int64_t q_stride_head,
                                  const void* key, int64_t key_stride_seq, int64_t key_stride_head,
                                  const void* value, int64_t value_stride_seq,
                                  int64_t value_stride_head, const void* rope_cos,
                                  const void* rope_sin, int64_t rope_rows, void* k_cache,
                                  void* v_cache,
                                  int64_t num_blocks, int32_t num_kv_heads, int32_t block_size,
                                  int32_t head_dim, const void* block_table,
                                  int32_t block_table_type, int64_t block_table_stride,
                                  int64_t blocks_per_seq, const void* context_lens,
                                  int32_t context_lens_type, int64_t max_context_len,
                                  int32_t batch, int32_t num_q_heads, float scale, void* out,
                                  int64_t out_stride_seq, int64_t out_stride_head, void* workspace,
                                  size_t workspace_bytes, int32_t pages_per_split, uint32_t flags,
                                  int32_t dtype, void* stream);

/*
 * Rotate-half RoPE of rows: out[b, h, t, :] = x * cos[p] + rotate_half(x) * sin[p]
 * at position p = start_b + t, each product and the sum rounded to the element
 * type as the reference's apply_rope computes them (src/micro_vllm/model.py:101-123,
 * called from model.py:214). x/out: [batch, heads, num_tokens, head_dim] with the
 * given element strides (feature stride 1); out may be x itself (in place).
 * cos/sin: [table_rows, head_dim] tables of the element type. positions: NULL
 * (start_b = start) or a device array read per positions_kind, as in
 * mv_write_paged_kv. A row whose position has no table row becomes NaN.
 * Replaces the reference's apply_rope for the batched path (no reference
 * native counterpart: the reference computes it with torch tensor operations).
 */
MV_API int mv_apply_rope(const void* x, int64_t x_stride_seq, int64_t x_stride_head,
                         int64_t x_stride_token, void* out, int64_t out_stride_seq,
                         int64_t out_stride_head, int64_t out_stride_token, int32_t batch,
                         int32_t heads, int32_t num_tokens, int32_t head_dim, const void* cos,
                         const void* sin, int64_t table_rows, const void* positions,
                         int32_t positions_type, int32_t positions_kind, int64_t start,
                         int32_t dtype, void* stream);

/*
 * Row operations of the batched runtime's decode step (the reference computes
 * them with torch tensor operations; no native counterpart).
 * mv_rms_norm: out[r] = weight * to_dtype(x[r] * rsqrt(mean(x[r]^2) + eps)) with
 * fp32 statistics (src/micro_vllm/model.py:25-41); rows of `hidden` elements at
 * the given element row strides.
 * mv_silu_mul: out[r] = to_dtype(silu(g)) * u for rows [g | u] of 2 * width
 * elements (a fused gate/up projection), each step rounded to the element type
 * as F.silu(gate) * up is (model.py:150-165).
 */
MV_API int mv_rms_norm(const void* x, int64_t x_stride_row, const void* weight, void* out,
                       int64_t out_stride_row, int64_t rows, int32_t hidden, float eps,
                       int32_t dtype, void* stream);
MV_API int mv_silu_mul(const void* gate_up, int64_t stride_row, void* out, int64_t out_stride_row,
                       int64_t rows, int32_t width, int32_t dtype, void* stream);

/*
 * mv_paged_decode for callers that cannot allocate device memory. No
 * counterpart in the reference (its kernel allocates its own output-sized
 * buffer). Some callers of a decode kernel may not call cudaMalloc: a plugin
 * whose host owns every device allocation (a serving engine that reserves all
 * memory up front and hands the plugin only inputs and outputs) has no
 * workspace to give and no right to take one. This entry point takes the same
 * arguments as mv_paged_decode minus the workspace and allocates nothing: its
 * split-KV scratch is a file-scope device array of MV_NOALLOC_SCRATCH_BYTES
 * that every GPU loading the library holds until the process exits.
 *   - Calls whose split plan needs more scratch than that (planned as the
 *     call itself would run, including the caches' alignment) are rejected
 *     with MV_ERR_UNSUPPORTED and a message naming the sizes;
 *     MV_FLAG_FUSED_MERGE is rejected too (its counters would have to start
 *     at zero).
 *   - A call outside stream capture looks up the array's device address
 *     (with the call's device current) and keeps it; a call inside a capture
 *     uses the kept one. So the first call on a device, and the first after
 *     a cudaDeviceReset of it, must come before any stream capture.
 *   - Every call shares the one array and leaves its partial results in it:
 *     calls that overlap on the GPU (other streams, other threads) race.
 */
#define MV_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

MV_API int mv_paged_decode_noalloc(const void* q, int64_t q_stride_seq, int64_t q_stride_head,
                                   const void* k_cache, const void* v_cache, int64_t num_blocks,
                                   int32_t num_kv_heads, int32_t block_size, int32_t head_dim,
                                   const void* block_table, int32_t block_table_type,
                                   int64_t block_table_stride, int64_t blocks_per_seq,
                                   const void* context_lens, int32_t context_lens_type,
                                   int64_t max_context_len, int32_t batch, int32_t num_q_heads,
                                   float scale, void* out, int64_t out_stride_seq,
                                   int64_t out_stride_head, int32_t pages_per_split,
                                   uint32_t flags, int32_t dtype, void* stream);

/*
 * The one-call decode step with its arguments in one struct: every field is
 * 8 bytes wide, in this order, with no padding. No reference counterpart: the
 * same call as mv_paged_decode_append (key and value non-NULL) or
 * mv_paged_decode (both NULL; the RoPE fields then unused), for bindings that
 * pay per marshalled argument (ctypes: ~0.4 us each, so a 35-argument call
 * costs more host time than a small decode step takes on the GPU). A caller
 * fills the struct once and changes only the fields that change per step.
 * The int64 fields standing for int32 arguments must fit in int32.
 */
typedef struct MvDecodeStepArgs {
    const void* q; int64_t q_stride_seq; int64_t q_stride_head;
    const void* key; int64_t key_stride_seq; int64_t key_stride_head;
    const void* value; int64_t value_stride_seq; int64_t value_stride_head;
    const void* rope_cos; const void* rope_sin; int64_t rope_rows;
    void* k_cache; void* v_cache; int64_t num_blocks; int64_t num_kv_heads; int64_t block_size;
    int64_t head_dim;
    const void* block_table; int64_t block_table_type; int64_t block_table_stride; int64_t blocks_per_seq;
    const void* context_lens; int64_t context_lens_type; int64_t max_context_len;
    int64_t batch; int64_t num_q_heads; double scale;
    void* out; int64_t out_stride_seq; int64_t out_stride_head;
    void* workspace; uint64_t workspace_bytes; int64_t pages_per_split; uint64_t flags; int64_t dtype;
} MvDecodeStepArgs;

MV_API int mv_paged_decode_step_args(const MvDecodeStepArgs* args, void* stream);

/*
 * Sticky MV_DEVICE_STATUS_* bits kernels have raised on `device` (a bounded
 * wait that gave up; a used page ID outside the pool). Reading synchronises with the device's legacy stream.
 */
MV_API int mv_device_status(int32_t device, uint32_t* status);
MV_API int mv_clear_device_status(int32_t device);

/*
 * Self-test of the failure path (no reference counterpart: the reference's
 * kernels have no bounded waits): launches one CTA on `stream` (current
 * device) that waits on a barrier phase nothing completes, with the kernels'
 * bounded wait shortened to limit_ns (at most 100 ms). The wait gives up, the
 * kernel raises MV_DEVICE_STATUS_WAIT_TIMEOUT exactly as a decode kernel
 * whose load never landed would, and returns; the context stays usable.
 */
MV_API int mv_selftest_wait_timeout(uint64_t limit_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MVDECODE_H_ */
