// Device-side building blocks shared by the decode and append kernels:
// launch parameters, index/length helpers, and thin inline-PTX wrappers for
// mbarriers, TMA tensor loads, ldmatrix, mma.sync and movmatrix on sm_100a.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

namespace mv {

// Sticky per-device error bits (MV_DEVICE_STATUS_*), raised by kernels whose
// bounded waits gave up. Zero at module load; cleared only by the host.
__device__ unsigned int g_device_status;

constexpr unsigned kStatusWaitTimeout = 1u;
constexpr unsigned kStatusBadPageId = 2u;

// A used block-table entry outside the pool: its rows become NaN (or its
// write is skipped); the sticky status records that it happened.
__device__ __forceinline__ void report_bad_page_id() { atomicOr(&g_device_status, kStatusBadPageId); }
// A bounded wait gives up after this long; nothing legitimate takes it.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

// Every non-empty workspace starts with this many zero-initialised unsigned
// counters (256 KiB); the kernels that use them leave them zero when they end.
constexpr int kCounterRegionSlots = 65536;

struct DecodeParams {
    const void* q;
    int64_t q_stride_seq;
    int64_t q_stride_head;
    const void* k_cache;
    const void* v_cache;
    int64_t num_blocks;
    int kv_heads;
    int block_size;
    int head_dim;
    int group;              // query heads per KV head
    int q_heads;
    int batch;
    const void* block_table;
    int table_i64;
    int64_t table_stride;
    int64_t blocks_per_seq;
    const void* context_lens;  // nullptr: every sequence has uniform_len tokens
    int lens_i64;
    int64_t uniform_len;
    int64_t max_context_len;
    float scale_log2;       // softmax scale * log2(e): scores live in the exp2 domain
    void* out;
    int64_t out_stride_seq;
    int64_t out_stride_head;
    float* part_o;          // [batch, q_heads, max_splits, head_dim]  normalised partial outputs
    float* part_lse;        // [batch, q_heads, max_splits]            log2-sum-exp of each split
    int pages_per_split;
    int max_splits;
    // Split grid: pages of split 0 when it is longer than the rest (0: every
    // split has pages_per_split pages). A nonzero value also orders the grid
    // split-major: every sequence's split 0 is dispatched before any split 1,
    // so the long first splits start in the first wave and the short later
    // ones fill the tail.
    int first_pages;
    int64_t* prefix_out;    // persistent schedule: per-sequence page prefix sums [batch + 1]
    int64_t persistent_warps;  // persistent schedule: warps in the grid
    unsigned int* counters; // split grid: per-(sequence, KV head) arrival counters, zero between calls
    int fused_merge;        // split grid: the last split CTA of a segment merges it
    // Split grid, fused append: this step's K/V row of every (sequence, KV
    // head), [batch, kv_heads] with feature stride 1, is written into the pool
    // at position len - 1 by the CTA that attends that page. nullptr: no append.
    const void* new_key;
    const void* new_value;
    int64_t new_key_stride[2];    // seq, head (elements)
    int64_t new_value_stride[2];
    // Fused RoPE (with the fused append): q and the new K rows arrive unrotated
    // and are rotated at position len - 1 with rows of these [rope_rows, D]
    // tables of the element type. nullptr: q and K are already rotated.
    const void* rope_cos;
    const void* rope_sin;
    int64_t rope_rows;
    // Contiguous caches (no block table; block_table is nullptr): token t of
    // KV head h of sequence b at k_cache + b*k_stride[0] + h*k_stride[1] +
    // t*k_stride[2] (V likewise with v_stride); "pages" are runs of
    // block_size tokens, and max_context_len never exceeds the cache length.
    int contiguous;
    int64_t k_stride[3];
    int64_t v_stride[3];
    // Query rows: `batch` counts rows, and row z is token t = z % q_tokens of
    // sequence z / q_tokens (a chunk of q_tokens new tokens per sequence; 1
    // for decode). Row t attends the first len - (q_tokens - 1 - t) tokens,
    // len being the sequence's length after the chunk; q and out of row z at
    // seq * *_stride_seq + t * *_stride_token.
    int q_tokens;
    int64_t q_stride_token;
    int64_t out_stride_token;
    // Split grid with first_pages: splits from the third on hold later_pages
    // pages (0: pages_per_split), so the splits dispatched last are shorter.
    int later_pages;
    // Split grid: CTAs whose dispatch index is below this (the first wave of
    // resident CTAs) warm L2 with their first prewait_pages pages per warp
    // before waiting for the previous grid (0: none).
    int prewait_ctas;
    int prewait_pages;
};

struct AppendParams {
    const void* key;
    const void* value;
    int64_t key_stride[3];    // seq, head, token (elements)
    int64_t value_stride[3];
    void* k_cache;
    void* v_cache;
    int64_t num_blocks;
    int kv_heads;
    int block_size;
    int row_bytes;            // head_dim * element size
    const void* block_table;
    int table_i64;
    int64_t table_stride;
    int64_t blocks_per_seq;
    const void* positions;
    int positions_i64;
    int positions_end;        // positions hold the end of the sequence, not the start
    int64_t start;
    int batch;
    int num_tokens;
    int elem_bytes;
};

__device__ __forceinline__ int64_t load_index(const void* base, int is64, int64_t i) {
    return is64 ? __ldg(static_cast<const long long*>(base) + i)
                : static_cast<int64_t>(__ldg(static_cast<const int*>(base) + i));
}

// An index read through L2 only (ld.global.cg: no L1 line is filled), for reads
// made before the grid-dependency wait: the value may predate the previous
// grid's writes, so it may only steer prefetches, and no later load of this
// kernel can hit a stale L1 copy of it.
__device__ __forceinline__ int64_t load_index_l2_hint(const void* base, int is64, int64_t i) {
    if (is64) {
        long long v;
        asm volatile("ld.global.cg.s64 %0, [%1];" : "=l"(v) : "l"(static_cast<const long long*>(base) + i));
        return v;
    }
    int v;
    asm volatile("ld.global.cg.s32 %0, [%1];" : "=r"(v) : "l"(static_cast<const int*>(base) + i));
    return v;
}

__device__ __forceinline__ int64_t row_seq(const DecodeParams& p, int64_t z) {
    return p.q_tokens > 1 ? z / p.q_tokens : z;
}

__device__ __forceinline__ int64_t row_q_offset(const DecodeParams& p, int64_t z) {
    if (p.q_tokens <= 1) return z * p.q_stride_seq;
    const int64_t b = z / p.q_tokens;
    return b * p.q_stride_seq + (z - b * p.q_tokens) * p.q_stride_token;
}

__device__ __forceinline__ int64_t row_out_offset(const DecodeParams& p, int64_t z) {
    if (p.q_tokens <= 1) return z * p.out_stride_seq;
    const int64_t b = z / p.q_tokens;
    return b * p.out_stride_seq + (z - b * p.q_tokens) * p.out_stride_token;
}

// How one query row's context is cut into split-KV chunks: a first split of
// first_pages pages (when set), then splits of pages_per_split pages.
struct SeqSplit {
    int64_t len;
    int64_t pages;
    int splits;
    int state;  // 0 attend, 1 empty (zeros), 2 invalid (NaN)
};

__device__ __forceinline__ SeqSplit seq_split(const DecodeParams& p, int b) {
    SeqSplit s;
    const int64_t seq = row_seq(p, b);
    s.len = p.context_lens ? load_index(p.context_lens, p.lens_i64, seq) : p.uniform_len;
    if (p.q_tokens > 1) s.len -= p.q_tokens - 1 - (b - seq * p.q_tokens);  // causal within the chunk
    const bool in_range = s.len >= 0 && s.len <= p.max_context_len &&
                          s.len <= p.blocks_per_seq * p.block_size;
    if (!in_range) {
        s.state = 2;
    } else if (s.len == 0) {
        s.state = 1;
    } else {
        s.state = 0;
    }
    s.pages = s.state == 0 ? (s.len + p.block_size - 1) / p.block_size : 0;
    // The last split is partial. Measured on B200, evening out the splits'
    // sizes was slower: the small last splits fill the tail of the grid.
    const int64_t later = p.later_pages > 0 ? p.later_pages : p.pages_per_split;
    const int64_t two = static_cast<int64_t>(p.first_pages) + p.pages_per_split;
    const int64_t splits = p.first_pages > 0
                               ? (s.pages <= p.first_pages ? 1
                                  : s.pages <= two        ? 2
                                                          : 2 + (s.pages - two + later - 1) / later)
                               : (s.pages + p.pages_per_split - 1) / p.pages_per_split;
    s.splits = splits < 1 ? 1 : static_cast<int>(splits);
    return s;
}

// First page of split `split`; it does not depend on the sequence's length.
__device__ __forceinline__ int64_t split_begin(const DecodeParams& p, int split) {
    if (p.first_pages > 0) {
        if (split <= 1) return split == 0 ? 0 : p.first_pages;
        const int64_t later = p.later_pages > 0 ? p.later_pages : p.pages_per_split;
        return p.first_pages + p.pages_per_split + static_cast<int64_t>(split - 2) * later;
    }
    return static_cast<int64_t>(split) * p.pages_per_split;
}

// Pages a full split `split` holds.
__device__ __forceinline__ int split_pages(const DecodeParams& p, int split) {
    if (p.first_pages <= 0 || split == 1) return p.pages_per_split;
    if (split == 0) return p.first_pages;
    return p.later_pages > 0 ? p.later_pages : p.pages_per_split;
}

// Pages [begin, end) of split `split` of a sequence.
__device__ __forceinline__ void split_range(const DecodeParams& p, const SeqSplit& s, int split, int64_t* begin,
                                            int64_t* end) {
    *begin = split_begin(p, split);
    const int64_t raw = *begin + split_pages(p, split);
    *end = raw < s.pages ? raw : s.pages;
}

template <typename T> __device__ __forceinline__ float to_float(T v);
template <> __device__ __forceinline__ float to_float<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_float<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 v) {
    return __bfloat162float(v);
}

template <typename T> __device__ __forceinline__ T from_float(float v);
template <> __device__ __forceinline__ float from_float<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_float<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}

// Rotate-half RoPE of one element, rounded like the reference's tensor
// expression x * cos + rotate_half(x) * sin in the element type
// (src/micro_vllm/model.py:101-123): each product is rounded to T, then their
// sum. `partner` is x[d + D/2] for the first half (rotate_half negates it)
// and x[d - D/2] for the second. No fused multiply-add.
template <typename T>
__device__ __forceinline__ float rope_element(float x, float partner, float c, float s, bool first_half) {
    const float a = to_float<T>(from_float<T>(__fmul_rn(x, c)));
    const float b = to_float<T>(from_float<T>(__fmul_rn(first_half ? -partner : partner, s)));
    return to_float<T>(from_float<T>(__fadd_rn(a, b)));
}

// The same for 8 packed 2-byte elements (one 16-byte chunk of a row).
template <typename T>
__device__ __forceinline__ uint4 rope_chunk(uint4 x, uint4 partner, uint4 c, uint4 s, bool first_half) {
    const T* xv = reinterpret_cast<const T*>(&x);
    const T* pv = reinterpret_cast<const T*>(&partner);
    const T* cv = reinterpret_cast<const T*>(&c);
    const T* sv = reinterpret_cast<const T*>(&s);
    uint4 out;
    T* ov = reinterpret_cast<T*>(&out);
#pragma unroll
    for (int e = 0; e < 8; ++e)
        ov[e] = from_float<T>(rope_element<T>(to_float<T>(xv[e]), to_float<T>(pv[e]), to_float<T>(cv[e]),
                                              to_float<T>(sv[e]), first_half));
    return out;
}

// Fill out[b, h*G + g, :] for every g of KV head h with one value (0 or NaN).
template <typename T>
__device__ void write_group_constant(const DecodeParams& p, int b, int h, float value) {
    T* out = static_cast<T*>(p.out);
    const int total = p.group * p.head_dim;
    for (int idx = threadIdx.x; idx < total; idx += blockDim.x) {
        const int g = idx / p.head_dim;
        const int d = idx - g * p.head_dim;
        out[row_out_offset(p, b) + (int64_t)(h * p.group + g) * p.out_stride_head + d] = from_float<T>(value);
    }
}

// Fused append for a sequence the decode does not attend (empty, or longer
// than max_context_len): the CTA's threads copy the new K/V row of head h to
// position len - 1 when the separate append kernel would have written it
// (position inside the table, page ID inside the pool). 16-byte chunks.
template <typename T>
__device__ inline void append_row_direct(const DecodeParams& p, int b, int h, int64_t len) {
    const int64_t pos = len - 1;
    if (pos < 0) return;
    if (p.rope_cos && pos >= p.rope_rows) return;  // no table row: nothing to write
    const int64_t logical = pos / p.block_size;
    if (logical >= p.blocks_per_seq) return;
    const int64_t id = load_index(p.block_table, p.table_i64, b * p.table_stride + logical);
    if (id < 0 || id >= p.num_blocks) {
        if (threadIdx.x == 0) report_bad_page_id();
        return;
    }
    const int chunks = p.head_dim / 8;  // 16-byte chunks of a 2-byte row
    const int64_t slot = pos - logical * p.block_size;
    for (int c = threadIdx.x; c < 2 * chunks; c += blockDim.x) {
        const int which = c >= chunks;
        const int cc = c - which * chunks;
        const int64_t* st = which ? p.new_value_stride : p.new_key_stride;
        const uint4* row = reinterpret_cast<const uint4*>(
            static_cast<const uint16_t*>(which ? p.new_value : p.new_key) + b * st[0] + h * st[1]);
        uint4 v = row[cc];
        if (p.rope_cos && !which) {
            const int64_t t = pos * (p.head_dim / 8) + cc;
            v = rope_chunk<T>(v, row[cc ^ (chunks / 2)], reinterpret_cast<const uint4*>(p.rope_cos)[t],
                              reinterpret_cast<const uint4*>(p.rope_sin)[t], cc < chunks / 2);
        }
        // The pools are written through the decode's const pointers: the caller passed them writable.
        uint4* dst = reinterpret_cast<uint4*>(const_cast<uint16_t*>(
                         static_cast<const uint16_t*>(which ? p.v_cache : p.k_cache)) +
                         ((id * p.kv_heads + h) * p.block_size + slot) * p.head_dim) +
                     cc;
        *dst = v;
    }
}

// Element-wise form of the fused append for kernels without 16-byte rows (any
// head_dim, alignment and element type): value row copied bit for bit, key row
// too or rotated (RoPE) at position len - 1. Skips exactly where the append
// kernel skips; `row` is the query row (one token per sequence).
template <typename T>
__device__ inline void append_row_elements(const DecodeParams& p, int b, int h, int64_t len) {
    using Raw = typename std::conditional<sizeof(T) == 2, uint16_t, uint32_t>::type;
    const int64_t pos = len - 1;
    if (pos < 0) return;
    if (p.rope_cos && pos >= p.rope_rows) return;
    const int64_t logical = pos / p.block_size;
    if (logical >= p.blocks_per_seq) return;
    const int64_t id = load_index(p.block_table, p.table_i64, b * p.table_stride + logical);
    if (id < 0 || id >= p.num_blocks) {
        if (threadIdx.x == 0) report_bad_page_id();
        return;
    }
    const int64_t dst = ((id * p.kv_heads + h) * p.block_size + (pos - logical * p.block_size)) * p.head_dim;
    const Raw* krow = static_cast<const Raw*>(p.new_key) + b * p.new_key_stride[0] + h * p.new_key_stride[1];
    const Raw* vrow = static_cast<const Raw*>(p.new_value) + b * p.new_value_stride[0] + h * p.new_value_stride[1];
    Raw* kpool = const_cast<Raw*>(static_cast<const Raw*>(p.k_cache));
    Raw* vpool = const_cast<Raw*>(static_cast<const Raw*>(p.v_cache));
    const int half = p.head_dim / 2;
    for (int d = threadIdx.x; d < p.head_dim; d += blockDim.x) {
        vpool[dst + d] = vrow[d];
        if (p.rope_cos) {
            const T* kr = reinterpret_cast<const T*>(krow);
            const bool first = d < half;
            const float x = to_float<T>(kr[d]);
            const float partner = to_float<T>(kr[first ? d + half : d - half]);
            const float c = to_float<T>(static_cast<const T*>(p.rope_cos)[pos * p.head_dim + d]);
            const float sn = to_float<T>(static_cast<const T*>(p.rope_sin)[pos * p.head_dim + d]);
            reinterpret_cast<T*>(kpool)[dst + d] = from_float<T>(rope_element<T>(x, partner, c, sn, first));
        } else {
            kpool[dst + d] = krow[d];
        }
    }
}

// Same for a split's partial result: NaN output and NaN log-sum-exp.
__device__ inline void write_group_partial_nan(const DecodeParams& p, int b, int h, int split) {
    const float nan = __int_as_float(0x7fffffff);
    const int total = p.group * p.head_dim;
    for (int idx = threadIdx.x; idx < total; idx += blockDim.x) {
        const int g = idx / p.head_dim;
        const int d = idx - g * p.head_dim;
        const int64_t row = ((int64_t)b * p.q_heads + h * p.group + g) * p.max_splits + split;
        p.part_o[row * p.head_dim + d] = nan;
        if (d == 0) p.part_lse[row] = nan;
    }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Programmatic dependent launch: every kernel here waits for the grid before
// it in the stream to finish (and flush) before reading any input, so it may
// be launched early, overlapping its launch and setup with that grid's tail;
// and it lets the next grid launch once it has finished its own setup.
__device__ __forceinline__ void wait_for_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_next_grid() { asm volatile("griddepcontrol.launch_dependents;" :::); }

__device__ __forceinline__ unsigned long long global_timer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (TMA) writes to the same buffer.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Wait for the barrier phase with the given parity; give up after limit_ns.
__device__ __forceinline__ bool mbar_wait_bounded_ns(uint32_t bar, uint32_t parity, unsigned long long limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long start = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - start > limit_ns) return false;
    }
}

// The kernels' waits: give up after kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    return mbar_wait_bounded_ns(bar, parity, kWaitLimitNs);
}

// --------------------------------------------------------------------- TMA

// 5-D tiled TMA load into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, int c4, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
        "r"(bar)
        : "memory");
}

// 5-D tiled prefetch of the same box into L2 only: no shared memory, no barrier.
__device__ __forceinline__ void tma_prefetch_l2_5d(const CUtensorMap* map, int c0, int c1, int c2,
                                                   int c3, int c4) {
    asm volatile(
        "cp.async.bulk.prefetch.tensor.5d.L2.global.tile [%0, {%1, %2, %3, %4, %5}];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
        : "memory");
}

__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// -------------------------------------------------------- warp-level MMA

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}

template <typename T> struct MmaOp;

template <> struct MmaOp<__nv_bfloat16> {
    __device__ __forceinline__ static void run(float (&c)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
            "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    // Two fp32 values -> packed pair; `lo` lands in the low half.
    __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
        uint32_t r;
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
        return r;
    }
};

template <> struct MmaOp<__half> {
    __device__ __forceinline__ static void run(float (&c)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
            "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
        uint32_t r;
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
        return r;
    }
};

}  // namespace mv
