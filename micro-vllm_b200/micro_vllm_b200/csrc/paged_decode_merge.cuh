// Split-KV (flash-decoding) second pass: combine the normalised partial
// outputs o_j and log2-sum-exp values lse_j of the pieces of one output row
// (sequence b, query head hq):
//   out = sum_j w_j o_j,  w_j = 2^(lse_j - lse_max) / sum_i 2^(lse_i - lse_max).
// Weights are normalised before the sum, so the result stays within max |o_j|
// (no overflow for large finite partials). A NaN partial (corrupted page ID,
// or a wait that gave up) poisons the row, as in the reference.
//
// One CTA per output row: the threads read the pieces' log-sum-exps in
// parallel, reduce them through shared memory, then each thread owns output
// columns and streams the pieces' partial rows with the weights read from
// shared memory, so the loads of every piece are independent and coalesced.
#pragma once

#include "mv_device.cuh"

namespace mv {

constexpr int kMergeThreads = 128;
constexpr int kMergeChunk = 256;  // pieces whose weights are staged at a time

template <typename T, typename RowOf>
__device__ __forceinline__ void merge_row(const DecodeParams& p, T* out, RowOf row_of, int n) {
    __shared__ float weights[kMergeChunk];
    __shared__ float red[kMergeThreads / 32];
    __shared__ int any_nan;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    if (n <= kMergeChunk) {
        // Two dependent rounds of loads: the log-sum-exps (kept in shared
        // memory for the max, the sum and the weights), then the partial rows.
        for (int j = tid; j < n; j += kMergeThreads) weights[j] = __ldcg(p.part_lse + row_of(j));
        __syncthreads();
        if (warp == 0) {
            float mx = -INFINITY;
            bool nan = false;
            for (int j = lane; j < n; j += 32) {
                nan |= isnan(weights[j]);
                mx = fmaxf(mx, weights[j]);
            }
            mx = warp_max(mx);
            nan = __any_sync(0xffffffffu, nan);
            float sum = 0.0f;
            for (int j = lane; j < n; j += 32) sum += fast_exp2(weights[j] - mx);
            const float inv = 1.0f / warp_sum(sum);
            __syncwarp();
            for (int j = lane; j < n; j += 32) weights[j] = nan ? __int_as_float(0x7fffffff)
                                                                 : fast_exp2(weights[j] - mx) * inv;
        }
        __syncthreads();
        for (int d = tid; d < p.head_dim; d += kMergeThreads) {
            float acc = 0.0f;
#pragma unroll 8
            for (int j = 0; j < n; ++j)
                acc = fmaf(weights[j], __ldcg(p.part_o + static_cast<int64_t>(row_of(j)) * p.head_dim + d), acc);
            out[d] = from_float<T>(acc);
        }
        return;
    }
    if (tid == 0) any_nan = 0;
    float mx = -INFINITY;
    for (int j = tid; j < n; j += kMergeThreads) {
        const float v = p.part_lse[row_of(j)];
        if (isnan(v)) any_nan = 1;
        mx = fmaxf(mx, v);
    }
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < kMergeThreads / 32; ++w) mx = fmaxf(mx, red[w]);
    if (any_nan) {
        for (int d = tid; d < p.head_dim; d += kMergeThreads) out[d] = from_float<T>(__int_as_float(0x7fffffff));
        return;
    }
    float sum = 0.0f;
    for (int j = tid; j < n; j += kMergeThreads) sum += fast_exp2(p.part_lse[row_of(j)] - mx);
    sum = warp_sum(sum);
    __syncthreads();  // red[] reads above are done
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    float total = 0.0f;
#pragma unroll
    for (int w = 0; w < kMergeThreads / 32; ++w) total += red[w];
    const float inv = 1.0f / total;

    for (int d0 = 0; d0 < p.head_dim; d0 += kMergeThreads) {
        const int d = d0 + tid;
        float acc = 0.0f;
        for (int j0 = 0; j0 < n; j0 += kMergeChunk) {
            const int count = n - j0 < kMergeChunk ? n - j0 : kMergeChunk;
            __syncthreads();  // previous chunk's weights are consumed
            for (int j = tid; j < count; j += kMergeThreads)
                weights[j] = fast_exp2(p.part_lse[row_of(j0 + j)] - mx) * inv;
            __syncthreads();
            if (d < p.head_dim) {
#pragma unroll 8
                for (int j = 0; j < count; ++j)
                    acc = fmaf(weights[j], p.part_o[static_cast<int64_t>(row_of(j0 + j)) * p.head_dim + d], acc);
            }
        }
        if (d < p.head_dim) out[d] = from_float<T>(acc);
    }
}

// Merge one (sequence, KV head) segment's n split partials into its G output
// rows, by the whole CTA. Split j of query row g is part row
// (b * q_heads + h * G + g) * max_splits + j. `weights` holds G * n floats
// of shared memory. Two dependent rounds of global loads: the G x n
// log-sum-exps (staged into `weights`), then the partial rows. Partials are
// read through L2 (ld.cg): other CTAs wrote them.
template <typename T>
__device__ void merge_segment(const DecodeParams& p, int b, int h, int n, float* weights) {
    const int G = p.group;
    const int D = p.head_dim;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nwarps = blockDim.x >> 5;
    const int64_t row0 = (static_cast<int64_t>(b) * p.q_heads + h * G) * p.max_splits;
    for (int idx = threadIdx.x; idx < G * n; idx += blockDim.x) {
        const int g = idx / n;
        weights[idx] = __ldcg(p.part_lse + row0 + static_cast<int64_t>(g) * p.max_splits + (idx - g * n));
    }
    __syncthreads();
    for (int g = warp; g < G; g += nwarps) {
        float* w = weights + g * n;
        float mx = -INFINITY;
        bool nan = false;
        for (int j = lane; j < n; j += 32) {
            nan |= isnan(w[j]);
            mx = fmaxf(mx, w[j]);
        }
        mx = warp_max(mx);
        nan = __any_sync(0xffffffffu, nan);
        float sum = 0.0f;
        for (int j = lane; j < n; j += 32) sum += fast_exp2(w[j] - mx);
        const float inv = nan ? __int_as_float(0x7fffffff) : 1.0f / warp_sum(sum);
        __syncwarp();
        for (int j = lane; j < n; j += 32) w[j] = fast_exp2(w[j] - mx) * inv;
    }
    __syncthreads();
    // Each thread owns a column and walks the rows four at a time, so the loads
    // of four rows x several splits are in flight together.
    T* out = static_cast<T*>(p.out) + row_out_offset(p, b);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        for (int g0 = 0; g0 < G; g0 += 4) {
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 2
            for (int j = 0; j < n; ++j) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int g = g0 + u;
                    if (g < G) {
                        const float* src = p.part_o + (row0 + static_cast<int64_t>(g) * p.max_splits + j) * D + d;
                        acc[u] = fmaf(weights[g * n + j], __ldcg(src), acc[u]);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (g0 + u < G)
                    out[static_cast<int64_t>(h * G + g0 + u) * p.out_stride_head + d] = from_float<T>(acc[u]);
            }
        }
    }
}

// Merge of one (sequence, KV head) segment's n <= kSegmentWarpBatch pieces
// by the CTA that finished it last, a warp per output row: lane j loads piece
// j's log-sum-exp and every lane its float4 column of every piece, for all the
// warp's rows at once -- one dependent round of loads (merge_segment takes two
// rounds, then one per few pieces). The arithmetic is the warp-per-row merge
// pass's below, in the same order, so both give the same bits. Needs head_dim
// 64 or 128 and at most two rows per warp.
constexpr int kSegmentWarpBatch = 8;

template <typename T>
__device__ void merge_segment_warps(const DecodeParams& p, int b, int h, int n) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nwarps = blockDim.x >> 5;
    const int c4n = p.head_dim >> 2;
    const bool col = lane < c4n;
    float lse[2];
    float4 v[2][kSegmentWarpBatch];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int g = warp + r * nwarps;
        const bool row = g < p.group;
        const int64_t base = (static_cast<int64_t>(b) * p.q_heads + h * p.group + (row ? g : 0)) * p.max_splits;
        const float4* src = reinterpret_cast<const float4*>(p.part_o + base * p.head_dim) + lane;
        lse[r] = row && lane < n ? __ldcg(p.part_lse + base + lane) : -INFINITY;
#pragma unroll
        for (int j = 0; j < kSegmentWarpBatch; ++j)
            v[r][j] = row && col && j < n ? __ldcg(src + static_cast<int64_t>(j) * c4n)
                                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int g = warp + r * nwarps;
        if (g >= p.group) break;
        const bool nan = __any_sync(0xffffffffu, isnan(lse[r]));
        const float mx = warp_max(lse[r]);
        const float e = lane < n ? fast_exp2(lse[r] - mx) : 0.0f;
        const float w = e * (1.0f / warp_sum(e));
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < kSegmentWarpBatch; ++j) {
            const float wj = __shfl_sync(0xffffffffu, w, j);
            if (j < n) {
                acc.x = fmaf(wj, v[r][j].x, acc.x);
                acc.y = fmaf(wj, v[r][j].y, acc.y);
                acc.z = fmaf(wj, v[r][j].z, acc.z);
                acc.w = fmaf(wj, v[r][j].w, acc.w);
            }
        }
        if (col) {
            const float q = __int_as_float(0x7fffffff);
            T* out = static_cast<T*>(p.out) + row_out_offset(p, b) +
                     static_cast<int64_t>(h * p.group + g) * p.out_stride_head + lane * 4;
            out[0] = from_float<T>(nan ? q : acc.x);
            out[1] = from_float<T>(nan ? q : acc.y);
            out[2] = from_float<T>(nan ? q : acc.z);
            out[3] = from_float<T>(nan ? q : acc.w);
        }
    }
}

// Merge of the fixed split grid, one CTA per output row (b, hq). Row (b, hq)
// has seq.splits pieces at part rows (b * q_heads + hq) * max_splits + j.
// Sequences that fit one split were finished by the first pass.
template <typename T>
__global__ void __launch_bounds__(kMergeThreads) paged_decode_merge_kernel(const DecodeParams p) {
    wait_for_prior_grid();
    allow_next_grid();
    const int hq = blockIdx.x;
    const int b = blockIdx.y;
    const SeqSplit seq = seq_split(p, b);
    if (seq.splits <= 1) return;
    T* out = static_cast<T*>(p.out) + row_out_offset(p, b) + static_cast<int64_t>(hq) * p.out_stride_head;
    const int64_t base = (static_cast<int64_t>(b) * p.q_heads + hq) * p.max_splits;
    merge_row<T>(p, out, [&](int j) -> long long { return base + j; }, seq.splits);
}

// Warp-per-row merge of the split grid for head_dim <= 128 (a multiple of 4)
// and at most 32 pieces: lane j holds piece j's log-sum-exp and every lane
// one float4 column of up to kWarpMergeBatch pieces' partial rows, all loaded
// together -- one dependent round of loads where the CTA-per-row merge takes
// two (log-sum-exps, then partials). The row's piece count reads only the
// caller's lengths, so it is computed before waiting for the first pass.
// Rows (warps) per CTA. Measured on B200 (Qwen2.5-7B geometry, batch 64, graphs
// of 8 steps): 1 / 2 / 4 / 8 / 16 / 32 rows 56.65-56.69 / 56.73-56.76 /
// 56.84-56.96 / 57.99 / 58.50 / 58.53 us per step -- the next step's decode
// launches once every merge CTA has started, and one-warp CTAs find room first.
#ifndef MV_WARP_MERGE_ROWS
#define MV_WARP_MERGE_ROWS 1
#endif
constexpr int kWarpMergeRows = MV_WARP_MERGE_ROWS;
constexpr int kWarpMergeBatch = 8;   // pieces whose partials are in flight together

template <typename T>
__global__ void __launch_bounds__(kWarpMergeRows * 32) paged_decode_merge_warp_kernel(const DecodeParams p) {
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpMergeRows + (threadIdx.x >> 5);  // z * q_heads + hq
    allow_next_grid();
    int n = 0;
    int64_t z = 0;
    if (row < static_cast<int64_t>(p.batch) * p.q_heads) {
        z = row / p.q_heads;
        n = seq_split(p, z).splits;
    }
    wait_for_prior_grid();
    if (n <= 1) return;
    const int hq = static_cast<int>(row - z * p.q_heads);
    const int c4n = p.head_dim >> 2;
    const int64_t base = row * p.max_splits;
    const float4* src = reinterpret_cast<const float4*>(p.part_o + base * p.head_dim) + lane;
    const bool col = lane < c4n;
    float lse = lane < n ? __ldcg(p.part_lse + base + lane) : -INFINITY;
    float4 v[kWarpMergeBatch];
#pragma unroll
    for (int j = 0; j < kWarpMergeBatch; ++j)
        v[j] = col && j < n ? __ldcg(src + static_cast<int64_t>(j) * c4n) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const bool nan = __any_sync(0xffffffffu, isnan(lse));
    const float mx = warp_max(lse);
    const float e = lane < n ? fast_exp2(lse - mx) : 0.0f;
    const float w = e * (1.0f / warp_sum(e));
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int j0 = 0; j0 < n; j0 += kWarpMergeBatch) {
        if (j0 > 0) {
#pragma unroll
            for (int j = 0; j < kWarpMergeBatch; ++j)
                v[j] = col && j0 + j < n ? __ldcg(src + static_cast<int64_t>(j0 + j) * c4n)
                                         : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int j = 0; j < kWarpMergeBatch; ++j) {
            const float wj = __shfl_sync(0xffffffffu, w, (j0 + j) & 31);
            if (j0 + j < n) {
                acc.x = fmaf(wj, v[j].x, acc.x);
                acc.y = fmaf(wj, v[j].y, acc.y);
                acc.z = fmaf(wj, v[j].z, acc.z);
                acc.w = fmaf(wj, v[j].w, acc.w);
            }
        }
    }
    if (!col) return;
    const float q = __int_as_float(0x7fffffff);
    T* out = static_cast<T*>(p.out) + row_out_offset(p, z) + static_cast<int64_t>(hq) * p.out_stride_head + lane * 4;
    out[0] = from_float<T>(nan ? q : acc.x);
    out[1] = from_float<T>(nan ? q : acc.y);
    out[2] = from_float<T>(nan ? q : acc.z);
    out[3] = from_float<T>(nan ? q : acc.w);
}

// The split grid's merge for rows of 33..kManyMergeMax pieces (long contexts),
// head_dim <= 128 and a multiple of 4: one CTA per row, its warps splitting the
// pieces (warp w: pieces w, w + 4, ...). Lane k of a warp loads the
// log-sum-exp of the warp's k-th piece and every lane a float4 column of up to
// kManyBatch of the warp's partial rows in the same round; the weights come
// from a CTA-wide max and sum, and the warps' column sums meet in shared
// memory in a fixed order. 64 pieces: one dependent round of loads (the
// CTA-per-row merge above takes one for the log-sum-exps and then eight
// rounds of 8 partial columns).
constexpr int kManyMergeWarps = 4;
constexpr int kManyBatch = 16;                                   // pieces per warp in flight at once
constexpr int kManyMergeMax = kManyMergeWarps * 2 * kManyBatch;  // 128

template <typename T>
__global__ void __launch_bounds__(kManyMergeWarps * 32) paged_decode_merge_many_kernel(const DecodeParams p) {
    __shared__ float red[2][kManyMergeWarps];
    __shared__ float4 sums[kManyMergeWarps][32];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int hq = blockIdx.x;
    const int b = blockIdx.y;
    allow_next_grid();
    const int n = seq_split(p, b).splits;  // reads only the caller's lengths
    wait_for_prior_grid();
    if (n <= 1) return;
    const int c4n = p.head_dim >> 2;
    const bool col = lane < c4n;
    const int64_t base = (static_cast<int64_t>(b) * p.q_heads + hq) * p.max_splits;
    const int mine = n > warp ? (n - warp + kManyMergeWarps - 1) / kManyMergeWarps : 0;  // <= 32
    const float4* src = reinterpret_cast<const float4*>(p.part_o + base * p.head_dim) + lane;
    const float lse = lane < mine ? __ldcg(p.part_lse + base + warp + kManyMergeWarps * lane) : -INFINITY;
    float4 v[kManyBatch];
#pragma unroll
    for (int k = 0; k < kManyBatch; ++k)
        v[k] = col && k < mine ? __ldcg(src + static_cast<int64_t>(warp + kManyMergeWarps * k) * c4n)
                               : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const bool nan_here = __any_sync(0xffffffffu, isnan(lse));
    const float wmax = warp_max(lse);
    if (lane == 0) red[0][warp] = nan_here ? __int_as_float(0x7fffffff) : wmax;
    __syncthreads();
    float mx = -INFINITY;
    bool nan = false;
#pragma unroll
    for (int w = 0; w < kManyMergeWarps; ++w) {
        nan |= isnan(red[0][w]);
        mx = fmaxf(mx, red[0][w]);
    }
    const float e = lane < mine ? fast_exp2(lse - mx) : 0.0f;
    const float wsum = warp_sum(e);
    if (lane == 0) red[1][warp] = wsum;
    __syncthreads();
    float total = 0.0f;
#pragma unroll
    for (int w = 0; w < kManyMergeWarps; ++w) total += red[1][w];
    const float wgt = e * (1.0f / total);
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int k0 = 0; k0 < mine; k0 += kManyBatch) {
        if (k0 > 0) {
#pragma unroll
            for (int k = 0; k < kManyBatch; ++k)
                v[k] = col && k0 + k < mine
                           ? __ldcg(src + static_cast<int64_t>(warp + kManyMergeWarps * (k0 + k)) * c4n)
                           : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int k = 0; k < kManyBatch; ++k) {
            const float wk = __shfl_sync(0xffffffffu, wgt, (k0 + k) & 31);
            if (k0 + k < mine) {
                acc.x = fmaf(wk, v[k].x, acc.x);
                acc.y = fmaf(wk, v[k].y, acc.y);
                acc.z = fmaf(wk, v[k].z, acc.z);
                acc.w = fmaf(wk, v[k].w, acc.w);
            }
        }
    }
    sums[warp][lane] = acc;
    __syncthreads();
    if (warp != 0 || !col) return;
    float4 r = sums[0][lane];
#pragma unroll
    for (int w = 1; w < kManyMergeWarps; ++w) {
        const float4 s = sums[w][lane];
        r.x += s.x;
        r.y += s.y;
        r.z += s.z;
        r.w += s.w;
    }
    const float q = __int_as_float(0x7fffffff);
    T* out = static_cast<T*>(p.out) + row_out_offset(p, b) + static_cast<int64_t>(hq) * p.out_stride_head + lane * 4;
    out[0] = from_float<T>(nan ? q : r.x);
    out[1] = from_float<T>(nan ? q : r.y);
    out[2] = from_float<T>(nan ? q : r.z);
    out[3] = from_float<T>(nan ? q : r.w);
}

// Merge of the persistent schedule. Row (b, hq) belongs to segment (b, h =
// hq / G). It writes the constant result of sequences with no pages (zeros or
// NaN), and for a segment cut across warps w0..w1 combines their partials.
// The segment's piece is partial slot 1 of w0 when the segment starts inside
// w0's range after w0's first piece, slot 0 otherwise. Segments inside one
// warp were written by that warp.
template <typename T, int GP>
__global__ void __launch_bounds__(kMergeThreads) paged_decode_persistent_merge_kernel(const DecodeParams p) {
    wait_for_prior_grid();
    allow_next_grid();
    const int hq = blockIdx.x;
    const int b = blockIdx.y;
    const int h = hq / p.group;
    const int g = hq - h * p.group;
    T* out = static_cast<T*>(p.out) + b * p.out_stride_seq + static_cast<int64_t>(hq) * p.out_stride_head;
    const SeqSplit seq = seq_split(p, b);
    if (seq.state != 0) {
        const float value = seq.state == 1 ? 0.0f : __int_as_float(0x7fffffff);
        for (int d = threadIdx.x; d < p.head_dim; d += blockDim.x) out[d] = from_float<T>(value);
        return;
    }
    const int64_t* prefix = p.prefix_out;
    const int64_t total = static_cast<int64_t>(p.kv_heads) * prefix[p.batch];
    const int64_t warps = p.persistent_warps < total ? p.persistent_warps : total;
    const int64_t pages = prefix[b + 1] - prefix[b];
    const int64_t start = static_cast<int64_t>(p.kv_heads) * prefix[b] + h * pages;
    const int64_t end = start + pages;
    const int64_t w0 = ((start + 1) * warps - 1) / total;  // warp owning page `start`
    const int64_t w1 = (end * warps - 1) / total;          // warp owning page end - 1
    if (w0 == w1) return;
    const int slot0 = (w0 * total / warps == start) ? 0 : 1;
    merge_row<T>(p, out,
                 [&](int j) -> long long { return ((w0 + j) * 2 + (j == 0 ? slot0 : 0)) * GP + g; },
                 static_cast<int>(w1 - w0 + 1));
}

}  // namespace mv
