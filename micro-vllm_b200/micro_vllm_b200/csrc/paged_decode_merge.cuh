// Split-KV (flash-decoding) second pass: combine the normalised partial
// outputs o_j and log2-sum-exp values lse_j of the pieces of one output row
// (sequence b, query head hq):
//   out = sum_j w_j o_j,  w_j = 2^(lse_j - lse_max) / sum_i 2^(lse_i - lse_max).
// Weights are normalised before the sum, so the result stays within max |o_j|
// (no overflow for large finite partials). A NaN partial (corrupted page ID,
// or a wait that gave up) poisons the row, as in the reference.
//
// One warp per output row, four rows per CTA: the lanes read the pieces'
// log-sum-exps in parallel, then stream the partial rows with lanes over the
// head dimension and the pieces' weights broadcast by shuffle, so every load
// of the second phase is independent of the others.
#pragma once

#include "mv_device.cuh"

namespace mv {

constexpr int kMergeThreads = 128;
constexpr int kMergeRowsPerCta = kMergeThreads / 32;

template <typename T, typename RowOf>
__device__ __forceinline__ void merge_row(const DecodeParams& p, T* out, RowOf row_of, int n, int lane) {
    float mx = -INFINITY;
    bool nan = false;
    for (int j = lane; j < n; j += 32) {
        const float v = p.part_lse[row_of(j)];
        nan |= isnan(v);
        mx = fmaxf(mx, v);
    }
    mx = warp_max(mx);
    if (__any_sync(0xffffffffu, nan)) {
        for (int d = lane; d < p.head_dim; d += 32) out[d] = from_float<T>(__int_as_float(0x7fffffff));
        return;
    }
    float sum = 0.0f;
    for (int j = lane; j < n; j += 32) sum += fast_exp2(p.part_lse[row_of(j)] - mx);
    const float inv = 1.0f / warp_sum(sum);

    constexpr int kCols = 4;  // columns per lane per pass: 128 columns per pass
    for (int d0 = 0; d0 < p.head_dim; d0 += 32 * kCols) {
        float acc[kCols];
#pragma unroll
        for (int c = 0; c < kCols; ++c) acc[c] = 0.0f;
        for (int j0 = 0; j0 < n; j0 += 32) {
            const int j = j0 + lane;
            const float wj = j < n ? fast_exp2(p.part_lse[row_of(j)] - mx) * inv : 0.0f;
            const long long rj = j < n ? row_of(j) : 0;
            const int count = n - j0 < 32 ? n - j0 : 32;
#pragma unroll 4
            for (int k = 0; k < count; ++k) {
                const float w = __shfl_sync(0xffffffffu, wj, k);
                const long long r = __shfl_sync(0xffffffffu, rj, k);
                const float* src = p.part_o + r * p.head_dim;
#pragma unroll
                for (int c = 0; c < kCols; ++c) {
                    const int d = d0 + c * 32 + lane;
                    if (d < p.head_dim) acc[c] = fmaf(w, src[d], acc[c]);
                }
            }
        }
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
            const int d = d0 + c * 32 + lane;
            if (d < p.head_dim) out[d] = from_float<T>(acc[c]);
        }
    }
}

// Merge of the fixed split grid: row (b, hq) has seq.splits pieces at
// part rows (b * q_heads + hq) * max_splits + j. Sequences that fit one split
// were finished by the first pass.
template <typename T>
__global__ void __launch_bounds__(kMergeThreads) paged_decode_merge_kernel(const DecodeParams p) {
    wait_for_prior_grid();
    allow_next_grid();
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kMergeRowsPerCta + (threadIdx.x >> 5);
    if (row >= static_cast<int64_t>(p.batch) * p.q_heads) return;
    const int b = static_cast<int>(row / p.q_heads);
    const int hq = static_cast<int>(row - static_cast<int64_t>(b) * p.q_heads);
    const SeqSplit seq = seq_split(p, b);
    if (seq.splits <= 1) return;
    T* out = static_cast<T*>(p.out) + b * p.out_stride_seq + static_cast<int64_t>(hq) * p.out_stride_head;
    const int64_t base = row * p.max_splits;
    merge_row<T>(p, out, [&](int j) -> long long { return base + j; }, seq.splits, lane);
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
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kMergeRowsPerCta + (threadIdx.x >> 5);
    if (row >= static_cast<int64_t>(p.batch) * p.q_heads) return;
    const int b = static_cast<int>(row / p.q_heads);
    const int hq = static_cast<int>(row - static_cast<int64_t>(b) * p.q_heads);
    const int h = hq / p.group;
    const int g = hq - h * p.group;
    T* out = static_cast<T*>(p.out) + b * p.out_stride_seq + static_cast<int64_t>(hq) * p.out_stride_head;
    const SeqSplit seq = seq_split(p, b);
    if (seq.state != 0) {
        const float value = seq.state == 1 ? 0.0f : __int_as_float(0x7fffffff);
        for (int d = lane; d < p.head_dim; d += 32) out[d] = from_float<T>(value);
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
                 static_cast<int>(w1 - w0 + 1), lane);
}

}  // namespace mv
