// Split-KV (flash-decoding) second pass: combine the normalised partial
// outputs o_s and log2-sum-exp values lse_s of a sequence's splits,
//   out = sum_s w_s o_s,  w_s = 2^(lse_s - lse_max) / sum_r 2^(lse_r - lse_max).
// One CTA per (query head, sequence); sequences that fit one split were
// finished by the first pass and are skipped. A NaN partial (corrupted page
// ID, or a wait that gave up) poisons the whole row, as in the reference.
#pragma once

#include "mv_device.cuh"

namespace mv {

constexpr int kMergeThreads = 128;

template <typename T>
__global__ void __launch_bounds__(kMergeThreads) paged_decode_merge_kernel(const DecodeParams p) {
    extern __shared__ float weights[];  // [max_splits]
    __shared__ float red[kMergeThreads / 32];
    __shared__ int any_nan;
    const int hq = blockIdx.x;
    const int b = blockIdx.y;
    wait_for_prior_grid();
    allow_next_grid();
    const SeqSplit seq = seq_split(p, b);
    if (seq.splits <= 1) return;
    const int n = seq.splits;
    const int tid = threadIdx.x;
    const int64_t row0 = (static_cast<int64_t>(b) * p.q_heads + hq) * p.max_splits;

    if (tid == 0) any_nan = 0;
    __syncthreads();
    float mx = -INFINITY;
    for (int s = tid; s < n; s += blockDim.x) {
        const float v = p.part_lse[row0 + s];
        weights[s] = v;
        if (isnan(v)) any_nan = 1;
        mx = fmaxf(mx, v);
    }
    mx = warp_max(mx);
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < kMergeThreads / 32; ++w) mx = fmaxf(mx, red[w]);

    T* out = static_cast<T*>(p.out) + b * p.out_stride_seq + static_cast<int64_t>(hq) * p.out_stride_head;
    if (any_nan) {
        for (int d = tid; d < p.head_dim; d += blockDim.x) out[d] = from_float<T>(__int_as_float(0x7fffffff));
        return;
    }
    __syncthreads();  // everyone has read red[] before it is reused
    float sum = 0.0f;
    for (int s = tid; s < n; s += blockDim.x) {
        const float w = fast_exp2(weights[s] - mx);
        weights[s] = w;
        sum += w;
    }
    sum = warp_sum(sum);
    if ((tid & 31) == 0) red[tid >> 5] = sum;
    __syncthreads();
    float total = 0.0f;
#pragma unroll
    for (int w = 0; w < kMergeThreads / 32; ++w) total += red[w];

    // Normalise the weights first: sum_s w_s o_s then stays within max |o_s|
    // (no overflow for large finite partials).
    const float inv_total = 1.0f / total;
    for (int s = tid; s < n; s += blockDim.x) weights[s] *= inv_total;
    __syncthreads();
    const float* part = p.part_o + row0 * p.head_dim;
    for (int d = tid; d < p.head_dim; d += blockDim.x) {
        float acc = 0.0f;
        for (int s = 0; s < n; ++s) acc = fmaf(weights[s], part[static_cast<int64_t>(s) * p.head_dim + d], acc);
        out[d] = from_float<T>(acc);
    }
}

// Merge pass of the persistent schedule. One CTA per (KV head h, sequence b):
// writes the constant result of sequences with no pages (zeros or NaN), and
// for a (b, h) segment cut across warps w0..w1 combines their partials. The
// segment's piece is partial slot 1 of w0 when the segment starts inside w0's
// range after w0's first piece, slot 0 otherwise. Segments inside one warp
// were written by that warp and are skipped.
template <typename T, int GP>
__global__ void __launch_bounds__(kMergeThreads) paged_decode_persistent_merge_kernel(const DecodeParams p) {
    const int h = blockIdx.x;
    const int b = blockIdx.y;
    wait_for_prior_grid();
    allow_next_grid();
    const SeqSplit seq = seq_split(p, b);
    if (seq.state != 0) {
        write_group_constant<T>(p, b, h, seq.state == 1 ? 0.0f : __int_as_float(0x7fffffff));
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
    const int n = static_cast<int>(w1 - w0 + 1);
    const int slot0 = (w0 * total / warps == start) ? 0 : 1;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    T* out = static_cast<T*>(p.out) + b * p.out_stride_seq;
    auto row_of = [&](int j) -> int64_t { return ((w0 + j) * 2 + (j == 0 ? slot0 : 0)) * GP; };
    for (int g = warp; g < p.group; g += kMergeThreads / 32) {
        float mx = -INFINITY;
        bool nan = false;
        for (int j = lane; j < n; j += 32) {
            const float v = p.part_lse[row_of(j) + g];
            nan |= isnan(v);
            mx = fmaxf(mx, v);
        }
        mx = warp_max(mx);
        nan = __any_sync(0xffffffffu, nan);
        T* row = out + static_cast<int64_t>(h * p.group + g) * p.out_stride_head;
        if (nan) {
            for (int d = lane; d < p.head_dim; d += 32) row[d] = from_float<T>(__int_as_float(0x7fffffff));
            continue;
        }
        float sum = 0.0f;
        for (int j = lane; j < n; j += 32) sum += fast_exp2(p.part_lse[row_of(j) + g] - mx);
        const float inv = 1.0f / warp_sum(sum);
        for (int d = lane; d < p.head_dim; d += 32) {
            float acc = 0.0f;
            for (int j = 0; j < n; ++j) {
                const int64_t r = row_of(j) + g;
                const float wgt = fast_exp2(p.part_lse[r] - mx) * inv;
                acc = fmaf(wgt, p.part_o[r * p.head_dim + d], acc);
            }
            row[d] = from_float<T>(acc);
        }
    }
}

}  // namespace mv
