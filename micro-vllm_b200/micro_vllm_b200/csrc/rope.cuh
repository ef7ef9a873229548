// Rotate-half RoPE of whole rows (the reference's apply_rope for the batched
// path): out[b, h, t, :] = RoPE(x[b, h, t, :]) at position start_b + t, with
// rows of caller-supplied cos/sin tables [table_rows, D] of the element type,
// rounded per operation as the reference's tensor expression is
// (src/micro_vllm/model.py:101-123; see rope_element). One thread per pair
// (d, d + D/2) of one row, so out may alias x exactly (in place).
#pragma once

#include "mv_device.cuh"

namespace mv {

constexpr int kRopeThreads = 256;

struct RopeParams {
    const void* x;
    int64_t x_stride[3];     // seq, head, token (elements)
    void* out;
    int64_t out_stride[3];
    int batch;
    int heads;
    int tokens;
    int head_dim;
    const void* cos;
    const void* sin;
    int64_t table_rows;
    const void* positions;   // nullptr: every sequence starts at `start`
    int positions_i64;
    int positions_end;       // positions hold the end of the sequence, not the start
    int64_t start;
};

template <typename T>
__global__ void __launch_bounds__(kRopeThreads) rope_rows_kernel(const RopeParams r, int64_t total) {
    wait_for_prior_grid();
    allow_next_grid();
    const int half = r.head_dim / 2;
    const int64_t stride = static_cast<int64_t>(blockDim.x) * gridDim.x;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total; idx += stride) {
        const int d = static_cast<int>(idx % half);
        int64_t row = idx / half;
        const int t = static_cast<int>(row % r.tokens);
        row /= r.tokens;
        const int h = static_cast<int>(row % r.heads);
        const int b = static_cast<int>(row / r.heads);
        int64_t start = r.start;
        if (r.positions) {
            start = load_index(r.positions, r.positions_i64, b);
            if (r.positions_end) start -= r.tokens;
        }
        const int64_t pos = start + t;
        const T* x = static_cast<const T*>(r.x) + b * r.x_stride[0] + h * r.x_stride[1] + t * r.x_stride[2];
        T* o = static_cast<T*>(r.out) + b * r.out_stride[0] + h * r.out_stride[1] + t * r.out_stride[2];
        if (pos < 0 || pos >= r.table_rows) {
            // No table row for this position: the row becomes NaN, nothing is read.
            o[d] = o[d + half] = from_float<T>(__int_as_float(0x7fffffff));
            continue;
        }
        const T* c = static_cast<const T*>(r.cos) + pos * r.head_dim;
        const T* s = static_cast<const T*>(r.sin) + pos * r.head_dim;
        const float x0 = to_float<T>(x[d]);
        const float x1 = to_float<T>(x[d + half]);
        const float y0 = rope_element<T>(x0, x1, to_float<T>(c[d]), to_float<T>(s[d]), true);
        const float y1 = rope_element<T>(x1, x0, to_float<T>(c[d + half]), to_float<T>(s[d + half]), false);
        o[d] = from_float<T>(y0);
        o[d + half] = from_float<T>(y1);
    }
}

// Two-byte types, head_dim a multiple of 16, 16-byte aligned rows and tables:
// one thread per (row, 16-byte chunk of the first half), rotating that chunk and
// its partner chunk D/2 away with the same rounding per element. Grid
// (token x chunk blocks, heads, sequences): 32-bit index arithmetic only.
template <typename T>
__global__ void __launch_bounds__(kRopeThreads) rope_rows_vec_kernel(const RopeParams r) {
    wait_for_prior_grid();
    allow_next_grid();
    const int half_chunks = r.head_dim / 16;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= r.tokens * half_chunks) return;
    const int t = i / half_chunks;
    const int c = i - t * half_chunks;
    const int h = blockIdx.y;
    const int b = blockIdx.z;
    int64_t start = r.start;
    if (r.positions) {
        start = load_index(r.positions, r.positions_i64, b);
        if (r.positions_end) start -= r.tokens;
    }
    const int64_t pos = start + t;
    const uint4* x = reinterpret_cast<const uint4*>(static_cast<const T*>(r.x) + b * r.x_stride[0] +
                                                    h * r.x_stride[1] + t * r.x_stride[2]);
    uint4* o = reinterpret_cast<uint4*>(static_cast<T*>(r.out) + b * r.out_stride[0] + h * r.out_stride[1] +
                                        t * r.out_stride[2]);
    if (pos < 0 || pos >= r.table_rows) {
        uint4 nan;
        T* ne = reinterpret_cast<T*>(&nan);
#pragma unroll
        for (int e = 0; e < 8; ++e) ne[e] = from_float<T>(__int_as_float(0x7fffffff));
        o[c] = nan;
        o[c + half_chunks] = nan;
        return;
    }
    const uint4* cs = reinterpret_cast<const uint4*>(static_cast<const T*>(r.cos) + pos * r.head_dim);
    const uint4* sn = reinterpret_cast<const uint4*>(static_cast<const T*>(r.sin) + pos * r.head_dim);
    const uint4 lo = x[c], hi = x[c + half_chunks];
    const uint4 out_lo = rope_chunk<T>(lo, hi, cs[c], sn[c], true);
    const uint4 out_hi = rope_chunk<T>(hi, lo, cs[c + half_chunks], sn[c + half_chunks], false);
    o[c] = out_lo;
    o[c + half_chunks] = out_hi;
}

}  // namespace mv
