// Row-wise operations around the decode step of the batched runtime:
//  * rms_norm_kernel: out = weight * to_T(x * rsqrt(mean(x^2) + eps)), the
//    statistics in fp32 (src/micro_vllm/model.py:25-41), one CTA per row;
//  * silu_mul_kernel: out = to_T(to_T(silu(g)) * u) for a row [g | u] of a
//    fused gate/up projection, rounded as F.silu(gate) * up is (model.py:150-165).
// Rows move as 16-byte chunks when the row width and alignment allow.
#pragma once

#include "mv_device.cuh"

namespace mv {

constexpr int kRowThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kRowThreads)
rms_norm_kernel(const T* x, int64_t x_stride, const T* weight, T* out, int64_t out_stride, int hidden, float eps) {
    wait_for_prior_grid();
    allow_next_grid();
    const T* row = x + blockIdx.x * x_stride;
    T* orow = out + blockIdx.x * out_stride;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        const float v = to_float<T>(row[i]);
        ss = __fmaf_rn(v, v, ss);
    }
    ss = warp_sum(ss);
    __shared__ float partial[kRowThreads / 32];
    __shared__ float scale;
    if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float total = 0.0f;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) total += partial[w];
        scale = rsqrtf(total / static_cast<float>(hidden) + eps);
    }
    __syncthreads();
    const float r = scale;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        const T normalized = from_float<T>(__fmul_rn(to_float<T>(row[i]), r));
        orow[i] = from_float<T>(__fmul_rn(to_float<T>(weight[i]), to_float<T>(normalized)));
    }
}

template <typename T>
__global__ void __launch_bounds__(kRowThreads)
silu_mul_kernel(const T* gate_up, int64_t stride, T* out, int64_t out_stride, int width, int64_t total) {
    wait_for_prior_grid();
    allow_next_grid();
    const int64_t step = static_cast<int64_t>(blockDim.x) * gridDim.x;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total; idx += step) {
        const int64_t r = idx / width;
        const int c = static_cast<int>(idx - r * width);
        const float g = to_float<T>(gate_up[r * stride + c]);
        const float u = to_float<T>(gate_up[r * stride + width + c]);
        const float silu = to_float<T>(from_float<T>(g / (1.0f + expf(-g))));
        out[r * out_stride + c] = from_float<T>(__fmul_rn(silu, u));
    }
}

// 16-byte vector forms (8 two-byte or 4 four-byte elements per chunk), used
// when widths, strides and addresses allow; same arithmetic per element.
template <typename T>
struct Chunk {
    static constexpr int kElems = 16 / sizeof(T);
};

// One CTA per row; the row stays in registers between the two passes
// (at most kMaxChunks 16-byte chunks per thread).
constexpr int kNormMaxChunks = 4;

template <typename T>
__global__ void __launch_bounds__(kRowThreads)
rms_norm_vec_kernel(const T* x, int64_t x_stride, const T* weight, T* out, int64_t out_stride, int hidden, float eps) {
    constexpr int E = Chunk<T>::kElems;
    wait_for_prior_grid();
    allow_next_grid();
    const uint4* row = reinterpret_cast<const uint4*>(x + blockIdx.x * x_stride);
    uint4* orow = reinterpret_cast<uint4*>(out + blockIdx.x * out_stride);
    const uint4* wrow = reinterpret_cast<const uint4*>(weight);
    const int chunks = hidden / E;
    uint4 v[kNormMaxChunks];
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < kNormMaxChunks; ++k) {
        const int c = threadIdx.x + k * kRowThreads;
        if (c < chunks) {
            v[k] = row[c];
            const T* e = reinterpret_cast<const T*>(&v[k]);
#pragma unroll
            for (int i = 0; i < E; ++i) {
                const float f = to_float<T>(e[i]);
                ss = __fmaf_rn(f, f, ss);
            }
        }
    }
    ss = warp_sum(ss);
    __shared__ float partial[kRowThreads / 32];
    __shared__ float scale;
    if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float total = 0.0f;
        for (int w = 0; w < kRowThreads / 32; ++w) total += partial[w];
        scale = rsqrtf(total / static_cast<float>(hidden) + eps);
    }
    __syncthreads();
    const float r = scale;
#pragma unroll
    for (int k = 0; k < kNormMaxChunks; ++k) {
        const int c = threadIdx.x + k * kRowThreads;
        if (c < chunks) {
            const uint4 wv = wrow[c];
            const T* e = reinterpret_cast<const T*>(&v[k]);
            const T* we = reinterpret_cast<const T*>(&wv);
            uint4 o;
            T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
            for (int i = 0; i < E; ++i) {
                const T normalized = from_float<T>(__fmul_rn(to_float<T>(e[i]), r));
                oe[i] = from_float<T>(__fmul_rn(to_float<T>(we[i]), to_float<T>(normalized)));
            }
            orow[c] = o;
        }
    }
}

// One warp per row for rows of up to 32 x kWarpNormChunks chunks (hidden <= 2048
// two-byte elements): the reduction stays in the warp, no shared memory or
// block barrier, and a CTA covers kRowThreads / 32 rows.
constexpr int kWarpNormChunks = 8;

template <typename T>
__global__ void __launch_bounds__(kRowThreads)
rms_norm_warp_kernel(const T* x, int64_t x_stride, const T* weight, T* out, int64_t out_stride, int hidden,
                     float eps, int64_t rows) {
    constexpr int E = Chunk<T>::kElems;
    wait_for_prior_grid();
    allow_next_grid();
    const int lane = threadIdx.x & 31;
    const int64_t r = static_cast<int64_t>(blockIdx.x) * (kRowThreads / 32) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const uint4* row = reinterpret_cast<const uint4*>(x + r * x_stride);
    uint4* orow = reinterpret_cast<uint4*>(out + r * out_stride);
    const uint4* wrow = reinterpret_cast<const uint4*>(weight);
    const int chunks = hidden / E;
    uint4 v[kWarpNormChunks];
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < kWarpNormChunks; ++k) {
        const int c = lane + 32 * k;
        if (c < chunks) {
            v[k] = row[c];
            const T* e = reinterpret_cast<const T*>(&v[k]);
#pragma unroll
            for (int i = 0; i < E; ++i) {
                const float f = to_float<T>(e[i]);
                ss = __fmaf_rn(f, f, ss);
            }
        }
    }
    const float scale = rsqrtf(warp_sum(ss) / static_cast<float>(hidden) + eps);
#pragma unroll
    for (int k = 0; k < kWarpNormChunks; ++k) {
        const int c = lane + 32 * k;
        if (c < chunks) {
            const uint4 wv = wrow[c];
            const T* e = reinterpret_cast<const T*>(&v[k]);
            const T* we = reinterpret_cast<const T*>(&wv);
            uint4 o;
            T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
            for (int i = 0; i < E; ++i) {
                const T normalized = from_float<T>(__fmul_rn(to_float<T>(e[i]), scale));
                oe[i] = from_float<T>(__fmul_rn(to_float<T>(we[i]), to_float<T>(normalized)));
            }
            orow[c] = o;
        }
    }
}

// Grid (chunk blocks, row blocks): no index division per element; rows beyond
// the grid's y extent are taken in steps of gridDim.y.
template <typename T>
__global__ void __launch_bounds__(kRowThreads)
silu_mul_vec_kernel(const T* gate_up, int64_t stride, T* out, int64_t out_stride, int width, int64_t rows) {
    constexpr int E = Chunk<T>::kElems;
    wait_for_prior_grid();
    allow_next_grid();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= width / E) return;
    for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
        const uint4 gv = *reinterpret_cast<const uint4*>(gate_up + r * stride + c * E);
        const uint4 uv = *reinterpret_cast<const uint4*>(gate_up + r * stride + width + c * E);
        const T* g = reinterpret_cast<const T*>(&gv);
        const T* u = reinterpret_cast<const T*>(&uv);
        uint4 o;
        T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int i = 0; i < E; ++i) {
            const float gf = to_float<T>(g[i]);
            const float silu = to_float<T>(from_float<T>(gf / (1.0f + expf(-gf))));
            oe[i] = from_float<T>(__fmul_rn(silu, to_float<T>(u[i])));
        }
        *reinterpret_cast<uint4*>(out + r * out_stride + c * E) = o;
    }
}

}  // namespace mv
