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

}  // namespace mv
