// Scalar helpers shared by the engine's support kernels: warp sums and the
// reference's RMS and sigmoid formulas in FP32 round-to-nearest.
#pragma once
#include <math.h>

#include "cq_gemv.cuh"

namespace nb200 {
namespace eng {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

// 1 / sqrt(mean(x^2) + 1e-6) from the sum of squares (engine.cpp:182).
__device__ __forceinline__ float rms_inv(float sumsq, int n) {
    return __fdiv_rn(1.f, sqrtf(__fadd_rn(__fdiv_rn(sumsq, (float)n), 1e-6f)));
}

// The reference's sigmoid, 1 / (1 + exp(-x)) (engine.cpp:36).
__device__ __forceinline__ float sigm(float x) { return __fdiv_rn(1.f, __fadd_rn(1.f, expf(-x))); }

// Sum of the K-split parts p[0], p[stride], ... of one GEMM output
// (1 <= parts <= kMaxKParts), added in part order.
__device__ __forceinline__ float part_sum(const float *__restrict__ p, int parts, long long stride) {
    float s = p[0];
#pragma unroll
    for (int i = 1; i < kMaxKParts; ++i)
        if (i < parts) s += p[i * stride];
    return s;
}

}  // namespace eng
}  // namespace nb200
