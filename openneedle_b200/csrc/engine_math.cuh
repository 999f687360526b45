// Scalar helpers shared by the engine's support kernels: warp sums and the
// reference's RMS and sigmoid formulas in FP32 round-to-nearest.
#pragma once
#include <math.h>

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

}  // namespace eng
}  // namespace nb200
