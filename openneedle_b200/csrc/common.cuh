// Shared device/host helpers for the needle2 B200 kernels (sm_100a only).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace nb200 {

// Thread-local error text behind needle2_b200_error(), the error channel that
// the reference's void entry points lack (needle2/csrc/cq.cpp:354-370).
void set_error(const std::string &msg);
void clear_error();
const char *last_error();

#define NB_CUDA_TRY(expr)                                                                  \
    do {                                                                                   \
        cudaError_t _e = (expr);                                                           \
        if (_e != cudaSuccess) {                                                           \
            ::nb200::set_error(std::string(#expr) + ": " + cudaGetErrorString(_e));        \
            return false;                                                                  \
        }                                                                                  \
    } while (0)

// Exact FP16 -> FP32 (the hardware conversion is exact for every half value,
// matching half_float of needle2/csrc/cq.cpp:14-28).
__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

// Round-half-to-even float -> int, i.e. std::nearbyint in the default mode.
__device__ __forceinline__ int rint_even(float v) { return __float2int_rn(v); }

__device__ __forceinline__ int clamp127(int v) { return v < -127 ? -127 : (v > 127 ? 127 : v); }

__host__ __device__ constexpr int ceil_div(int a, int b) { return (a + b - 1) / b; }

}  // namespace nb200
