// Persistent CQ2/CQ4 GEMV (see cq_gemv.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace nb200 {

constexpr int kGemvV2MaxSmem = 200 * 1024;

struct GemvV2Params {
    const uint8_t *packed;   // [out][rowbytes]
    const uint16_t *norms;   // [out][groups] FP16 bits
    int out, groups, rowbytes, padded, M, rpr;
    const float *rot;        // FP32 mode activations [M][padded]
    const int8_t *q;         // SDOT activations [M][padded]
    const float *xs;         // SDOT scales [M][groups]
    float *y;
    int ldy;
    int32_t *partials;       // SDOT debug [M][out][groups] or null
    float lut[16];
    uint32_t ctab[4];
    float cs;
};

// Rows of activations one launch can take for this geometry (0: unsupported).
int gemv_v2_max_rows(int bits, int group, int groups, bool i8);
bool launch_gemv_v2(const GemvV2Params &p, int bits, int group, bool i8, cudaStream_t st);

}  // namespace nb200
