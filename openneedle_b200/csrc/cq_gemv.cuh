// Persistent CQ2/CQ4 GEMV over one or several matrices (see cq_gemv.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace nb200 {

constexpr int kGemvMaxMats = 32;    // matrices fused into one launch
constexpr int kGemvMaxSmem = 200 * 1024;

struct GemvMatrix {
    const uint8_t *packed;   // [out][rowbytes]
    const uint16_t *norms;   // [out][groups] FP16 bits
    const uint16_t *norms8;  // [out][groups rounded up to 8] FP16 bits (int8 mode)
    float *y;                // [M][out]
    int out;
};

// Matrices of one launch share the input geometry (in, group, bits) and the
// codebook, so one prepared activation serves them all (the fused projections
// of needle2/csrc/engine.cpp:560-606 and cq_linear_many, cq.cpp:291-340).
struct GemvBatch {
    int nmat;
    GemvMatrix mat[kGemvMaxMats];
    int bits, group, groups, rowbytes, padded, M;
    const float *rot;        // FP32 mode activations [M][padded]
    const int8_t *q;         // SDOT activations [M][padded] (CQ2: bit-plane order)
    const float *xs;         // SDOT scales [M][groups]
    int32_t *partials;       // SDOT debug [M][out][groups] (single matrix) or null
    float lut[16];           // FP32 mode: value of each stored index
    uint32_t ctab[4];        // SDOT: int8 centroids, four per word
    uint32_t ntab[2];        // SDOT CQ4 sign split: |centroid| of entries 0-7
    uint32_t ptab[2];        // SDOT CQ4 sign split: centroid of entries 8-15
    int split;               // SDOT CQ4: entries 0-7 <= 0 <= entries 8-15
    float cs;                // SDOT: centroid scale
};

// Activation rows one launch can take for this geometry (0: not supported).
int gemv_max_rows(int bits, int group, int groups, bool i8);
bool launch_gemv(const GemvBatch &b, bool i8, cudaStream_t st);
// int8 (SDOT) GEMV with the products on the tensor cores (cq_gemv_mma.cu);
// launch_gemv routes int8 batches here.
int gemv_mma_max_rows(int bits, int group, int groups);
bool launch_gemv_mma(const GemvBatch &b, cudaStream_t st);
// Fault flag of kernels with bounded waits (0 when none ran out); clears it.
int read_and_clear_gemv_fault();

}  // namespace nb200
