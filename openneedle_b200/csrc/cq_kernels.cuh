// Launchers for the CQ matrix kernels (FP32 mode, SDOT int8 mode, row gather).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace nb200 {

// Largest group handled on the GPU (warp FWHT up to 1024, CTA FWHT above).
constexpr int kMaxGroup = 16384;
// Activation rows per GEMV pass; larger batches run several passes.
constexpr int kGemvMaxRows = 16;

struct CQDevice {
    int out, in, bits, group, padded, groups, storage_bits, rowbytes;
    const uint8_t *packed;    // [out][rowbytes] device
    const uint16_t *norms;    // [out][groups] FP16 bits, device
    const uint16_t *norms8;   // SDOT: norms with rows padded to a multiple of 8 groups (== norms when aligned)
    const uint8_t *frag;      // SDOT: fragment-order copy for the warp-MMA kernel, or null
    const uint16_t *normsF;   // SDOT: norms in fragment order, or null
    const uint8_t *blocked;   // FP32: row-block copy for the row GEMV kernels (see blocked_bytes), or null
    const uint16_t *normsB;   // FP32: norms of the row-block copy, or null
    float lut[16];            // FP32 mode: value of each stored index
    uint32_t ctab[4];         // SDOT: int8 centroids, four per word
    uint32_t ntab[2], ptab[2];   // SDOT CQ4 sign split: |c| of entries 0-7, c of entries 8-15
    int split;                // SDOT CQ4: entries 0-7 <= 0 <= entries 8-15 (sign-split decode applies)
    float centroid_scale;     // SDOT: max|cb|/127
};

// Rotation of activations x[M][in] (zero padded): rot[M][padded] FP32.
bool launch_rotate(const CQDevice &w, const float *x, int M, float *rot, cudaStream_t s);
// The rotation straight into the FP32-mode GEMM's bf16 operands: hilo[M][padded]
// = bf16(rot), then hilo[M*padded + ...] = bf16(rot - hi) (groups 8 to 1024).
bool launch_rotate_hilo(const CQDevice &w, const float *x, int M, uint16_t *hilo, cudaStream_t s);
// SDOT quantiser: q[M][padded] int8 (CQ2: bit-plane order of each 16-element
// block) and xs[M][groups].
bool launch_quantize(const CQDevice &w, const float *x, int M, int8_t *q, float *xs, cudaStream_t s);
// y[m*ldy + r] for m < M, FP32 mode from rot.
bool launch_gemv_f32(const CQDevice &w, const float *rot, int M, float *y, int ldy, cudaStream_t s);
// y from q/xs (SDOT mode); optional partials[M][out][groups] int32.
bool launch_gemv_i8(const CQDevice &w, const int8_t *q, const float *xs, int M, float *y, int ldy,
                    int32_t *partials, cudaStream_t s);
// Dequantised rows: y[c][in] for ids[c].
bool launch_rows(const CQDevice &w, const int64_t *ids, int count, float *y, cudaStream_t s);

bool gemv_fast_path(const CQDevice &w);
// The engine's fake activation quantiser, in place on x[rows][dim] (per row).
bool launch_activation_quant(float *x, int rows, int dim, int bits, cudaStream_t st);
// The decode loop's greedy token of each logits row: out[r] = first index of
// the row's maximum (NaNs never win; 0 when the first logit is NaN).
bool launch_argmax(const float *x, int rows, int vocab, int ld, int *out, cudaStream_t st);

struct GemvBatch;
// A one-matrix GEMV batch description of w (activations and outputs unset).
GemvBatch single_batch(const CQDevice &w);

}  // namespace nb200
