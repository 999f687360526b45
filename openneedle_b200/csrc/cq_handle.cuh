// Internal access to CQ handles (cq_abi.cu) for the engine: the device view of
// a handle's matrix, its prepared activations, and an int8 twin of an FP32
// handle.  Not part of the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "cq_kernels.cuh"

namespace nb200 {

struct QkvgEpilogue;
struct KParts;

// Device view of handle's matrix (null when handle is null).
const CQDevice *handle_matrix(void *handle);
bool handle_is_sdot(void *handle);
int handle_device(void *handle);
// Rotate (FP32 handle) or rotate and quantise (int8 handle) x[batch][in] into
// the handle's scratch and return it: rot [batch][padded] (FP32), or q
// [batch][padded] (CQ2 in bit-plane order) and xs [batch][groups] (int8).
bool handle_prepare(void *handle, const float *x, int batch, const float **rot, const int8_t **q, const float **xs,
                    cudaStream_t st);
// Whether y_i = W_i x for these FP32 handles and `batch` rows runs the
// tensor-core GEMM on activations rotated and split into bf16 hi/lo (true:
// *group and *scale are the rotation's group size and 1/sqrt(group)).
bool handle_hilo_gemm(void *const *hs, int count, int batch, int *group, float *scale);
// That GEMM on activations the caller rotated and split: a_hilo [batch][in]
// bf16 hi, then [batch][in] lo (in = the matrices' padded width).
// epi / epi_done: the decode epilogue of launch_gemm_f32x3_multi (optional);
// kp: its K-split partial outputs (optional; ys[i] + p * kp->pstride, the
// output's rows of width out_i).
bool handle_many_hilo(void *const *hs, int count, const uint16_t *a_hilo, float *const *ys, int batch,
                      cudaStream_t st, const QkvgEpilogue *epi = nullptr, bool *epi_done = nullptr,
                      const KParts *kp = nullptr);
// A new int8 (SDOT) handle over the same packed matrix as the FP32 handle
// `cq` (its device copy read back once), or null with the error set.
void *handle_make_sdot(void *cq);

}  // namespace nb200
