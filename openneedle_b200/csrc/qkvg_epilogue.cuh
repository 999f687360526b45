// Decode-step epilogue of the fused Q/K/V/gate GEMM: the work of
// qk_rope_store_kernel (engine_kernels.cu) done where the GEMM's 64-wide output
// tiles leave TMEM, one head of one row per thread.  Q and K heads get the
// RMS norm with (1 + norm) and the rotary embedding at the row's position
// (needle2/csrc/engine.cpp:994-1000); K and V heads are stored into the KV
// cache row of the row's token (engine.cpp:1001-1021: scale max/127 or 1,
// values rint(x * (127 / max)) clamped to +-127, or FP32 as is).
#pragma once
#include <stdint.h>

#include "kv_pool.cuh"

namespace nb200 {

struct QkvgEpilogue {
    int active;                    // 1: the launch's four segments are q, k, v and gate of decode rows
    int heads, kvheads, hd;        // hd must equal the GEMM's tile width
    const float *q_norm, *k_norm;  // [hd]
    const float *cos_t, *sin_t;    // [table_len][hd / 2]: cosf / sinf of position / divisor[j]
    int table_len;
    const float *divisor;          // [hd / 2], for positions past the table
    const int *pos;                // [rows]: position of each row's token
    KVStoreTarget kv;              // where each row's K and V heads go (one token per row)
};

// cos/sin tables of the rotary embedding: angle = position / divisor[j]
// (engine.cpp:997-999), the formula qk_norm_rope_kernel evaluates per call.
bool launch_rope_table(const float *divisor, int half, int positions, float *cos_t, float *sin_t, cudaStream_t st);

}  // namespace nb200
