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
    const uint8_t *frag;     // int8 mode: fragment-order copy (build_frag_layout), or null
    const uint16_t *normsF;  // int8 mode: norms [16-row tile][group][row g: (g, g + 8)], or null
    const uint8_t *blocked;  // FP32 mode: row-block copy (build_blocked_layout), or null
    const uint16_t *normsB;  // FP32 mode: norms [32-row block][group][32 rows], or null
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
// FP32-mode GEMV with one output row per lane (cq_gemv_rows.cu) for up to
// gemv_rows_max_rows activation rows; launch_gemv routes FP32 batches there
// when every matrix carries the row-block copy: rows in blocks of 32; per
// block and group, the group's packed bytes in units of U bytes (32 where a
// group's bytes are a multiple of 32, else 16), unit c of all 32 rows stored
// one after another, so one warp load reads one contiguous span of 32 * U
// bytes; rows past the matrix are zero.  normsB holds per block and group the
// 32 rows' norms.
size_t blocked_bytes(int out, int groups, int group, int bits);
size_t blocked_norm_count(int out, int groups);
bool build_blocked_layout(const uint8_t *packed, const uint16_t *norms, int out, int groups, int group, int bits,
                          int rowbytes, uint8_t *blocked, uint16_t *normsB, cudaStream_t st);
int gemv_rows_max_rows(int bits, int group, int groups);
bool launch_gemv_rows(const GemvBatch &b, cudaStream_t st);
// Which FP32 GEMV kernel launch_gemv uses: 0 automatic (for one activation row
// the product-table cluster kernel where its table fits, else the row kernel
// where it fits), 1 the slot-per-lane kernel of cq_gemv.cu, 2 the row kernel
// without the product table.
void set_f32_gemv_kernel(int kind);
int f32_gemv_kernel();
// int8 GEMV with weights as the mma.sync A operand (cq_gemv_frag.cu).  The
// fragment-order copy: 16-row tiles; per tile and group one block of
// 32 lanes x (gb / 2) bytes; lane (g, t) holds, for every 32-wide K step s,
// the indices of rows g and g + 8 at k = 32s + 4t..4t+3 (nibbles / crumbs 0-3)
// and 32s + 16 + 4t..4t+3 (4-7); CQ2 words carry two K steps.  normsF holds
// per tile and group the pairs (row g, row g + 8), g = 0..7.
size_t frag_bytes(int out, int groups, int group, int bits);
size_t frag_norm_count(int out, int groups);
bool build_frag_layout(const uint8_t *packed, const uint16_t *norms, int out, int groups, int group, int bits,
                       int rowbytes, uint8_t *frag, uint16_t *normsF, cudaStream_t st);
int gemv_frag_max_rows(int bits, int group, int groups);
bool launch_gemv_frag(const GemvBatch &b, cudaStream_t st);
// int8 prefill GEMM on tcgen05 (cq_gemm_tc.cu) for group size 128: weights
// decoded once to int8 W8[out][padded] (activation element order) and group
// scales nsT[groups][out rounded up to the tile width].
size_t gemm_w8_bytes(int out, int padded);
size_t gemm_ns_count(int out, int groups);
bool gemm_supported(int bits, int group, int padded);
bool gemm_prepare(const uint8_t *packed, const uint16_t *norms, int out, int groups, int group, int bits, int rowbytes,
                  int padded, const uint32_t ctab[4], float cs, int8_t *w8, float *nsT, cudaStream_t st);
bool launch_gemm_i8(const int8_t *q, const float *xs, int M, const int8_t *w8, const float *nsT, int N, int padded,
                    int groups, float *y, int ldy, cudaStream_t st);
// The same GEMM writing every output element to each of dsts[0..ndst) (the
// columns this matrix covers in several [M][ldy] buffers, e.g. every rank's
// output of an N-sharded matrix: the all-gather fused into the epilogue).
constexpr int kMaxGemmOutputs = 8;
bool launch_gemm_i8_multi(const int8_t *q, const float *xs, int M, const int8_t *w8, const float *nsT, int N,
                          int padded, int groups, float *const *dsts, int ndst, int ldy, cudaStream_t st);
// FP32-mode prefill GEMM on tcgen05 (cq_gemm_tc.cu): weights W' = half(norm) *
// lut[idx] split once to bf16 hi/lo [2][out][padded], activations split per
// call, three bf16 MMAs per K step into an f32 accumulator.
bool gemm_f32_supported(int storage_bits, int padded);
size_t gemm_f32_weight_elems(int out, int padded);
bool gemm_f32_prepare(const uint8_t *packed, const uint16_t *norms, int out, int groups, int group, int storage_bits,
                      int rowbytes, int padded, const float lut[16], uint16_t *w_hilo, cudaStream_t st);
bool launch_split_bf16(const float *x, long long n, uint16_t *hilo, cudaStream_t st);
bool launch_gemm_f32x3(const uint16_t *a_hilo, int M, const uint16_t *w_hilo, int N, int padded, float *y, int ldy,
                       cudaStream_t st);
// Several matrices against the same split activations in one launch (the
// fused projections): y_i[M][ldy_i] = A . W_i^T.
struct F32Out {
    const uint16_t *w_hilo;
    int N;
    float *y;
    int ldy;
};
struct QkvgEpilogue;
// Partial outputs of a launch split along K (decode-sized launches whose few
// output tiles would leave most SMs idle): the launch may split K into up to
// max_parts parts (a power of two); part p of output i is written to
// y_i + p * pstride (part 0 included) and *parts receives how many were
// written, so that the consumer adds them in order.
struct KParts {
    int max_parts;
    long long pstride;
    int *parts;
};
constexpr int kMaxKParts = 8;   // most K parts of one launch
// epi (optional, four segments q, k, v, gate): the decode-step epilogue of
// qkvg_epilogue.cuh, applied when the launch runs 64-wide tiles of one head
// each; *epi_done tells whether it ran (else the caller still has to do it).
// kp (optional, not with epi): K-split partial outputs as above.
bool launch_gemm_f32x3_multi(const uint16_t *a_hilo, int M, int padded, const F32Out *outs, int count,
                             cudaStream_t st, const QkvgEpilogue *epi = nullptr, bool *epi_done = nullptr,
                             const KParts *kp = nullptr);
// Activation rows from which int8 products run as the tensor-core GEMM.
constexpr int kGemmMinRows = 64;

// Fault flag of kernels with bounded waits (0 when none ran out); clears it.
int read_and_clear_gemv_fault();

}  // namespace nb200
