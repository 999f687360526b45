// SDOT (int8) CQ2/CQ4 prefill GEMM on the sm_100a tensor cores:
// y[m][n] = sum_g ((float(d[m,n,g]) * ns[n,g]) * xs[m,g]) in group order, with
// d[m,n,g] the exact int32 dot of group g (needle2/csrc/sdot.cpp:108-149).
//
// The weights are decoded once per matrix (lazily, at the first prefill) to an
// int8 copy W8[N][padded] in the activations' element order, and the group
// scales ns[n,g] = half(norm) * cs to nsT[g][N'] (N' = N rounded up to 192).
// One persistent CTA per SM walks 128 x 192 output tiles (15 warps, 128
// registers a thread; 192 columns also pack the SMs' waves better than 256 at
// the usual sizes), its pipelines running on across tile boundaries:
//   * warp 0 (one lane): TMA loads of the group's activation tile (128 x 128
//     bytes) and weight tile (192 x 128 bytes), 128-byte swizzled, into a
//     5-stage ring, and a bulk copy of the group's 192 scales into an 8-deep
//     ring;
//   * warp 1 (one lane): per group four tcgen05.mma kind::i8 (M = 128,
//     N = 192, K = 32) into one of two TMEM accumulators, then commits; the
//     accumulators hold a bias (see biased_pair) that the MMAs add onto;
//   * warps 2-13: thread = accumulator lane (activation row) x 64 columns;
//     per group it reads its int32 dots back (tcgen05.ld) and adds the group
//     terms to its 64 running sums in registers, in group order (paired FP32
//     instructions, exact per element); the finished tile leaves through
//     shared memory in coalesced rows.
// All waits are bounded; on timeout the CTA raises the device fault flag.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "cq_gemv.cuh"
#include "qkvg_epilogue.cuh"
#include "tcgen05.cuh"

namespace nb200 {

extern __device__ int g_gemv_fault;

namespace {

constexpr int kBM = 128, kBN = 192, kBK = 128;   // tile rows, columns, K per group step
constexpr int kDCols = 256;                       // TMEM columns between the two accumulators
constexpr int kStages = 5, kNsRing = 8;
constexpr int kEpiWarps = kBN / 64 * 4;           // 12: four lane quarters x 64-column slices
constexpr int kXsWarp = 2 + kEpiWarps;            // 14: loads the activation scales
constexpr int kThreads = (3 + kEpiWarps) * 32;    // 480
constexpr int kStageA = kBM * kBK, kStageB = kBN * kBK, kStageBytes = kStageA + kStageB;
constexpr size_t kSmem = (size_t)kStages * kStageBytes + (size_t)kNsRing * (kBN + kBM) * 4 + 1024;
constexpr uint32_t kWaitLimit = 1u << 24;

__device__ __forceinline__ bool gwait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    const uint32_t a = smem_addr(bar);
    {
        // a phase that has already completed is the common case: the
        // non-blocking test answers it without try_wait's suspend latency
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
        if ((i & 1023) == 1023 && *abort_flag) return false;
    }
    *abort_flag = 1;
    atomicExch(&g_gemv_fault, 1);
    return false;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// Paired FP32 arithmetic (sm_100): two IEEE round-to-nearest results per
// instruction, element by element identical to the scalar forms.
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    unsigned long long r, x, y;
    memcpy(&x, &a, 8);
    memcpy(&y, &b, 8);
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
    float2 o;
    memcpy(&o, &r, 8);
    return o;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    unsigned long long r, x, y;
    memcpy(&x, &a, 8);
    memcpy(&y, &b, 8);
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
    float2 o;
    memcpy(&o, &r, 8);
    return o;
}

// acc + t with one rounding, written as fma(t, one, acc) where one == 1.0f
// arrives as a kernel argument. A paired multiply feeding a paired add may be
// fused into a paired FMA by the assembler (measured: it changes the rounding
// of about 4 in 10 terms), which the running sums must not see; the product
// here is an FMA's multiplicand, which cannot be fused any further, and the
// assembler cannot fold a multiplier it does not know.
__device__ __forceinline__ float2 fma_one2(float2 t, float2 one, float2 acc) {
    unsigned long long r, x, y, z;
    memcpy(&x, &t, 8);
    memcpy(&y, &one, 8);
    memcpy(&z, &acc, 8);
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(x), "l"(y), "l"(z));
    float2 o;
    memcpy(&o, &r, 8);
    return o;
}

// Two int32 dots to float, exactly. The accumulator starts every group at the
// bit pattern of 1.5 * 2^23 (kBias), so the MMA leaves kBias + d there; with
// |d| <= 128 * 127 * 127 < 2^22 that integer is the float 1.5 * 2^23 + d (same
// binade, spacing 1), and subtracting 1.5 * 2^23 leaves d itself. This costs
// one paired subtract per two elements instead of two quarter-rate
// int-to-float conversions.
constexpr uint32_t kBias = 0x4B400000u;   // 12582912.0f
// true: the accumulators are reset to kBias in TMEM after each read (a TMEM
// store per chunk); false: they start at zero and the bias is added here.
constexpr bool kBiasInTmem = false;
__device__ __forceinline__ float2 biased_pair(uint32_t a, uint32_t b) {
    if (!kBiasInTmem) {
        a += kBias;
        b += kBias;
    }
    return fadd2(make_float2(__uint_as_float(a), __uint_as_float(b)), make_float2(-12582912.0f, -12582912.0f));
}

// Adds one group's terms for one 16x256b chunk (two column blocks of two rows):
// acc += (d * ns) * xs per element, in that order, one rounding per operation.
// v[0..1] / v[2..3] are rows 0 / 8 of block 0, v[4..7] the same of block 1.
__device__ __forceinline__ void chunk_terms(const uint32_t (&v)[8], const float2 (&ns2)[2], float2 xs_a, float2 xs_b,
                                            float2 one2, float2 *acc_a, float2 *acc_b) {
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        acc_a[b] = fma_one2(fmul2(fmul2(biased_pair(v[4 * b], v[4 * b + 1]), ns2[b]), xs_a), one2, acc_a[b]);
        acc_b[b] = fma_one2(fmul2(fmul2(biased_pair(v[4 * b + 2], v[4 * b + 3]), ns2[b]), xs_b), one2, acc_b[b]);
    }
}

// K-major, 128-byte swizzled operand: 8-row atoms of 1 KB (SBO = 1024).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

struct GemmArgs {
    int M, N, groups, ldy;
    const float *xs;    // [M][groups]
    const float *nsT;   // [groups][N rounded up to 256]
    int nstride;        // N rounded up to 256
    float *y;           // [M][ldy]
    float one;          // 1.0f, passed at run time: see fma_one2
    // outputs: y[m][n] is written to dst[i] + m * ldy + n for every i < ndst (the
    // caller's own buffer, or the same columns of every rank's full output
    // buffer when an all-gather is fused into the epilogue)
    float *dst[kMaxGemmOutputs];
    int ndst;
    int mtiles, tiles;   // tile t covers rows (t % mtiles) * 128 and columns (t / mtiles) * 192
};

// 15 warps: at most four per SM sub-partition, so 128 registers per thread.
__global__ void __launch_bounds__(kThreads, 1)
    cq_gemm_i8_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                      const __grid_constant__ GemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *ns_ring = reinterpret_cast<float *>(smem + (size_t)kStages * kStageBytes);   // [kNsRing][kBN]
    float *xs_ring = ns_ring + (size_t)kNsRing * kBN;                                  // [kNsRing][kBM]
    __shared__ __align__(8) uint64_t full[kStages], empty[kStages], dfull[2], dfree[2], nsfull[kNsRing],
        nsfree[kNsRing];
    __shared__ uint32_t tmem_s;
    __shared__ volatile int abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.groups;

    if (warp == 1) tc::alloc(&tmem_s, 512);
    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int d = 0; d < 2; ++d) {
            mbar_init(&dfull[d], 1);
            mbar_init(&dfree[d], kEpiWarps);
        }
        for (int r = 0; r < kNsRing; ++r) {
            mbar_init(&nsfull[r], 1 + 32);   // the scale copy, and each lane of the activation-scale warp
            mbar_init(&nsfree[r], kEpiWarps);
        }
        fence_barrier_init();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = tmem_s;

    // persistent: CTA b takes tiles b, b + gridDim.x, ...; every ring, TMEM
    // accumulator and barrier phase runs on the CTA's group counter gg, which
    // continues across tiles, so the next tile's loads and MMAs overlap the
    // previous tile's last groups and its output
    if (warp == 0) {
        if (lane == 0) {
            pdl_wait();   // the activations come from the preceding kernel
            int gg = 0;
            bool stop = false;
            for (int tile = blockIdx.x; tile < a.tiles && !stop; tile += gridDim.x) {
                const int m0 = (tile % a.mtiles) * kBM, n0 = (tile / a.mtiles) * kBN;
                for (int g = 0; g < G; ++g, ++gg) {
                    const int s = gg % kStages;
                    if (abort_flag ||
                        (gg >= kStages && !gwait(&empty[s], (uint32_t)((gg / kStages) - 1) & 1, &abort_flag))) {
                        stop = true;
                        break;
                    }
                    uint8_t *st = smem + (size_t)s * kStageBytes;
                    mbar_arrive_expect_tx(&full[s], kStageBytes);
                    tma_load_2d(st, &ta, g * kBK, m0, &full[s]);
                    tma_load_2d(st + kStageA, &tb, g * kBK, n0, &full[s]);
                    const int r = gg % kNsRing;
                    if (gg >= kNsRing && !gwait(&nsfree[r], (uint32_t)((gg / kNsRing) - 1) & 1, &abort_flag)) {
                        stop = true;
                        break;
                    }
                    mbar_arrive_expect_tx(&nsfull[r], kBN * 4);
                    bulk_g2s(ns_ring + (size_t)r * kBN, a.nsT + (size_t)g * a.nstride + n0, kBN * 4, &nsfull[r]);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_s8(kBM, kBN);
            int gg = 0;
            bool stop = false;
            for (int tile = blockIdx.x; tile < a.tiles && !stop; tile += gridDim.x) {
                for (int g = 0; g < G; ++g, ++gg) {
                    const int s = gg % kStages, d = gg & 1;
                    if (abort_flag || !gwait(&full[s], (uint32_t)(gg / kStages) & 1, &abort_flag) ||
                        !gwait(&dfree[d], (uint32_t)(gg / 2) & 1, &abort_flag)) {
                        stop = true;
                        break;
                    }
                    tc::fence_after();
                    const uint32_t sa = smem_addr(smem + (size_t)s * kStageBytes), sb = sa + kStageA;
#pragma unroll
                    for (int kk = 0; kk < kBK / 32; ++kk)
                        tc::mma_i8_ss(tmem + (uint32_t)(d * kDCols), sw128_desc(sa + kk * 32),
                                      sw128_desc(sb + kk * 32), idesc, kBiasInTmem || kk > 0);
                    tc::commit(&empty[s]);
                    tc::commit(&dfull[d]);
                }
            }
        }
        __syncwarp();
    } else if (warp == kXsWarp) {
        // each group's 128 activation scales of the tile into the ring slot that
        // also takes the group's column scales; the epilogue then never waits on
        // a global load (lanes: rows lane + 32 j)
        pdl_wait();
        int gg = 0;
        bool stop = false;
        for (int tile = blockIdx.x; tile < a.tiles && !stop; tile += gridDim.x) {
            const int m0 = (tile % a.mtiles) * kBM;
            for (int g = 0; g < G; ++g, ++gg) {
                const int r = gg % kNsRing;
                if (abort_flag ||
                    (gg >= kNsRing && !gwait(&nsfree[r], (uint32_t)((gg / kNsRing) - 1) & 1, &abort_flag))) {
                    stop = true;
                    break;
                }
#pragma unroll
                for (int j = 0; j < kBM / 32; ++j) {
                    const int row = m0 + lane + 32 * j;
                    xs_ring[(size_t)r * kBM + lane + 32 * j] = row < a.M ? a.xs[(size_t)row * G + g] : 0.f;
                }
                mbar_arrive(&nsfull[r]);
            }
        }
    } else {
        // epilogue: warp (q, slice) owns accumulator lanes 32q..32q+31 (activation
        // rows) x 64 columns, read in the 16x256b shape: thread t holds rows
        // 32q + t/4 + {0, 8, 16, 24} x columns 8b + 2(t%4) + {0, 1} (b = 0..7),
        // so per group it needs 4 row scales and 16 column scales.
        const int q = warp & 3, slice = (warp - 2) >> 2;
        const int col0 = slice * 64, cpair = 2 * (lane & 3);
        const int rbase = 32 * q + (lane >> 2);   // tile-local row of r = 0; r adds 8 r
        const uint32_t quarter = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)col0;
        // both accumulators start at the bias; the MMA warp waits for this
        if (kBiasInTmem) {
            for (int d = 0; d < 2; ++d)
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    tc::fill16x256_x2(
                        quarter + ((uint32_t)(16 * (i & 1)) << 16) + (uint32_t)(d * kDCols + 16 * (i >> 1)), kBias);
            tc::wait_st();
        }
        tc::fence_before();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&dfree[0]);
            mbar_arrive(&dfree[1]);
        }
        int gg = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < a.tiles && ok; tile += gridDim.x) {
            const int m0 = (tile % a.mtiles) * kBM, n0 = (tile / a.mtiles) * kBN;
            float2 acc[4][8];   // [row][column block], a column pair each
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int b = 0; b < 8; ++b) acc[r][b] = make_float2(0.f, 0.f);
            for (int g = 0; g < G; ++g, ++gg) {
                const int d = gg & 1, ri = gg % kNsRing;
                if (!gwait(&dfull[d], (uint32_t)(gg / 2) & 1, &abort_flag) ||
                    !gwait(&nsfull[ri], (uint32_t)(gg / kNsRing) & 1, &abort_flag)) {
                    ok = false;
                    break;
                }
                tc::fence_after();
                float2 xs2[4];
    #pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const float x = xs_ring[(size_t)ri * kBM + rbase + 8 * r];
                    xs2[r] = make_float2(x, x);
                }
                const float *nsr = ns_ring + (size_t)ri * kBN + col0 + cpair;
                const float2 one2 = make_float2(a.one, a.one);
                const uint32_t dq = quarter + (uint32_t)(d * kDCols);
                // chunk i: lanes +16 (i & 1), columns 16 (i >> 1) .. +15 (blocks 2c, 2c + 1);
                // read it, reset it to the bias for group g + 2, and keep the next
                // chunk's read in flight while this one is summed
                uint32_t va[8], vb[8];
                float2 ns2[2];
                tc::ld16x256_x2(dq, va);
    #pragma unroll
                for (int i = 0; i < 8; i += 2) {
                    const int c = i >> 1;
                    const uint32_t lo = dq + (uint32_t)(16 * c), hi = lo + (16u << 16);
                    ns2[0] = *reinterpret_cast<const float2 *>(nsr + 16 * c);
                    ns2[1] = *reinterpret_cast<const float2 *>(nsr + 16 * c + 8);
                    tc::wait_ld();
                    tc::hold8(va);
                    if (kBiasInTmem) tc::fill16x256_x2(lo, kBias);
                    tc::ld16x256_x2(hi, vb);
                    chunk_terms(va, ns2, xs2[0], xs2[1], one2, acc[0] + 2 * c, acc[1] + 2 * c);
                    tc::wait_ld();
                    tc::hold8(vb);
                    if (kBiasInTmem) tc::fill16x256_x2(hi, kBias);
                    if (i + 2 < 8) tc::ld16x256_x2(lo + 16, va);
                    chunk_terms(vb, ns2, xs2[2], xs2[3], one2, acc[2] + 2 * c, acc[3] + 2 * c);
                }
                if (kBiasInTmem) tc::wait_st();
                tc::fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&dfree[d]);
                    mbar_arrive(&nsfree[ri]);
                }
            }
            if (!ok) break;
            // the tile's rows straight from registers: for each (row, block) the four
            // lanes of a row write one 32-byte sector
            for (int di = 0; di < a.ndst; ++di) {
                float *const y = a.dst[di];
                const bool vec = (a.ldy & 1) == 0 && (reinterpret_cast<uintptr_t>(y) & 7) == 0;
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int row = m0 + rbase + 8 * r;
                    if (row >= a.M) continue;
                    float *yr = y + (size_t)row * a.ldy + n0 + col0 + cpair;
#pragma unroll
                    for (int b = 0; b < 8; ++b) {
                        const int col = n0 + col0 + 8 * b + cpair;
                        if (vec && col + 1 < a.N) {
                            *reinterpret_cast<float2 *>(yr + 8 * b) = acc[r][b];
                        } else {
                            if (col < a.N) yr[8 * b] = acc[r][b].x;
                            if (col + 1 < a.N) yr[8 * b + 1] = acc[r][b].y;
                        }
                    }
                }
            }
        }
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == 1) tc::dealloc(tmem, 512);
}

// Decoded int8 weights in the activations' element order (CQ2 activations are
// stored per 16 elements as evens then odds) and transposed group scales.
__global__ void gemm_prepare_kernel(const uint8_t *__restrict__ packed, const uint16_t *__restrict__ norms, int out,
                                    int groups, int G, int bits, int rowbytes, int padded, uint4 ctab, float cs,
                                    int nstride, int8_t *__restrict__ w8, float *__restrict__ nsT) {
    const int8_t *tab = reinterpret_cast<const int8_t *>(&ctab);
    const long long total = (long long)out * padded;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int n = (int)(i / padded), p = (int)(i % padded);
        int e = p;   // element stored at position p
        if (bits == 2) {
            const int r = p & 15;
            e = (p & ~15) | (r < 8 ? 2 * r : 2 * (r - 8) + 1);
        }
        const uint8_t *rp = packed + (size_t)n * rowbytes;
        const int idx = bits == 4 ? ((rp[e >> 1] >> (4 * (e & 1))) & 15) : ((rp[e >> 2] >> (2 * (e & 3))) & 3);
        w8[i] = tab[idx];
    }
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < (long long)groups * nstride;
         i += (long long)gridDim.x * blockDim.x) {
        const int g = (int)(i / nstride), n = (int)(i % nstride);
        nsT[i] = n < out ? __fmul_rn(half_bits_to_float(norms[(size_t)n * groups + g]), cs) : 0.f;
    }
    (void)G;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

bool make_map(CUtensorMap *map, const void *base, int rows, int cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled is not available from the driver");
        return false;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed for the prefill GEMM operands");
        return false;
    }
    return true;
}

// ---------------------------------------------------------------------------
// FP32-mode prefill GEMM: y[m][r] = sum_k W'[r][k] * rot[m][k] with
// W'[r][k] = half(norm[r, k / G]) * lut[idx[r][k]] (needle2/csrc/cq.cpp:75-109;
// the per-group norm folded into the weights, a reassociation well inside the
// FP32 tolerance).  Operands are split into bf16 pairs, v = hi + lo with
// hi = bf16(v) and lo = bf16(v - hi), and each K step issues three
// kind::f16 MMAs, A_hi B_hi + A_lo B_hi + A_hi B_lo, into one f32 accumulator
// (about 2^-16 relative error per product; bf16 keeps FP32's exponent range).
// 128 x 256 tiles with K = 64 (one 128-byte row of bf16) per stage, two
// stages of 96 KB; or, for decode-sized launches, 128 x 64 tiles with two
// stages of 48 KB (two CTAs per SM) or, where the grid fits one CTA per SM,
// four, so that half of a K = 512 product is in flight at once.
// Warp 0 issues the TMA loads (the weight tiles of the first stages before the
// kernel waits for its predecessor, which produces only the activations),
// warp 1 the MMAs, warps 2-5 read the accumulator (32 rows each) and store y.
constexpr int kFBM = 128, kFBK = 64;
constexpr int kFPartA = kFBM * kFBK * 2;   // bytes of one bf16 part of the activation tile
constexpr int kFThreads = 6 * 32;
template <int BN, int ST>
struct FTile {
    static constexpr int kStages = ST;
    static constexpr int kPartB = BN * kFBK * 2;
    static constexpr int kStageBytes = 2 * kFPartA + 2 * kPartB;
    static constexpr size_t kSmem = (size_t)kStages * kStageBytes + 1024;
};

// One output matrix of a launch: its bf16 hi/lo weight maps, y[M][ldy] and
// the first of its tiles along grid y.
struct F32Seg {
    CUtensorMap bh, bl;
    float *y;
    int N, ldy, tile0;
};
constexpr int kF32MaxSegs = 4;
struct GemmF32Args {
    F32Seg seg[kF32MaxSegs];
    int nseg, M, ksteps;   // ksteps: K steps of one CTA (of one part along grid z)
    long long pstride;     // floats between the partial outputs of consecutive parts
    QkvgEpilogue epi;      // used by the EPI instantiations only
};

// Norm, rotary embedding and KV store of one 64-wide head held by one thread
// (QkvgEpilogue): segment seg (0 q, 1 k, 2 v, 3 gate), head `head` of it,
// output row `row`; y receives the (roped) head.
__device__ __forceinline__ void qkvg_head(const QkvgEpilogue &E, int seg, int head, int row, float (&h)[64],
                                          float *yr) {
    if (seg <= 1) {
        const float *nrm = seg == 0 ? E.q_norm : E.k_norm;
        // four interleaved partial sums: a quarter of the dependent chain
        float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 64; ++i) s4[i & 3] = fmaf(h[i], h[i], s4[i & 3]);
        const float s = (s4[0] + s4[1]) + (s4[2] + s4[3]);
        const float inv = __fdiv_rn(1.f, sqrtf(__fadd_rn(__fdiv_rn(s, 64.f), 1e-6f)));
#pragma unroll
        for (int i = 0; i < 64; ++i) h[i] = __fmul_rn(__fmul_rn(h[i], inv), __fadd_rn(1.f, nrm[i]));
        const int p = E.pos[row];
        const bool tab = p < E.table_len;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            float co, si;
            if (tab) {
                co = E.cos_t[(size_t)p * 32 + j];
                si = E.sin_t[(size_t)p * 32 + j];
            } else {
                const float ang = __fdiv_rn((float)p, E.divisor[j]);
                co = cosf(ang);
                si = sinf(ang);
            }
            const float a = h[j], c = h[j + 32];
            h[j] = __fsub_rn(__fmul_rn(a, co), __fmul_rn(c, si));
            h[j + 32] = __fadd_rn(__fmul_rn(c, co), __fmul_rn(a, si));
        }
    }
#pragma unroll
    for (int i = 0; i < 64; i += 4) *reinterpret_cast<float4 *>(yr + i) = make_float4(h[i], h[i + 1], h[i + 2], h[i + 3]);
    if (seg != 1 && seg != 2) return;
    const KVDest &d = E.kv.dest;
    const int sess = d.session[row], p = d.position[row];
    const bool pinned = p < d.prefix;
    const size_t krow = pinned ? (size_t)head * d.prefix + p
                               : ((size_t)sess * E.kvheads + head) * d.rows +
                                     (d.window ? (p - d.prefix) % d.window : p - d.prefix);
    const bool isv = seg == 2;
    if (E.kv.fp32) {
        float *dst = (isv ? (pinned ? d.pvf : E.kv.vf) : (pinned ? d.pkf : E.kv.kf)) + krow * 64;
#pragma unroll
        for (int i = 0; i < 64; i += 4) *reinterpret_cast<float4 *>(dst + i) = make_float4(h[i], h[i + 1], h[i + 2], h[i + 3]);
        return;
    }
    float m4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 64; ++i) m4[i & 3] = fmaxf(m4[i & 3], fabsf(h[i]));
    const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
    const float sc = mx > 0.f ? __fdiv_rn(mx, 127.f) : 1.f;
    const float iv = mx > 0.f ? __fdiv_rn(127.f, mx) : 0.f;
    int8_t *dst = (isv ? (pinned ? d.pv : E.kv.v8) : (pinned ? d.pk : E.kv.k8)) + krow * 64;
    float *sdst = isv ? (pinned ? d.pvs : E.kv.vs) : (pinned ? d.pks : E.kv.ks);
#pragma unroll
    for (int i = 0; i < 64; i += 16) {
        uint32_t w[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            uint32_t word = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                int qv = __float2int_rn(__fmul_rn(h[i + 4 * b + e], iv));
                qv = qv < -127 ? -127 : (qv > 127 ? 127 : qv);
                word |= (uint32_t)(uint8_t)(int8_t)qv << (8 * e);
            }
            w[b] = word;
        }
        *reinterpret_cast<uint4 *>(dst + i) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    sdst[krow] = sc;
}

// grid: (M tiles, total N tiles of all segments, K parts); tile width BN (256
// for prefill-sized launches, 64 or 128 when that leaves too few CTAs for the
// machine).  Part z of a K-split launch takes K steps [z ksteps, (z + 1)
// ksteps) and writes its partial tile to y + z pstride; the consumer adds the
// parts in order.
template <int BN, int ST, int ACC, bool EPI>
__global__ void __launch_bounds__(kFThreads, 1)
    cq_gemm_f32x3_kernel(const __grid_constant__ CUtensorMap tah, const __grid_constant__ CUtensorMap tal,
                         const __grid_constant__ GemmF32Args a) {
    constexpr int kPartB = FTile<BN, ST>::kPartB, kStageBytes = FTile<BN, ST>::kStageBytes;
    constexpr int kFStages = ST;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t full[kFStages], empty[kFStages], dfull;
    __shared__ uint32_t tmem_s;
    __shared__ volatile int abort_flag;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int si = 0;
    while (si + 1 < a.nseg && (int)blockIdx.y >= a.seg[si + 1].tile0) ++si;
    const F32Seg &sg = a.seg[si];
    const int m0 = blockIdx.x * kFBM, n0 = ((int)blockIdx.y - sg.tile0) * BN;
    const int S = a.ksteps, k0 = (int)blockIdx.z * S;
    float *const yout = sg.y + (size_t)blockIdx.z * a.pstride;

    if (warp == 1) tc::alloc(&tmem_s, BN * ACC);
    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < kFStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&dfull, 1);
        fence_barrier_init();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = tmem_s;

    if (warp == 0) {
        if (lane == 0) {
            // weights of the first stages: they do not depend on the preceding kernel
            const int pre = S < kFStages ? S : kFStages;
            for (int k = 0; k < pre; ++k) {
                uint8_t *st = smem + (size_t)k * kStageBytes;
                mbar_arrive_expect_tx(&full[k], kStageBytes);
                const int x = (k0 + k) * kFBK * 2;
                tma_load_2d(st + 2 * kFPartA, &sg.bh, x, n0, &full[k]);
                tma_load_2d(st + 2 * kFPartA + kPartB, &sg.bl, x, n0, &full[k]);
            }
            pdl_wait();
            for (int k = 0; k < S && !abort_flag; ++k) {
                const int s = k % kFStages;
                uint8_t *st = smem + (size_t)s * kStageBytes;
                const int x = (k0 + k) * kFBK * 2;   // byte column of this K step
                if (k >= kFStages) {
                    if (!gwait(&empty[s], (uint32_t)((k / kFStages) - 1) & 1, &abort_flag)) break;
                    mbar_arrive_expect_tx(&full[s], kStageBytes);
                    tma_load_2d(st + 2 * kFPartA, &sg.bh, x, n0, &full[s]);
                    tma_load_2d(st + 2 * kFPartA + kPartB, &sg.bl, x, n0, &full[s]);
                }
                tma_load_2d(st, &tah, x, m0, &full[s]);
                tma_load_2d(st + kFPartA, &tal, x, m0, &full[s]);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_bf16(kFBM, BN);
            for (int k = 0; k < S && !abort_flag; ++k) {
                const int s = k % kFStages;
                if (!gwait(&full[s], (uint32_t)(k / kFStages) & 1, &abort_flag)) break;
                tc::fence_after();
                const uint32_t ah = smem_addr(smem + (size_t)s * kStageBytes), al = ah + kFPartA;
                const uint32_t bh = ah + 2 * kFPartA, bl = bh + kPartB;
#pragma unroll
                for (int kk = 0; kk < kFBK / 16; ++kk) {   // 16 bf16 = 32 bytes per MMA
                    const uint32_t o = kk * 32;
                    // MMA i of the tile goes to accumulator i % ACC (independent chains)
                    const int i0 = 3 * (k * (kFBK / 16) + kk);
                    const uint32_t d0 = tmem + (uint32_t)((i0 % ACC) * BN);
                    const uint32_t d1 = tmem + (uint32_t)(((i0 + 1) % ACC) * BN);
                    const uint32_t d2 = tmem + (uint32_t)(((i0 + 2) % ACC) * BN);
                    tc::mma_bf16_ss(d0, sw128_desc(ah + o), sw128_desc(bh + o), idesc, i0 >= ACC);
                    tc::mma_bf16_ss(d1, sw128_desc(al + o), sw128_desc(bh + o), idesc, i0 + 1 >= ACC);
                    tc::mma_bf16_ss(d2, sw128_desc(ah + o), sw128_desc(bl + o), idesc, i0 + 2 >= ACC);
                }
                tc::commit(&empty[s]);
            }
            tc::commit(&dfull);
        }
        __syncwarp();
    } else {
        // warps 2-5: TMEM lanes 32 (warp % 4) .. +31 = tile rows; the ACC
        // accumulators added in order
        const int q = warp & 3;
        const int row = m0 + 32 * q + lane;
        const bool ok = gwait(&dfull, 0, &abort_flag);
        tc::fence_after();
        if constexpr (EPI) {
            static_assert(BN == 64, "the decode epilogue takes one 64-wide head per tile");
            if (ok) {
                float h[64];
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t v[32];
                    tc::ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(32 * c), v);
                    tc::wait_ld();
#pragma unroll
                    for (int x = 1; x < ACC; ++x) {
                        uint32_t w[32];
                        tc::ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(x * BN + 32 * c), w);
                        tc::wait_ld();
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(w[j]));
                    }
#pragma unroll
                    for (int j = 0; j < 32; ++j) h[32 * c + j] = __uint_as_float(v[j]);
                }
                if (row < a.M) qkvg_head(a.epi, si, n0 / 64, row, h, sg.y + (size_t)row * sg.ldy + n0);
            }
        } else if (ok) {
            const bool vec = (sg.ldy & 3) == 0 && (reinterpret_cast<uintptr_t>(yout) & 15) == 0;
            float *yr = yout + (size_t)min(row, a.M - 1) * sg.ldy + n0;
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t v[32];
                tc::ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(32 * c), v);
                tc::wait_ld();
#pragma unroll
                for (int x = 1; x < ACC; ++x) {
                    uint32_t w[32];
                    tc::ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(x * BN + 32 * c), w);
                    tc::wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(w[j]));
                }
                if (row < a.M) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        const int col = 32 * c + j;
                        if (vec && n0 + col + 3 < sg.N) {
                            *reinterpret_cast<float4 *>(yr + col) = make_float4(
                                __uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                                __uint_as_float(v[j + 3]));
                        } else {
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                if (n0 + col + e < sg.N) yr[col + e] = __uint_as_float(v[j + e]);
                        }
                    }
                }
            }
        }
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == 1) tc::dealloc(tmem, BN * ACC);
}

constexpr int kDecodeAcc = 1;     // accumulators per 64-wide tile
constexpr int kPartWidth = 64;     // tile width of K-split launches (measured: 64 < 128 < 256)

struct Lut16 {
    float v[16];
};

// W'[r][k] split to bf16 hi [out][padded] and lo (the next out * padded values).
__global__ void gemm_f32_prepare_kernel(const uint8_t *__restrict__ packed, const uint16_t *__restrict__ norms,
                                        int out, int groups, int group, int sbits, int rowbytes, int padded, Lut16 lut,
                                        uint16_t *__restrict__ hi, uint16_t *__restrict__ lo) {
    const long long total = (long long)out * padded;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / padded), e = (int)(i % padded);
        const uint8_t *rp = packed + (size_t)r * rowbytes;
        const int idx = sbits == 4 ? ((rp[e >> 1] >> (4 * (e & 1))) & 15) : ((rp[e >> 2] >> (2 * (e & 3))) & 3);
        const float w = __fmul_rn(half_bits_to_float(norms[(size_t)r * groups + e / group]), lut.v[idx]);
        const __nv_bfloat16 h = __float2bfloat16_rn(w);
        hi[i] = __bfloat16_as_ushort(h);
        lo[i] = __bfloat16_as_ushort(__float2bfloat16_rn(__fsub_rn(w, __bfloat162float(h))));
    }
}

// rot[n] -> bf16 hi[n], lo[n]
__global__ void split_bf16_kernel(const float *__restrict__ x, long long n, uint16_t *__restrict__ hi,
                                  uint16_t *__restrict__ lo) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float v = x[i];
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        hi[i] = __bfloat16_as_ushort(h);
        lo[i] = __bfloat16_as_ushort(__float2bfloat16_rn(__fsub_rn(v, __bfloat162float(h))));
    }
}

}  // namespace

size_t gemm_w8_bytes(int out, int padded) { return (size_t)out * padded; }
size_t gemm_ns_count(int out, int groups) { return (size_t)groups * ((out + kBN - 1) / kBN * kBN); }

bool gemm_prepare(const uint8_t *packed, const uint16_t *norms, int out, int groups, int group, int bits, int rowbytes,
                  int padded, const uint32_t ctab[4], float cs, int8_t *w8, float *nsT, cudaStream_t st) {
    uint4 t;
    std::memcpy(&t, ctab, 16);
    const int nstride = (out + kBN - 1) / kBN * kBN;
    gemm_prepare_kernel<<<148 * 8, 256, 0, st>>>(packed, norms, out, groups, group, bits, rowbytes, padded, t, cs,
                                                nstride, w8, nsT);
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool gemm_supported(int bits, int group, int padded) {
    return (bits == 2 || bits == 4) && group == kBK && padded % kBK == 0 && padded >= kBK;
}

bool launch_gemm_i8(const int8_t *q, const float *xs, int M, const int8_t *w8, const float *nsT, int N, int padded,
                    int groups, float *y, int ldy, cudaStream_t st) {
    return launch_gemm_i8_multi(q, xs, M, w8, nsT, N, padded, groups, &y, 1, ldy, st);
}

bool launch_gemm_i8_multi(const int8_t *q, const float *xs, int M, const int8_t *w8, const float *nsT, int N,
                          int padded, int groups, float *const *dsts, int ndst, int ldy, cudaStream_t st) {
    if (M <= 0 || N <= 0) return true;
    if (ndst < 1 || ndst > kMaxGemmOutputs) {
        set_error("prefill GEMM: 1 to 8 output buffers");
        return false;
    }
    if (padded % kBK || groups * kBK != padded) {
        set_error("prefill GEMM requires group size 128");
        return false;
    }
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(w8)) & 15) {
        set_error("prefill GEMM operands must be 16-byte aligned");
        return false;
    }
    CUtensorMap ta, tb;
    if (!make_map(&ta, q, M, padded, kBM) || !make_map(&tb, w8, N, padded, kBN)) return false;
    GemmArgs args{};
    args.M = M;
    args.N = N;
    args.groups = groups;
    args.ldy = ldy;
    args.xs = xs;
    args.nsT = nsT;
    args.nstride = (N + kBN - 1) / kBN * kBN;
    args.y = nullptr;
    args.one = 1.0f;
    for (int i = 0; i < ndst; ++i) args.dst[i] = dsts[i];
    args.ndst = ndst;
    static bool configured[64] = {};
    int dev = 0;
    NB_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        NB_CUDA_TRY(cudaFuncSetAttribute(cq_gemm_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    cudaLaunchConfig_t cfg{};
    static int sms[64] = {};
    if (dev >= 0 && dev < 64 && !sms[dev]) NB_CUDA_TRY(cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev));
    const int nsm = dev >= 0 && dev < 64 && sms[dev] > 0 ? sms[dev] : 148;
    args.mtiles = (M + kBM - 1) / kBM;
    args.tiles = args.mtiles * ((N + kBN - 1) / kBN);
    cfg.gridDim = dim3(std::min(args.tiles, nsm));   // one persistent CTA per SM
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NB_CUDA_TRY(cudaLaunchKernelEx(&cfg, cq_gemm_i8_kernel, ta, tb, args));
    return true;
}

bool gemm_f32_supported(int storage_bits, int padded) {
    return (storage_bits == 2 || storage_bits == 4) && padded % kFBK == 0 && padded >= kFBK;
}

size_t gemm_f32_weight_elems(int out, int padded) { return 2 * (size_t)out * padded; }

bool gemm_f32_prepare(const uint8_t *packed, const uint16_t *norms, int out, int groups, int group, int storage_bits,
                      int rowbytes, int padded, const float lut[16], uint16_t *w_hilo, cudaStream_t st) {
    Lut16 l;
    std::memcpy(l.v, lut, sizeof(l.v));
    gemm_f32_prepare_kernel<<<148 * 8, 256, 0, st>>>(packed, norms, out, groups, group, storage_bits, rowbytes, padded,
                                                    l, w_hilo, w_hilo + (size_t)out * padded);
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_split_bf16(const float *x, long long n, uint16_t *hilo, cudaStream_t st) {
    if (n <= 0) return true;
    split_bf16_kernel<<<148 * 4, 256, 0, st>>>(x, n, hilo, hilo + n);
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_gemm_f32x3_multi(const uint16_t *a_hilo, int M, int padded, const F32Out *outs, int count,
                             cudaStream_t st, const QkvgEpilogue *epi, bool *epi_done, const KParts *kp) {
    if (epi_done) *epi_done = false;
    if (kp && kp->parts) *kp->parts = 1;
    if (M <= 0 || count <= 0) return true;
    if (padded % kFBK) {
        set_error("FP32 prefill GEMM requires the padded width to be a multiple of 64");
        return false;
    }
    if (count > kF32MaxSegs) {
        for (int i = 0; i < count; i += kF32MaxSegs)
            if (!launch_gemm_f32x3_multi(a_hilo, M, padded, outs + i, std::min(kF32MaxSegs, count - i), st)) return false;
        return true;
    }
    int dev = 0, sms = 148;
    NB_CUDA_TRY(cudaGetDevice(&dev));
    static int sm_count[64] = {};
    if (dev >= 0 && dev < 64) {
        if (!sm_count[dev]) NB_CUDA_TRY(cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev));
        sms = sm_count[dev];
    }
    const int mtiles = (M + kFBM - 1) / kFBM;
    auto tiles_of = [&](int bn) {
        int t = 0;
        for (int i = 0; i < count; ++i) t += (outs[i].N + bn - 1) / bn;
        return t;
    };
    // 128 x 256 tiles where they fill the machine; 64-wide tiles (four times
    // the CTAs) where they do not
    const bool narrow = (long long)mtiles * tiles_of(256) < 2LL * sms;
    // the decode epilogue: four segments (q, k, v, gate) of whole 64-wide heads
    const bool with_epi = narrow && epi && epi->active && count == 4 && epi->hd == 64;
    // K split into parts where the caller adds partial outputs: each CTA then
    // issues a fraction of the tile's MMAs (a 128-row MMA costs about the
    // same whatever its width up to 256, so one CTA's chain of MMAs bounds a
    // decode-sized launch), as many parts as keep the grid within one CTA per SM
    const int steps = padded / kFBK;
    int parts = 1;
    if (narrow && !with_epi && kp && kp->max_parts > 1 && kp->pstride > 0) {
        const long long grid = (long long)mtiles * tiles_of(kPartWidth);
        while (2 * parts <= kp->max_parts && 2 * parts <= kMaxKParts && steps % (2 * parts) == 0 &&
               grid * 2 * parts <= sms)
            parts *= 2;
    }
    const int BN = parts > 1 ? kPartWidth : narrow ? 64 : 256;
    const size_t an = (size_t)M * padded;
    CUtensorMap tah, tal;
    // bf16 rows seen as bytes: 2 * padded bytes per row, 128-byte (64-element) boxes
    if (!make_map(&tah, a_hilo, M, 2 * padded, kFBM) || !make_map(&tal, a_hilo + an, M, 2 * padded, kFBM)) return false;
    GemmF32Args args{};
    args.nseg = count;
    args.M = M;
    args.ksteps = steps / parts;
    args.pstride = parts > 1 ? kp->pstride : 0;
    int tiles = 0;
    for (int i = 0; i < count; ++i) {
        const F32Out &o = outs[i];
        const size_t wn = (size_t)o.N * padded;
        if (!make_map(&args.seg[i].bh, o.w_hilo, o.N, 2 * padded, BN) ||
            !make_map(&args.seg[i].bl, o.w_hilo + wn, o.N, 2 * padded, BN))
            return false;
        args.seg[i].y = o.y;
        args.seg[i].N = o.N;
        args.seg[i].ldy = o.ldy;
        args.seg[i].tile0 = tiles;
        tiles += (o.N + BN - 1) / BN;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(mtiles, tiles, parts);
    cfg.blockDim = dim3(kFThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    static bool configured[7][64] = {};
    auto launch = [&](auto kernel, size_t smem, int which) -> bool {
        if (dev < 0 || dev >= 64 || !configured[which][dev]) {
            NB_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            if (dev >= 0 && dev < 64) configured[which][dev] = true;
        }
        cfg.dynamicSmemBytes = smem;
        NB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, tah, tal, args));
        return true;
    };
    if (parts > 1) {
        if (kp->parts) *kp->parts = parts;
        return launch(cq_gemm_f32x3_kernel<kPartWidth, 2, 1, false>, FTile<kPartWidth, 2>::kSmem, 3);
    }
    if (!narrow) return launch(cq_gemm_f32x3_kernel<256, 2, 1, false>, FTile<256, 2>::kSmem, 0);
    if (with_epi) {
        args.epi = *epi;
        if (epi_done) *epi_done = true;
    }
    // one CTA per SM with the deep pipeline while the grid fits the machine
    if ((long long)mtiles * tiles <= sms)
        return with_epi ? launch(cq_gemm_f32x3_kernel<64, 4, kDecodeAcc, true>, FTile<64, 4>::kSmem, 4)
                        : launch(cq_gemm_f32x3_kernel<64, 4, kDecodeAcc, false>, FTile<64, 4>::kSmem, 1);
    return with_epi ? launch(cq_gemm_f32x3_kernel<64, 2, kDecodeAcc, true>, FTile<64, 2>::kSmem, 5)
                    : launch(cq_gemm_f32x3_kernel<64, 2, kDecodeAcc, false>, FTile<64, 2>::kSmem, 2);
}

bool launch_gemm_f32x3(const uint16_t *a_hilo, int M, const uint16_t *w_hilo, int N, int padded, float *y, int ldy,
                       cudaStream_t st) {
    const F32Out o{w_hilo, N, y, ldy};
    return launch_gemm_f32x3_multi(a_hilo, M, padded, &o, 1, st);
}

}  // namespace nb200
