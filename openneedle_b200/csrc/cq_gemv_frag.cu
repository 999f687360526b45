// SDOT (int8) CQ2/CQ4 GEMV for small activation batches (M <= 16): weights
// as the 16-row A operand of mma.sync.m16n8k32 (s8 x s8 -> s32), activations
// as the 8-column B operand.
//
// A warp owns a tile of 16 consecutive weight rows and walks its groups in
// order.  The matrix is stored in fragment order (built once at create time,
// see frag_layout in cq_gemv.cuh): the 16 rows x one group form one contiguous
// block in which lane (g, t) finds, word by word, exactly the packed indices
// of its A fragments (rows g and g+8, k = 4t..4t+3 and 16+4t..16+4t+3 of every
// 32-wide K step).  A warp therefore loads 32 contiguous bytes per lane per
// group (one coalesced 1 KB block for CQ4 / group 128), decodes them in
// registers to int8 centroids (byte permutes over the 16- or 4-entry table)
// and issues G/32 MMAs per group, twice with a sign-split codebook (positive
// and negative halves into separate accumulators, subtracted afterwards).
//
// The C fragment after a group is the reference's int32 group dot d[m, r, g]
// (needle2/csrc/sdot.cpp:108-137) for rows g, g+8 and activations 2t, 2t+1, so
// each lane adds (float(d) * (half(norm) * cs)) * xs to its own rows' running
// sums in group order (sdot.cpp:142-149): bit-identical to the reference, no
// cross-lane reduction.  Group blocks stream through a register ring PF groups
// ahead of the decode, across tile boundaries.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "cq_gemv.cuh"
#include "sm100_async.cuh"

namespace nb200 {
namespace {

constexpr int kFragMaxSmem = 225 * 1024;

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

template <int K>
__device__ __forceinline__ uint32_t shr_mul(uint32_t x) {
    return __umulhi(x, 1u << (32 - K));
}

// CQ4 word -> int8 centroids of nibbles 0..3 (lo) and 4..7 (hi).
__device__ __forceinline__ void dec4(uint32_t w, const uint32_t (&t)[4], uint32_t &lo, uint32_t &hi) {
    const uint32_t sel = w & 0x77777777u;
    const uint32_t comb = (shr_mul<1>(w) & 0x44444444u) | 0x32103210u;
    lo = prmt(prmt(t[0], t[1], sel), prmt(t[2], t[3], sel), comb);
    const uint32_t sel2 = shr_mul<16>(sel), comb2 = shr_mul<16>(comb);
    hi = prmt(prmt(t[0], t[1], sel2), prmt(t[2], t[3], sel2), comb2);
}

// CQ4 sign-split decode: |centroid| where the index is 0-7 and centroid where
// it is 8-15, zero elsewhere (a selector nibble with bit 3 set returns the sign
// of a non-negative byte, i.e. 0).
__device__ __forceinline__ void dec4_split(uint32_t w, const uint32_t (&nt)[2], const uint32_t (&pt)[2],
                                           uint32_t &nlo, uint32_t &nhi, uint32_t &plo, uint32_t &phi) {
    const uint32_t wx = w ^ 0x88888888u;
    nlo = prmt(nt[0], nt[1], w);
    nhi = prmt(nt[0], nt[1], shr_mul<16>(w));
    plo = prmt(pt[0], pt[1], wx);
    phi = prmt(pt[0], pt[1], shr_mul<16>(wx));
}

// CQ2 word (16 crumbs) -> centroids of crumbs 0,2,4,6 | 8..14 even | 1,3,5,7 |
// 9..15 odd; the fragment layout puts K step 2p in the first two and 2p+1 in
// the last two.
__device__ __forceinline__ void dec2(uint32_t w, uint32_t t, uint32_t (&r)[4]) {
    const uint32_t e = w & 0x33333333u, o = shr_mul<2>(w) & 0x33333333u;
    r[0] = prmt(t, t, e);
    r[1] = prmt(t, t, shr_mul<16>(e));
    r[2] = prmt(t, t, o);
    r[3] = prmt(t, t, shr_mul<16>(o));
}

// First K step of a group: D = A x B (zero accumulator input).
__device__ __forceinline__ void mma_s8_first(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int BITS, int G>
struct FragGeo {
    static constexpr int KK = G / 32;                     // K steps per group
    static constexpr int LW = BITS == 4 ? 2 * KK : KK;    // 32-bit words per lane per group
    static constexpr int LB = 4 * LW;                     // bytes per lane per group
    static constexpr int SLOT = 32 * (LB + 4);            // one ring slot: the lanes' words, then their norm pairs
    // ring depth: about 6 KB of weights per warp (deeper rings measured no faster)
    static constexpr int PF = 6144 / (32 * LB) < 4 ? 4 : (6144 / (32 * LB) > 16 ? 16 : 6144 / (32 * LB));
};

// Shared memory: activations [NB][padded + 32] (each 32-wide K step stored in
// B-fragment order: lane t's k = 4t..4t+3, 16+4t..16+4t+3 adjacent), the
// scales [NB][groups], then per warp a ring of pf slots.
__host__ __device__ inline size_t frag_smem(int padded, int groups, int nb, int slot_bytes, int pf, int warps) {
    const size_t head = ((size_t)nb * (padded + 32) + 4 * (size_t)nb * groups + 127) / 128 * 128;
    return head + (size_t)warps * pf * slot_bytes;
}

// MT: exact activation rows for MT <= 4, an upper bound (rows in b.M) for 8 / 16.
// PF: ring slots per warp.  NT: threads per CTA.  DBG: also write the int32
// group dots to b.partials.
template <int BITS, int G, int MT, bool SPLIT, int PF, int NT, bool DBG, bool PAIR>
__global__ void __launch_bounds__(NT, 1)
    cq_gemv_frag_kernel(const __grid_constant__ GemvBatch b, const int total_tiles) {
    static_assert(!PAIR || PF % 2 == 0, "paired groups need an even ring");
    constexpr int kFragThreads = NT, kFragWarps = NT / 32;
    using Geo = FragGeo<BITS, G>;
    constexpr int KK = Geo::KK, LW = Geo::LW, LB = Geo::LB, SLOT = Geo::SLOT;
    constexpr int NB = MT <= 8 ? 8 : 16;
    constexpr int NP = NB / 8;   // B passes per K step
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int tile_base[kGemvMaxMats + 1];

    const int gpr = b.groups, M = MT <= 4 ? MT : b.M;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int astride = b.padded + 32;
    uint8_t *act = smem;
    float *xs_s = reinterpret_cast<float *>(smem + (size_t)NB * astride);
    const size_t head = ((size_t)NB * astride + 4 * (size_t)NB * gpr + 127) / 128 * 128;
    // slot s: lane l's LB bytes at s*SLOT + l*LB (each lane copies and reads its own bytes; measured faster
    // than a bank-conflict-free chunk-major order), its norm pair at s*SLOT + 32*LB + 4*l
    uint8_t *ring = smem + head + (size_t)warp * PF * SLOT;

    const int s0 = (int)((long long)total_tiles * blockIdx.x / gridDim.x);
    const int s1 = (int)((long long)total_tiles * (blockIdx.x + 1) / gridDim.x);

    pdl_launch_dependents();
    if (tid == 0) {
        int acc = 0;
        for (int j = 0; j < b.nmat; ++j) {
            tile_base[j] = acc;
            acc += (b.mat[j].out + 15) / 16;
        }
        tile_base[b.nmat] = acc;
    }
    __syncthreads();

    // load cursor: tiles s0 + warp, s0 + warp + kFragWarps, ...; one commit group per group block
    int ltile = s0 + warp, lj = 0, lmat = 0, lslot = 0;
    const uint8_t *lw = nullptr;
    const uint32_t *ln = nullptr;
    auto lseek = [&]() {
        if (ltile < s1) {
            while (lmat + 1 < b.nmat && ltile >= tile_base[lmat + 1]) ++lmat;
            const size_t lt = (size_t)(ltile - tile_base[lmat]);
            lw = b.mat[lmat].frag + (lt * gpr) * 32 * LB + (size_t)lane * LB;
            ln = reinterpret_cast<const uint32_t *>(b.mat[lmat].normsF) + lt * gpr * 8 + g;
        }
    };
    // one commit group per group block, or per two consecutive blocks of a tile
    // (PAIR: the row's group count is even) in two consecutive slots
    constexpr int GB = PAIR ? 2 : 1;        // group blocks per commit group
    constexpr int AHEAD = PF / GB - 1;      // commit groups in flight ahead of the consumer
    auto issue = [&]() {
        if (ltile < s1) {
#pragma unroll
            for (int h = 0; h < GB; ++h) {
                uint8_t *dst = ring + (size_t)(lslot + h) * SLOT;
                if constexpr (LB >= 16) {
#pragma unroll
                    for (int c = 0; c < LB / 16; ++c)
                        cp_async<16>(dst + lane * LB + 16 * c, lw + h * 32 * LB + 16 * c);
                } else {
                    cp_async<LB>(dst + lane * LB, lw + h * 32 * LB);
                }
                cp_async<4>(dst + 32 * LB + 4 * lane, ln + 8 * h);
            }
            lw += GB * 32 * LB;
            ln += 8 * GB;
            lj += GB;
            if (lj == gpr) {
                lj = 0;
                ltile += kFragWarps;
                lseek();
            }
        }
        cp_async_commit();
        lslot = lslot + GB == PF ? 0 : lslot + GB;
    };
    lseek();
    // the weights do not depend on the preceding kernel: start streaming them first
    for (int p = 0; p < AHEAD; ++p) issue();

    pdl_wait();
    // one thread per 32-wide K step of one activation row: the natural element
    // words w0..w7 (w_i = elements 4i..4i+3) go out as w0 w4 w1 w5 w2 w6 w3 w7,
    // so lane t finds k = 4t..4t+3 and 16+4t..16+4t+3 in one 8-byte load
    for (int i = tid; i < NB * (b.padded / 32); i += kFragThreads) {
        const int n = i / (b.padded / 32), c = i % (b.padded / 32);
        uint32_t w[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
        if (n < M) {
            const uint4 *src = reinterpret_cast<const uint4 *>(b.q + (size_t)n * b.padded + (size_t)c * 32);
            const uint4 u0 = src[0], u1 = src[1];
            if (BITS == 4) {
                w[0] = u0.x; w[1] = u0.y; w[2] = u0.z; w[3] = u0.w;
                w[4] = u1.x; w[5] = u1.y; w[6] = u1.z; w[7] = u1.w;
            } else {
                // CQ2 activations are stored per 16 elements as evens then odds
                w[0] = prmt(u0.x, u0.z, 0x5140u); w[1] = prmt(u0.x, u0.z, 0x7362u);
                w[2] = prmt(u0.y, u0.w, 0x5140u); w[3] = prmt(u0.y, u0.w, 0x7362u);
                w[4] = prmt(u1.x, u1.z, 0x5140u); w[5] = prmt(u1.x, u1.z, 0x7362u);
                w[6] = prmt(u1.y, u1.w, 0x5140u); w[7] = prmt(u1.y, u1.w, 0x7362u);
            }
        }
        uint4 *dst = reinterpret_cast<uint4 *>(act + (size_t)n * astride + (size_t)c * 32);
        dst[0] = make_uint4(w[0], w[4], w[1], w[5]);
        dst[1] = make_uint4(w[2], w[6], w[3], w[7]);
    }
    for (int i = tid; i < NB * gpr; i += kFragThreads) xs_s[i] = i < M * gpr ? b.xs[i] : 0.f;
    __syncthreads();

    const uint32_t ctab[4] = {b.ctab[0], b.ctab[1], b.ctab[2], b.ctab[3]};
    const uint32_t ntab[2] = {b.ntab[0], b.ntab[1]}, ptab[2] = {b.ptab[0], b.ptab[1]};
    const float cs = b.cs;

    // consume side: the warp's tiles in order, each group by group
    const uint8_t *abase = act + (size_t)g * astride + t * 8;
    int cslot = 0, cmat = 0;
    for (int ctile = s0 + warp; ctile < s1; ctile += kFragWarps) {
        while (cmat + 1 < b.nmat && ctile >= tile_base[cmat + 1]) ++cmat;
        const int row0 = (ctile - tile_base[cmat]) * 16;
        float acc[NP][4];
#pragma unroll
        for (int q = 0; q < NP; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
        const uint8_t *ab = abase;
        // one group: its block from ring slot `slot`, activations at `ab`
        auto group = [&](const uint8_t *slot, int cj, const uint8_t *ab) {
            uint32_t wv[LW];
            if constexpr (LB >= 16) {
    #pragma unroll
                for (int c = 0; c < LB / 16; ++c) {
                    const uint4 u = *reinterpret_cast<const uint4 *>(slot + lane * LB + 16 * c);
                    wv[4 * c] = u.x; wv[4 * c + 1] = u.y; wv[4 * c + 2] = u.z; wv[4 * c + 3] = u.w;
                }
            } else {
                const uint2 u = *reinterpret_cast<const uint2 *>(slot + lane * LB);
                wv[0] = u.x; wv[1] = u.y;
            }
            const uint32_t nv = *reinterpret_cast<const uint32_t *>(slot + 32 * LB + 4 * lane);
            int cp[NP][4], cn[SPLIT ? NP : 1][4];
            if constexpr (BITS == 4) {
    #pragma unroll
                for (int s = 0; s < KK; ++s) {
                    uint32_t a0, a1, a2, a3, n0 = 0, n1 = 0, n2 = 0, n3 = 0;
                    if constexpr (SPLIT) {
                        dec4_split(wv[2 * s], ntab, ptab, n0, n2, a0, a2);
                        dec4_split(wv[2 * s + 1], ntab, ptab, n1, n3, a1, a3);
                    } else {
                        dec4(wv[2 * s], ctab, a0, a2);
                        dec4(wv[2 * s + 1], ctab, a1, a3);
                    }
    #pragma unroll
                    for (int q = 0; q < NP; ++q) {
                        const uint2 bx = *reinterpret_cast<const uint2 *>(ab + (size_t)q * 8 * astride + s * 32);
                        if (s == 0) {
                            mma_s8_first(cp[q], a0, a1, a2, a3, bx.x, bx.y);
                            if constexpr (SPLIT) mma_s8_first(cn[q], n0, n1, n2, n3, bx.x, bx.y);
                        } else {
                            mma_s8(cp[q], a0, a1, a2, a3, bx.x, bx.y);
                            if constexpr (SPLIT) mma_s8(cn[q], n0, n1, n2, n3, bx.x, bx.y);
                        }
                    }
                }
            } else {
    #pragma unroll
                for (int pp = 0; pp < KK / 2; ++pp) {
                    uint32_t r0[4], r1[4];
                    dec2(wv[2 * pp], ctab[0], r0);
                    dec2(wv[2 * pp + 1], ctab[0], r1);
    #pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int s = 2 * pp + h;
    #pragma unroll
                        for (int q = 0; q < NP; ++q) {
                            const uint2 bx = *reinterpret_cast<const uint2 *>(ab + (size_t)q * 8 * astride + s * 32);
                            if (s == 0)
                                mma_s8_first(cp[q], r0[2 * h], r1[2 * h], r0[2 * h + 1], r1[2 * h + 1], bx.x, bx.y);
                            else
                                mma_s8(cp[q], r0[2 * h], r1[2 * h], r0[2 * h + 1], r1[2 * h + 1], bx.x, bx.y);
                        }
                    }
                }
            }
            // epilogue of group cj: rows g (c0, c1) and g + 8 (c2, c3), activations 2t, 2t + 1 (+8 per pass)
            const float nsa = __fmul_rn(half_bits_to_float((uint16_t)(nv & 0xffffu)), cs);
            const float nsb = __fmul_rn(half_bits_to_float((uint16_t)(nv >> 16)), cs);
#pragma unroll
            for (int q = 0; q < NP; ++q) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int a = 8 * q + 2 * t + (e & 1);
                    if (MT <= 4 ? a < MT : a < M) {
                        int d = cp[q][e];
                        if constexpr (SPLIT) d -= cn[q][e];
                        const float ns = e < 2 ? nsa : nsb;
                        acc[q][e] = __fadd_rn(acc[q][e], __fmul_rn(__fmul_rn(__int2float_rn(d), ns), xs_s[a * gpr + cj]));
                        if constexpr (DBG) {
                            const int row = row0 + g + (e < 2 ? 0 : 8);
                            if (row < b.mat[cmat].out) b.partials[((size_t)a * b.mat[cmat].out + row) * gpr + cj] = d;
                        }
                    }
                }
            }
                };
        for (int cj = 0; cj < gpr; cj += GB, ab += GB * KK * 32) {
            issue();                        // AHEAD commit groups ahead (their slots were consumed last iteration)
            cp_async_wait<AHEAD>();         // this commit group's blocks have landed
#pragma unroll
            for (int h = 0; h < GB; ++h) group(ring + (size_t)(cslot + h) * SLOT, cj + h, ab + h * KK * 32);
            cslot = cslot + GB == PF ? 0 : cslot + GB;
        }
        const GemvMatrix &mat = b.mat[cmat];
#pragma unroll
        for (int q = 0; q < NP; ++q) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int a = 8 * q + 2 * t + (e & 1);
                const int row = row0 + g + (e < 2 ? 0 : 8);
                if ((MT <= 4 ? a < MT : a < M) && row < mat.out) mat.y[(size_t)a * mat.out + row] = acc[q][e];
            }
        }
    }
    cp_async_wait<0>();
}

template <int BITS, int G, int MT, bool SPLIT, int PF, int NT, bool DBG = false, bool PAIR = false>
bool launch_frag_pf(const GemvBatch &b, size_t smem, cudaStream_t st) {
    auto kernel = cq_gemv_frag_kernel<BITS, G, MT, SPLIT, PF, NT, DBG, PAIR>;
    static bool configured[64] = {};
    static int sms[64] = {};
    int dev = 0;
    NB_CUDA_TRY(cudaGetDevice(&dev));
    const bool cached = dev >= 0 && dev < 64;
    if (!cached || !configured[dev]) {
        NB_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFragMaxSmem));
        int n = 148;
        NB_CUDA_TRY(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        if (cached) {
            configured[dev] = true;
            sms[dev] = n;
        }
    }
    constexpr int warps = NT / 32;
    int total = 0;
    for (int j = 0; j < b.nmat; ++j) total += (b.mat[j].out + 15) / 16;
    const int grid = std::max(1, std::min((total + warps - 1) / warps, cached ? sms[dev] : 148));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, b, total));
    return true;
}

// Warps per CTA from the work: every 16-row tile is one warp's, so a launch
// with few tiles uses 8 warps per CTA (spreading them over all SMs, two CTAs per
// SM), a large one 32 warps with a 4-slot ring (measured fastest for one to
// four activation rows and groups up to 128; 64 registers per thread), else 16
// warps with the full ring, or half of it when shared memory is short.  With an
// even group count (and ring), copies go out two group blocks at a time.
template <int BITS, int G, int MT, bool SPLIT>
bool launch_frag(const GemvBatch &b, cudaStream_t st) {
    using Geo = FragGeo<BITS, G>;
    const int nb = MT <= 8 ? 8 : 16;
    if (b.partials) {   // debug export of the int32 group dots: 16 warps
        const size_t full = frag_smem(b.padded, b.groups, nb, Geo::SLOT, Geo::PF, 16);
        if (full <= (size_t)kFragMaxSmem) return launch_frag_pf<BITS, G, MT, SPLIT, Geo::PF, 512, true>(b, full, st);
        return launch_frag_pf<BITS, G, MT, SPLIT, Geo::PF / 2, 512, true>(
            b, frag_smem(b.padded, b.groups, nb, Geo::SLOT, Geo::PF / 2, 16), st);
    }
    int tiles = 0;
    for (int j = 0; j < b.nmat; ++j) tiles += (b.mat[j].out + 15) / 16;
    const bool pair = b.groups % 2 == 0;   // two group blocks per copy batch
    if (tiles <= 148 * 8) {
        const size_t narrow = frag_smem(b.padded, b.groups, nb, Geo::SLOT, Geo::PF, 8);
        if (narrow <= (size_t)kFragMaxSmem) {
            if constexpr (Geo::PF % 2 == 0)
                if (pair) return launch_frag_pf<BITS, G, MT, SPLIT, Geo::PF, 256, false, true>(b, narrow, st);
            return launch_frag_pf<BITS, G, MT, SPLIT, Geo::PF, 256>(b, narrow, st);
        }
    }
    if constexpr (MT <= 4 && G <= 128) {
        const size_t wide = frag_smem(b.padded, b.groups, nb, Geo::SLOT, 4, 32);
        if (tiles > 148 * 16 && wide <= (size_t)kFragMaxSmem) {
            // an even group count: two group blocks per copy batch
            if (pair) return launch_frag_pf<BITS, G, MT, SPLIT, 4, 1024, false, true>(b, wide, st);
            return launch_frag_pf<BITS, G, MT, SPLIT, 4, 1024>(b, wide, st);
        }
    }
    const size_t full = frag_smem(b.padded, b.groups, nb, Geo::SLOT, Geo::PF, 16);
    if (full <= (size_t)kFragMaxSmem) {
        if constexpr (Geo::PF % 2 == 0)
            if (pair) return launch_frag_pf<BITS, G, MT, SPLIT, Geo::PF, 512, false, true>(b, full, st);
        return launch_frag_pf<BITS, G, MT, SPLIT, Geo::PF, 512>(b, full, st);
    }
    return launch_frag_pf<BITS, G, MT, SPLIT, Geo::PF / 2, 512>(
        b, frag_smem(b.padded, b.groups, nb, Geo::SLOT, Geo::PF / 2, 16), st);
}

template <int BITS, int G, bool SPLIT>
bool launch_frag_m(const GemvBatch &b, cudaStream_t st) {
    switch (b.M) {
        case 1: return launch_frag<BITS, G, 1, SPLIT>(b, st);
        case 2: return launch_frag<BITS, G, 2, SPLIT>(b, st);
        case 3: return launch_frag<BITS, G, 3, SPLIT>(b, st);
        case 4: return launch_frag<BITS, G, 4, SPLIT>(b, st);
        default: return b.M <= 8 ? launch_frag<BITS, G, 8, SPLIT>(b, st) : launch_frag<BITS, G, 16, SPLIT>(b, st);
    }
}

template <int G>
bool launch_frag_cq4(const GemvBatch &b, cudaStream_t st) {
    return b.split ? launch_frag_m<4, G, true>(b, st) : launch_frag_m<4, G, false>(b, st);
}

int slot_bytes_of(int bits, int group) { return 32 * (group * bits / 16 + 4); }
int ring_depth_of(int bits, int group) {
    const int lb = group * bits / 16, pf = 6144 / (32 * lb);
    return pf < 4 ? 4 : (pf > 16 ? 16 : pf);
}

// One thread per 32-bit word of the fragment-order copy (see frag layout in
// cq_gemv.cuh), read from the row-major packed matrix on the device.
template <int BITS>
__global__ void frag_repack_kernel(const uint8_t *__restrict__ packed, const uint16_t *__restrict__ norms, int out,
                                   int groups, int G, int rowbytes, uint32_t *__restrict__ frag,
                                   uint16_t *__restrict__ normsF, long long total_words) {
    const int KK = G / 32, LW = BITS == 4 ? 2 * KK : KK;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total_words;
         i += (long long)gridDim.x * blockDim.x) {
        const long long blk = i / (32 * LW);
        const int rem = (int)(i % (32 * LW)), l = rem / LW, w = rem % LW;
        const int T = (int)(blk / groups), j = (int)(blk % groups), g = l >> 2, t = l & 3;
        const int h = w & 1, row = 16 * T + g + 8 * h;
        uint32_t word = 0;
        if (row < out) {
            const uint8_t *rp = packed + (size_t)row * rowbytes;
            if (BITS == 4) {
                const int s = w >> 1;
                for (int n = 0; n < 8; ++n) {
                    const int e = j * G + 32 * s + (n < 4 ? 4 * t + n : 12 + 4 * t + n);
                    const uint32_t byte = rp[e >> 1];
                    word |= ((e & 1) ? byte >> 4 : byte & 15u) << (4 * n);
                }
            } else {
                const int pp = w >> 1;
                for (int c = 0; c < 16; ++c) {
                    const int s = 2 * pp + (c & 1), ii = (c >> 1) & 3;
                    const int e = j * G + 32 * s + (c >= 8 ? 16 : 0) + 4 * t + ii;
                    word |= ((uint32_t)(rp[e >> 2] >> (2 * (e & 3))) & 3u) << (2 * c);
                }
            }
        }
        frag[i] = word;
        if (w == 0 && t == 0)
            for (int hh = 0; hh < 2; ++hh) {
                const int r = 16 * T + g + 8 * hh;
                normsF[((size_t)blk * 8 + g) * 2 + hh] = r < out ? norms[(size_t)r * groups + j] : (uint16_t)0;
            }
    }
}

}  // namespace

size_t frag_bytes(int out, int groups, int group, int bits) {
    return ((size_t)out + 15) / 16 * groups * 16 * (size_t)(group * bits / 8);
}
size_t frag_norm_count(int out, int groups) { return ((size_t)out + 15) / 16 * groups * 16; }

bool build_frag_layout(const uint8_t *packed, const uint16_t *norms, int out, int groups, int group, int bits,
                       int rowbytes, uint8_t *frag, uint16_t *normsF, cudaStream_t st) {
    const long long words = (long long)(frag_bytes(out, groups, group, bits) / 4);
    const int threads = 256;
    const int blocks = (int)std::min<long long>((words + threads - 1) / threads, 148 * 16);
    if (bits == 4)
        frag_repack_kernel<4><<<blocks, threads, 0, st>>>(packed, norms, out, groups, group, rowbytes,
                                                          reinterpret_cast<uint32_t *>(frag), normsF, words);
    else
        frag_repack_kernel<2><<<blocks, threads, 0, st>>>(packed, norms, out, groups, group, rowbytes,
                                                          reinterpret_cast<uint32_t *>(frag), normsF, words);
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

int gemv_frag_max_rows(int bits, int group, int groups) {
    if ((bits != 2 && bits != 4) || (group != 64 && group != 128 && group != 256) || groups < 1) return 0;
    for (int m : {16, 8})
        if (frag_smem(group * groups, groups, m <= 8 ? 8 : 16, slot_bytes_of(bits, group), ring_depth_of(bits, group) / 2,
                      16) <=
            (size_t)kFragMaxSmem)
            return m;
    return 0;
}

bool launch_gemv_frag(const GemvBatch &b, cudaStream_t st) {
    if (b.nmat < 1 || b.nmat > kGemvMaxMats || b.M < 1 || b.M > gemv_frag_max_rows(b.bits, b.group, b.groups) ||
        (b.partials && b.nmat != 1)) {
        set_error("int8 GEMV launch outside the fragment-order kernel's envelope");
        return false;
    }
    for (int j = 0; j < b.nmat; ++j)
        if (!b.mat[j].frag || !b.mat[j].normsF) {
            set_error("int8 GEMV launch without the fragment-order weight layout");
            return false;
        }
    if (b.bits == 4) {
        if (b.group == 64) return launch_frag_cq4<64>(b, st);
        if (b.group == 128) return launch_frag_cq4<128>(b, st);
        return launch_frag_cq4<256>(b, st);
    }
    if (b.group == 64) return launch_frag_m<2, 64, false>(b, st);
    if (b.group == 128) return launch_frag_m<2, 128, false>(b, st);
    return launch_frag_m<2, 256, false>(b, st);
}

}  // namespace nb200
