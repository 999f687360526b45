// Persistent CQ2/CQ4 GEMV for B200 (sm_100a), FP32 and SDOT (int8) modes.
//
// One CTA per SM streams a balanced, contiguous range of weight rows.  The CTA
// works in rounds: thread t always owns the same (row offset, group) unit of a
// round, so its activation slice is fixed for the whole launch (registers for
// a single SDOT row, padded shared memory otherwise) and no index arithmetic
// depends on runtime division inside the loop.  The next round's packed bytes
// are loaded before the current round is computed.
//
// Per unit the thread produces the group term of the reference:
//   FP32: sum_i cb[idx]*rot[i], times half(norm)      (needle2/csrc/cq.cpp:157-164)
//   SDOT: (float(int32 dot) * (half(norm)*cs)) * xs   (needle2/csrc/sdot.cpp:142-149)
// Terms land in shared memory (double buffered); after one barrier per round,
// one thread per output row adds its terms in group order, as the reference
// does, so SDOT outputs are bit-identical to it.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "cq_gemv.cuh"

namespace nb200 {
namespace {

constexpr int kThreadsV2 = 512;

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// CQ4 word (8 nibbles) -> int8 centroids of elements 0..3 (lo4) and 4..7 (hi4).
__device__ __forceinline__ void dec4(uint32_t w, const uint32_t (&t)[4], uint32_t &lo4, uint32_t &hi4) {
    const uint32_t sel = w & 0x77777777u;
    const uint32_t hb = (w >> 1) & 0x44444444u;
    uint32_t a = prmt(t[0], t[1], sel), b = prmt(t[2], t[3], sel);
    lo4 = prmt(a, b, (hb & 0xffffu) | 0x3210u);
    const uint32_t sel2 = sel >> 16, hb2 = hb >> 16;
    a = prmt(t[0], t[1], sel2);
    b = prmt(t[2], t[3], sel2);
    hi4 = prmt(a, b, hb2 | 0x3210u);
}

// CQ2 word (16 crumbs) -> centroids in bit-plane order (even elements of the
// word first, then odd), matching the SDOT activation layout.
__device__ __forceinline__ void dec2(uint32_t w, uint32_t t, uint32_t (&r)[4]) {
    const uint32_t e = w & 0x33333333u, o = (w >> 2) & 0x33333333u;
    r[0] = prmt(t, t, e);
    r[1] = prmt(t, t, e >> 16);
    r[2] = prmt(t, t, o);
    r[3] = prmt(t, t, o >> 16);
}

template <int BITS, int G>
struct Unit {
    static constexpr int BYTES = G * BITS / 8;      // packed bytes of one group
    static constexpr int CHUNKS = BYTES / 16;       // 16-byte loads per unit
    static constexpr int EPC = 128 / BITS;          // elements per chunk
};

template <bool I8, int BITS, int G, int MT>
__global__ void __launch_bounds__(kThreadsV2, 1) cq_gemv_v2(const GemvV2Params p) {
    using U = Unit<BITS, G>;
    constexpr bool XREG = I8 && MT == 1 && G <= 128;   // activation slice lives in registers
    extern __shared__ __align__(16) unsigned char smem[];
    // layout: [terms: 2][MT][rpr][gpr+1] float | [xs: MT][groups] float | [x]
    const int gpr = p.groups, tstride = gpr + 1;
    float *terms = reinterpret_cast<float *>(smem);
    const int tbuf = p.M * p.rpr * tstride;
    float *xs_s = terms + 2 * tbuf;
    const int head = 2 * tbuf + (I8 ? p.M * gpr : 0);            // floats before the x region
    unsigned char *x_s = smem + 4 * ((head + 3) & ~3);           // 16-byte aligned
    // per-group activation stride in shared memory, padded by 16 bytes so that
    // threads of consecutive groups hit distinct banks
    constexpr int XG = I8 ? G + 16 : 4 * G + 16;
    __shared__ float lut[16];

    const int tid = threadIdx.x;
    const int r0 = (int)((long long)p.out * blockIdx.x / gridDim.x);
    const int r1 = (int)((long long)p.out * (blockIdx.x + 1) / gridDim.x);

    // activations of this pass into shared memory
    if (I8) {
        for (int i = tid; i < p.M * gpr; i += kThreadsV2) xs_s[i] = p.xs[i];
        const int n16 = G / 16;
        for (int i = tid; i < p.M * gpr * n16; i += kThreadsV2) {
            const int m = i / (gpr * n16), rem = i % (gpr * n16), g = rem / n16, c = rem % n16;
            *reinterpret_cast<int4 *>(x_s + ((size_t)m * gpr + g) * XG + 16 * c) =
                *reinterpret_cast<const int4 *>(p.q + (size_t)m * p.padded + (size_t)g * G + 16 * c);
        }
    } else {
        if (tid < 16) lut[tid] = p.lut[tid];
        const int n4 = G / 4;
        for (int i = tid; i < p.M * gpr * n4; i += kThreadsV2) {
            const int m = i / (gpr * n4), rem = i % (gpr * n4), g = rem / n4, c = rem % n4;
            *reinterpret_cast<float4 *>(x_s + ((size_t)m * gpr + g) * XG + 16 * c) =
                *reinterpret_cast<const float4 *>(p.rot + (size_t)m * p.padded + (size_t)g * G + 4 * c);
        }
    }
    __syncthreads();

    // this thread's fixed unit
    const int units = p.rpr * gpr;
    const bool active = tid < units;
    const int roff = active ? tid / gpr : 0, g = active ? tid % gpr : 0;
    uint32_t ctab[4] = {p.ctab[0], p.ctab[1], p.ctab[2], p.ctab[3]};

    int xr[XREG ? G / 4 : 1];
    if (XREG) {
#pragma unroll
        for (int i = 0; i < G / 16; ++i) {
            const int4 v = *reinterpret_cast<const int4 *>(x_s + (size_t)g * XG + 16 * i);
            xr[4 * i] = v.x; xr[4 * i + 1] = v.y; xr[4 * i + 2] = v.z; xr[4 * i + 3] = v.w;
        }
    }

    const int rounds = (r1 - r0 + p.rpr - 1) / p.rpr;
    uint4 cur[U::CHUNKS], nxt[U::CHUNKS];
    auto load = [&](int round, uint4(&buf)[U::CHUNKS]) {
        const int row = r0 + round * p.rpr + roff;
        if (active && row < r1) {
            const uint4 *src = reinterpret_cast<const uint4 *>(p.packed + (size_t)row * p.rowbytes + (size_t)g * U::BYTES);
#pragma unroll
            for (int c = 0; c < U::CHUNKS; ++c) buf[c] = __ldg(src + c);
        }
    };
    if (rounds > 0) load(0, cur);

    for (int round = 0; round < rounds; ++round) {
        if (round + 1 < rounds) load(round + 1, nxt);
        const int rowbase = r0 + round * p.rpr;
        const int row = rowbase + roff;
        float *tb = terms + (round & 1) * tbuf;
        if (active && row < r1) {
            const float nv = half_bits_to_float(__ldg(p.norms + (size_t)row * gpr + g));
            if (I8) {
                int acc[MT];
#pragma unroll
                for (int m = 0; m < MT; ++m) acc[m] = 0;
#pragma unroll
                for (int c = 0; c < U::CHUNKS; ++c) {
                    uint32_t d[U::EPC / 4];
                    const uint32_t w[4] = {cur[c].x, cur[c].y, cur[c].z, cur[c].w};
                    if (BITS == 4) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) dec4(w[i], ctab, d[2 * i], d[2 * i + 1]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            uint32_t r4[4];
                            dec2(w[i], ctab[0], r4);
#pragma unroll
                            for (int k = 0; k < 4; ++k) d[4 * i + k] = r4[k];
                        }
                    }
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        if (m < p.M) {
#pragma unroll
                            for (int i = 0; i < U::EPC / 16; ++i) {
                                int4 xv;
                                if (XREG) {
                                    const int base = (c * U::EPC + 16 * i) / 4;
                                    xv = make_int4(xr[base], xr[base + 1], xr[base + 2], xr[base + 3]);
                                } else {
                                    xv = *reinterpret_cast<const int4 *>(x_s + ((size_t)m * gpr + g) * XG +
                                                                         c * U::EPC + 16 * i);
                                }
                                acc[m] = __dp4a((int)d[4 * i + 0], xv.x, acc[m]);
                                acc[m] = __dp4a((int)d[4 * i + 1], xv.y, acc[m]);
                                acc[m] = __dp4a((int)d[4 * i + 2], xv.z, acc[m]);
                                acc[m] = __dp4a((int)d[4 * i + 3], xv.w, acc[m]);
                            }
                        }
                    }
                }
                const float ns = __fmul_rn(nv, p.cs);
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m < p.M) {
                        tb[(m * p.rpr + roff) * tstride + g] =
                            __fmul_rn(__fmul_rn(__int2float_rn(acc[m]), ns), xs_s[m * gpr + g]);
                        if (p.partials) p.partials[((size_t)m * p.out + row) * gpr + g] = acc[m];
                    }
                }
            } else {
                float acc[MT];
#pragma unroll
                for (int m = 0; m < MT; ++m) acc[m] = 0.f;
                constexpr unsigned mask = (1u << BITS) - 1u;
#pragma unroll
                for (int c = 0; c < U::CHUNKS; ++c) {
                    const uint32_t w[4] = {cur[c].x, cur[c].y, cur[c].z, cur[c].w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        constexpr int EPW = 32 / BITS;  // elements per word
                        float wv[EPW];
#pragma unroll
                        for (int e = 0; e < EPW; ++e) wv[e] = lut[(w[i] >> (BITS * e)) & mask];
#pragma unroll
                        for (int m = 0; m < MT; ++m) {
                            if (m < p.M) {
                                const float *xp = reinterpret_cast<const float *>(
                                    x_s + ((size_t)m * gpr + g) * XG + 4 * (c * U::EPC + i * EPW));
#pragma unroll
                                for (int e4 = 0; e4 < EPW / 4; ++e4) {
                                    const float4 xv = *reinterpret_cast<const float4 *>(xp + 4 * e4);
                                    acc[m] = fmaf(wv[4 * e4 + 0], xv.x, acc[m]);
                                    acc[m] = fmaf(wv[4 * e4 + 1], xv.y, acc[m]);
                                    acc[m] = fmaf(wv[4 * e4 + 2], xv.z, acc[m]);
                                    acc[m] = fmaf(wv[4 * e4 + 3], xv.w, acc[m]);
                                }
                            }
                        }
                    }
                }
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    if (m < p.M) tb[(m * p.rpr + roff) * tstride + g] = __fmul_rn(acc[m], nv);
            }
        }
        __syncthreads();
        // ordered sums of this round's rows
        const int nrows = min(p.rpr, r1 - rowbase);
        for (int idx = tid; idx < p.M * nrows; idx += kThreadsV2) {
            const int m = idx / nrows, rl = idx - m * nrows;
            const float *tr = tb + (m * p.rpr + rl) * tstride;
            float v = 0.f;
            for (int gg = 0; gg < gpr; ++gg) v = __fadd_rn(v, tr[gg]);
            p.y[(size_t)m * p.ldy + rowbase + rl] = v;
        }
#pragma unroll
        for (int c = 0; c < U::CHUNKS; ++c) cur[c] = nxt[c];
    }
}

int num_sms() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

template <bool I8, int BITS, int G, int MT>
bool launch_v2(const GemvV2Params &p, size_t smem, cudaStream_t st) {
    auto kernel = cq_gemv_v2<I8, BITS, G, MT>;
    static bool configured[64] = {};
    int dev = 0;
    NB_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        NB_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvV2MaxSmem));
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    static int sms[64] = {};
    if (dev >= 0 && dev < 64 && !sms[dev]) sms[dev] = num_sms();
    const int grid = std::max(1, std::min(p.out, dev >= 0 && dev < 64 ? sms[dev] : 148));
    kernel<<<grid, kThreadsV2, smem, st>>>(p);
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

template <bool I8, int BITS, int G>
bool dispatch_mt(const GemvV2Params &p, size_t smem, cudaStream_t st) {
    if (p.M <= 1) return launch_v2<I8, BITS, G, 1>(p, smem, st);
    if (p.M <= 2) return launch_v2<I8, BITS, G, 2>(p, smem, st);
    if (p.M <= 4) return launch_v2<I8, BITS, G, 4>(p, smem, st);
    if (p.M <= 8) return launch_v2<I8, BITS, G, 8>(p, smem, st);
    return launch_v2<I8, BITS, G, 16>(p, smem, st);
}

template <bool I8>
bool dispatch(const GemvV2Params &p, int bits, int group, size_t smem, cudaStream_t st) {
    if (bits == 4) {
        if (group == 64) return dispatch_mt<I8, 4, 64>(p, smem, st);
        if (group == 128) return dispatch_mt<I8, 4, 128>(p, smem, st);
        return dispatch_mt<I8, 4, 256>(p, smem, st);
    }
    if (group == 64) return dispatch_mt<I8, 2, 64>(p, smem, st);
    if (group == 128) return dispatch_mt<I8, 2, 128>(p, smem, st);
    return dispatch_mt<I8, 2, 256>(p, smem, st);
}

}  // namespace

namespace {

// Dynamic shared memory of one launch; the same layout as in cq_gemv_v2.
size_t gemv_v2_smem(int M, int groups, int group, int rpr, bool i8) {
    const size_t head = 2 * (size_t)M * rpr * (groups + 1) + (i8 ? (size_t)M * groups : 0);
    const size_t x = (size_t)M * groups * (i8 ? group + 16 : 4 * group + 16);
    return 4 * ((head + 3) & ~size_t(3)) + x;
}

}  // namespace

int gemv_v2_max_rows(int bits, int group, int groups, bool i8) {
    if ((bits != 2 && bits != 4) || (group != 64 && group != 128 && group != 256)) return 0;
    if (groups < 1 || groups > kThreadsV2) return 0;
    const int rpr = kThreadsV2 / groups;
    for (int m : {16, 8, 4, 2, 1})
        if (gemv_v2_smem(m, groups, group, rpr, i8) <= (size_t)kGemvV2MaxSmem) return m;
    return 0;
}

bool launch_gemv_v2(const GemvV2Params &p0, int bits, int group, bool i8, cudaStream_t st) {
    GemvV2Params p = p0;
    const int cap = gemv_v2_max_rows(bits, group, p.groups, i8);
    if (cap < p.M || p.M < 1) {
        set_error("GEMV shape outside the persistent kernel's envelope");
        return false;
    }
    p.rpr = kThreadsV2 / p.groups;
    const size_t smem = gemv_v2_smem(p.M, p.groups, group, p.rpr, i8);
    return i8 ? dispatch<true>(p, bits, group, smem, st) : dispatch<false>(p, bits, group, smem, st);
}

}  // namespace nb200
