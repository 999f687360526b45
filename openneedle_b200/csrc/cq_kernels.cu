// CQ packed-weight kernels for B200 (sm_100a).
//
//  * rotate / quantize: per-(row, group) normalised Walsh-Hadamard transform of
//    the activations, optionally followed by the SDOT int8 quantiser
//    (needle2/csrc/cq.cpp:30-46,153-156; needle2/csrc/sdot.cpp:47-103).
//  * cq_gemv: y = W x for a CQ2/CQ4 matrix streamed once from HBM in 16-byte
//    chunks; FP32 mode (codebook lookup + FMA) or SDOT mode (prmt-decoded int8
//    centroids + dp4a, exact int32 per group) — needle2/csrc/cq.cpp:157-197,
//    needle2/csrc/sdot.cpp:108-149.  Each group's partial becomes one term and
//    the terms of a row are added in group order by one thread, as the
//    reference does, so the SDOT output is bit-identical.
//  * rows: dequantised rows (needle2/csrc/cq.cpp:276-284).
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "pdl.cuh"
#include "cq_gemv.cuh"
#include "sm100_async.cuh"
#include <cuda_bf16.h>

#include "cq_kernels.cuh"

namespace nb200 {

namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// Destination of element e (within a group) in the CQ2 SDOT activation layout:
// each 16-element block holds its even elements first, then its odd ones, the
// order in which decode_cq2_i8 produces centroids.
__device__ __forceinline__ int cq2_plane_index(int e) {
    int r = e & 15;
    return (e & ~15) | ((r & 1) ? 8 + (r >> 1) : (r >> 1));
}

// ------------------------------------------------------------------- FWHT

template <int G>
struct WarpShape {
    static constexpr int E = G >= 32 ? G / 32 : 1;       // elements per lane
    static constexpr int LANES = G >= 32 ? 32 : G;       // lanes per group
    static constexpr int PER_WARP = 32 / LANES;          // groups per warp
};

// Radix-2 butterflies with strides 1, 2, ..., G/2 then one multiply by
// `scale`.  Element (lane_in_group*E + j).  Every stage computes exactly the
// reference's a+b / a-b, so the result is bit-identical to
// needle2/csrc/cq.cpp:30-46.
template <int G>
__device__ __forceinline__ void warp_fwht(float (&v)[WarpShape<G>::E], int lane_in_group, float scale) {
    constexpr int E = WarpShape<G>::E;
#pragma unroll
    for (int h = 1; h < E; h <<= 1) {
#pragma unroll
        for (int j = 0; j < E; ++j) {
            if (!(j & h)) {
                float a = v[j], b = v[j + h];
                v[j] = __fadd_rn(a, b);
                v[j + h] = __fsub_rn(a, b);
            }
        }
    }
#pragma unroll
    for (int h = E; h < G; h <<= 1) {
        const int lb = h / E;
        const bool upper = (lane_in_group & lb) != 0;
#pragma unroll
        for (int j = 0; j < E; ++j) {
            float other = __shfl_xor_sync(kFull, v[j], lb);
            v[j] = upper ? __fsub_rn(other, v[j]) : __fadd_rn(v[j], other);
        }
    }
#pragma unroll
    for (int j = 0; j < E; ++j) v[j] = __fmul_rn(v[j], scale);
}

// One CTA-wide FWHT over s[0..G) in shared memory (G > 1024).
__device__ void block_fwht(float *s, int G, float scale) {
    for (int h = 1; h < G; h <<= 1) {
        __syncthreads();
        for (int i = threadIdx.x; i < G / 2; i += blockDim.x) {
            int j = (i / h) * 2 * h + (i % h);
            float a = s[j], b = s[j + h];
            s[j] = __fadd_rn(a, b);
            s[j + h] = __fsub_rn(a, b);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G; i += blockDim.x) s[i] = __fmul_rn(s[i], scale);
    __syncthreads();
}

// SDOT scale of one group: absmax/127, 1 when absmax is 0, absmax when the
// quotient underflows (needle2/csrc/sdot.cpp:78-79).
__device__ __forceinline__ float sdot_scale(float absmax) {
    float sc = absmax > 0.f ? __fdiv_rn(absmax, 127.f) : 1.f;
    if (sc == 0.f) sc = absmax;
    return sc;
}

// FP32 mode writes rot[M][padded], or (hilo not null) the bf16 operands of
// the FP32-mode GEMM directly: hilo[i] = bf16(v), hilo[lo_off + i] =
// bf16(v - hi), as split_bf16_kernel makes them from rot.
template <int G, bool QUANT>
__global__ void __launch_bounds__(256) rotate_warp_kernel(const float *__restrict__ x, int M, int in, int padded,
                                                          float scale, float *__restrict__ rot,
                                                          int8_t *__restrict__ q, float *__restrict__ xs,
                                                          int cq2_planes, uint16_t *__restrict__ hilo,
                                                          long long lo_off) {
    using S = WarpShape<G>;
    pdl_launch_dependents();
    pdl_wait();   // x may be produced by the preceding kernel in the stream
    const int groups = padded / G;
    const int lane = threadIdx.x & 31;
    const int lig = lane % S::LANES, sub = lane / S::LANES;
    const long long total = (long long)M * groups;
    const long long warps = (long long)gridDim.x * (blockDim.x / 32);
    for (long long base = ((long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * S::PER_WARP;
         base < total; base += warps * S::PER_WARP) {
        const long long item = base + sub;
        const bool valid = item < total;
        const int m = valid ? (int)(item / groups) : 0, g = valid ? (int)(item % groups) : 0;
        float v[S::E];
#pragma unroll
        for (int j = 0; j < S::E; ++j) {
            int e = g * G + lig * S::E + j;
            v[j] = (valid && e < in) ? __ldg(x + (size_t)m * in + e) : 0.f;
        }
        warp_fwht<G>(v, lig, scale);
        if (!QUANT) {
            if (valid && hilo) {
                const size_t o = (size_t)m * padded + (size_t)g * G + lig * S::E;
#pragma unroll
                for (int j = 0; j < S::E; ++j) {
                    const __nv_bfloat16 h = __float2bfloat16_rn(v[j]);
                    hilo[o + j] = __bfloat16_as_ushort(h);
                    hilo[lo_off + o + j] = __bfloat16_as_ushort(__float2bfloat16_rn(__fsub_rn(v[j], __bfloat162float(h))));
                }
            } else if (valid) {
                float *dst = rot + (size_t)m * padded + (size_t)g * G + lig * S::E;
#pragma unroll
                for (int j = 0; j < S::E; ++j) dst[j] = v[j];
            }
        } else {
            float amax = 0.f;
#pragma unroll
            for (int j = 0; j < S::E; ++j) amax = fmaxf(amax, fabsf(v[j]));
#pragma unroll
            for (int o = S::LANES / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, o));
            const float sc = sdot_scale(amax);
            if (valid) {
                if (lig == 0) xs[(size_t)m * groups + g] = sc;
                int8_t *dst = q + (size_t)m * padded + (size_t)g * G;
#pragma unroll
                for (int j = 0; j < S::E; ++j) {
                    int e = lig * S::E + j;
                    dst[cq2_planes ? cq2_plane_index(e) : e] = (int8_t)clamp127(rint_even(__fdiv_rn(v[j], sc)));
                }
            }
        }
    }
}

template <bool QUANT>
__global__ void __launch_bounds__(1024) rotate_block_kernel(const float *__restrict__ x, int in, int padded, int G,
                                                            float scale, float *__restrict__ rot,
                                                            int8_t *__restrict__ q, float *__restrict__ xs,
                                                            int cq2_planes) {
    extern __shared__ float s[];
    __shared__ float red[32];
    const int groups = padded / G;
    const int m = blockIdx.x / groups, g = blockIdx.x % groups;
    for (int i = threadIdx.x; i < G; i += blockDim.x) {
        int e = g * G + i;
        s[i] = e < in ? __ldg(x + (size_t)m * in + e) : 0.f;
    }
    block_fwht(s, G, scale);
    if (!QUANT) {
        for (int i = threadIdx.x; i < G; i += blockDim.x) rot[(size_t)m * padded + (size_t)g * G + i] = s[i];
        return;
    }
    float amax = 0.f;
    for (int i = threadIdx.x; i < G; i += blockDim.x) amax = fmaxf(amax, fabsf(s[i]));
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = amax;
    __syncthreads();
    if (threadIdx.x < 32) {
        amax = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, o));
        if (threadIdx.x == 0) red[0] = amax;
    }
    __syncthreads();
    const float sc = sdot_scale(red[0]);
    if (threadIdx.x == 0) xs[(size_t)m * groups + g] = sc;
    int8_t *dst = q + (size_t)m * padded + (size_t)g * G;
    for (int i = threadIdx.x; i < G; i += blockDim.x)
        dst[cq2_planes ? cq2_plane_index(i) : i] = (int8_t)clamp127(rint_even(__fdiv_rn(s[i], sc)));
}

template <bool QUANT>
bool launch_rotate_impl(const CQDevice &w, const float *x, int M, float *rot, int8_t *q, float *xs,
                        int cq2_planes, cudaStream_t st, uint16_t *hilo = nullptr) {
    const float scale = 1.0f / sqrtf((float)w.group);  // host: same expression as the reference
    const long long items = (long long)M * w.groups;
    if (items == 0) return true;
    auto warp_launch = [&](auto kernel, int per_warp) {
        long long warps = (items + per_warp - 1) / per_warp;
        int blocks = (int)std::min<long long>((warps + 7) / 8, 65535);
        // programmatic dependent launch: may start while the previous kernel drains
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(blocks);
        cfg.blockDim = dim3(256);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaLaunchKernelEx(&cfg, kernel, x, M, w.in, w.padded, scale, rot, q, xs, cq2_planes, hilo,
                           (long long)M * w.padded);
    };
    if (hilo && (w.group < 8 || w.group > 1024)) {
        set_error("the direct bf16 split needs a group of 8 to 1024");
        return false;
    }
    switch (w.group) {
        case 8: warp_launch(rotate_warp_kernel<8, QUANT>, 4); break;
        case 16: warp_launch(rotate_warp_kernel<16, QUANT>, 2); break;
        case 32: warp_launch(rotate_warp_kernel<32, QUANT>, 1); break;
        case 64: warp_launch(rotate_warp_kernel<64, QUANT>, 1); break;
        case 128: warp_launch(rotate_warp_kernel<128, QUANT>, 1); break;
        case 256: warp_launch(rotate_warp_kernel<256, QUANT>, 1); break;
        case 512: warp_launch(rotate_warp_kernel<512, QUANT>, 1); break;
        case 1024: warp_launch(rotate_warp_kernel<1024, QUANT>, 1); break;
        default: {
            if (w.group > kMaxGroup || items > 0x7fffffffLL) {
                set_error("group size above 16384 is not supported by the GPU build");
                return false;
            }
            size_t smem = sizeof(float) * (size_t)w.group;
            NB_CUDA_TRY(cudaFuncSetAttribute(rotate_block_kernel<QUANT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            rotate_block_kernel<QUANT><<<(unsigned)items, 1024, smem, st>>>(x, w.in, w.padded, w.group, scale, rot,
                                                                           q, xs, cq2_planes);
        }
    }
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

// ------------------------------------------------------------------- GEMV

struct GemvParams {
    const uint8_t *packed;
    const uint16_t *norms;
    int out, groups, rowbytes, cpr, gpc, rows_per_tile, tiles, M;
    int padded;
    const float *rot;      // FP32 mode activations [M][padded]
    const int8_t *q;       // SDOT activations [M][padded]
    const float *xs;       // SDOT scales [M][groups]
    float *y;
    int ldy;
    int32_t *partials;     // SDOT debug output [M][out][groups] or null
    float lut[16];
    uint32_t ctab[4];
    float cs;
};

constexpr int kThreads = 256;
constexpr int kChunksPerThread = 4;
constexpr int kTileChunks = kThreads * kChunksPerThread;  // 16 KB of packed weights

// 16 int8 centroids of a CQ4 chunk word: nibble i -> byte i of lo4 (i<4) or hi4.
__device__ __forceinline__ void decode_cq4_i8(uint32_t w, const uint32_t (&t)[4], uint32_t &lo4, uint32_t &hi4) {
    const uint32_t sel = w & 0x77777777u;             // low three index bits per nibble
    const uint32_t hb = (w >> 1) & 0x44444444u;       // index bit 3 moved to nibble bit 2
    uint32_t a = prmt(t[0], t[1], sel), b = prmt(t[2], t[3], sel);
    lo4 = prmt(a, b, (hb & 0xffffu) | 0x3210u);       // byte i from a (bit3 = 0) or b
    const uint32_t sel2 = sel >> 16, hb2 = hb >> 16;
    a = prmt(t[0], t[1], sel2);
    b = prmt(t[2], t[3], sel2);
    hi4 = prmt(a, b, hb2 | 0x3210u);
}

// CQ2 word (16 crumbs) -> four words of int8 centroids in plane order:
// r0 = elements 0,2,4,6; r1 = 8..14 even; r2 = 1,3,5,7; r3 = 9..15 odd.
__device__ __forceinline__ void decode_cq2_i8(uint32_t w, uint32_t t, uint32_t (&r)[4]) {
    const uint32_t e = w & 0x33333333u, o = (w >> 2) & 0x33333333u;
    r[0] = prmt(t, t, e);
    r[1] = prmt(t, t, e >> 16);
    r[2] = prmt(t, t, o);
    r[3] = prmt(t, t, o >> 16);
}

__device__ __forceinline__ uint4 ldg_stream(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

template <bool I8, int BITS>
__global__ void __launch_bounds__(kThreads) cq_gemv_kernel(const GemvParams p) {
    extern __shared__ float terms[];  // [M][rows_per_tile][groups]
    __shared__ float lut[16];
    constexpr int EPC = 128 / BITS;   // elements per 16-byte chunk
    if (!I8 && threadIdx.x < 16) lut[threadIdx.x] = p.lut[threadIdx.x];
    uint32_t ctab[4] = {p.ctab[0], p.ctab[1], p.ctab[2], p.ctab[3]};
    __syncthreads();

    const int tid = threadIdx.x, lane = tid & 31;
    const int t0 = (int)((long long)p.tiles * blockIdx.x / gridDim.x);
    const int t1 = (int)((long long)p.tiles * (blockIdx.x + 1) / gridDim.x);
    const int R = p.rows_per_tile;

    uint4 cur[kChunksPerThread], nxt[kChunksPerThread];
    auto load_tile = [&](int tile, uint4(&buf)[kChunksPerThread]) {
        const int row0 = tile * R;
        const int nch = min(R, p.out - row0) * p.cpr;
        const uint4 *src = reinterpret_cast<const uint4 *>(p.packed + (size_t)row0 * p.rowbytes);
#pragma unroll
        for (int j = 0; j < kChunksPerThread; ++j) {
            const int c = tid + j * kThreads;
            buf[j] = c < nch ? ldg_stream(src + c) : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    if (t0 < t1) load_tile(t0, cur);

    for (int tile = t0; tile < t1; ++tile) {
        if (tile + 1 < t1) load_tile(tile + 1, nxt);
        const int row0 = tile * R;
        const int nrows = min(R, p.out - row0);
        const int nch = nrows * p.cpr;
#pragma unroll
        for (int j = 0; j < kChunksPerThread; ++j) {
            const int c = tid + j * kThreads;
            const bool valid = c < nch;
            const int rl = c / p.cpr, kc = c - rl * p.cpr, g = kc / p.gpc;
            const bool leader = valid && (lane % p.gpc) == 0;
            const uint32_t wd[4] = {cur[j].x, cur[j].y, cur[j].z, cur[j].w};
            if (I8) {
                uint32_t dec[EPC / 4];
                if (BITS == 4) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) decode_cq4_i8(wd[i], ctab, dec[2 * i], dec[2 * i + 1]);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        uint32_t r[4];
                        decode_cq2_i8(wd[i], ctab[0], r);
#pragma unroll
                        for (int k = 0; k < 4; ++k) dec[4 * i + k] = r[k];
                    }
                }
                for (int m = 0; m < p.M; ++m) {
                    const int4 *xq = reinterpret_cast<const int4 *>(p.q + (size_t)m * p.padded + (size_t)kc * EPC);
                    int acc = 0;
#pragma unroll
                    for (int i = 0; i < EPC / 16; ++i) {
                        const int4 xv = valid ? __ldg(xq + i) : make_int4(0, 0, 0, 0);
                        acc = __dp4a((int)dec[4 * i + 0], xv.x, acc);
                        acc = __dp4a((int)dec[4 * i + 1], xv.y, acc);
                        acc = __dp4a((int)dec[4 * i + 2], xv.z, acc);
                        acc = __dp4a((int)dec[4 * i + 3], xv.w, acc);
                    }
                    for (int o = p.gpc >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
                    if (leader) {
                        const int row = row0 + rl;
                        const float ns = __fmul_rn(half_bits_to_float(__ldg(p.norms + (size_t)row * p.groups + g)), p.cs);
                        const float t = __fmul_rn(__fmul_rn(__int2float_rn(acc), ns), __ldg(p.xs + (size_t)m * p.groups + g));
                        terms[((size_t)m * R + rl) * p.groups + g] = t;
                        if (p.partials) p.partials[((size_t)m * p.out + row) * p.groups + g] = acc;
                    }
                }
            } else {
                for (int m = 0; m < p.M; ++m) {
                    const float4 *xr = reinterpret_cast<const float4 *>(p.rot + (size_t)m * p.padded + (size_t)kc * EPC);
                    float acc = 0.f;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
#pragma unroll
                        for (int k = 0; k < EPC / 16; ++k) {
                            const float4 xv = valid ? __ldg(xr + i * (EPC / 16) + k) : make_float4(0.f, 0.f, 0.f, 0.f);
                            const int sh = k * 4 * BITS;
                            constexpr unsigned mask = (1u << BITS) - 1u;
                            acc = fmaf(lut[(wd[i] >> (sh + 0 * BITS)) & mask], xv.x, acc);
                            acc = fmaf(lut[(wd[i] >> (sh + 1 * BITS)) & mask], xv.y, acc);
                            acc = fmaf(lut[(wd[i] >> (sh + 2 * BITS)) & mask], xv.z, acc);
                            acc = fmaf(lut[(wd[i] >> (sh + 3 * BITS)) & mask], xv.w, acc);
                        }
                    }
                    for (int o = p.gpc >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
                    if (leader) {
                        const int row = row0 + rl;
                        const float nv = half_bits_to_float(__ldg(p.norms + (size_t)row * p.groups + g));
                        terms[((size_t)m * R + rl) * p.groups + g] = __fmul_rn(acc, nv);
                    }
                }
            }
        }
        __syncthreads();
        for (int idx = tid; idx < p.M * nrows; idx += kThreads) {
            const int m = idx / nrows, rl = idx - m * nrows;
            const float *tr = terms + ((size_t)m * R + rl) * p.groups;
            float v = 0.f;
            for (int g = 0; g < p.groups; ++g) v = __fadd_rn(v, tr[g]);
            p.y[(size_t)m * p.ldy + row0 + rl] = v;
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kChunksPerThread; ++j) cur[j] = nxt[j];
    }
}

struct Lut16 {
    float v[16];
};

// Generic FP32 path (CQ3, ternary, tiny groups, very long rows): one thread per
// (activation row, output row) in the reference's own operation order.
__global__ void cq_gemv_generic_kernel(const uint8_t *__restrict__ packed, const uint16_t *__restrict__ norms,
                                       int out, int groups, int group, int padded, int storage_bits, int rowbytes,
                                       const float *__restrict__ rot, int M, float *__restrict__ y, int ldy,
                                       const Lut16 lut_in) {
    __shared__ float lut[16];
    if (threadIdx.x < 16) lut[threadIdx.x] = lut_in.v[threadIdx.x];
    __syncthreads();
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)M * out) return;
    const int m = (int)(idx / out), r = (int)(idx % out);
    const uint8_t *p = packed + (size_t)r * rowbytes;
    const float *xr = rot + (size_t)m * padded;
    const unsigned mask = (1u << storage_bits) - 1u;
    float sum = 0.f;
    for (int g = 0; g < groups; ++g) {
        float gs = 0.f;
        for (int i = 0; i < group; ++i) {
            const int e = g * group + i, bit = e * storage_bits, byte = bit >> 3, shift = bit & 7;
            unsigned word = p[byte];
            if (shift + storage_bits > 8) word |= (unsigned)p[byte + 1] << 8;
            gs = __fadd_rn(gs, __fmul_rn(lut[(word >> shift) & mask], xr[e]));
        }
        sum = __fadd_rn(sum, __fmul_rn(gs, half_bits_to_float(norms[(size_t)r * groups + g])));
    }
    y[(size_t)m * ldy + r] = sum;
}

// Generic SDOT path (groups whose packed bytes exceed one warp's 32 chunks):
// one thread per (activation row, output row), exact int32 per group, terms
// added in group order (needle2/csrc/sdot.cpp:133-148).
__global__ void cq_gemv_i8_generic_kernel(const uint8_t *__restrict__ packed, const uint16_t *__restrict__ norms,
                                          int out, int groups, int group, int padded, int bits, int rowbytes,
                                          const int8_t *__restrict__ q, const float *__restrict__ xs, int M,
                                          float *__restrict__ y, int ldy, int32_t *__restrict__ partials,
                                          uint4 ctab, float cs) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)M * out) return;
    const int m = (int)(idx / out), r = (int)(idx % out);
    int8_t cent[16];
    memcpy(cent, &ctab, 16);
    const uint8_t *p = packed + (size_t)r * rowbytes;
    const int8_t *xq = q + (size_t)m * padded;
    const unsigned mask = (1u << bits) - 1u;
    float value = 0.f;
    for (int g = 0; g < groups; ++g) {
        int acc = 0;
        for (int i = 0; i < group; ++i) {
            const int e = g * group + i, bit = e * bits;
            const unsigned idx4 = (p[bit >> 3] >> (bit & 7)) & mask;
            const int d = bits == 2 ? cq2_plane_index(i) : i;
            acc += (int)cent[idx4] * (int)xq[(size_t)g * group + d];
        }
        const float ns = __fmul_rn(half_bits_to_float(norms[(size_t)r * groups + g]), cs);
        value = __fadd_rn(value, __fmul_rn(__fmul_rn(__int2float_rn(acc), ns), xs[(size_t)m * groups + g]));
        if (partials) partials[((size_t)m * out + r) * groups + g] = acc;
    }
    y[(size_t)m * ldy + r] = value;
}

int device_sms() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

template <bool I8, int BITS>
bool launch_gemv_fast(const CQDevice &w, GemvParams &p, cudaStream_t st) {
    p.cpr = w.rowbytes / 16;
    p.gpc = w.group * BITS / 8 / 16;
    p.rows_per_tile = std::max(1, kTileChunks / p.cpr);
    p.tiles = ceil_div(w.out, p.rows_per_tile);
    const size_t smem = sizeof(float) * (size_t)p.M * p.rows_per_tile * w.groups;
    auto kernel = cq_gemv_kernel<I8, BITS>;
    static bool configured[64] = {};  // per device ordinal
    int dev = 0;
    NB_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        NB_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    int per_sm = 1;
    NB_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem));
    const int grid = std::max(1, std::min(p.tiles, device_sms() * std::max(1, per_sm)));
    kernel<<<grid, kThreads, smem, st>>>(p);
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

}  // namespace

bool gemv_fast_path(const CQDevice &w) {
    if (w.bits != 2 && w.bits != 4 && w.bits != 5) return false;
    const int sb = w.storage_bits;
    const int group_bytes = w.group * sb / 8;
    if (group_bytes < 16 || group_bytes % 16) return false;
    const int gpc = group_bytes / 16;
    if (gpc > 32 || w.rowbytes % 16) return false;
    return w.rowbytes / 16 <= kTileChunks;
}

bool launch_rotate(const CQDevice &w, const float *x, int M, float *rot, cudaStream_t s) {
    return launch_rotate_impl<false>(w, x, M, rot, nullptr, nullptr, 0, s);
}

bool launch_rotate_hilo(const CQDevice &w, const float *x, int M, uint16_t *hilo, cudaStream_t s) {
    return launch_rotate_impl<false>(w, x, M, nullptr, nullptr, nullptr, 0, s, hilo);
}

bool launch_quantize(const CQDevice &w, const float *x, int M, int8_t *q, float *xs, cudaStream_t s) {
    return launch_rotate_impl<true>(w, x, M, nullptr, q, xs, w.bits == 2 ? 1 : 0, s);
}

GemvBatch single_batch(const CQDevice &w) {
    GemvBatch b{};
    b.nmat = 1;
    b.mat[0].packed = w.packed;
    b.mat[0].norms = w.norms;
    b.mat[0].norms8 = w.norms8;
    b.mat[0].frag = w.frag;
    b.mat[0].normsF = w.normsF;
    b.mat[0].blocked = w.blocked;
    b.mat[0].normsB = w.normsB;
    b.mat[0].out = w.out;
    b.bits = w.bits;
    b.group = w.group;
    b.groups = w.groups;
    b.rowbytes = w.rowbytes;
    b.padded = w.padded;
    for (int i = 0; i < 16; ++i) b.lut[i] = w.lut[i];
    for (int i = 0; i < 4; ++i) b.ctab[i] = w.ctab[i];
    for (int i = 0; i < 2; ++i) {
        b.ntab[i] = w.ntab[i];
        b.ptab[i] = w.ptab[i];
    }
    b.split = w.split;
    b.cs = w.centroid_scale;
    return b;
}

bool launch_gemv_f32(const CQDevice &w, const float *rot, int M, float *y, int ldy, cudaStream_t s) {
    if (M <= 0 || w.out <= 0) return true;
    if (!gemv_fast_path(w)) {
        Lut16 lut;
        for (int i = 0; i < 16; ++i) lut.v[i] = w.lut[i];
        const long long n = (long long)M * w.out;
        cq_gemv_generic_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(w.packed, w.norms, w.out, w.groups, w.group,
                                                                          w.padded, w.storage_bits, w.rowbytes, rot,
                                                                          M, y, ldy, lut);
        NB_CUDA_TRY(cudaGetLastError());
        return true;
    }
    if (w.bits != 5 && ldy == w.out) {
        const int cap = gemv_max_rows(w.bits, w.group, w.groups, false);
        if (cap > 0) {
            for (int m0 = 0; m0 < M; m0 += cap) {
                GemvBatch b = single_batch(w);
                b.M = std::min(cap, M - m0);
                b.rot = rot + (size_t)m0 * w.padded;
                b.mat[0].y = y + (size_t)m0 * ldy;
                if (!launch_gemv(b, false, s)) return false;
            }
            return true;
        }
    }
    for (int m0 = 0; m0 < M; m0 += kGemvMaxRows) {
        GemvParams p{};
        p.packed = w.packed;
        p.norms = w.norms;
        p.out = w.out;
        p.groups = w.groups;
        p.rowbytes = w.rowbytes;
        p.padded = w.padded;
        p.M = std::min(kGemvMaxRows, M - m0);
        p.rot = rot + (size_t)m0 * w.padded;
        p.y = y + (size_t)m0 * ldy;
        p.ldy = ldy;
        for (int i = 0; i < 16; ++i) p.lut[i] = w.lut[i];
        bool ok = w.storage_bits == 4 ? launch_gemv_fast<false, 4>(w, p, s) : launch_gemv_fast<false, 2>(w, p, s);
        if (!ok) return false;
    }
    return true;
}

bool launch_gemv_i8(const CQDevice &w, const int8_t *q, const float *xs, int M, float *y, int ldy,
                    int32_t *partials, cudaStream_t s) {
    if (M <= 0 || w.out <= 0) return true;
    if (w.bits != 2 && w.bits != 4) {
        set_error("SDOT requires CQ2/CQ4 with group size between 64 and 131072");
        return false;
    }
    if (ldy == w.out) {
        const int cap = gemv_max_rows(w.bits, w.group, w.groups, true);
        if (cap > 0) {
            for (int m0 = 0; m0 < M; m0 += cap) {
                GemvBatch b = single_batch(w);
                b.M = std::min(cap, M - m0);
                b.q = q + (size_t)m0 * w.padded;
                b.xs = xs + (size_t)m0 * w.groups;
                b.mat[0].y = y + (size_t)m0 * ldy;
                b.partials = partials ? partials + (size_t)m0 * w.out * w.groups : nullptr;
                if (!launch_gemv(b, true, s)) return false;
            }
            return true;
        }
    }
    if (!gemv_fast_path(w)) {
        uint4 ctab;
        memcpy(&ctab, w.ctab, 16);
        const long long n = (long long)M * w.out;
        cq_gemv_i8_generic_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(
            w.packed, w.norms, w.out, w.groups, w.group, w.padded, w.bits, w.rowbytes, q, xs, M, y, ldy, partials,
            ctab, w.centroid_scale);
        NB_CUDA_TRY(cudaGetLastError());
        return true;
    }
    for (int m0 = 0; m0 < M; m0 += kGemvMaxRows) {
        GemvParams p{};
        p.packed = w.packed;
        p.norms = w.norms;
        p.out = w.out;
        p.groups = w.groups;
        p.rowbytes = w.rowbytes;
        p.padded = w.padded;
        p.M = std::min(kGemvMaxRows, M - m0);
        p.q = q + (size_t)m0 * w.padded;
        p.xs = xs + (size_t)m0 * w.groups;
        p.y = y + (size_t)m0 * ldy;
        p.ldy = ldy;
        p.partials = partials ? partials + (size_t)m0 * w.out * w.groups : nullptr;
        for (int i = 0; i < 4; ++i) p.ctab[i] = w.ctab[i];
        p.cs = w.centroid_scale;
        bool ok = w.bits == 4 ? launch_gemv_fast<true, 4>(w, p, s) : launch_gemv_fast<true, 2>(w, p, s);
        if (!ok) return false;
    }
    return true;
}

// ------------------------------------------------------------------- rows

namespace {

template <int G>
__global__ void __launch_bounds__(256) rows_warp_kernel(const uint8_t *__restrict__ packed,
                                                        const uint16_t *__restrict__ norms, int in, int groups,
                                                        int storage_bits, int rowbytes, const int64_t *__restrict__ ids,
                                                        int count, float scale, float *__restrict__ y,
                                                        const float4 lut0, const float4 lut1, const float4 lut2,
                                                        const float4 lut3) {
    using S = WarpShape<G>;
    __shared__ float lut[16];
    if (threadIdx.x < 16) {
        const float4 l = threadIdx.x < 4 ? lut0 : threadIdx.x < 8 ? lut1 : threadIdx.x < 12 ? lut2 : lut3;
        const int k = threadIdx.x & 3;
        lut[threadIdx.x] = k == 0 ? l.x : k == 1 ? l.y : k == 2 ? l.z : l.w;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int lig = lane % S::LANES, sub = lane / S::LANES;
    const long long total = (long long)count * groups;
    const long long warps = (long long)gridDim.x * (blockDim.x / 32);
    const unsigned mask = (1u << storage_bits) - 1u;
    for (long long base = ((long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * S::PER_WARP;
         base < total; base += warps * S::PER_WARP) {
        const long long item = base + sub;
        const bool valid = item < total;
        const int c = valid ? (int)(item / groups) : 0, g = valid ? (int)(item % groups) : 0;
        const int64_t r = valid ? ids[c] : 0;
        const uint8_t *p = packed + (size_t)r * rowbytes;
        const float nv = valid ? half_bits_to_float(norms[(size_t)r * groups + g]) : 0.f;
        float v[S::E];
#pragma unroll
        for (int j = 0; j < S::E; ++j) {
            float wv = 0.f;
            if (valid) {
                const int e = g * G + lig * S::E + j, bit = e * storage_bits, byte = bit >> 3, shift = bit & 7;
                unsigned word = p[byte];
                if (shift + storage_bits > 8) word |= (unsigned)p[byte + 1] << 8;
                wv = lut[(word >> shift) & mask];
            }
            v[j] = __fmul_rn(wv, nv);
        }
        warp_fwht<G>(v, lig, scale);
        if (valid) {
#pragma unroll
            for (int j = 0; j < S::E; ++j) {
                const int e = g * G + lig * S::E + j;
                if (e < in) y[(size_t)c * in + e] = v[j];
            }
        }
    }
}

__global__ void __launch_bounds__(1024) rows_block_kernel(const uint8_t *__restrict__ packed,
                                                          const uint16_t *__restrict__ norms, int in, int groups,
                                                          int G, int storage_bits, int rowbytes,
                                                          const int64_t *__restrict__ ids, float scale,
                                                          float *__restrict__ y, const float *__restrict__ lut) {
    extern __shared__ float s[];
    const int c = blockIdx.x / groups, g = blockIdx.x % groups;
    const int64_t r = ids[c];
    const uint8_t *p = packed + (size_t)r * rowbytes;
    const float nv = half_bits_to_float(norms[(size_t)r * groups + g]);
    const unsigned mask = (1u << storage_bits) - 1u;
    for (int i = threadIdx.x; i < G; i += blockDim.x) {
        const int e = g * G + i, bit = e * storage_bits, byte = bit >> 3, shift = bit & 7;
        unsigned word = p[byte];
        if (shift + storage_bits > 8) word |= (unsigned)p[byte + 1] << 8;
        s[i] = __fmul_rn(lut[(word >> shift) & mask], nv);
    }
    block_fwht(s, G, scale);
    for (int i = threadIdx.x; i < G; i += blockDim.x) {
        const int e = g * G + i;
        if (e < in) y[(size_t)c * in + e] = s[i];
    }
}

}  // namespace

bool launch_rows(const CQDevice &w, const int64_t *ids, int count, float *y, cudaStream_t st) {
    if (count <= 0) return true;
    const float scale = 1.0f / sqrtf((float)w.group);
    const long long items = (long long)count * w.groups;
    const float4 l0 = make_float4(w.lut[0], w.lut[1], w.lut[2], w.lut[3]);
    const float4 l1 = make_float4(w.lut[4], w.lut[5], w.lut[6], w.lut[7]);
    const float4 l2 = make_float4(w.lut[8], w.lut[9], w.lut[10], w.lut[11]);
    const float4 l3 = make_float4(w.lut[12], w.lut[13], w.lut[14], w.lut[15]);
    auto warp_launch = [&](auto kernel, int per_warp) {
        long long warps = (items + per_warp - 1) / per_warp;
        int blocks = (int)std::min<long long>((warps + 7) / 8, 65535);
        kernel<<<blocks, 256, 0, st>>>(w.packed, w.norms, w.in, w.groups, w.storage_bits, w.rowbytes, ids, count,
                                       scale, y, l0, l1, l2, l3);
    };
    switch (w.group) {
        case 8: warp_launch(rows_warp_kernel<8>, 4); break;
        case 16: warp_launch(rows_warp_kernel<16>, 2); break;
        case 32: warp_launch(rows_warp_kernel<32>, 1); break;
        case 64: warp_launch(rows_warp_kernel<64>, 1); break;
        case 128: warp_launch(rows_warp_kernel<128>, 1); break;
        case 256: warp_launch(rows_warp_kernel<256>, 1); break;
        case 512: warp_launch(rows_warp_kernel<512>, 1); break;
        case 1024: warp_launch(rows_warp_kernel<1024>, 1); break;
        default: {
            if (w.group > kMaxGroup || items > 0x7fffffffLL) {
                set_error("group size above 16384 is not supported by the GPU build");
                return false;
            }
            float *lut = nullptr;
            NB_CUDA_TRY(cudaMallocAsync(&lut, sizeof(float) * 16, st));
            NB_CUDA_TRY(cudaMemcpyAsync(lut, w.lut, sizeof(float) * 16, cudaMemcpyHostToDevice, st));
            size_t smem = sizeof(float) * (size_t)w.group;
            NB_CUDA_TRY(cudaFuncSetAttribute(rows_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            rows_block_kernel<<<(unsigned)items, 1024, smem, st>>>(w.packed, w.norms, w.in, w.groups, w.group,
                                                                  w.storage_bits, w.rowbytes, ids, scale, y, lut);
            NB_CUDA_TRY(cudaFreeAsync(lut, st));
        }
    }
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

namespace {

// One warp per row: a = max|x|; unchanged when a == 0; otherwise
// x = clamp(round_half_even(x / scale), -maxq - 1, maxq) * scale with
// scale = a / maxq, maxq = 2^(bits-1) - 1 (needle2/csrc/engine.cpp:185-191;
// IEEE divide and multiply, so the result is the reference's bit for bit).
__global__ void activation_quant_kernel(float *__restrict__ x, int rows, int dim, int bits) {
    pdl_enter();
    const int warp = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (warp >= rows) return;
    float *xr = x + (size_t)warp * dim;
    float a = 0.f;
    for (int i = lane; i < dim; i += 32) a = fmaxf(a, fabsf(xr[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (!(a > 0.f)) return;
    const int maxq = (1 << (bits - 1)) - 1;
    const float scale = __fdiv_rn(a, (float)maxq), hi = (float)maxq, lo = (float)(-maxq - 1);
    for (int i = lane; i < dim; i += 32) {
        const float r = rintf(__fdiv_rn(xr[i], scale));
        xr[i] = __fmul_rn(fmaxf(lo, fminf(hi, r)), scale);
    }
}

}  // namespace

namespace {

// (value, index) candidates of the greedy scan: the larger value wins, an equal
// one the smaller index; NaN never wins (index INT_MAX marks "none yet").
__device__ __forceinline__ void better(float &v, int &i, float ov, int oi) {
    if (ov > v || (ov == v && oi < i)) {
        v = ov;
        i = oi;
    }
}

// One CTA per row: the reference's sequential scan (best = 0, then every index
// strictly greater than the best so far, needle2/csrc/engine.cpp:1434-1442)
// gives the first index of the maximum over the non-NaN logits, or 0 when
// logits[0] is NaN.  Each thread scans its indices in increasing order, then
// the candidates are reduced with the same order.
__global__ void argmax_kernel(const float *__restrict__ x, int vocab, int ld, int *__restrict__ out) {
    pdl_enter();
    __shared__ float sv[32];
    __shared__ int si[32];
    const float *row = x + (size_t)blockIdx.x * ld;
    const float x0 = row[0];
    if (x0 != x0) {   // NaN first: nothing is ever greater
        if (threadIdx.x == 0) out[blockIdx.x] = 0;
        return;
    }
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
        const float y = row[i];
        if (y > v || (y == v && idx == 0x7fffffff)) {   // first candidate of this thread, or a strictly larger one
            v = y;
            idx = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        better(v, idx, ov, oi);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (lane == 0) {
        sv[warp] = v;
        si[warp] = idx;
    }
    __syncthreads();
    if (warp == 0) {
        v = lane < nw ? sv[lane] : -INFINITY;
        idx = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
            better(v, idx, ov, oi);
        }
        if (lane == 0) out[blockIdx.x] = idx;   // x0 is a candidate, so idx is set
    }
}

}  // namespace

// The same scan with 16-byte loads (rows 16-byte aligned, vocab a multiple of
// 4): thread t of 256 takes the 4-element pieces t, t + 256, ... in increasing
// order, eight loads in flight; the reduction is argmax_kernel's.
__global__ void __launch_bounds__(256) argmax_vec_kernel(const float *__restrict__ x, int vocab, int ld,
                                                         int *__restrict__ out) {
    pdl_enter();
    __shared__ float sv[8];
    __shared__ int si[8];
    const float *row = x + (size_t)blockIdx.x * ld;
    if (row[0] != row[0]) {   // NaN first: nothing is ever greater
        if (threadIdx.x == 0) out[blockIdx.x] = 0;
        return;
    }
    const float4 *r4 = reinterpret_cast<const float4 *>(row);
    const int pieces = vocab / 4;
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int b = threadIdx.x; b < pieces; b += 8 * 256) {
        float4 c[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int k = b + u * 256;
            c[u] = k < pieces ? __ldg(r4 + k) : make_float4(NAN, NAN, NAN, NAN);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i0 = 4 * (b + u * 256);
            const float e[4] = {c[u].x, c[u].y, c[u].z, c[u].w};
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (e[q] > v || (e[q] == v && idx == 0x7fffffff)) {
                    v = e[q];
                    idx = i0 + q;
                }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        better(v, idx, ov, oi);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = v;
        si[warp] = idx;
    }
    __syncthreads();
    if (warp == 0) {
        v = lane < 8 ? sv[lane] : -INFINITY;
        idx = lane < 8 ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
            better(v, idx, ov, oi);
        }
        if (lane == 0) out[blockIdx.x] = idx;   // x0 is a candidate, so idx is set
    }
}

bool launch_argmax(const float *x, int rows, int vocab, int ld, int *out, cudaStream_t st) {
    if (rows <= 0) return true;
    if (vocab % 4 == 0 && ld % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        NB_CUDA_TRY(launch_pdl(argmax_vec_kernel, rows, 256, 0, st, x, vocab, ld, out));
        NB_CUDA_TRY(cudaGetLastError());
        return true;
    }
    NB_CUDA_TRY(launch_pdl(argmax_kernel, rows, 1024, 0, st, x, vocab, ld, out));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_activation_quant(float *x, int rows, int dim, int bits, cudaStream_t st) {
    if (rows <= 0 || dim <= 0 || bits == 0) return true;
    const long long threads = (long long)rows * 32;
    NB_CUDA_TRY(launch_pdl(activation_quant_kernel, (unsigned)((threads + 255) / 256), 256, 0, st, x, rows, dim, bits));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

}  // namespace nb200
