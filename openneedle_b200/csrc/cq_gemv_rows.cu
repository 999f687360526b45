// FP32-mode CQ2/CQ4 GEMV for decode batches (up to 4 activation rows), one
// output row per lane.
//
//   t_g = sum_i lut[idx_i] * rot[i]      y_r = sum_g half(norm_rg) * t_g
// (CQ::linear's FP32 loop, needle2/csrc/cq.cpp:157-164), in FP32 with a different
// association: even and odd elements of a group in the two halves of a paired
// FMA, the row's groups split over S warps whose partial sums are added in
// split order.
//
// Work unit: a row block of 32 consecutive rows of one matrix.  The S warps of
// a unit each walk a contiguous range of gpr / S groups for all 32 rows (lane l
// = row l), so at every step all lanes of a warp multiply by the same activation
// elements: the activation reads are shared-memory broadcasts, and the only
// per-lane shared-memory traffic left is the codebook lookup (a 16-entry table
// in 16 banks, conflict-free).  Each lane keeps the packed bytes of D groups in
// flight in registers.  The S partial sums meet in shared memory (double
// buffered, one CTA barrier per unit) and split 0's warp stores the row.
//
// The slot-per-lane kernel of cq_gemv.cu gives every lane a different group,
// so each of its activation reads is a distinct 16-byte load and the lookups
// and activation reads together hold it to about a fifth of HBM bandwidth.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "cq_gemv.cuh"
#include "sm100_async.cuh"

namespace nb200 {
namespace {

constexpr int kRowsThreads = 256;
constexpr int kRowsWarps = kRowsThreads / 32;
constexpr size_t kRowsMaxX = 96 * 1024;   // activation bytes staged per CTA (two CTAs per SM)

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long r, x, y, z;
    memcpy(&x, &a, 8);
    memcpy(&y, &b, 8);
    memcpy(&z, &c, 8);
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(x), "l"(y), "l"(z));
    float2 o;
    memcpy(&o, &r, 8);
    return o;
}

// Codebook value at byte offset `off` (4 * index) of the shared table.
__device__ __forceinline__ float lut_at(const float *lut, uint32_t off) {
    return *reinterpret_cast<const float *>(reinterpret_cast<const char *>(lut) + off);
}

// Byte k of v, zero-extended.
template <int K>
__device__ __forceinline__ uint32_t byte_of(uint32_t v) {
    return prmt(v, 0u, 0x4440u | K);
}

// Two 16-byte chunks in one 256-bit read-only load (32-byte aligned source):
// a warp's load then touches each of its 32 rows once instead of twice.
__device__ __forceinline__ void ldg_pair(const uint4 *src, uint4 &a, uint4 &b) {
    asm("ld.global.nc.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(a.x), "=r"(a.y), "=r"(a.z), "=r"(a.w), "=r"(b.x), "=r"(b.y), "=r"(b.z), "=r"(b.w)
        : "l"(src));
}

// Largest power of two <= 8 that divides the groups of a row.
__host__ __device__ inline int rows_splits(int groups) {
    int s = 8;
    while (groups % s) s >>= 1;
    return s;
}

template <int BITS, int G, int MT, int D, bool V8>
__global__ void __launch_bounds__(kRowsThreads, 2) cq_gemv_rows_kernel(const GemvBatch b, const int total_blocks) {
    constexpr int BYTES = G * BITS / 8;   // packed bytes of one group of one row
    constexpr int CHUNKS = BYTES / 16;
    constexpr int EPW = 32 / BITS;        // elements per 32-bit word
    extern __shared__ __align__(16) float x_s[];   // [MT][padded]
    __shared__ __align__(16) float lut[16];
    __shared__ float part[2][kRowsWarps][MT][32];
    __shared__ int blk_base[kGemvMaxMats + 1];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gpr = b.groups, S = rows_splits(gpr), ng = gpr / S, RBC = kRowsWarps / S;
    const int split = warp % S, slot = warp / S;
    const int g0 = split * ng;
    const int stride = gridDim.x * RBC;
    const int first = blockIdx.x * RBC;
    const int niters = first < total_blocks ? (total_blocks - first + stride - 1) / stride : 0;

    pdl_launch_dependents();
    if (tid == 0) {
        int acc = 0;
        for (int j = 0; j < b.nmat; ++j) {
            blk_base[j] = acc;
            acc += (b.mat[j].out + 31) / 32;
        }
        blk_base[b.nmat] = acc;
    }
    __syncthreads();

    // row block u -> matrix and first row
    auto locate = [&](int u, int &j, int &rowbase) {
        j = 0;
        while (j + 1 < b.nmat && blk_base[j + 1] <= u) ++j;
        rowbase = (u - blk_base[j]) * 32;
    };

    // load side: iteration l_it, group l_gi of this warp's range
    int l_it = 0, l_gi = 0;
    bool l_ok = false;
    const uint8_t *l_row = nullptr;
    const uint16_t *l_norm = nullptr;
    auto seek = [&]() {
        l_ok = false;
        const int u = first + l_it * stride + slot;
        if (l_it < niters && u < total_blocks) {
            int j, rowbase;
            locate(u, j, rowbase);
            const int row = rowbase + lane;
            if (row < b.mat[j].out) {
                l_ok = true;
                l_row = b.mat[j].packed + (size_t)row * b.rowbytes + (size_t)g0 * BYTES;
                l_norm = b.mat[j].norms + (size_t)row * gpr + g0;
            }
        }
    };
    auto load = [&](uint4 (&bf)[CHUNKS], float &nv) {
        if (l_it >= niters) return;
        if (l_ok) {
            const uint4 *src = reinterpret_cast<const uint4 *>(l_row + (size_t)l_gi * BYTES);
#pragma unroll
            for (int c = 0; c < CHUNKS; c += V8 ? 2 : 1) {
                if constexpr (V8)
                    ldg_pair(src + c, bf[c], bf[c + 1]);
                else
                    bf[c] = __ldg(src + c);
            }
            nv = half_bits_to_float(__ldg(l_norm + l_gi));
        } else {
            nv = 0.f;
        }
        if (++l_gi == ng) {
            l_gi = 0;
            ++l_it;
            seek();
        }
    };

    uint4 buf[D][CHUNKS];
    float nv[D];
    seek();
#pragma unroll
    for (int d = 0; d < D; ++d) {
        nv[d] = 0.f;
#pragma unroll
        for (int c = 0; c < CHUNKS; ++c) buf[d][c] = make_uint4(0u, 0u, 0u, 0u);
        load(buf[d], nv[d]);
    }

    // activations come from the preceding kernel in the stream
    pdl_wait();
    if (tid < 16) lut[tid] = b.lut[tid];
    {
        const int n4 = MT * b.padded / 4;
        const int rows = min(MT, b.M);
        for (int i = tid; i < n4; i += kRowsThreads) {
            const int m = (4 * i) / b.padded;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m < rows) v = *reinterpret_cast<const float4 *>(b.rot + 4 * (size_t)i);
            reinterpret_cast<float4 *>(x_s)[i] = v;
        }
    }
    __syncthreads();

    float p[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) p[m] = 0.f;
    int c_it = 0, c_gi = 0, par = 0;

    // one group of the 32 rows: t_g per row, accumulated into p
    auto compute = [&](const uint4 (&bf)[CHUNKS], float n) {
        const float *xg = x_s + (size_t)(g0 + c_gi) * G;
        float2 acc[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] = make_float2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < CHUNKS; ++c) {
            const uint32_t words[4] = {bf[c].x, bf[c].y, bf[c].z, bf[c].w};
#pragma unroll
            for (int jw = 0; jw < 4; ++jw) {
                const uint32_t w = words[jw];
                const int e0 = (4 * c + jw) * EPW;   // first element of the word in the group
                if (BITS == 4) {
                    // byte k of a / o: 4 * index of element 2k / 2k + 1 of the word
                    const uint32_t a = (w << 2) & 0x3C3C3C3Cu, o = (w >> 2) & 0x3C3C3C3Cu;
                    const float2 w01 = make_float2(lut_at(lut, byte_of<0>(a)), lut_at(lut, byte_of<0>(o)));
                    const float2 w23 = make_float2(lut_at(lut, byte_of<1>(a)), lut_at(lut, byte_of<1>(o)));
                    const float2 w45 = make_float2(lut_at(lut, byte_of<2>(a)), lut_at(lut, byte_of<2>(o)));
                    const float2 w67 = make_float2(lut_at(lut, byte_of<3>(a)), lut_at(lut, byte_of<3>(o)));
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        const float4 xa = *reinterpret_cast<const float4 *>(xg + (size_t)m * b.padded + e0);
                        const float4 xb = *reinterpret_cast<const float4 *>(xg + (size_t)m * b.padded + e0 + 4);
                        acc[m] = ffma2(w01, make_float2(xa.x, xa.y), acc[m]);
                        acc[m] = ffma2(w23, make_float2(xa.z, xa.w), acc[m]);
                        acc[m] = ffma2(w45, make_float2(xb.x, xb.y), acc[m]);
                        acc[m] = ffma2(w67, make_float2(xb.z, xb.w), acc[m]);
                    }
                } else {
                    // byte k of q0..q3: 4 * index of element 4k + 0..3 of the word
                    const uint32_t q0 = (w << 2) & 0x0C0C0C0Cu, q1 = w & 0x0C0C0C0Cu;
                    const uint32_t q2 = (w >> 2) & 0x0C0C0C0Cu, q3 = (w >> 4) & 0x0C0C0C0Cu;
                    float2 wv[8];
                    wv[0] = make_float2(lut_at(lut, byte_of<0>(q0)), lut_at(lut, byte_of<0>(q1)));
                    wv[1] = make_float2(lut_at(lut, byte_of<0>(q2)), lut_at(lut, byte_of<0>(q3)));
                    wv[2] = make_float2(lut_at(lut, byte_of<1>(q0)), lut_at(lut, byte_of<1>(q1)));
                    wv[3] = make_float2(lut_at(lut, byte_of<1>(q2)), lut_at(lut, byte_of<1>(q3)));
                    wv[4] = make_float2(lut_at(lut, byte_of<2>(q0)), lut_at(lut, byte_of<2>(q1)));
                    wv[5] = make_float2(lut_at(lut, byte_of<2>(q2)), lut_at(lut, byte_of<2>(q3)));
                    wv[6] = make_float2(lut_at(lut, byte_of<3>(q0)), lut_at(lut, byte_of<3>(q1)));
                    wv[7] = make_float2(lut_at(lut, byte_of<3>(q2)), lut_at(lut, byte_of<3>(q3)));
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
#pragma unroll
                        for (int h = 0; h < 4; ++h) {
                            const float4 xv =
                                *reinterpret_cast<const float4 *>(xg + (size_t)m * b.padded + e0 + 4 * h);
                            acc[m] = ffma2(wv[2 * h], make_float2(xv.x, xv.y), acc[m]);
                            acc[m] = ffma2(wv[2 * h + 1], make_float2(xv.z, xv.w), acc[m]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) p[m] = fmaf(acc[m].x + acc[m].y, n, p[m]);
    };

    // end of a unit: the S partial sums of each row, added in split order
    auto finish_unit = [&]() {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            part[par][warp][m][lane] = p[m];
            p[m] = 0.f;
        }
        __syncthreads();
        const int u = first + c_it * stride + slot;
        if (split == 0 && u < total_blocks) {
            int j, rowbase;
            locate(u, j, rowbase);
            const int row = rowbase + lane, out = b.mat[j].out;
            if (row < out) {
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m < b.M) {
                        float v = part[par][warp][m][lane];
                        for (int s = 1; s < S; ++s) v += part[par][warp + s][m][lane];
                        b.mat[j].y[(size_t)m * out + row] = v;
                    }
                }
            }
        }
        par ^= 1;
    };

    const int steps = niters * ng;
    for (int t0 = 0; t0 < steps; t0 += D) {
#pragma unroll
        for (int d = 0; d < D; ++d) {
            if (t0 + d < steps) {   // the same for every thread of the CTA
                compute(buf[d], nv[d]);
                load(buf[d], nv[d]);
                if (++c_gi == ng) {
                    finish_unit();
                    c_gi = 0;
                    ++c_it;
                }
            }
        }
    }
}

template <int BITS, int G, int MT, bool V8>
bool launch_rows(const GemvBatch &b, cudaStream_t st) {
    constexpr int D = G * BITS / 8 >= 64 ? 2 : (G * BITS / 8 >= 32 ? 3 : 4);
    auto kernel = cq_gemv_rows_kernel<BITS, G, MT, D, V8>;
    static bool configured[64] = {};
    static int sms[64] = {};
    int dev = 0;
    NB_CUDA_TRY(cudaGetDevice(&dev));
    const bool cached = dev >= 0 && dev < 64;
    if (!cached || !configured[dev]) {
        NB_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRowsMaxX));
        int n = 148;
        NB_CUDA_TRY(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        if (cached) {
            configured[dev] = true;
            sms[dev] = n;
        }
    }
    int total = 0;
    for (int j = 0; j < b.nmat; ++j) total += (b.mat[j].out + 31) / 32;
    const int rbc = kRowsWarps / rows_splits(b.groups);
    const int grid = std::max(1, std::min((total + rbc - 1) / rbc, 2 * (cached ? sms[dev] : 148)));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kRowsThreads);
    cfg.dynamicSmemBytes = sizeof(float) * (size_t)MT * b.padded;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, b, total));
    return true;
}

template <int BITS, int G, bool V8>
bool rows_mt(const GemvBatch &b, cudaStream_t st) {
    if (b.M <= 1) return launch_rows<BITS, G, 1, V8>(b, st);
    if (b.M <= 2) return launch_rows<BITS, G, 2, V8>(b, st);
    return launch_rows<BITS, G, 4, V8>(b, st);
}

// 256-bit weight loads where every row's group bytes start on a 32-byte
// boundary (groups of at least 32 packed bytes, 32-byte rows and bases).
template <int BITS, int G>
bool rows_v8(const GemvBatch &b, cudaStream_t st) {
    bool v8 = G * BITS / 8 >= 32 && b.rowbytes % 32 == 0;
    for (int j = 0; j < b.nmat && v8; ++j) v8 = reinterpret_cast<uintptr_t>(b.mat[j].packed) % 32 == 0;
    if constexpr (G * BITS / 8 >= 32) {
        if (v8) return rows_mt<BITS, G, true>(b, st);
    }
    return rows_mt<BITS, G, false>(b, st);
}

int g_f32_gemv_kind = 0;

}  // namespace

void set_f32_gemv_kernel(int kind) { g_f32_gemv_kind = kind; }
int f32_gemv_kernel() { return g_f32_gemv_kind; }

int gemv_rows_max_rows(int bits, int group, int groups) {
    if ((bits != 2 && bits != 4) || (group != 64 && group != 128 && group != 256) || groups < 1) return 0;
    for (int m : {4, 2, 1})
        if (sizeof(float) * (size_t)m * groups * group <= kRowsMaxX) return m;
    return 0;
}

bool launch_gemv_rows(const GemvBatch &b, cudaStream_t st) {
    if (b.nmat < 1 || b.nmat > kGemvMaxMats || b.M < 1 || b.M > gemv_rows_max_rows(b.bits, b.group, b.groups) ||
        b.rowbytes % 16 || b.padded != b.groups * b.group) {
        set_error("FP32 row GEMV launch outside its envelope");
        return false;
    }
    if (b.bits == 4) {
        if (b.group == 64) return rows_v8<4, 64>(b, st);
        if (b.group == 128) return rows_v8<4, 128>(b, st);
        return rows_v8<4, 256>(b, st);
    }
    if (b.group == 64) return rows_v8<2, 64>(b, st);
    if (b.group == 128) return rows_v8<2, 128>(b, st);
    return rows_v8<2, 256>(b, st);
}

}  // namespace nb200
