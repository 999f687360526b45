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

// Unit of the row-block copy: 32 bytes where a group's packed bytes are a
// multiple of 32 (one 256-bit load), else 16.
__host__ __device__ constexpr int blocked_unit(int group_bytes) { return group_bytes % 32 == 0 ? 32 : 16; }

// Row-block copy, 16 bytes per thread: byte o of the copy is byte k of unit c
// of row 32 * block + lane, group g (see blocked_bytes); rows past `out` zero.
__global__ void build_blocked_kernel(const uint8_t *__restrict__ packed, const uint16_t *__restrict__ norms,
                                     int out, int groups, int gbytes, int rowbytes, uint8_t *__restrict__ blocked,
                                     uint16_t *__restrict__ normsB, size_t n16, size_t nnorm) {
    const int unit = blocked_unit(gbytes);
    const size_t step = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += step) {
        const size_t o = 16 * i, bg = o / (32 * (size_t)gbytes);
        const int rem = (int)(o % (32 * (size_t)gbytes));
        const int c = rem / (32 * unit), lane = (rem % (32 * unit)) / unit, k = rem % unit;
        const int r = (int)(bg / groups) * 32 + lane, g = (int)(bg % groups);
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r < out)
            v = *reinterpret_cast<const uint4 *>(packed + (size_t)r * rowbytes + (size_t)g * gbytes + c * unit + k);
        *reinterpret_cast<uint4 *>(blocked + o) = v;
    }
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nnorm; i += step) {
        const size_t bg = i / 32;
        const int r = (int)(bg / groups) * 32 + (int)(i % 32), g = (int)(bg % groups);
        normsB[i] = r < out ? norms[(size_t)r * groups + g] : (uint16_t)0;
    }
}

template <int BITS, int G, int MT, int D>
__global__ void __launch_bounds__(kRowsThreads, 2) cq_gemv_rows_kernel(const GemvBatch b, const int total_blocks) {
    constexpr int BYTES = G * BITS / 8;   // packed bytes of one group of one row
    constexpr int CHUNKS = BYTES / 16;
    constexpr int BU = blocked_unit(BYTES);
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
            // the row-block copy holds zero rows past the matrix: all lanes load
            const size_t bg = (size_t)(rowbase / 32) * gpr + g0;
            l_ok = true;
            l_row = b.mat[j].blocked + bg * 32 * BYTES + (size_t)lane * BU;
            l_norm = b.mat[j].normsB + bg * 32 + lane;
        }
    };
    auto load = [&](uint4 (&bf)[CHUNKS], float &nv) {
        if (l_it >= niters) return;
        if (l_ok) {
            const uint8_t *src = l_row + (size_t)l_gi * 32 * BYTES;
#pragma unroll
            for (int c = 0; c < BYTES / BU; ++c) {
                if constexpr (BU == 32)
                    ldg_pair(reinterpret_cast<const uint4 *>(src + c * 32 * BU), bf[2 * c], bf[2 * c + 1]);
                else
                    bf[c] = __ldg(reinterpret_cast<const uint4 *>(src + c * 32 * BU));
            }
            nv = half_bits_to_float(__ldg(l_norm + (size_t)l_gi * 32));
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

// ---- one activation row: product table, one cluster per row block set ----
//
// For a single activation row every group's products lut[c] * rot[i] can be
// tabulated once: P[i][c] (16 entries per element for CQ4, 4 for CQ2).  A
// lane's element term is then one table read (the 16 entries of an element sit
// in 16 consecutive banks, so the lanes of a warp, all at the same element,
// never conflict) and one add; the activation reads and the multiplies leave
// the loop.  The table of all groups does not fit one CTA, so each CTA of a
// cluster of S owns one split of gpr / S groups (its table built once) and
// all S CTAs walk the same row blocks; after each set of 8 row blocks the
// cluster synchronises and rank 0 adds the S partial sums of each row, reading
// the other CTAs' shared memory, in rank order.  Each warp takes kPtabBlocks
// row blocks between two cluster barriers.

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The float at the same shared-memory offset as `local` in cluster CTA `rank`.
__device__ __forceinline__ float ld_cluster(const float *local, uint32_t rank) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(local));
    uint32_t r;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(r) : "memory");
    return v;
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

constexpr size_t kPtabMax = 96 * 1024;   // product-table bytes per CTA (two CTAs per SM)

// CTAs per SM the table kernel is compiled for: as many as fit without
// register spills for the group's register buffers (occupancy hides the
// weight loads' latency; 4 CTAs = 64 registers a thread).
__host__ __device__ constexpr int ptab_min_blocks(int bits, int group) {
    return group * bits / 8 >= 128 ? 2 : (bits == 4 || group == 64 ? 4 : 3);
}
constexpr int kPtabBlocks = 4;           // row blocks a warp takes between two cluster barriers

template <int BITS, int G, int D>
__global__ void __launch_bounds__(kRowsThreads, ptab_min_blocks(BITS, G)) cq_gemv_ptab_kernel(const GemvBatch b, const int total_blocks) {
    constexpr int BYTES = G * BITS / 8;
    constexpr int CHUNKS = BYTES / 16;
    constexpr int BU = blocked_unit(BYTES);
    constexpr int EPW = 32 / BITS;
    constexpr int NC = 1 << BITS;              // table entries per element
    extern __shared__ __align__(16) float ptab_raw[];   // [ng][G][NC] from the first 256-byte boundary
    __shared__ __align__(16) float lut[16];
    __shared__ float part[2][kRowsWarps][kPtabBlocks][32];
    __shared__ int blk_base[kGemvMaxMats + 1];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gpr = b.groups, S = rows_splits(gpr), ng = gpr / S;
    const int split = static_cast<int>(cluster_rank());
    const int g0 = split * ng;
    const int cid = blockIdx.x / S, ncl = gridDim.x / S;
    // a unit: kPtabBlocks consecutive row blocks of one warp
    const int total_units = (total_blocks + kPtabBlocks - 1) / kPtabBlocks;
    const int stride = ncl * kRowsWarps, first = cid * kRowsWarps;
    const int niters = first < total_units ? (total_units - first + stride - 1) / stride : 0;

    pdl_launch_dependents();
    if (tid == 0) {
        int acc = 0;
        for (int j = 0; j < b.nmat; ++j) {
            blk_base[j] = acc;
            acc += (b.mat[j].out + 31) / 32;
        }
        blk_base[b.nmat] = acc;
    }
    if (tid < 16) lut[tid] = b.lut[tid];
    __syncthreads();

    auto locate = [&](int u, int &j, int &rowbase) {
        j = 0;
        while (j + 1 < b.nmat && blk_base[j + 1] <= u) ++j;
        rowbase = (u - blk_base[j]) * 32;
    };

    int l_it = 0, l_k = 0, l_gi = 0;
    bool l_ok = false;
    const uint8_t *l_row = nullptr;
    const uint16_t *l_norm = nullptr;
    auto seek = [&]() {
        l_ok = false;
        const int u = (first + l_it * stride + warp) * kPtabBlocks + l_k;
        if (l_it < niters && u < total_blocks) {
            int j, rowbase;
            locate(u, j, rowbase);
            // the row-block copy holds zero rows past the matrix: all lanes load
            const size_t bg = (size_t)(rowbase / 32) * gpr + g0;
            l_ok = true;
            l_row = b.mat[j].blocked + bg * 32 * BYTES + (size_t)lane * BU;
            l_norm = b.mat[j].normsB + bg * 32 + lane;
        }
    };
    auto load = [&](uint4 (&bf)[CHUNKS], float &nv) {
        if (l_it >= niters) return;
        if (l_ok) {
            const uint8_t *src = l_row + (size_t)l_gi * 32 * BYTES;
#pragma unroll
            for (int c = 0; c < BYTES / BU; ++c) {
                if constexpr (BU == 32)
                    ldg_pair(reinterpret_cast<const uint4 *>(src + c * 32 * BU), bf[2 * c], bf[2 * c + 1]);
                else
                    bf[c] = __ldg(reinterpret_cast<const uint4 *>(src + c * 32 * BU));
            }
            nv = half_bits_to_float(__ldg(l_norm + (size_t)l_gi * 32));
        } else {
            nv = 0.f;
        }
        if (++l_gi == ng) {
            l_gi = 0;
            if (++l_k == kPtabBlocks) {
                l_k = 0;
                ++l_it;
            }
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

    // the table starts on a 256-byte boundary, so a table address is the
    // group's base with the entry offset (< 256) in its low byte
    const uint32_t raw32 = static_cast<uint32_t>(__cvta_generic_to_shared(ptab_raw));
    const uint32_t ptab32 = (raw32 + 255u) & ~255u;
    float *ptab = ptab_raw + (ptab32 - raw32) / 4;

    // the activation row comes from the preceding kernel in the stream
    pdl_wait();
    for (int i = tid; i < ng * G * NC / 4; i += kRowsThreads) {
        const int e = (4 * i) / NC, c = (4 * i) % NC;
        const float xv = b.rot[(size_t)g0 * G + e];
        reinterpret_cast<float4 *>(ptab)[i] =
            make_float4(lut[c] * xv, lut[c + 1] * xv, lut[c + 2] * xv, lut[c + 3] * xv);
    }
    __syncthreads();

    float p = 0.f;
    int c_it = 0, c_k = 0, c_gi = 0, par = 0;

    auto compute = [&](const uint4 (&bf)[CHUNKS], float n) {
        const uint32_t pbase = ptab32 + (uint32_t)c_gi * (G * NC * 4);
        float2 acc = make_float2(0.f, 0.f);
        // table entry of element e whose offset (4 * index) is byte k of `offs`:
        // one byte permute puts it into the low byte of the group's base
        auto at = [&](int e, uint32_t offs, uint32_t k) {
            const uint32_t addr = prmt(offs, pbase, 0x7650u | k) + 4 * NC * e;
            float v;
            asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
            return v;
        };
#pragma unroll
        for (int c = 0; c < CHUNKS; ++c) {
            const uint32_t words[4] = {bf[c].x, bf[c].y, bf[c].z, bf[c].w};
#pragma unroll
            for (int jw = 0; jw < 4; ++jw) {
                const uint32_t w = words[jw];
                const int e0 = (4 * c + jw) * EPW;
                if (BITS == 4) {
                    const uint32_t a = (w << 2) & 0x3C3C3C3Cu, o = (w >> 2) & 0x3C3C3C3Cu;
                    acc = fadd2(acc, make_float2(at(e0 + 0, a, 0), at(e0 + 1, o, 0)));
                    acc = fadd2(acc, make_float2(at(e0 + 2, a, 1), at(e0 + 3, o, 1)));
                    acc = fadd2(acc, make_float2(at(e0 + 4, a, 2), at(e0 + 5, o, 2)));
                    acc = fadd2(acc, make_float2(at(e0 + 6, a, 3), at(e0 + 7, o, 3)));
                } else {
                    const uint32_t q0 = (w << 2) & 0x0C0C0C0Cu, q1 = w & 0x0C0C0C0Cu;
                    const uint32_t q2 = (w >> 2) & 0x0C0C0C0Cu, q3 = (w >> 4) & 0x0C0C0C0Cu;
                    acc = fadd2(acc, make_float2(at(e0 + 0, q0, 0), at(e0 + 1, q1, 0)));
                    acc = fadd2(acc, make_float2(at(e0 + 2, q2, 0), at(e0 + 3, q3, 0)));
                    acc = fadd2(acc, make_float2(at(e0 + 4, q0, 1), at(e0 + 5, q1, 1)));
                    acc = fadd2(acc, make_float2(at(e0 + 6, q2, 1), at(e0 + 7, q3, 1)));
                    acc = fadd2(acc, make_float2(at(e0 + 8, q0, 2), at(e0 + 9, q1, 2)));
                    acc = fadd2(acc, make_float2(at(e0 + 10, q2, 2), at(e0 + 11, q3, 2)));
                    acc = fadd2(acc, make_float2(at(e0 + 12, q0, 3), at(e0 + 13, q1, 3)));
                    acc = fadd2(acc, make_float2(at(e0 + 14, q2, 3), at(e0 + 15, q3, 3)));
                }
            }
        }
        p = fmaf(acc.x + acc.y, n, p);
    };

    auto finish_unit = [&]() {
        cluster_sync();
        for (int k = 0; k < kPtabBlocks; ++k) {
            const int u = (first + c_it * stride + warp) * kPtabBlocks + k;
            if (split == 0 && u < total_blocks) {
                int j, rowbase;
                locate(u, j, rowbase);
                const int row = rowbase + lane, out = b.mat[j].out;
                if (row < out) {
                    float v = part[par][warp][k][lane];
                    for (int s = 1; s < S; ++s) v += ld_cluster(&part[par][warp][k][lane], (uint32_t)s);
                    b.mat[j].y[row] = v;
                }
            }
        }
        par ^= 1;
    };

    const int steps = niters * kPtabBlocks * ng;
    for (int t0 = 0; t0 < steps; t0 += D) {
#pragma unroll
        for (int d = 0; d < D; ++d) {
            if (t0 + d < steps) {   // the same for every thread of the cluster
                compute(buf[d], nv[d]);
                load(buf[d], nv[d]);
                if (++c_gi == ng) {
                    c_gi = 0;
                    part[par][warp][c_k][lane] = p;
                    p = 0.f;
                    if (++c_k == kPtabBlocks) {
                        finish_unit();
                        c_k = 0;
                        ++c_it;
                    }
                }
            }
        }
    }
    // no CTA leaves while rank 0 may still read its partial sums
    cluster_sync();
}

template <int BITS, int G>
bool launch_ptab(const GemvBatch &b, cudaStream_t st) {
    constexpr int D = G * BITS / 8 >= 64 ? 2 : (G * BITS / 8 >= 32 ? 3 : 4);
    auto kernel = cq_gemv_ptab_kernel<BITS, G, D>;
    static bool configured[64] = {};
    int dev = 0;
    NB_CUDA_TRY(cudaGetDevice(&dev));
    const bool cached = dev >= 0 && dev < 64;
    if (!cached || !configured[dev]) {
        NB_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPtabMax + 256));
        if (cached) configured[dev] = true;
    }
    const int S = rows_splits(b.groups);
    const size_t smem = sizeof(float) * (size_t)(b.groups / S) * G * (1 << BITS) + 256;
    int total = 0;
    for (int j = 0; j < b.nmat; ++j) total += (b.mat[j].out + 31) / 32;
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(kRowsThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    // clusters resident at once for this cluster size and table (cached per device)
    static int max_clusters[64][4] = {};
    static size_t max_smem[64][4] = {};
    const int si = S == 8 ? 3 : (S == 4 ? 2 : (S == 2 ? 1 : 0));
    int maxc = cached ? max_clusters[dev][si] : 0;
    if (!cached || max_smem[dev][si] != smem || maxc <= 0) {
        cfg.gridDim = dim3(S);
        NB_CUDA_TRY(cudaOccupancyMaxActiveClusters(&maxc, kernel, &cfg));
        if (maxc <= 0) {
            set_error("FP32 product-table GEMV: no cluster fits on this device");
            return false;
        }
        if (cached) {
            max_clusters[dev][si] = maxc;
            max_smem[dev][si] = smem;
        }
    }
    const int units = (total + kPtabBlocks - 1) / kPtabBlocks;
    const int clusters = std::max(1, std::min((units + kRowsWarps - 1) / kRowsWarps, maxc));
    cfg.gridDim = dim3(clusters * S);
    NB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, b, total));
    return true;
}

template <int BITS, int G, int MT>
bool launch_rows(const GemvBatch &b, cudaStream_t st) {
    constexpr int D = G * BITS / 8 >= 64 ? 2 : (G * BITS / 8 >= 32 ? 3 : 4);
    auto kernel = cq_gemv_rows_kernel<BITS, G, MT, D>;
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

template <int BITS, int G>
bool rows_mt(const GemvBatch &b, cudaStream_t st) {
    if (b.M <= 1) return launch_rows<BITS, G, 1>(b, st);
    if (b.M <= 2) return launch_rows<BITS, G, 2>(b, st);
    return launch_rows<BITS, G, 4>(b, st);
}

bool ptab_fits(const GemvBatch &b) {
    const int S = rows_splits(b.groups);
    return b.M == 1 && sizeof(float) * (size_t)(b.groups / S) * b.group * (1 << b.bits) <= kPtabMax;
}

int g_f32_gemv_kind = 0;

template <int BITS, int G>
bool rows_pick(const GemvBatch &b, cudaStream_t st) {
    if (g_f32_gemv_kind == 0 && ptab_fits(b)) return launch_ptab<BITS, G>(b, st);
    return rows_mt<BITS, G>(b, st);
}

}  // namespace

void set_f32_gemv_kernel(int kind) { g_f32_gemv_kind = kind; }
int f32_gemv_kernel() { return g_f32_gemv_kind; }

size_t blocked_bytes(int out, int groups, int group, int bits) {
    return (size_t)((out + 31) / 32) * 32 * groups * (group * bits / 8);
}

size_t blocked_norm_count(int out, int groups) { return (size_t)((out + 31) / 32) * 32 * groups; }

bool build_blocked_layout(const uint8_t *packed, const uint16_t *norms, int out, int groups, int group, int bits,
                          int rowbytes, uint8_t *blocked, uint16_t *normsB, cudaStream_t st) {
    const int gbytes = group * bits / 8;
    if (gbytes % 16 || rowbytes % 16 || (size_t)rowbytes < (size_t)groups * gbytes) {
        set_error("row-block copy needs 16-byte groups and rows");
        return false;
    }
    build_blocked_kernel<<<148 * 8, 256, 0, st>>>(packed, norms, out, groups, gbytes, rowbytes, blocked, normsB,
                                                   blocked_bytes(out, groups, group, bits) / 16,
                                                   blocked_norm_count(out, groups));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

int gemv_rows_max_rows(int bits, int group, int groups) {
    if ((bits != 2 && bits != 4) || (group != 64 && group != 128 && group != 256) || groups < 1) return 0;
    for (int m : {4, 2, 1})
        if (sizeof(float) * (size_t)m * groups * group <= kRowsMaxX) return m;
    return 0;
}

bool launch_gemv_rows(const GemvBatch &b, cudaStream_t st) {
    bool blocked = true;
    for (int j = 0; j < b.nmat; ++j) blocked = blocked && b.mat[j].blocked && b.mat[j].normsB;
    if (b.nmat < 1 || b.nmat > kGemvMaxMats || b.M < 1 || b.M > gemv_rows_max_rows(b.bits, b.group, b.groups) ||
        b.padded != b.groups * b.group || !blocked) {
        set_error("FP32 row GEMV launch outside its envelope");
        return false;
    }
    if (b.bits == 4) {
        if (b.group == 64) return rows_pick<4, 64>(b, st);
        if (b.group == 128) return rows_pick<4, 128>(b, st);
        return rows_pick<4, 256>(b, st);
    }
    if (b.group == 64) return rows_pick<2, 64>(b, st);
    if (b.group == 128) return rows_pick<2, 128>(b, st);
    return rows_pick<2, 256>(b, st);
}

}  // namespace nb200
