// SDOT (int8) CQ2/CQ4 GEMV for small activation batches (M <= 16) with the
// int8 products on the tensor cores.
//
// Work unit: one weight row, walked in batches of eight consecutive groups.
// In a batch, lane (g, t) of a warp (g = lane / 4, t = lane % 4) loads the
// t-th quarter of group 8*batch + g of the row, so one warp load reads one
// contiguous span of the row (512 bytes for CQ4 / group 128) and a row is
// streamed front to back by consecutive loads of the same warp.  Each lane
// decodes its words in registers to int8 centroids (byte permutes over a 16-
// or 4-entry table); the result is, as it stands, the B fragment of
// mma.sync.m16n8k32 s8 x s8 -> s32 whose column n is group 8*batch + n of the
// row.  Row n of the A operand holds that same group's int8 activations (of
// activation row 2p for A rows 0-7 and 2p+1 for A rows 8-15), read from
// shared memory in the matching k order.  The diagonal of the 16 x 8 result
// is then exactly the int32 group dot d[m, r, g] of the reference
// (needle2/csrc/sdot.cpp:108-137); the off-diagonal products are discarded.
//
// The lane holding a diagonal entry forms the group term
// (float(d) * (half(norm) * cs)) * xs (sdot.cpp:142-149) and parks it in a
// per-warp shared buffer; every few rows the warp sums each row's terms in
// group order, one lane per (activation, row), so outputs are bit-identical
// to the reference.  Weight loads run PF batches ahead across row boundaries.
//
// The tensor-core shape is the legacy warp MMA because the operand is born in
// registers by the decode; the weights stream from HBM once, so the kernel is
// bound by memory and by the integer permutes of the decode, not by MMA rate.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "cq_gemv.cuh"
#include "sm100_async.cuh"

namespace nb200 {
namespace {

constexpr int kMmaThreads = 512;
constexpr int kMmaWarps = kMmaThreads / 32;

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// x >> K as the high half of a product (keeps the shift off the integer pipe,
// which the byte permutes of the decode saturate).
template <int K>
__device__ __forceinline__ uint32_t shr_mul(uint32_t x) {
    return __umulhi(x, 1u << (32 - K));
}

// CQ4 word -> int8 centroids of elements 0..3 (lo4) and 4..7 (hi4).  Two
// permutes pick from entries 0-7 and 8-15, a third selects by index bit 3.
__device__ __forceinline__ void dec4(uint32_t w, const uint32_t (&t)[4], uint32_t &lo4, uint32_t &hi4) {
    const uint32_t sel = w & 0x77777777u;
    const uint32_t comb = (shr_mul<1>(w) & 0x44444444u) | 0x32103210u;  // byte i: i + 4*bit3
    lo4 = prmt(prmt(t[0], t[1], sel), prmt(t[2], t[3], sel), comb);
    const uint32_t sel2 = shr_mul<16>(sel), comb2 = shr_mul<16>(comb);
    hi4 = prmt(prmt(t[0], t[1], sel2), prmt(t[2], t[3], sel2), comb2);
}

// CQ2 word (16 crumbs) -> centroids in bit-plane order: r0 = elements
// 0,2,4,6; r1 = 8..14 even; r2 = 1,3,5,7; r3 = 9..15 odd (the order in which
// the activation quantiser stores CQ2 activations).
__device__ __forceinline__ void dec2(uint32_t w, uint32_t t, uint32_t (&r)[4]) {
    const uint32_t e = w & 0x33333333u, o = shr_mul<2>(w) & 0x33333333u;
    r[0] = prmt(t, t, e);
    r[1] = prmt(t, t, shr_mul<16>(e));
    r[2] = prmt(t, t, o);
    r[3] = prmt(t, t, shr_mul<16>(o));
}

__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// CQ4 word -> the two halves of a sign-split decode: neg = |centroid| of
// elements whose index is 0-7 (0 elsewhere), pos = centroid of elements whose
// index is 8-15 (0 elsewhere), for elements 0..3 (lo) and 4..7 (hi).  A
// permute selector nibble with bit 3 set yields the sign of the selected byte,
// which is 0 for the non-negative tables, so no select step is needed; the
// group dot is then dot(x, pos) - dot(x, neg).
__device__ __forceinline__ void dec4_split(uint32_t w, const uint32_t (&nt)[2], const uint32_t (&pt)[2],
                                           uint32_t &nlo, uint32_t &nhi, uint32_t &plo, uint32_t &phi) {
    const uint32_t wx = w ^ 0x88888888u;
    nlo = prmt(nt[0], nt[1], w);
    nhi = prmt(nt[0], nt[1], shr_mul<16>(w));
    plo = prmt(pt[0], pt[1], wx);
    phi = prmt(pt[0], pt[1], shr_mul<16>(wx));
}

template <int N>
__device__ __forceinline__ void cp_async(void *dst, const void *src, bool valid) {
    const uint32_t d = smem_addr(dst);
    const int n = valid ? N : 0;   // 0: fill with zeros, read nothing
    if constexpr (N == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;" ::"r"(d), "l"(src), "n"(N), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Geometry of one (bits, group) instantiation.
template <int BITS, int G>
struct Geo {
    static constexpr int GB = G * BITS / 8;        // packed bytes of one row-group
    static constexpr int LB = GB / 4;              // bytes of one lane's quarter
    static constexpr int W = LB / 4;               // 32-bit words per lane quarter
    static constexpr int XP = BITS == 4 ? 2 : 4;   // pad words per staged activation group (banks)
    static constexpr int XG = G / 4 + XP;          // staged activation words per group
    static constexpr int XL = BITS == 4 ? 2 * W : 4 * W;   // activation words per lane quarter
    // batches in flight per warp: about 6 KB of weights
    static constexpr int PF = 6144 / (32 * LB) < 4 ? 4 : (6144 / (32 * LB) > 16 ? 16 : 6144 / (32 * LB));
};

template <int W>
struct Words {
    uint32_t v[W];
};

template <int W>
__device__ __forceinline__ Words<W> lds_words(const uint8_t *p) {
    Words<W> r;
    if constexpr (W == 1) {
        r.v[0] = *reinterpret_cast<const uint32_t *>(p);
    } else if constexpr (W == 2) {
        const uint2 u = *reinterpret_cast<const uint2 *>(p);
        r.v[0] = u.x; r.v[1] = u.y;
    } else {
#pragma unroll
        for (int i = 0; i < W; i += 4) {
            const uint4 u = reinterpret_cast<const uint4 *>(p)[i / 4];
            r.v[i] = u.x; r.v[i + 1] = u.y; r.v[i + 2] = u.z; r.v[i + 3] = u.w;
        }
    }
    return r;
}

// Shared memory of one launch, in bytes from the start: per warp a weight ring
// [PF][32 lanes][LB] and a norm ring [PF][8] words; staged activations
// [2*MP][groups][XG] words; scales [2*MP][groups]; per warp a term buffer
// [M*R][groups + 1] and the R row ids it belongs to.
struct MmaSmem {
    size_t ring, nring, x, xs, terms, frow, total, terms_per_warp;
};

__host__ __device__ inline MmaSmem mma_smem(int G, int bits, int groups, int mp, int M, int R) {
    MmaSmem s;
    const int lb = G * bits / 32;
    const int pf = 6144 / (32 * lb) < 4 ? 4 : (6144 / (32 * lb) > 16 ? 16 : 6144 / (32 * lb));
    const int xg = G / 4 + (bits == 4 ? 2 : 4);
    s.terms_per_warp = (size_t)M * R * (groups + 1);
    s.ring = 0;
    s.nring = s.ring + (size_t)kMmaWarps * pf * 32 * lb;
    s.x = s.nring + (size_t)kMmaWarps * pf * 8 * 4;
    s.xs = s.x + 4 * (size_t)2 * mp * groups * xg;
    s.terms = s.xs + 4 * (size_t)2 * mp * groups;
    s.frow = s.terms + 4 * (size_t)kMmaWarps * s.terms_per_warp;
    s.total = s.frow + 4 * (size_t)kMmaWarps * R;
    return s;
}

// MT: the exact number of activation rows for MT <= 4, an upper bound (rows
// in b.M) for MT = 8 or 16.  SPLIT: sign-split CQ4 decode.
template <int BITS, int G, int MT, bool SPLIT>
__global__ void __launch_bounds__(kMmaThreads, 1)
    cq_gemv_mma_kernel(const __grid_constant__ GemvBatch b, const int total_rows, const int R) {
    using Gm = Geo<BITS, G>;
    constexpr int W = Gm::W, LB = Gm::LB, PF = Gm::PF;
    constexpr int MP = (MT + 1) / 2;   // activation-row pairs (A rows 0-7 / 8-15)
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ int row_base[kGemvMaxMats + 1];

    const int gpr = b.groups, M = MT <= 4 ? MT : b.M;
    const int nb = (gpr + 7) >> 3;   // batches per row
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const bool diag = t == (g >> 1);   // lane holding C[g][g]: element g & 1 of c0/c1 (c2/c3 for A rows 8-15)
    const MmaSmem L = mma_smem(G, BITS, gpr, MP, M, R);
    const int xrow = gpr * Gm::XG;
    uint8_t *wring = smem + L.ring + (size_t)warp * PF * 32 * LB + lane * LB;   // + slot * 32 * LB
    uint32_t *nring = reinterpret_cast<uint32_t *>(smem + L.nring) + warp * PF * 8 + g;   // + slot * 8
    const uint32_t *x_s = reinterpret_cast<const uint32_t *>(smem + L.x);
    float *xs_s = reinterpret_cast<float *>(smem + L.xs);
    float *terms = reinterpret_cast<float *>(smem + L.terms) + (size_t)warp * L.terms_per_warp;
    int *frow = reinterpret_cast<int *>(smem + L.frow) + warp * R;
    const int tst = gpr + 1;

    const int s0 = (int)((long long)total_rows * blockIdx.x / gridDim.x);
    const int s1 = (int)((long long)total_rows * (blockIdx.x + 1) / gridDim.x);

    pdl_launch_dependents();
    if (tid == 0) {
        int acc = 0;
        for (int j = 0; j < b.nmat; ++j) {
            row_base[j] = acc;
            acc += b.mat[j].out;
        }
        row_base[b.nmat] = acc;
    }
    __syncthreads();

    // Load cursor: rows s0 + warp, s0 + warp + kMmaWarps, ...; PF batches
    // ahead of the consumer.  One commit group per batch (empty past the end).
    int lrow = s0 + warp, ljb = 0, lmat = 0, lslot = 0;
    const uint8_t *lw = nullptr, *lw0 = nullptr;
    const uint32_t *ln = nullptr;
    auto lseek = [&]() {
        if (lrow < s1) {
            while (lmat + 1 < b.nmat && lrow >= row_base[lmat + 1]) ++lmat;
            const GemvMatrix &m = b.mat[lmat];
            const size_t r = (size_t)(lrow - row_base[lmat]);
            lw0 = m.packed + r * b.rowbytes + t * LB;
            lw = lw0 + g * Gm::GB;
            ln = reinterpret_cast<const uint32_t *>(m.norms8 + r * (size_t)(nb * 8)) + (g >> 1);
        }
    };
    auto issue = [&]() {
        if (lrow < s1) {
            const bool ok = ljb * 8 + g < gpr;
            uint8_t *dst = wring + (size_t)lslot * 32 * LB;
            const uint8_t *src = ok ? lw : lw0;
#pragma unroll
            for (int c = 0; c < (LB > 16 ? LB / 16 : 1); ++c) {
                constexpr int N = LB > 16 ? 16 : LB;
                cp_async<N>(dst + c * 16, src + c * 16, ok);
            }
            if (diag) cp_async<4>(nring + lslot * 8, ln, true);
            lw += 8 * Gm::GB;
            ln += 4;
            if (++ljb == nb) {
                ljb = 0;
                lrow += kMmaWarps;
                lseek();
            }
        }
        cp_async_commit();
        lslot = lslot + 1 == PF ? 0 : lslot + 1;
    };
    lseek();
    // the weights do not depend on the preceding kernel: start streaming them
    // before waiting for its activations
    for (int p = 0; p < PF; ++p) issue();

    pdl_wait();
    {
        uint32_t *xw = reinterpret_cast<uint32_t *>(smem + L.x);
        const int cpg = G / 16;   // 16-byte chunks per group
        for (int i = tid; i < 2 * MP * gpr * cpg; i += kMmaThreads) {
            const int m = i / (gpr * cpg), rem = i % (gpr * cpg), grp = rem / cpg, c = rem % cpg;
            int4 v = make_int4(0, 0, 0, 0);
            if (m < M) v = *reinterpret_cast<const int4 *>(b.q + (size_t)m * b.padded + (size_t)grp * G + 16 * c);
            uint32_t *d = xw + (size_t)m * xrow + grp * Gm::XG + 4 * c;
            reinterpret_cast<uint2 *>(d)[0] = make_uint2((uint32_t)v.x, (uint32_t)v.y);
            reinterpret_cast<uint2 *>(d)[1] = make_uint2((uint32_t)v.z, (uint32_t)v.w);
        }
        for (int i = tid; i < 2 * MP * gpr; i += kMmaThreads) xs_s[i] = i < M * gpr ? b.xs[i] : 0.f;
    }
    __syncthreads();

    const uint32_t ctab[4] = {b.ctab[0], b.ctab[1], b.ctab[2], b.ctab[3]};
    const uint32_t ntab[2] = {b.ntab[0], b.ntab[1]}, ptab[2] = {b.ptab[0], b.ptab[1]};
    const float cs = b.cs;

    int crow = s0 + warp, cjb = 0, cslot = 0, nrows = 0;
    while (crow < s1) {
        cp_async_wait<PF - 1>();
        const Words<W> wv = lds_words<W>(wring + (size_t)cslot * 32 * LB);
        const uint32_t nw = nring[cslot * 8];
        const int grp = cjb * 8 + g;
        const uint32_t *xp = x_s + min(grp, gpr - 1) * Gm::XG + t * Gm::XL;
        int c[MP][4], cn[SPLIT ? MP : 1][4];
#pragma unroll
        for (int q = 0; q < MP; ++q) {
            c[q][0] = c[q][1] = c[q][2] = c[q][3] = 0;
            if (SPLIT) cn[q][0] = cn[q][1] = cn[q][2] = cn[q][3] = 0;
        }
#pragma unroll
        for (int i = 0; i < W; ++i) {
            if constexpr (BITS == 4) {
                uint32_t lo, hi, nlo = 0, nhi = 0;
                if constexpr (SPLIT)
                    dec4_split(wv.v[i], ntab, ptab, nlo, nhi, lo, hi);
                else
                    dec4(wv.v[i], ctab, lo, hi);
#pragma unroll
                for (int q = 0; q < MP; ++q) {
                    const uint2 x0 = *reinterpret_cast<const uint2 *>(xp + (size_t)(2 * q) * xrow + 2 * i);
                    const bool second = MT <= 4 ? 2 * q + 1 < MT : 2 * q + 1 < M;
                    const uint2 x1 = second ? *reinterpret_cast<const uint2 *>(xp + (size_t)(2 * q + 1) * xrow + 2 * i)
                                            : make_uint2(0u, 0u);
                    mma_s8(c[q], x0.x, x1.x, x0.y, x1.y, lo, hi);
                    if constexpr (SPLIT) mma_s8(cn[q], x0.x, x1.x, x0.y, x1.y, nlo, nhi);
                }
            } else {
                uint32_t r[4];
                dec2(wv.v[i], ctab[0], r);
#pragma unroll
                for (int q = 0; q < MP; ++q) {
                    const uint4 x0 = *reinterpret_cast<const uint4 *>(xp + (size_t)(2 * q) * xrow + 4 * i);
                    const bool second = MT <= 4 ? 2 * q + 1 < MT : 2 * q + 1 < M;
                    const uint4 x1 = second ? *reinterpret_cast<const uint4 *>(xp + (size_t)(2 * q + 1) * xrow + 4 * i)
                                            : make_uint4(0u, 0u, 0u, 0u);
                    mma_s8(c[q], x0.x, x1.x, x0.y, x1.y, r[0], r[1]);
                    mma_s8(c[q], x0.z, x1.z, x0.w, x1.w, r[2], r[3]);
                }
            }
        }
        // the slot's words and norm are in registers and used: refill it
        const float nv = half_bits_to_float((uint16_t)((g & 1) ? nw >> 16 : nw & 0xffffu));
        issue();
        cslot = cslot + 1 == PF ? 0 : cslot + 1;
        if (diag && grp < gpr) {
            const float ns = __fmul_rn(nv, cs);
#pragma unroll
            for (int q = 0; q < MP; ++q) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int m = 2 * q + h;
                    if (MT <= 4 ? m < MT : m < M) {
                        int d = (g & 1) ? c[q][2 * h + 1] : c[q][2 * h];
                        if constexpr (SPLIT) d -= (g & 1) ? cn[q][2 * h + 1] : cn[q][2 * h];
                        terms[(m * R + nrows) * tst + grp] =
                            __fmul_rn(__fmul_rn(__int2float_rn(d), ns), xs_s[m * gpr + grp]);
                        if (b.partials) b.partials[((size_t)m * b.mat[0].out + crow) * gpr + grp] = d;
                    }
                }
            }
        }
        if (++cjb == nb) {
            cjb = 0;
            if (lane == 0) frow[nrows] = crow;
            ++nrows;
            crow += kMmaWarps;
            if (nrows == R || crow >= s1) {
                __syncwarp();
                // one lane per (activation row, weight row): the group terms in order
                for (int l = lane; l < M * nrows; l += 32) {
                    const int m = l / nrows, r = l % nrows;
                    const float *tr = terms + (m * R + r) * tst;
                    float v = 0.f;
#pragma unroll 4
                    for (int j = 0; j < gpr; ++j) v = __fadd_rn(v, tr[j]);
                    const int row = frow[r];
                    int mi = 0;
                    while (mi + 1 < b.nmat && row >= row_base[mi + 1]) ++mi;
                    const GemvMatrix &mat = b.mat[mi];
                    mat.y[(size_t)m * mat.out + (row - row_base[mi])] = v;
                }
                __syncwarp();
                nrows = 0;
            }
        }
    }
    cp_async_wait<0>();
}

// Activation-row pairs per MMA, rows summed per flush and the shared memory
// they need, for M activation rows (false: does not fit).
bool mma_plan(int G, int bits, int groups, int M, int &mt, int &R, size_t &smem) {
    mt = M <= 4 ? M : M <= 8 ? 8 : 16;
    for (int r : {8, 4, 2, 1}) {
        if (M * r > 32 && r > 1) continue;
        const MmaSmem s = mma_smem(G, bits, groups, (mt + 1) / 2, M, r);
        if (s.total <= (size_t)kGemvMaxSmem) {
            R = r;
            smem = s.total;
            return true;
        }
    }
    return false;
}

template <int BITS, int G, int MT, bool SPLIT>
bool launch_mma(const GemvBatch &b, int R, size_t smem, cudaStream_t st) {
    auto kernel = cq_gemv_mma_kernel<BITS, G, MT, SPLIT>;
    static bool configured[64] = {};
    static int sms[64] = {};
    int dev = 0;
    NB_CUDA_TRY(cudaGetDevice(&dev));
    const bool cached = dev >= 0 && dev < 64;
    if (!cached || !configured[dev]) {
        NB_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxSmem));
        int n = 148;
        NB_CUDA_TRY(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        if (cached) {
            configured[dev] = true;
            sms[dev] = n;
        }
    }
    int total = 0;
    for (int j = 0; j < b.nmat; ++j) total += b.mat[j].out;
    const int grid = std::max(1, std::min((total + kMmaWarps - 1) / kMmaWarps, cached ? sms[dev] : 148));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kMmaThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, b, total, R));
    return true;
}

template <int BITS, int G, bool SPLIT>
bool launch_mma_rows(const GemvBatch &b, int mt, int R, size_t smem, cudaStream_t st) {
    switch (mt) {
        case 1: return launch_mma<BITS, G, 1, SPLIT>(b, R, smem, st);
        case 2: return launch_mma<BITS, G, 2, SPLIT>(b, R, smem, st);
        case 3: return launch_mma<BITS, G, 3, SPLIT>(b, R, smem, st);
        case 4: return launch_mma<BITS, G, 4, SPLIT>(b, R, smem, st);
        case 8: return launch_mma<BITS, G, 8, SPLIT>(b, R, smem, st);
        default: return launch_mma<BITS, G, 16, SPLIT>(b, R, smem, st);
    }
}

template <int G>
bool launch_mma_cq4(const GemvBatch &b, int mt, int R, size_t smem, cudaStream_t st) {
    return b.split ? launch_mma_rows<4, G, true>(b, mt, R, smem, st) : launch_mma_rows<4, G, false>(b, mt, R, smem, st);
}

}  // namespace

int gemv_mma_max_rows(int bits, int group, int groups) {
    if ((bits != 2 && bits != 4) || (group != 64 && group != 128 && group != 256) || groups < 1) return 0;
    for (int m : {16, 8, 4, 2, 1}) {
        int mt, R;
        size_t smem;
        if (mma_plan(group, bits, groups, m, mt, R, smem)) return m;
    }
    return 0;
}

bool launch_gemv_mma(const GemvBatch &b, cudaStream_t st) {
    int mt = 0, R = 0;
    size_t smem = 0;
    if (b.nmat < 1 || b.nmat > kGemvMaxMats || b.M < 1 || b.M > gemv_mma_max_rows(b.bits, b.group, b.groups) ||
        b.rowbytes % 16 || (b.partials && b.nmat != 1) || !mma_plan(b.group, b.bits, b.groups, b.M, mt, R, smem)) {
        set_error("int8 GEMV launch outside the tensor-core kernel's envelope");
        return false;
    }
    for (int j = 0; j < b.nmat; ++j)
        if (!b.mat[j].norms8) {
            set_error("int8 GEMV launch without the 8-group norm layout");
            return false;
        }
    if (b.bits == 4) {
        if (b.group == 64) return launch_mma_cq4<64>(b, mt, R, smem, st);
        if (b.group == 128) return launch_mma_cq4<128>(b, mt, R, smem, st);
        return launch_mma_cq4<256>(b, mt, R, smem, st);
    }
    if (b.group == 64) return launch_mma_rows<2, 64, false>(b, mt, R, smem, st);
    if (b.group == 128) return launch_mma_rows<2, 128, false>(b, mt, R, smem, st);
    return launch_mma_rows<2, 256, false>(b, mt, R, smem, st);
}

}  // namespace nb200
