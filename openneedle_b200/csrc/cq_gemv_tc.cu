// SDOT (int8) CQ2/CQ4 GEMV for small activation batches (M <= 16) on the
// sm_100a tensor cores (tcgen05.mma kind::i8, A in tensor memory).
//
// Work unit: a tile of 128 consecutive weight rows of one matrix, walked group
// by group.  A CTA runs two independent pipelines (one per tile stream), each
// of six warps:
//   * producer warp: 1-D bulk copies (cp.async.bulk) of the tile's packed rows,
//     a stage of SG groups at a time, into padded shared-memory rows (a row's
//     bytes of one stage arrive as one contiguous request);
//   * four decode warps: thread r owns tile row r, which is TMEM lane r.  Per
//     group it decodes its row's packed bytes to int8 centroids (byte permutes
//     over the 16- or 4-entry table) and stores them with tcgen05.st as the A
//     operand (128 rows x G int8) in a TMEM slot;
//   * MMA warp: one thread issues G/32 MMAs D[128 x NB] = A x B per group, B the
//     int8 activations (NB rows, K-major, resident in shared memory), into the
//     slot's own D columns, then commits to the slot's barrier.
// D is exactly the reference's int32 group dot d[m, r, g]
// (needle2/csrc/sdot.cpp:108-137).  Some groups later the decode thread reads
// its lane of D back (tcgen05.ld) and adds (float(d) * (half(norm) * cs)) * xs
// to its row's running sums in group order (sdot.cpp:142-149): outputs are
// bit-identical to the reference and need no cross-thread reduction.
//
// With a sign-split int8 codebook (entries 0-7 <= 0 <= entries 8-15) the CQ4
// decode writes two A halves, |centroid| of the negative entries and the
// positive entries, and the MMA adds A_pos x B + A_neg x (-B).
//
// Every mbarrier wait is bounded; on timeout the CTA raises the device fault
// flag, stops its pipelines and frees its tensor memory.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "cq_gemv.cuh"
#include "tcgen05.cuh"

namespace nb200 {

extern __device__ int g_gemv_fault;

namespace {

constexpr int kPipes = 2;
constexpr int kWarpsPerPipe = 6;                      // 4 decode, 1 producer, 1 MMA
constexpr int kThreads = kPipes * kWarpsPerPipe * 32;  // 384
constexpr int kTile = 128;                             // rows per tile = TMEM lanes
constexpr int kMaxStages = 8;
constexpr int kMaxASlots = 4;
constexpr int kMaxDSlots = 8;
constexpr int kTmemCols = 512;                         // 256 per pipe
constexpr size_t kMaxSmem = 225 * 1024;   // dynamic; the static barriers and ids take about 1 KB more
constexpr uint32_t kWaitLimit = 1u << 23;

// Per pipe: TMEM holds a ring of QA decoded-weight (A) slots followed by a
// ring of QD accumulator (D) slots; the epilogue of group item e runs QD items
// after its decode, so QD >= QA keeps every barrier within one phase of its
// waiter.
struct TcPlan {
    int SG;            // groups per stage
    int S;             // stages per pipe
    int QA, QD;        // A slots, D slots per pipe (QD >= max(QA, 3))
    int dcols;         // D columns per slot: NB, or 2*NB (positive and negative halves)
    int total_tiles;
    uint32_t off_b, off_xs, off_nbuf, off_stage, stage_bytes;   // stage: SG x 128 x gb weights, then SG x 128 norms
    size_t smem;
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

template <int K>
__device__ __forceinline__ uint32_t shr_mul(uint32_t x) {
    return __umulhi(x, 1u << (32 - K));
}

// CQ4 word -> int8 centroids of elements 0..3 (lo) and 4..7 (hi).
__device__ __forceinline__ void dec4(uint32_t w, const uint32_t (&t)[4], uint32_t &lo, uint32_t &hi) {
    const uint32_t sel = w & 0x77777777u;
    const uint32_t comb = (shr_mul<1>(w) & 0x44444444u) | 0x32103210u;
    lo = prmt(prmt(t[0], t[1], sel), prmt(t[2], t[3], sel), comb);
    const uint32_t sel2 = shr_mul<16>(sel), comb2 = shr_mul<16>(comb);
    hi = prmt(prmt(t[0], t[1], sel2), prmt(t[2], t[3], sel2), comb2);
}

// CQ4 sign-split decode: |centroid| where the index is 0-7, centroid where it
// is 8-15, zero elsewhere (a selector nibble with bit 3 set returns the sign of
// a non-negative byte, i.e. 0).
__device__ __forceinline__ void dec4_split(uint32_t w, const uint32_t (&nt)[2], const uint32_t (&pt)[2],
                                           uint32_t &nlo, uint32_t &nhi, uint32_t &plo, uint32_t &phi) {
    const uint32_t wx = w ^ 0x88888888u;
    nlo = prmt(nt[0], nt[1], w);
    nhi = prmt(nt[0], nt[1], shr_mul<16>(w));
    plo = prmt(pt[0], pt[1], wx);
    phi = prmt(pt[0], pt[1], shr_mul<16>(wx));
}

// CQ2 word (16 crumbs) -> centroids in bit-plane order (elements 0,2,4,6 |
// 8..14 even | 1,3,5,7 | 9..15 odd), the order of the stored CQ2 activations.
__device__ __forceinline__ void dec2(uint32_t w, uint32_t t, uint32_t *r) {
    const uint32_t e = w & 0x33333333u, o = shr_mul<2>(w) & 0x33333333u;
    r[0] = prmt(t, t, e);
    r[1] = prmt(t, t, shr_mul<16>(e));
    r[2] = prmt(t, t, o);
    r[3] = prmt(t, t, shr_mul<16>(o));
}

__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    const uint32_t a = smem_addr(bar);
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

__device__ __forceinline__ void named_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

template <int BITS, int G, int NB, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    cq_gemv_tc_kernel(const __grid_constant__ GemvBatch b, const __grid_constant__ TcPlan p) {
    constexpr int GB = G * BITS / 8;                 // packed bytes of one row-group
    constexpr int GW = GB / 4;                       // packed words of one row-group
    constexpr int KK = G / 32;                       // MMA K steps per group
    constexpr int AH = G / 4;                        // A columns of one decode half
    constexpr int ACOLS = (SPLIT ? 2 : 1) * AH;
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ __align__(8) uint64_t bars[kPipes][2 * kMaxStages + kMaxASlots + kMaxDSlots];
    __shared__ uint32_t tmem_base_s;
    __shared__ int tile_base[kGemvMaxMats + 1];
    __shared__ volatile int abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pipe = warp / kWarpsPerPipe, role = warp % kWarpsPerPipe;
    const int gpr = b.groups, M = b.M;
    uint64_t *full = bars[pipe], *empty = full + kMaxStages, *afull = empty + kMaxStages, *mdone = afull + kMaxASlots;

    pdl_launch_dependents();
    if (warp == 0) tc::alloc(&tmem_base_s, kTmemCols);
    if (tid == 0) {
        abort_flag = 0;
        int acc = 0;
        for (int j = 0; j < b.nmat; ++j) {
            tile_base[j] = acc;
            acc += (b.mat[j].out + kTile - 1) / kTile;
        }
        tile_base[b.nmat] = acc;
        for (int q = 0; q < kPipes; ++q) {
            uint64_t *bq = bars[q];
            for (int s = 0; s < p.S; ++s) {
                mbar_init(&bq[s], 1);                // producer arrive + transaction bytes
                mbar_init(&bq[kMaxStages + s], 4);   // one arrive per decode warp
            }
            for (int s = 0; s < p.QA; ++s) mbar_init(&bq[2 * kMaxStages + s], 4);               // A slot written
            for (int s = 0; s < p.QD; ++s) mbar_init(&bq[2 * kMaxStages + kMaxASlots + s], 1);  // MMA commit
        }
        fence_barrier_init();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = tmem_base_s + (uint32_t)(pipe * (kTmemCols / kPipes));
    const uint32_t dbase = (uint32_t)(p.QA * ACOLS);   // first D column of the pipe

    const int tile0 = blockIdx.x * kPipes + pipe, tstep = gridDim.x * kPipes;
    const int ntiles = tile0 < p.total_tiles ? (p.total_tiles - 1 - tile0) / tstep + 1 : 0;
    const int spt = (gpr + p.SG - 1) / p.SG;   // stages per tile
    const int g8 = (gpr + 7) / 8 * 8;
    uint8_t *ring = smem + p.off_stage + (size_t)pipe * p.S * p.stage_bytes;

    if (role == 4) {
        // ---- producer: the weights do not depend on the preceding kernel.  One
        // stage = SG groups of the tile: one contiguous block of the tile-major
        // weights and one of the tile-major norms.
        if (lane == 0) {
            int seq = 0, mi = 0;
            for (int k = 0; k < ntiles && !abort_flag; ++k) {
                const int tile = tile0 + k * tstep;
                while (mi + 1 < b.nmat && tile >= tile_base[mi + 1]) ++mi;
                const GemvMatrix &mat = b.mat[mi];
                const size_t lt = (size_t)(tile - tile_base[mi]);
                for (int sg = 0; sg < spt; ++sg, ++seq) {
                    const int st = seq % p.S;
                    if (seq >= p.S && !wait_bar(&empty[st], (uint32_t)((seq / p.S) - 1) & 1, &abort_flag)) break;
                    const int j0 = sg * p.SG, ng = min(p.SG, gpr - j0);
                    const uint32_t wbytes = (uint32_t)ng * kTile * GB, nbytes = (uint32_t)ng * kTile * 2;
                    mbar_arrive_expect_tx(&full[st], wbytes + nbytes);
                    uint8_t *dst = ring + (size_t)st * p.stage_bytes;
                    bulk_g2s(dst, mat.tiled + ((lt * g8 + j0) * kTile) * GB, wbytes, &full[st]);
                    bulk_g2s(dst + (size_t)p.SG * kTile * GB, mat.normsT + (lt * g8 + j0) * kTile, nbytes, &full[st]);
                }
            }
        }
        __syncwarp();
    } else {
        // ---- decode and MMA warps: stage the activations once (K-major, no swizzle)
        if (role < 4) {
            pdl_wait();
            const int dt = pipe * 128 + role * 32 + lane;   // 0..255 over both pipes' decode warps
            const int cpr = b.padded / 16;                  // 16-byte chunks per activation row
            uint8_t *bs = smem + p.off_b;
            for (int i = dt; i < NB * cpr; i += 256) {
                // consecutive threads fill consecutive 16-byte rows of one core matrix
                const int blk = i / (8 * cpr), rem = i % (8 * cpr), c = rem / 8, n = blk * 8 + rem % 8;
                int4 v = make_int4(0, 0, 0, 0);
                if (n < M) v = *reinterpret_cast<const int4 *>(b.q + (size_t)n * b.padded + 16 * (size_t)c);
                *reinterpret_cast<int4 *>(bs + (size_t)(n & 7) * 16 + (size_t)blk * 8 * b.padded + (size_t)c * 128) = v;
            }
            float *xs_s = reinterpret_cast<float *>(smem + p.off_xs);
            for (int i = dt; i < M * gpr; i += 256) xs_s[i] = b.xs[i];
            fence_proxy_async();
        }
        named_sync(1, kPipes * 5 * 32);

        if (role == 5) {
            // ---- MMA issue (one thread)
            if (lane == 0) {
                const uint32_t idesc = tc::idesc_s8(kTile, NB);
                const uint32_t bsm = smem_addr(smem + p.off_b);
                const uint32_t sbo = 8u * (uint32_t)b.padded;
                int it = 0;
                for (int k = 0; k < ntiles && !abort_flag; ++k) {
                    for (int j = 0; j < gpr; ++j, ++it) {
                        const int sa = it % p.QA, sd = it % p.QD;
                        if (!wait_bar(&afull[sa], (uint32_t)(it / p.QA) & 1, &abort_flag)) break;
                        tc::fence_after();
                        const uint32_t a = tmem + (uint32_t)(sa * ACOLS), d = tmem + dbase + (uint32_t)(sd * p.dcols);
#pragma unroll
                        for (int kk = 0; kk < KK; ++kk) {
                            const uint64_t bd = tc::sdesc(bsm + (uint32_t)(j * (G / 16) + 2 * kk) * 128u, 128, sbo);
                            tc::mma_i8_ts(d, a + kk * 8, bd, idesc, kk > 0);
                            if (SPLIT) tc::mma_i8_ts(d + NB, a + AH + kk * 8, bd, idesc, kk > 0);
                        }
                        tc::commit(&mdone[sd]);
                    }
                }
            }
            __syncwarp();
        } else {
            // ---- decode + epilogue: thread = tile row = TMEM lane
            const int rl = 32 * (warp & 3) + lane;
            const uint32_t lane_bits = (uint32_t)(32 * (warp & 3)) << 16;
            const float *xs_s = reinterpret_cast<const float *>(smem + p.off_xs);
            float *nbuf = reinterpret_cast<float *>(smem + p.off_nbuf) + ((size_t)pipe * kTile + rl) * p.QD;
            const uint32_t ctab[4] = {b.ctab[0], b.ctab[1], b.ctab[2], b.ctab[3]};
            const uint32_t ntab[2] = {b.ntab[0], b.ntab[1]}, ptab[2] = {b.ptab[0], b.ptab[1]};
            const float cs = b.cs;

            // epilogue cursor (items it - QD ...): tile ek, group ej
            int ek = 0, ej = 0, emi = 0;
            int e_row = 0, e_out = 0;
            bool e_valid = false;
            float *e_y = nullptr;
            float accm[NB];
#pragma unroll
            for (int m = 0; m < NB; ++m) accm[m] = 0.f;
            auto e_seek = [&]() {
                if (ek < ntiles) {
                    const int tile = tile0 + ek * tstep;
                    while (emi + 1 < b.nmat && tile >= tile_base[emi + 1]) ++emi;
                    e_out = b.mat[emi].out;
                    e_row = (tile - tile_base[emi]) * kTile + rl;
                    e_valid = e_row < e_out;
                    e_y = b.mat[emi].y;
                }
            };
            e_seek();
            // group dot of item `item` for every activation row, its norm, then the terms
            auto epilogue = [&](int item) {
                const int sd = item % p.QD;
                const uint32_t daddr = tmem + lane_bits + dbase + (uint32_t)(sd * p.dcols);
                int dv[NB];
                if constexpr (NB == 8 && !SPLIT) {
                    uint32_t t[8];
                    tc::ld8(daddr, t);
                    tc::wait_ld();
#pragma unroll
                    for (int m = 0; m < 8; ++m) dv[m] = (int)t[m];
                } else if constexpr (NB == 8) {
                    uint32_t t[16];
                    tc::ld16(daddr, t);
                    tc::wait_ld();
#pragma unroll
                    for (int m = 0; m < 8; ++m) dv[m] = (int)t[m] - (int)t[8 + m];
                } else if constexpr (!SPLIT) {
                    uint32_t t[16];
                    tc::ld16(daddr, t);
                    tc::wait_ld();
#pragma unroll
                    for (int m = 0; m < 16; ++m) dv[m] = (int)t[m];
                } else {
                    uint32_t t[16], u[16];
                    tc::ld16(daddr, t);
                    tc::ld16(daddr + 16, u);
                    tc::wait_ld();
#pragma unroll
                    for (int m = 0; m < 16; ++m) dv[m] = (int)t[m] - (int)u[m];
                }
                const float ns = nbuf[sd];
#pragma unroll
                for (int m = 0; m < NB; ++m)
                    if (m < M)
                        accm[m] = __fadd_rn(accm[m], __fmul_rn(__fmul_rn(__int2float_rn(dv[m]), ns), xs_s[m * gpr + ej]));
                if (b.partials && e_valid) {
#pragma unroll
                    for (int m = 0; m < NB; ++m)
                        if (m < M) b.partials[((size_t)m * e_out + e_row) * gpr + ej] = (int32_t)dv[m];
                }
                if (++ej == gpr) {
                    if (e_valid) {
#pragma unroll
                        for (int m = 0; m < NB; ++m)
                            if (m < M) e_y[(size_t)m * e_out + e_row] = accm[m];
                    }
#pragma unroll
                    for (int m = 0; m < NB; ++m) accm[m] = 0.f;
                    ej = 0;
                    ++ek;
                    e_seek();
                }
            };

            int it = 0, seq = 0;
            bool ok = true;
            const int rows_per_128 = GB < 128 ? 128 / GB : 1;
            const int swz = (rl / rows_per_128) & (GB / 16 - 1);   // this row's chunk swizzle
            for (int k = 0; k < ntiles && ok; ++k) {
                for (int sg = 0; sg < spt && ok; ++sg, ++seq) {
                    const int st = seq % p.S;
                    if (!wait_bar(&full[st], (uint32_t)(seq / p.S) & 1, &abort_flag)) { ok = false; break; }
                    const uint8_t *sbase = ring + (size_t)st * p.stage_bytes;
                    const uint16_t *snorm = reinterpret_cast<const uint16_t *>(sbase + (size_t)p.SG * kTile * GB) + rl;
                    const int ng = min(p.SG, gpr - sg * p.SG);
                    for (int jj = 0; jj < ng; ++jj, ++it) {
                        const int sa = it % p.QA, sd = it % p.QD;
                        if (it >= p.QD) {
                            // D slot sd holds item it - QD, whose MMA is done
                            if (!wait_bar(&mdone[sd], (uint32_t)((it - p.QD) / p.QD) & 1, &abort_flag)) { ok = false; break; }
                            tc::fence_after();
                            epilogue(it - p.QD);
                        }
                        nbuf[sd] = __fmul_rn(half_bits_to_float(snorm[jj * kTile]), cs);
                        if (it >= p.QA) {
                            // A slot sa was read by the MMA of item it - QA
                            const int prev = it - p.QA;
                            if (!wait_bar(&mdone[prev % p.QD], (uint32_t)(prev / p.QD) & 1, &abort_flag)) { ok = false; break; }
                            tc::fence_after();
                        }
                        const uint32_t abase = tmem + lane_bits + (uint32_t)(sa * ACOLS);
                        const uint8_t *src = sbase + ((size_t)jj * kTile + rl) * GB;
#pragma unroll
                        for (int c0 = 0; c0 < GW; c0 += 8) {   // 8 packed words per store batch
                            uint32_t w[8];
#pragma unroll
                            for (int c = 0; c < 8; c += 4) {
                                if (c0 + c < GW) {
                                    const uint4 v =
                                        *reinterpret_cast<const uint4 *>(src + 16 * (((c0 + c) / 4) ^ swz));
                                    w[c] = v.x; w[c + 1] = v.y; w[c + 2] = v.z; w[c + 3] = v.w;
                                } else {
                                    w[c] = w[c + 1] = w[c + 2] = w[c + 3] = 0u;
                                }
                            }
                            if constexpr (BITS == 4) {
                                uint32_t pc[16], nc[16];
#pragma unroll
                                for (int i = 0; i < 8; ++i) {
                                    if constexpr (SPLIT)
                                        dec4_split(w[i], ntab, ptab, nc[2 * i], nc[2 * i + 1], pc[2 * i], pc[2 * i + 1]);
                                    else
                                        dec4(w[i], ctab, pc[2 * i], pc[2 * i + 1]);
                                }
                                tc::st16(abase + (uint32_t)(2 * c0), pc);
                                if (SPLIT) tc::st16(abase + (uint32_t)(AH + 2 * c0), nc);
                            } else {
                                uint32_t pc[32];
#pragma unroll
                                for (int i = 0; i < 8; ++i) dec2(w[i], ctab[0], pc + 4 * i);
                                if (GW - c0 >= 8)
                                    tc::st32(abase + (uint32_t)(4 * c0), reinterpret_cast<const uint32_t(&)[32]>(pc));
                                else
                                    tc::st16(abase + (uint32_t)(4 * c0), pc);
                            }
                        }
                        tc::wait_st();
                        tc::fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&afull[sa]);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[st]);
                }
            }
            if (ok) {
                for (int e = max(0, it - p.QD); e < it; ++e) {
                    if (!wait_bar(&mdone[e % p.QD], (uint32_t)(e / p.QD) & 1, &abort_flag)) break;
                    tc::fence_after();
                    epilogue(e);
                }
            }
        }
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (warp == 0) tc::dealloc(tmem_base_s, kTmemCols);
}

bool make_plan(int bits, int G, int padded, int groups, int M, int total_tiles, bool split, TcPlan &p, int &nb) {
    if (M > 16) return false;
    nb = M <= 8 ? 8 : 16;
    const int gb = G * bits / 8;
    const int acols = (split ? 2 : 1) * G / 4;
    p.dcols = (split ? 2 : 1) * nb;
    const int budget = kTmemCols / kPipes;
    p.QA = 0;
    for (int qa = kMaxASlots; qa >= 2; --qa)
        if (qa * acols + std::max(qa, 4) * p.dcols <= budget) {
            p.QA = qa;
            break;
        }
    if (!p.QA) return false;
    p.QD = std::max(p.QA, std::min(kMaxDSlots, (budget - p.QA * acols) / p.dcols));
    if (p.QD < 3) return false;
    p.total_tiles = total_tiles;
    // most bytes in flight per pipe ((S - 1) stages) that fit in shared memory
    size_t best = 0;
    TcPlan bestp = p;
    const int sg0 = std::max(1, 256 / gb);
    for (int sg = sg0; sg >= 1; sg /= 2) {
        for (int S = kMaxStages; S >= 2; --S) {
            TcPlan q = p;
            size_t off = 0;
            q.off_b = 0;
            off += (size_t)nb * padded;
            q.off_xs = (uint32_t)off;
            off += (size_t)4 * nb * groups;
            off = (off + 15) / 16 * 16;
            q.off_nbuf = (uint32_t)off;
            off += (size_t)4 * kPipes * kTile * q.QD;
            off = (off + 127) / 128 * 128;
            q.off_stage = (uint32_t)off;
            q.SG = sg;
            q.S = S;
            q.stage_bytes = (uint32_t)(((size_t)sg * kTile * (gb + 2) + 127) / 128 * 128);
            off += (size_t)kPipes * S * q.stage_bytes;
            if (off > kMaxSmem) continue;
            q.smem = off;
            const size_t inflight = (size_t)(S - 1) * q.stage_bytes;
            if (inflight > best) {
                best = inflight;
                bestp = q;
            }
            break;   // the largest S that fits for this stage size
        }
        if (sg == 1) break;
    }
    if (!best) return false;
    p = bestp;
    return true;
}

template <int BITS, int G, int NB, bool SPLIT>
bool launch_tc(const GemvBatch &b, const TcPlan &p, cudaStream_t st) {
    auto kernel = cq_gemv_tc_kernel<BITS, G, NB, SPLIT>;
    static bool configured[64] = {};
    static int sms[64] = {};
    int dev = 0;
    NB_CUDA_TRY(cudaGetDevice(&dev));
    const bool cached = dev >= 0 && dev < 64;
    if (!cached || !configured[dev]) {
        NB_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem));
        int n = 148;
        NB_CUDA_TRY(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        if (cached) {
            configured[dev] = true;
            sms[dev] = n;
        }
    }
    const int grid = std::max(1, std::min((p.total_tiles + kPipes - 1) / kPipes, cached ? sms[dev] : 148));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, b, p));
    return true;
}

template <int BITS, int G>
bool launch_tc_geo(const GemvBatch &b, const TcPlan &p, int nb, bool split, cudaStream_t st) {
    if constexpr (BITS == 4) {
        if (split) return nb == 8 ? launch_tc<BITS, G, 8, true>(b, p, st) : launch_tc<BITS, G, 16, true>(b, p, st);
    }
    return nb == 8 ? launch_tc<BITS, G, 8, false>(b, p, st) : launch_tc<BITS, G, 16, false>(b, p, st);
}

int total_tiles_of(const GemvBatch &b) {
    int t = 0;
    for (int j = 0; j < b.nmat; ++j) t += (b.mat[j].out + kTile - 1) / kTile;
    return t;
}

}  // namespace

int gemv_tc_max_rows(int bits, int group, int groups) {
    if ((bits != 2 && bits != 4) || (group != 64 && group != 128 && group != 256) || groups < 1) return 0;
    for (int m : {16, 8}) {
        TcPlan p;
        int nb;
        if (make_plan(bits, group, group * groups, groups, m, 1, false, p, nb)) return m;
    }
    return 0;
}

bool launch_gemv_tc(const GemvBatch &b, cudaStream_t st) {
    if (b.nmat < 1 || b.nmat > kGemvMaxMats || b.M < 1 || (b.partials && b.nmat != 1) || b.rowbytes % 16) {
        set_error("int8 GEMV launch outside the tcgen05 kernel's envelope");
        return false;
    }
    for (int j = 0; j < b.nmat; ++j)
        if (!b.mat[j].tiled || !b.mat[j].normsT) {
            set_error("int8 GEMV launch without the tile-major weight layout");
            return false;
        }
    TcPlan p;
    int nb = 8;
    bool split = b.bits == 4 && b.split;
    const int tiles = total_tiles_of(b);
    if (split && !make_plan(b.bits, b.group, b.padded, b.groups, b.M, tiles, true, p, nb)) split = false;
    if (!split && !make_plan(b.bits, b.group, b.padded, b.groups, b.M, tiles, false, p, nb)) {
        set_error("int8 GEMV geometry does not fit the tcgen05 kernel's shared memory");
        return false;
    }
    if (b.bits == 4) {
        if (b.group == 64) return launch_tc_geo<4, 64>(b, p, nb, split, st);
        if (b.group == 128) return launch_tc_geo<4, 128>(b, p, nb, split, st);
        return launch_tc_geo<4, 256>(b, p, nb, split, st);
    }
    if (b.group == 64) return launch_tc_geo<2, 64>(b, p, nb, false, st);
    if (b.group == 128) return launch_tc_geo<2, 128>(b, p, nb, false, st);
    return launch_tc_geo<2, 256>(b, p, nb, false, st);
}

}  // namespace nb200
