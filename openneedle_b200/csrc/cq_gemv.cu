// Persistent CQ2/CQ4 GEMV for B200 (sm_100a), FP32 and SDOT (int8) modes,
// over one matrix or several matrices sharing the input (one launch).
//
// Work unit: one group (G elements) of one row; a "slot" is the rows that one
// warp covers with one unit per lane (32 units: a whole row at 32 groups,
// eight rows at four groups ...).  The slots of all matrices form one list;
// each CTA (one per SM) owns a balanced contiguous range of it and its warps
// take slots from a shared counter.  A warp keeps D slots of packed bytes in
// flight in registers (128-bit read-only loads), computes the group terms of
// the reference,
//   FP32: sum_i cb[idx]*rot[i], times half(norm)      (needle2/csrc/cq.cpp:157-164)
//   SDOT: (float(int32 dot) * (half(norm)*cs)) * xs   (needle2/csrc/sdot.cpp:142-149)
// and one lane per output row adds the row's terms in group order, as the
// reference does (bit-identical SDOT outputs).  No CTA-wide barrier is taken
// after the prologue; the weight loads of the first slots are issued before
// the kernel waits for the preceding (quantise) kernel, whose results it
// needs only for the activations (programmatic dependent launch).
//
// SDOT weights are decoded in registers: CQ4 nibbles index a 16-entry int8
// table through two byte permutes plus a select permute, CQ2 crumbs a
// 4-entry table through one permute; products are dp4a (exact int32).
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "cq_gemv.cuh"
#include "sm100_async.cuh"

namespace nb200 {

__device__ int g_gemv_fault = 0;

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// Right shift by k as the high word of a multiply by 2^(32-k): it issues on
// the multiply-add pipe, leaving the integer pipe (which carries the byte
// permutes and is the decode's bottleneck) to the permutes.
template <int K>
__device__ __forceinline__ uint32_t shr_mul(uint32_t x) {
    return __umulhi(x, 1u << (32 - K));
}

// CQ4 word (8 nibbles, element e in bits 4e..4e+3) -> int8 centroids of
// elements 0..3 (lo4) and 4..7 (hi4).  Two permutes pick from entries 0-7 and
// 8-15 by the low three index bits; a third selects per byte by bit 3.
__device__ __forceinline__ void dec4(uint32_t w, const uint32_t (&t)[4], uint32_t &lo4, uint32_t &hi4) {
    const uint32_t sel = w & 0x77777777u;
    const uint32_t comb = (shr_mul<1>(w) & 0x44444444u) | 0x32103210u;  // byte i: i + 4*bit3
    lo4 = prmt(prmt(t[0], t[1], sel), prmt(t[2], t[3], sel), comb);
    const uint32_t sel2 = shr_mul<16>(sel), comb2 = shr_mul<16>(comb);
    hi4 = prmt(prmt(t[0], t[1], sel2), prmt(t[2], t[3], sel2), comb2);
}

// CQ2 word (16 crumbs) -> centroids in bit-plane order (even elements of the
// word first, then odd), matching the SDOT activation layout.
__device__ __forceinline__ void dec2(uint32_t w, uint32_t t, uint32_t (&r)[4]) {
    const uint32_t e = w & 0x33333333u, o = shr_mul<2>(w) & 0x33333333u;
    r[0] = prmt(t, t, e);
    r[1] = prmt(t, t, shr_mul<16>(e));
    r[2] = prmt(t, t, o);
    r[3] = prmt(t, t, shr_mul<16>(o));
}

template <int BITS, int G>
struct Unit {
    static constexpr int BYTES = G * BITS / 8;  // packed bytes of one group
    static constexpr int CHUNKS = BYTES / 16;   // 16-byte loads of a unit
    static constexpr int EPC = 128 / BITS;      // elements per 16 bytes
};

struct SlotRef {
    int mat, rowbase, nrows;
};

__device__ __forceinline__ SlotRef locate(const GemvBatch &b, const int *base, int s, int rps) {
    int j = 0;
    while (j + 1 < b.nmat && s >= base[j + 1]) ++j;
    SlotRef r;
    r.mat = j;
    r.rowbase = (s - base[j]) * rps;
    r.nrows = min(rps, b.mat[j].out - r.rowbase);
    return r;
}

template <bool I8, int BITS, int G, int MT, int THREADS = kThreads, int D = 2>
__global__ void __launch_bounds__(THREADS, 1) cq_gemv_kernel(const GemvBatch b, const int total_slots,
                                                             const int rps) {
    using U = Unit<BITS, G>;
    constexpr bool XREG = I8 && MT == 1 && G <= 128;   // activation slice held in registers
    constexpr int XG = I8 ? G + 16 : 4 * G + 16;       // padded per-group activation stride (bytes)
    constexpr int BATCH = 4;                           // slots taken from the counter at once
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ float lut[16];
    __shared__ int next_slot;
    __shared__ int slot_base[kGemvMaxMats + 1];

    const int gpr = b.groups, tstride = gpr + 1;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // terms of up to RB buffered rows per activation row; one lane folds each
    const int RB = max(32 / b.M, rps);
    unsigned char *x_s = smem;
    float *xs_s = reinterpret_cast<float *>(x_s + (size_t)b.M * gpr * XG);
    float *terms = xs_s + (I8 ? b.M * gpr : 0) + (size_t)warp * b.M * RB * tstride;

    const int s0 = (int)((long long)total_slots * blockIdx.x / gridDim.x);
    const int s1 = (int)((long long)total_slots * (blockIdx.x + 1) / gridDim.x);

    pdl_launch_dependents();
    if (tid == 0) {
        next_slot = s0;
        int acc = 0;
        for (int j = 0; j < b.nmat; ++j) {
            slot_base[j] = acc;
            acc += (b.mat[j].out + rps - 1) / rps;
        }
        slot_base[b.nmat] = acc;
    }
    __syncthreads();

    const bool active = lane < rps * gpr;
    const int roff = active ? lane / gpr : 0, g = active ? lane % gpr : 0;

    // this warp's slot supply: batches of consecutive slots from the counter
    int batch_pos = 0, batch_end = 0;
    auto next_id = [&]() -> int {
        if (batch_pos >= batch_end) {
            int base = 0;
            if (lane == 0) base = atomicAdd(&next_slot, BATCH);
            base = __shfl_sync(0xffffffffu, base, 0);
            batch_pos = min(base, s1);
            batch_end = min(base + BATCH, s1);
            if (batch_pos >= batch_end) return s1;
        }
        return batch_pos++;
    };
    auto load = [&](int s, SlotRef &r, uint4 (&buf)[U::CHUNKS], float &nv) {
        if (s >= s1) return;
        r = locate(b, slot_base, s, rps);
        if (active && roff < r.nrows) {
            const GemvMatrix &m = b.mat[r.mat];
            const int row = r.rowbase + roff;
            const uint4 *src = reinterpret_cast<const uint4 *>(m.packed + (size_t)row * b.rowbytes + g * U::BYTES);
#pragma unroll
            for (int c = 0; c < U::CHUNKS; ++c) buf[c] = __ldg(src + c);
            nv = half_bits_to_float(__ldg(m.norms + (size_t)row * gpr + g));
        }
    };

    // ring of D slots in flight
    int sid[D];
    SlotRef ref[D];
    uint4 buf[D][U::CHUNKS];
    float nv[D];
#pragma unroll
    for (int d = 0; d < D; ++d) {
        sid[d] = next_id();
        ref[d] = SlotRef{};
        nv[d] = 0.f;
        load(sid[d], ref[d], buf[d], nv[d]);
    }

    // activations come from the preceding kernel in the stream
    pdl_wait();
    if (I8) {
        for (int i = tid; i < b.M * gpr; i += THREADS) xs_s[i] = b.xs[i];
        const int n16 = G / 16;
        for (int i = tid; i < b.M * gpr * n16; i += THREADS) {
            const int m = i / (gpr * n16), rem = i % (gpr * n16), gg = rem / n16, c = rem % n16;
            *reinterpret_cast<int4 *>(x_s + ((size_t)m * gpr + gg) * XG + 16 * c) =
                *reinterpret_cast<const int4 *>(b.q + (size_t)m * b.padded + (size_t)gg * G + 16 * c);
        }
    } else {
        if (tid < 16) lut[tid] = b.lut[tid];
        const int n4 = G / 4;
        for (int i = tid; i < b.M * gpr * n4; i += THREADS) {
            const int m = i / (gpr * n4), rem = i % (gpr * n4), gg = rem / n4, c = rem % n4;
            *reinterpret_cast<float4 *>(x_s + ((size_t)m * gpr + gg) * XG + 16 * c) =
                *reinterpret_cast<const float4 *>(b.rot + (size_t)m * b.padded + (size_t)gg * G + 4 * c);
        }
    }
    __syncthreads();

    const uint32_t ctab[4] = {b.ctab[0], b.ctab[1], b.ctab[2], b.ctab[3]};
    int xr[XREG ? U::CHUNKS * U::EPC / 4 : 1];
    if (XREG) {
#pragma unroll
        for (int i = 0; i < U::CHUNKS * U::EPC / 16; ++i) {
            const int4 v = *reinterpret_cast<const int4 *>(x_s + (size_t)g * XG + 16 * i);
            xr[4 * i] = v.x; xr[4 * i + 1] = v.y; xr[4 * i + 2] = v.z; xr[4 * i + 3] = v.w;
        }
    }

    // buffered rows: lane l remembers (matrix, row) of buffered row l
    int nbuf = 0, my_mat = 0, my_row = 0;
    auto fold = [&]() {
        __syncwarp();
        const int total = b.M * nbuf;
        for (int base = 0; base < total; base += 32) {
            const int idx = base + lane;
            const int m = idx < total ? idx / nbuf : 0, rb = idx < total ? idx - m * nbuf : 0;
            const int mm = __shfl_sync(0xffffffffu, my_mat, rb), rr = __shfl_sync(0xffffffffu, my_row, rb);
            if (idx < total) {
                const float *tr = terms + (m * RB + rb) * tstride;
                float v = 0.f;
                int gg = 0;
                for (; gg + 8 <= gpr; gg += 8) {
                    float t[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) t[j] = tr[gg + j];
#pragma unroll
                    for (int j = 0; j < 8; ++j) v = __fadd_rn(v, t[j]);
                }
                for (; gg < gpr; ++gg) v = __fadd_rn(v, tr[gg]);
                const GemvMatrix &mat = b.mat[mm];
                mat.y[(size_t)m * mat.out + rr] = v;
            }
        }
        __syncwarp();
        nbuf = 0;
    };

    auto compute = [&](const SlotRef &r, const uint4 (&buf)[U::CHUNKS], float nvv) {
        // rows of this slot take buffer rows nbuf .. nbuf + r.nrows - 1
        if (lane >= nbuf && lane < nbuf + r.nrows) {
            my_mat = r.mat;
            my_row = r.rowbase + lane - nbuf;
        }
        if (active && roff < r.nrows) {
            const int row = r.rowbase + roff, rb = nbuf + roff;
            if (I8) {
                int acc[MT];
#pragma unroll
                for (int m = 0; m < MT; ++m) acc[m] = 0;
#pragma unroll
                for (int c = 0; c < U::CHUNKS; ++c) {
                    const uint32_t w[4] = {buf[c].x, buf[c].y, buf[c].z, buf[c].w};
                    uint32_t dd[U::EPC / 4];
                    if (BITS == 4) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) dec4(w[i], ctab, dd[2 * i], dd[2 * i + 1]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            uint32_t q4[4];
                            dec2(w[i], ctab[0], q4);
#pragma unroll
                            for (int k = 0; k < 4; ++k) dd[4 * i + k] = q4[k];
                        }
                    }
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        if (m < b.M) {
#pragma unroll
                            for (int k = 0; k < U::EPC / 16; ++k) {
                                int4 xv;
                                if (XREG) {
                                    const int base = c * U::EPC / 4 + 4 * k;
                                    xv = make_int4(xr[base], xr[base + 1], xr[base + 2], xr[base + 3]);
                                } else {
                                    xv = *reinterpret_cast<const int4 *>(x_s + ((size_t)m * gpr + g) * XG +
                                                                         c * U::EPC + 16 * k);
                                }
                                acc[m] = __dp4a((int)dd[4 * k + 0], xv.x, acc[m]);
                                acc[m] = __dp4a((int)dd[4 * k + 1], xv.y, acc[m]);
                                acc[m] = __dp4a((int)dd[4 * k + 2], xv.z, acc[m]);
                                acc[m] = __dp4a((int)dd[4 * k + 3], xv.w, acc[m]);
                            }
                        }
                    }
                }
                const float ns = __fmul_rn(nvv, b.cs);
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m < b.M) {
                        terms[(m * RB + rb) * tstride + g] =
                            __fmul_rn(__fmul_rn(__int2float_rn(acc[m]), ns), xs_s[m * gpr + g]);
                        if (b.partials) b.partials[((size_t)m * b.mat[0].out + row) * gpr + g] = acc[m];
                    }
                }
            } else {
                float acc[MT];
#pragma unroll
                for (int m = 0; m < MT; ++m) acc[m] = 0.f;
                constexpr unsigned mask = (1u << BITS) - 1u;
                constexpr int EPW = 32 / BITS;  // elements per 32-bit word
#pragma unroll
                for (int c = 0; c < U::CHUNKS; ++c) {
                    const uint32_t w[4] = {buf[c].x, buf[c].y, buf[c].z, buf[c].w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float wf[EPW];
#pragma unroll
                        for (int e = 0; e < EPW; ++e) wf[e] = lut[(w[j] >> (BITS * e)) & mask];
#pragma unroll
                        for (int m = 0; m < MT; ++m) {
                            if (m < b.M) {
                                const float *xp = reinterpret_cast<const float *>(
                                    x_s + ((size_t)m * gpr + g) * XG + 4 * (c * U::EPC + j * EPW));
#pragma unroll
                                for (int e4 = 0; e4 < EPW / 4; ++e4) {
                                    const float4 xv = *reinterpret_cast<const float4 *>(xp + 4 * e4);
                                    acc[m] = fmaf(wf[4 * e4 + 0], xv.x, acc[m]);
                                    acc[m] = fmaf(wf[4 * e4 + 1], xv.y, acc[m]);
                                    acc[m] = fmaf(wf[4 * e4 + 2], xv.z, acc[m]);
                                    acc[m] = fmaf(wf[4 * e4 + 3], xv.w, acc[m]);
                                }
                            }
                        }
                    }
                }
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    if (m < b.M) terms[(m * RB + rb) * tstride + g] = __fmul_rn(acc[m], nvv);
            }
        }
        nbuf += r.nrows;
    };

    // compute the oldest slot, then refill its buffer with the next one
    bool more = sid[0] < s1;
    while (more) {
#pragma unroll
        for (int d = 0; d < D; ++d) {
            if (sid[d] >= s1) {
                more = false;
                break;
            }
            if (nbuf + ref[d].nrows > RB) fold();
            compute(ref[d], buf[d], nv[d]);
            sid[d] = next_id();
            load(sid[d], ref[d], buf[d], nv[d]);
        }
    }
    if (nbuf) fold();
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Shared-memory staged variant: every lane copies its own unit of the next
// slots with cp.async (16-byte pieces) into a per-warp ring of D slot
// buffers, so loads in flight hold no registers and more warps fit per SM.
// A lane only ever reads the bytes it copied itself: no warp-level
// synchronisation is needed between copy and use.  Pieces are read back in a
// lane-rotated order so that the 16-byte shared loads of a warp do not
// collide in banks.
template <bool I8, int BITS, int G, int MT, int THREADS, int D>
__global__ void __launch_bounds__(THREADS, 1) cq_gemv_staged(const GemvBatch b, const int total_slots,
                                                             const int rps) {
    using U = Unit<BITS, G>;
    constexpr int NW = THREADS / 32;
    constexpr bool XREG = I8 && MT == 1 && G <= 128;
    constexpr int XG = I8 ? G + 16 : 4 * G + 16;
    constexpr int BATCH = 4;
    constexpr int SWZ = U::BYTES >= 128 ? 0 : U::BYTES == 64 ? 1 : U::BYTES == 32 ? 2 : 3;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ float lut[16];
    __shared__ int next_slot;
    __shared__ int slot_base[kGemvMaxMats + 1];

    const int gpr = b.groups, tstride = gpr + 1;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int RB = max(16 / b.M, rps);
    // layout: [ring: NW][D][32 lanes][U::BYTES] | x | xs | terms [NW][M][RB][gpr+1]
    unsigned char *ring = smem + (size_t)warp * D * 32 * U::BYTES;
    unsigned char *x_s = smem + (size_t)NW * D * 32 * U::BYTES;
    float *xs_s = reinterpret_cast<float *>(x_s + (size_t)b.M * gpr * XG);
    float *terms = xs_s + (I8 ? b.M * gpr : 0) + (size_t)warp * b.M * RB * tstride;

    const int s0 = (int)((long long)total_slots * blockIdx.x / gridDim.x);
    const int s1 = (int)((long long)total_slots * (blockIdx.x + 1) / gridDim.x);

    pdl_launch_dependents();
    if (tid == 0) {
        next_slot = s0;
        int acc = 0;
        for (int j = 0; j < b.nmat; ++j) {
            slot_base[j] = acc;
            acc += (b.mat[j].out + rps - 1) / rps;
        }
        slot_base[b.nmat] = acc;
    }
    __syncthreads();

    const bool active = lane < rps * gpr;
    const int roff = active ? lane / gpr : 0, g = active ? lane % gpr : 0;
    const int swz = (lane >> SWZ) & (U::CHUNKS - 1);

    int batch_pos = 0, batch_end = 0;
    auto next_id = [&]() -> int {
        if (batch_pos >= batch_end) {
            int base = 0;
            if (lane == 0) base = atomicAdd(&next_slot, BATCH);
            base = __shfl_sync(0xffffffffu, base, 0);
            batch_pos = min(base, s1);
            batch_end = min(base + BATCH, s1);
            if (batch_pos >= batch_end) return s1;
        }
        return batch_pos++;
    };
    // start the copies of slot s into ring buffer d (one commit group per slot)
    auto issue = [&](int s, int d, SlotRef &r, float &nv) {
        if (s < s1) {
            r = locate(b, slot_base, s, rps);
            if (active && roff < r.nrows) {
                const GemvMatrix &m = b.mat[r.mat];
                const int row = r.rowbase + roff;
                const unsigned char *src = m.packed + (size_t)row * b.rowbytes + g * U::BYTES;
                unsigned char *dst = ring + ((size_t)d * 32 + lane) * U::BYTES;
#pragma unroll
                for (int c = 0; c < U::CHUNKS; ++c) cp_async16(dst + 16 * c, src + 16 * c);
                nv = half_bits_to_float(__ldg(m.norms + (size_t)row * gpr + g));
            }
        }
        cp_async_commit();
    };

    int sid[D];
    SlotRef ref[D];
    float nv[D];
#pragma unroll
    for (int d = 0; d < D; ++d) {
        sid[d] = next_id();
        ref[d] = SlotRef{};
        nv[d] = 0.f;
        issue(sid[d], d, ref[d], nv[d]);
    }

    pdl_wait();
    if (I8) {
        for (int i = tid; i < b.M * gpr; i += THREADS) xs_s[i] = b.xs[i];
        const int n16 = G / 16;
        for (int i = tid; i < b.M * gpr * n16; i += THREADS) {
            const int m = i / (gpr * n16), rem = i % (gpr * n16), gg = rem / n16, c = rem % n16;
            *reinterpret_cast<int4 *>(x_s + ((size_t)m * gpr + gg) * XG + 16 * c) =
                *reinterpret_cast<const int4 *>(b.q + (size_t)m * b.padded + (size_t)gg * G + 16 * c);
        }
    } else {
        if (tid < 16) lut[tid] = b.lut[tid];
        const int n4 = G / 4;
        for (int i = tid; i < b.M * gpr * n4; i += THREADS) {
            const int m = i / (gpr * n4), rem = i % (gpr * n4), gg = rem / n4, c = rem % n4;
            *reinterpret_cast<float4 *>(x_s + ((size_t)m * gpr + gg) * XG + 16 * c) =
                *reinterpret_cast<const float4 *>(b.rot + (size_t)m * b.padded + (size_t)gg * G + 4 * c);
        }
    }
    __syncthreads();

    const uint32_t ctab[4] = {b.ctab[0], b.ctab[1], b.ctab[2], b.ctab[3]};
    // this lane's activation pieces, in its rotated piece order
    int xr[XREG ? U::CHUNKS * U::EPC / 4 : 1];
    if (XREG) {
#pragma unroll
        for (int c = 0; c < U::CHUNKS; ++c) {
            const unsigned char *xp = x_s + (size_t)g * XG + (c ^ swz) * U::EPC;
#pragma unroll
            for (int i = 0; i < U::EPC / 16; ++i) {
                const int4 v = *reinterpret_cast<const int4 *>(xp + 16 * i);
                const int base = c * U::EPC / 4 + 4 * i;
                xr[base] = v.x; xr[base + 1] = v.y; xr[base + 2] = v.z; xr[base + 3] = v.w;
            }
        }
    }

    int nbuf = 0, my_mat = 0, my_row = 0;
    auto fold = [&]() {
        __syncwarp();
        const int total = b.M * nbuf;
        for (int base = 0; base < total; base += 32) {
            const int idx = base + lane;
            const int m = idx < total ? idx / nbuf : 0, rb = idx < total ? idx - m * nbuf : 0;
            const int mm = __shfl_sync(0xffffffffu, my_mat, rb), rr = __shfl_sync(0xffffffffu, my_row, rb);
            if (idx < total) {
                const float *tr = terms + (m * RB + rb) * tstride;
                float v = 0.f;
                int gg = 0;
                for (; gg + 8 <= gpr; gg += 8) {
                    float t[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) t[j] = tr[gg + j];
#pragma unroll
                    for (int j = 0; j < 8; ++j) v = __fadd_rn(v, t[j]);
                }
                for (; gg < gpr; ++gg) v = __fadd_rn(v, tr[gg]);
                const GemvMatrix &mat = b.mat[mm];
                mat.y[(size_t)m * mat.out + rr] = v;
            }
        }
        __syncwarp();
        nbuf = 0;
    };

    auto compute = [&](int d, const SlotRef &r, float nvv) {
        if (lane >= nbuf && lane < nbuf + r.nrows) {
            my_mat = r.mat;
            my_row = r.rowbase + lane - nbuf;
        }
        if (active && roff < r.nrows) {
            const int row = r.rowbase + roff, rb = nbuf + roff;
            const unsigned char *ub = ring + ((size_t)d * 32 + lane) * U::BYTES;
            if (I8) {
                // four independent int32 chains per row (exact: integer sums
                // do not depend on order), added together at the end
                int acc4[MT][4];
#pragma unroll
                for (int m = 0; m < MT; ++m)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc4[m][j] = 0;
#pragma unroll
                for (int c = 0; c < U::CHUNKS; ++c) {
                    const int cc = c ^ swz;
                    const uint4 wv = *reinterpret_cast<const uint4 *>(ub + 16 * cc);
                    const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
                    uint32_t dd[U::EPC / 4];
                    if (BITS == 4) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) dec4(w[i], ctab, dd[2 * i], dd[2 * i + 1]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            uint32_t q4[4];
                            dec2(w[i], ctab[0], q4);
#pragma unroll
                            for (int k = 0; k < 4; ++k) dd[4 * i + k] = q4[k];
                        }
                    }
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        if (m < b.M) {
#pragma unroll
                            for (int k = 0; k < U::EPC / 16; ++k) {
                                int4 xv;
                                if (XREG) {
                                    const int base = c * U::EPC / 4 + 4 * k;
                                    xv = make_int4(xr[base], xr[base + 1], xr[base + 2], xr[base + 3]);
                                } else {
                                    xv = *reinterpret_cast<const int4 *>(x_s + ((size_t)m * gpr + g) * XG +
                                                                         cc * U::EPC + 16 * k);
                                }
                                acc4[m][0] = __dp4a((int)dd[4 * k + 0], xv.x, acc4[m][0]);
                                acc4[m][1] = __dp4a((int)dd[4 * k + 1], xv.y, acc4[m][1]);
                                acc4[m][2] = __dp4a((int)dd[4 * k + 2], xv.z, acc4[m][2]);
                                acc4[m][3] = __dp4a((int)dd[4 * k + 3], xv.w, acc4[m][3]);
                            }
                        }
                    }
                }
                const float ns = __fmul_rn(nvv, b.cs);
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m < b.M) {
                        const int acc = (acc4[m][0] + acc4[m][1]) + (acc4[m][2] + acc4[m][3]);
                        terms[(m * RB + rb) * tstride + g] =
                            __fmul_rn(__fmul_rn(__int2float_rn(acc), ns), xs_s[m * gpr + g]);
                        if (b.partials) b.partials[((size_t)m * b.mat[0].out + row) * gpr + g] = acc;
                    }
                }
            } else {
                float acc[MT];
#pragma unroll
                for (int m = 0; m < MT; ++m) acc[m] = 0.f;
                constexpr unsigned mask = (1u << BITS) - 1u;
                constexpr int EPW = 32 / BITS;
#pragma unroll
                for (int c = 0; c < U::CHUNKS; ++c) {
                    const int cc = c ^ swz;
                    const uint4 wv = *reinterpret_cast<const uint4 *>(ub + 16 * cc);
                    const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float wf[EPW];
#pragma unroll
                        for (int e = 0; e < EPW; ++e) wf[e] = lut[(w[j] >> (BITS * e)) & mask];
#pragma unroll
                        for (int m = 0; m < MT; ++m) {
                            if (m < b.M) {
                                const float *xp = reinterpret_cast<const float *>(
                                    x_s + ((size_t)m * gpr + g) * XG + 4 * (cc * U::EPC + j * EPW));
#pragma unroll
                                for (int e4 = 0; e4 < EPW / 4; ++e4) {
                                    const float4 xv = *reinterpret_cast<const float4 *>(xp + 4 * e4);
                                    acc[m] = fmaf(wf[4 * e4 + 0], xv.x, acc[m]);
                                    acc[m] = fmaf(wf[4 * e4 + 1], xv.y, acc[m]);
                                    acc[m] = fmaf(wf[4 * e4 + 2], xv.z, acc[m]);
                                    acc[m] = fmaf(wf[4 * e4 + 3], xv.w, acc[m]);
                                }
                            }
                        }
                    }
                }
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    if (m < b.M) terms[(m * RB + rb) * tstride + g] = __fmul_rn(acc[m], nvv);
            }
        }
        nbuf += r.nrows;
    };

    bool more = sid[0] < s1;
    while (more) {
#pragma unroll
        for (int d = 0; d < D; ++d) {
            if (sid[d] >= s1) {
                more = false;
                break;
            }
            cp_async_wait<D - 1>();   // this lane's copies of the oldest slot have landed
            if (nbuf + ref[d].nrows > RB) fold();
            compute(d, ref[d], nv[d]);
            sid[d] = next_id();
            issue(sid[d], d, ref[d], nv[d]);
        }
    }
    cp_async_wait<0>();
    if (nbuf) fold();
}

int rows_per_slot(int groups) { return 32 / groups; }

size_t smem_bytes(int M, int groups, int group, bool i8, int warps = kWarps) {
    const size_t x = (size_t)M * groups * (i8 ? group + 16 : 4 * group + 16);
    const size_t xs = i8 ? 4 * (size_t)M * groups : 0;
    const int rb = std::max(32 / M, rows_per_slot(groups));
    const size_t terms = 4 * (size_t)warps * M * rb * (groups + 1);
    return x + xs + terms;
}

// Dynamic shared memory of cq_gemv_staged (same layout as in the kernel).
size_t staged_smem_bytes(int M, int groups, int group, int bits, bool i8, int warps, int depth) {
    const size_t ring = (size_t)warps * depth * 32 * (group * bits / 8);
    const size_t x = (size_t)M * groups * (i8 ? group + 16 : 4 * group + 16);
    const size_t xs = i8 ? 4 * (size_t)M * groups : 0;
    const int rb = std::max(16 / M, rows_per_slot(groups));
    const size_t terms = 4 * (size_t)warps * M * rb * (groups + 1);
    return ring + x + xs + terms;
}

template <bool I8, int BITS, int G, int MT>
bool launch_one(const GemvBatch &b, cudaStream_t st) {
    auto kernel = cq_gemv_kernel<I8, BITS, G, MT>;
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
    const int rps = rows_per_slot(b.groups);
    int total = 0;
    for (int j = 0; j < b.nmat; ++j) total += (b.mat[j].out + rps - 1) / rps;
    const int grid = std::max(1, std::min(total, cached ? sms[dev] : 148));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes(b.M, b.groups, G, I8);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    NB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, b, total, rps));
    return true;
}

template <bool I8, int BITS, int G>
bool dispatch_mt(const GemvBatch &b, cudaStream_t st) {
    if (b.M <= 1) return launch_one<I8, BITS, G, 1>(b, st);
    if (b.M <= 2) return launch_one<I8, BITS, G, 2>(b, st);
    if (b.M <= 4) return launch_one<I8, BITS, G, 4>(b, st);
    return launch_one<I8, BITS, G, 8>(b, st);
}

template <bool I8>
bool dispatch(const GemvBatch &b, cudaStream_t st) {
    if (b.bits == 4) {
        if (b.group == 64) return dispatch_mt<I8, 4, 64>(b, st);
        if (b.group == 128) return dispatch_mt<I8, 4, 128>(b, st);
        return dispatch_mt<I8, 4, 256>(b, st);
    }
    if (b.group == 64) return dispatch_mt<I8, 2, 64>(b, st);
    if (b.group == 128) return dispatch_mt<I8, 2, 128>(b, st);
    return dispatch_mt<I8, 2, 256>(b, st);
}

}  // namespace

int gemv_max_rows(int bits, int group, int groups, bool i8) {
    if (i8) return gemv_frag_max_rows(bits, group, groups);
    if ((bits != 2 && bits != 4) || (group != 64 && group != 128 && group != 256)) return 0;
    if (groups < 1 || groups > 32) return 0;
    for (int m : {8, 4, 2, 1})
        if (smem_bytes(m, groups, group, i8) <= (size_t)kGemvMaxSmem) return m;
    return 0;
}

bool launch_gemv(const GemvBatch &b, bool i8, cudaStream_t st) {
    if (b.nmat < 1 || b.nmat > kGemvMaxMats || b.M < 1 || b.M > gemv_max_rows(b.bits, b.group, b.groups, i8) ||
        b.rowbytes % 16 || (b.partials && b.nmat != 1)) {
        set_error("GEMV launch outside the persistent kernel's envelope");
        return false;
    }
    if (!i8) {
        bool blocked = true;
        for (int j = 0; j < b.nmat; ++j) blocked = blocked && b.mat[j].blocked && b.mat[j].normsB;
        if (f32_gemv_kernel() != 1 && blocked && b.M <= gemv_rows_max_rows(b.bits, b.group, b.groups))
            return launch_gemv_rows(b, st);
        return dispatch<false>(b, st);
    }
    for (int j = 0; j < b.nmat; ++j)
        if (!b.mat[j].frag || !b.mat[j].normsF) {
            set_error("int8 GEMV needs the fragment-order copy of every matrix");
            return false;
        }
    return launch_gemv_frag(b, st);
}

int read_and_clear_gemv_fault() {
    int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemv_fault, sizeof(int)) != cudaSuccess) return -1;
    if (v) cudaMemcpyToSymbol(g_gemv_fault, &zero, sizeof(int));
    return v;
}

}  // namespace nb200
