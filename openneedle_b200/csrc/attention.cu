// INT8 KV-cache attention for B200 (sm_100a): quantise-store, split-K
// flash-decode, and causal prefill over a shared, read-only cached prefix.
//
// Semantics follow OpenNeedle's Engine (needle2/csrc/engine.cpp):
//  * store (1005-1021): per token and KV head, scale = max|k|/127 (1 if 0),
//    k_i8 = clamp(round-half-even(k * (127/max)), -127, 127); same for v;
//  * slots (500, 898-911): prefix sinks [0, P) are pinned; other positions
//    cycle through `window` slots (or are linear without a window); a query at
//    pos sees the sinks, then max(P, pos-window+1) .. pos;
//  * scores (949-960): s = (q . float(k_i8)) * k_scale * (1/sqrt(HD)),
//    softmax over the visible slots, out = sum p * v_scale * float(v_i8).
//  * prefill (1170-1210): each token stores its K/V, then attends.  Here a
//    prefill chunk attends over older slots plus the chunk's own freshly
//    quantised K/V (a staging copy), and the ring is written afterwards, which
//    is the same visible set and values as the token-by-token order.
//
// Device layout (head-major, so one (sequence, KV head) is one contiguous
// stream):  prefix  k/v [KV][P][HD] int8, scales [KV][P];  per session
// k/v [S][KV][Cs][HD], scales [S][KV][Cs], Cs = window ? window : max_seq - P.
#include <cuda_bf16.h>
#include <math.h>

#include <algorithm>
#include <cstring>

#include "attention.cuh"
#include "common.cuh"
#include "engine_math.cuh"
#include "pdl.cuh"
#include "sm100_async.cuh"

namespace nb200 {

namespace {

constexpr unsigned kFull = 0xffffffffu;

// The engine's output gate, o * sigmoid(g) with sigmoid(g) = 1 / (1 + exp(-g))
// (needle2/csrc/engine.cpp:36,123-129), applied as attention writes its output.
__device__ __forceinline__ float gated(const AttnParams &p, size_t i, float o) {
    return p.gate ? __fmul_rn(o, __fdiv_rn(1.f, __fadd_rn(1.f, expf(-p.gate[i])))) : o;
}

// One warp per (token, KV head): quantise head_dim values of k and v.
__global__ void kv_quantize_kernel(const float *__restrict__ k, const float *__restrict__ v, int tokens, int kvheads,
                                   int hd, int8_t *__restrict__ ko, int8_t *__restrict__ vo, float *__restrict__ ks,
                                   float *__restrict__ vs, KVDest dest) {
    pdl_enter();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= tokens * kvheads) return;
    const int t = warp / kvheads, kh = warp % kvheads;
    const float *kp = k + ((size_t)t * kvheads + kh) * hd, *vp = v + ((size_t)t * kvheads + kh) * hd;
    float mk = 0.f, mv = 0.f;
    for (int d = lane; d < hd; d += 32) {
        mk = fmaxf(mk, fabsf(kp[d]));
        mv = fmaxf(mv, fabsf(vp[d]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mk = fmaxf(mk, __shfl_xor_sync(kFull, mk, o));
        mv = fmaxf(mv, __shfl_xor_sync(kFull, mv, o));
    }
    const float sk = mk > 0.f ? __fdiv_rn(mk, 127.f) : 1.f, sv = mv > 0.f ? __fdiv_rn(mv, 127.f) : 1.f;
    const float ik = mk > 0.f ? __fdiv_rn(127.f, mk) : 0.f, iv = mv > 0.f ? __fdiv_rn(127.f, mv) : 0.f;
    // destination row
    size_t row;
    if (dest.mode == KVDest::kLinear) {
        row = (size_t)kh * dest.rows + t;                      // [KV][rows] (prefix or staging)
    } else {
        const int e = t / dest.tokens_per_entry, tt = t % dest.tokens_per_entry;
        const int s = dest.session[e], pos = dest.position[e] + tt;
        if (tt < dest.min_t && pos >= dest.prefix) return;   // overwritten later in the chunk's window
        if (pos < dest.prefix) {
            // a pinned prefix position (the prefix itself being prefilled)
            row = (size_t)kh * dest.prefix + pos;              // [KV][P]
            ko = dest.pk; vo = dest.pv; ks = dest.pks; vs = dest.pvs;
        } else {
            const int slot = dest.window ? (pos - dest.prefix) % dest.window : pos - dest.prefix;
            row = ((size_t)s * kvheads + kh) * dest.rows + slot;   // [S][KV][Cs]
        }
    }
    for (int d = lane; d < hd; d += 32) {
        ko[row * hd + d] = (int8_t)clamp127(rint_even(__fmul_rn(kp[d], ik)));
        vo[row * hd + d] = (int8_t)clamp127(rint_even(__fmul_rn(vp[d], iv)));
    }
    if (lane == 0) {
        ks[row] = sk;
        vs[row] = sv;
    }
}

// FP32 cache store: one warp per (token, KV head), rows as kv_quantize_kernel.
__global__ void kv_store_f32_kernel(const float *__restrict__ k, const float *__restrict__ v, int tokens, int kvheads,
                                    int hd, float *__restrict__ ko, float *__restrict__ vo, KVDest dest) {
    pdl_enter();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= tokens * kvheads) return;
    const int t = warp / kvheads, kh = warp % kvheads;
    const float *kp = k + ((size_t)t * kvheads + kh) * hd, *vp = v + ((size_t)t * kvheads + kh) * hd;
    size_t row;
    if (dest.mode == KVDest::kLinear) {
        row = (size_t)kh * dest.rows + t;
    } else {
        const int e = t / dest.tokens_per_entry, tt = t % dest.tokens_per_entry;
        const int s = dest.session[e], pos = dest.position[e] + tt;
        if (tt < dest.min_t && pos >= dest.prefix) return;
        if (pos < dest.prefix) {
            row = (size_t)kh * dest.prefix + pos;
            ko = dest.pkf; vo = dest.pvf;
        } else {
            const int slot = dest.window ? (pos - dest.prefix) % dest.window : pos - dest.prefix;
            row = ((size_t)s * kvheads + kh) * dest.rows + slot;
        }
    }
    for (int d = lane; d < hd; d += 32) {
        ko[row * hd + d] = kp[d];
        vo[row * hd + d] = vp[d];
    }
}

// Exact int8 -> float for four packed bytes.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float &a, float &b, float &c, float &d) {
    a = (float)(int8_t)(w & 0xff);
    b = (float)(int8_t)((w >> 8) & 0xff);
    c = (float)(int8_t)((w >> 16) & 0xff);
    d = (float)(int8_t)(w >> 24);
}

template <typename T>
struct Row {
    const T *k, *v;
    float ks, vs;
};

// Visible index i of query (session s, position pos) -> K/V row.  A prefill
// chunk's own rows come from the staging area even where the chunk lies inside
// the pinned prefix (the prefix itself being prefilled).
template <typename T>
__device__ __forceinline__ Row<T> visible_row(const AttnParams &p, int s, int pos, int kh, int i, int prefix_count,
                                              int start, int entry, int chunk_start) {
    int position;
    if (i < prefix_count) {
        position = i;
    } else {
        position = start + (i - prefix_count);
    }
    Row<T> r;
    size_t row;
    int where;   // 0 staged chunk, 1 pinned prefix, 2 session slots
    const bool staged = sizeof(T) == 1 ? p.stage_k != nullptr : p.stage_kf != nullptr;
    if (staged && position >= chunk_start) {
        row = (size_t)kh * p.stage_rows + (size_t)entry * p.tokens + (position - chunk_start);
        where = 0;
    } else if (position < p.prefix) {
        row = (size_t)kh * p.prefix + position;
        where = 1;
    } else {
        const int slot = p.window ? (position - p.prefix) % p.window : position - p.prefix;
        row = ((size_t)s * p.kvheads + kh) * p.cs + slot;
        where = 2;
    }
    if constexpr (sizeof(T) == 1) {
        const int8_t *kb = where == 0 ? p.stage_k : where == 1 ? p.pk : p.sk;
        const int8_t *vb = where == 0 ? p.stage_v : where == 1 ? p.pv : p.sv;
        const float *ksb = where == 0 ? p.stage_ks : where == 1 ? p.pks : p.sks;
        const float *vsb = where == 0 ? p.stage_vs : where == 1 ? p.pvs : p.svs;
        r.k = kb + row * p.hd;
        r.v = vb + row * p.hd;
        r.ks = ksb[row];
        r.vs = vsb[row];
    } else {
        // FP32 cache: no scales (the reference's FP32 KV arithmetic, engine.cpp:918-929)
        const float *kb = where == 0 ? p.stage_kf : where == 1 ? p.pkf : p.skf;
        const float *vb = where == 0 ? p.stage_vf : where == 1 ? p.pvf : p.svf;
        r.k = kb + row * p.hd;
        r.v = vb + row * p.hd;
        r.ks = 1.f;
        r.vs = 1.f;
    }
    return r;
}

// One CTA = (query, KV head, split): the R = heads/kvheads query heads of the
// group over a contiguous range of the visible slots.  Lane-per-slot scores,
// online softmax per warp, lane-per-dimension value accumulation.
template <int HD, bool EXACT, typename T>
__global__ void __launch_bounds__(128) attn_split_kernel(const AttnParams p) {
    pdl_enter();
    constexpr int NW = 4;
    const int hd = EXACT ? HD : p.hd;
    constexpr int DPL = (HD + 31) / 32;   // dims per lane in the PV phase
    __shared__ float qs[kMaxQueryGroup * HD];
    __shared__ float wm[NW][kMaxQueryGroup], wl[NW][kMaxQueryGroup];
    __shared__ float wacc[NW][kMaxQueryGroup][HD];

    const int split = blockIdx.x, kh = blockIdx.y, query = blockIdx.z;
    const int entry = query / p.tokens, t = query % p.tokens;
    const int s = p.session[entry];
    const int chunk_start = p.position[entry];
    const int pos = chunk_start + t;
    const int R = p.heads / p.kvheads;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int prefix_count = p.window ? min(p.prefix, pos + 1) : 0;
    const int start = p.window ? max(p.prefix, pos - p.window + 1) : 0;
    const int len = prefix_count + max(0, pos - start + 1);
    const int per = (len + p.splits - 1) / p.splits;
    const int i0 = split * per, i1 = min(len, i0 + per);

    for (int idx = threadIdx.x; idx < R * hd; idx += blockDim.x) {
        const int r = idx / hd, d = idx % hd;
        qs[r * HD + d] = p.q[((size_t)query * p.heads + kh * R + r) * hd + d];
    }
    __syncthreads();

    const float inv_sqrt = p.inv_sqrt_hd;
    float m[kMaxQueryGroup], l[kMaxQueryGroup], acc[kMaxQueryGroup][DPL];
#pragma unroll
    for (int r = 0; r < kMaxQueryGroup; ++r) {
        m[r] = -INFINITY;
        l[r] = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[r][j] = 0.f;
    }

    for (int base = i0 + warp * 32; base < i1; base += NW * 32) {
        const int i = base + lane;
        const bool valid = i < i1;
        Row<T> row{};
        float sc[kMaxQueryGroup];
#pragma unroll
        for (int r = 0; r < kMaxQueryGroup; ++r) sc[r] = -INFINITY;
        if (valid) {
            row = visible_row<T>(p, s, pos, kh, i, prefix_count, start, entry, chunk_start);
            float dot[kMaxQueryGroup];
#pragma unroll
            for (int r = 0; r < kMaxQueryGroup; ++r) dot[r] = 0.f;
            if constexpr (sizeof(T) == 4) {
                for (int d = 0; d < hd; ++d) {
                    const float kf = __ldg(reinterpret_cast<const float *>(row.k) + d);
#pragma unroll
                    for (int r = 0; r < kMaxQueryGroup; ++r)
                        if (r < R) dot[r] = fmaf(qs[r * HD + d], kf, dot[r]);
                }
            } else if (hd % 4 == 0) {
                const uint32_t *kw = reinterpret_cast<const uint32_t *>(row.k);
#pragma unroll 4
                for (int d4 = 0; d4 < hd / 4; ++d4) {
                    float a, b, c, e;
                    i8x4_to_f32(__ldg(kw + d4), a, b, c, e);
#pragma unroll
                    for (int r = 0; r < kMaxQueryGroup; ++r) {
                        if (r < R) {
                            const float4 qv = *reinterpret_cast<const float4 *>(qs + r * HD + 4 * d4);
                            dot[r] = fmaf(qv.x, a, dot[r]);
                            dot[r] = fmaf(qv.y, b, dot[r]);
                            dot[r] = fmaf(qv.z, c, dot[r]);
                            dot[r] = fmaf(qv.w, e, dot[r]);
                        }
                    }
                }
            } else {
                for (int d = 0; d < hd; ++d) {
                    const float kf = (float)row.k[d];
#pragma unroll
                    for (int r = 0; r < kMaxQueryGroup; ++r)
                        if (r < R) dot[r] = fmaf(qs[r * HD + d], kf, dot[r]);
                }
            }
#pragma unroll
            for (int r = 0; r < kMaxQueryGroup; ++r) sc[r] = __fmul_rn(__fmul_rn(dot[r], row.ks), inv_sqrt);
        }
        // online softmax update per head
        float pr[kMaxQueryGroup];
#pragma unroll
        for (int r = 0; r < kMaxQueryGroup; ++r) {
            if (r >= R) { pr[r] = 0.f; continue; }
            float bm = sc[r];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, o));
            const float mn = fmaxf(m[r], bm);
            const float corr = m[r] == -INFINITY ? 0.f : expf(m[r] - mn);
            pr[r] = valid ? expf(sc[r] - mn) : 0.f;
            float ps = pr[r];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(kFull, ps, o);
            l[r] = l[r] * corr + ps;
            m[r] = mn;
#pragma unroll
            for (int j = 0; j < DPL; ++j) acc[r][j] *= corr;
            pr[r] *= valid ? row.vs : 0.f;     // fold the value scale into the weight
        }
        // values: lane owns dims lane + 32*j
        const int nvalid = min(32, i1 - base);
        for (int jt = 0; jt < nvalid; ++jt) {
            const T *vrow = reinterpret_cast<const T *>(
                __shfl_sync(kFull, reinterpret_cast<unsigned long long>(row.v), jt));
            float w[kMaxQueryGroup];
#pragma unroll
            for (int r = 0; r < kMaxQueryGroup; ++r) w[r] = __shfl_sync(kFull, pr[r], jt);
#pragma unroll
            for (int j = 0; j < DPL; ++j) {
                const int d = lane + 32 * j;
                if (d < hd) {
                    const float vf = (float)__ldg(vrow + d);
#pragma unroll
                    for (int r = 0; r < kMaxQueryGroup; ++r)
                        if (r < R) acc[r][j] = fmaf(w[r], vf, acc[r][j]);
                }
            }
        }
    }
    // combine the warps of this CTA
#pragma unroll
    for (int r = 0; r < kMaxQueryGroup; ++r) {
        if (r >= R) continue;
        if (lane == 0) {
            wm[warp][r] = m[r];
            wl[warp][r] = l[r];
        }
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
            const int d = lane + 32 * j;
            if (d < hd) wacc[warp][r][d] = acc[r][j];
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < R * hd; idx += blockDim.x) {
        const int r = idx / hd, d = idx % hd;
        float mm = -INFINITY;
        for (int w = 0; w < NW; ++w) mm = fmaxf(mm, wm[w][r]);
        float ll = 0.f, aa = 0.f;
        for (int w = 0; w < NW; ++w) {
            if (wm[w][r] == -INFINITY) continue;
            const float f = expf(wm[w][r] - mm);
            ll += wl[w][r] * f;
            aa += wacc[w][r][d] * f;
        }
        const int h = kh * R + r;
        if (p.splits == 1) {
            const size_t oi = ((size_t)query * p.heads + h) * hd + d;
            p.out[oi] = gated(p, oi, ll > 0.f ? aa / ll : 0.f);
        } else {
            const size_t prow = ((size_t)query * p.heads + h) * p.splits + split;
            p.part_acc[prow * hd + d] = aa;
            if (d == 0) {
                p.part_m[prow] = mm;
                p.part_l[prow] = ll;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Streaming decode/prefill kernel for HD = 64 or 128 (the fast path).
//
// A warp walks a contiguous range of visible slots, 8 slots per step: lane
// (j = lane / 4, c = lane % 4) owns slot base + j and dimensions
// [c * HD/4, (c + 1) * HD/4), so a step's K rows (and V rows) arrive as 16-byte
// coalesced loads.  int8 values become floats exactly through a byte permute
// into the bit pattern of 2^23 + (b + 128) and one subtraction.  Scores are
// reduced over the slot's four lanes; each chunk of CH steps updates the
// running max once (per query head), and values accumulate per lane over its
// slots, reduced across the warp at the end.  The R query heads of the KV group
// share every K/V read.

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
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    unsigned long long r, x, y;
    memcpy(&x, &a, 8);
    memcpy(&y, &b, 8);
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
    float2 o;
    memcpy(&o, &r, 8);
    return o;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    unsigned long long r, x, y;
    memcpy(&x, &a, 8);
    memcpy(&y, &b, 8);
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
    float2 o;
    memcpy(&o, &r, 8);
    return o;
}

// Four int8 (one word) -> exact floats, as pairs (bytes 0,1) and (2,3).
__device__ __forceinline__ void i8x4_pairs(uint32_t w, float2 &lo, float2 &hi) {
    const uint32_t u = w ^ 0x80808080u;   // b + 128, as unsigned bytes
    const uint32_t top = 0x4B000000u;     // 2^23
    const float2 off = make_float2(-8388736.f, -8388736.f);   // -(2^23 + 128)
    lo = fadd2(make_float2(__uint_as_float(prmt(u, top, 0x7540)), __uint_as_float(prmt(u, top, 0x7541))), off);
    hi = fadd2(make_float2(__uint_as_float(prmt(u, top, 0x7542)), __uint_as_float(prmt(u, top, 0x7543))), off);
}

// Global addresses of visible index i's K/V rows and scales, and how many
// visible indices from i on map to consecutive rows of the same array (up to the
// end of the prefix, of the staged chunk, or of the ring before it wraps).
struct RowPtr {
    const int8_t *k, *v;
    const float *ks, *vs;
    int run;
};
__device__ __forceinline__ RowPtr visible_ptr(const AttnParams &p, int s, int kh, int i, int prefix_count, int start,
                                              int entry, int chunk_start) {
    constexpr int kLong = 1 << 30;
    const int position = i < prefix_count ? i : start + (i - prefix_count);
    size_t row;
    RowPtr r;
    if (p.stage_k && position >= chunk_start) {
        row = (size_t)kh * p.stage_rows + (size_t)entry * p.tokens + (position - chunk_start);
        r.k = p.stage_k; r.v = p.stage_v; r.ks = p.stage_ks; r.vs = p.stage_vs;
        r.run = chunk_start + p.tokens - position;
    } else if (position < p.prefix) {
        row = (size_t)kh * p.prefix + position;
        r.k = p.pk; r.v = p.pv; r.ks = p.pks; r.vs = p.pvs;
        r.run = i < prefix_count ? prefix_count - i : p.prefix - position;
        if (p.stage_k) r.run = min(r.run, chunk_start - position);
    } else {
        const int slot = p.window ? (position - p.prefix) % p.window : position - p.prefix;
        row = ((size_t)s * p.kvheads + kh) * p.cs + slot;
        r.k = p.sk; r.v = p.sv; r.ks = p.sks; r.vs = p.svs;
        r.run = p.window ? p.window - slot : kLong;
        if (p.stage_k) r.run = min(r.run, chunk_start - position);
    }
    r.k += row * p.hd;
    r.v += row * p.hd;
    r.ks += row;
    r.vs += row;
    return r;
}

// Decode prologue of a CTA of attn_stream_kernel when the new token's
// projections arrive as K-split parts (AttnParams::qkv_*): the parts added in
// order, the CTA's R query heads RMS-normed (1 + q_norm) and roped into qs,
// and -- where `own` (the CTA's slots include the token's) -- the KV head's K
// (normed, roped) and V quantised and stored in the token's cache row.  The
// arithmetic is qk_rope_store_kernel's (engine.cpp:994-1021).  Lane holds
// elements lane + 32 e; the rotary pairs (j, j + HD / 2) sit in one lane.
template <int HD, int R, int NWARPS>
__device__ __forceinline__ void qkv_prologue(const AttnParams &p, int query, int kh, int pos, int s, bool own,
                                             float *qs, int warp, int lane) {
    constexpr int E = HD / 32, half = HD / 2;
    // units: R query heads; where own, the KV head's K and V, then the gate of the R query heads
    const int units = R + (own ? 2 + (p.qkv_g ? R : 0) : 0);
#pragma unroll
    for (int u0 = 0; u0 < 2 * R + 2; u0 += NWARPS) {
        const int u = u0 + warp;
        if (u >= units) break;
        if (u >= R + 2) {   // a gate head: the parts' sum, read back by this query's epilogue
            const size_t o = ((size_t)query * p.heads + kh * R + (u - R - 2)) * HD;
#pragma unroll
            for (int e = 0; e < E; ++e)
                const_cast<float *>(p.gate)[o + lane + 32 * e] =
                    eng::part_sum(p.qkv_g + o + lane + 32 * e, p.qkv_parts, p.qkv_pstride);
            continue;
        }
        const bool isq = u < R, isv = u == R + 1;
        const size_t off = isq ? ((size_t)query * p.heads + kh * R + u) * HD : ((size_t)query * p.kvheads + kh) * HD;
        const float *src = (isq ? p.qkv_q : isv ? p.qkv_v : p.qkv_k) + off;
        float h[E];
#pragma unroll
        for (int e = 0; e < E; ++e) h[e] = eng::part_sum(src + lane + 32 * e, p.qkv_parts, p.qkv_pstride);
        if (!isv) {
            const float *nrm = isq ? p.q_norm : p.k_norm;
            float ss = 0.f;
#pragma unroll
            for (int e = 0; e < E; ++e) ss = fmaf(h[e], h[e], ss);
            const float inv = eng::rms_inv(eng::warp_sum(ss), HD);
#pragma unroll
            for (int e = 0; e < E; ++e) h[e] = __fmul_rn(__fmul_rn(h[e], inv), __fadd_rn(1.f, nrm[lane + 32 * e]));
            const bool tab = p.rope_cos && pos < p.rope_len;
#pragma unroll
            for (int e = 0; e < E / 2; ++e) {
                const int j = lane + 32 * e;
                float co, si;
                if (tab) {
                    co = p.rope_cos[(size_t)pos * half + j];
                    si = p.rope_sin[(size_t)pos * half + j];
                } else {
                    const float ang = __fdiv_rn((float)pos, p.rope_div[j]);
                    co = cosf(ang);
                    si = sinf(ang);
                }
                const float a = h[e], c = h[e + E / 2];
                h[e] = __fsub_rn(__fmul_rn(a, co), __fmul_rn(c, si));
                h[e + E / 2] = __fadd_rn(__fmul_rn(c, co), __fmul_rn(a, si));
            }
        }
        if (isq) {
#pragma unroll
            for (int e = 0; e < E; ++e) qs[u * HD + lane + 32 * e] = h[e];
            continue;
        }
        const bool pinned = pos < p.prefix;
        const size_t row = pinned ? (size_t)kh * p.prefix + pos
                                  : ((size_t)s * p.kvheads + kh) * p.cs +
                                        (p.window ? (pos - p.prefix) % p.window : pos - p.prefix);
        float mx = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) mx = fmaxf(mx, fabsf(h[e]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
        const float sc = mx > 0.f ? __fdiv_rn(mx, 127.f) : 1.f;
        const float iv = mx > 0.f ? __fdiv_rn(127.f, mx) : 0.f;
        int8_t *dst = const_cast<int8_t *>(isv ? (pinned ? p.pv : p.sv) : (pinned ? p.pk : p.sk)) + row * HD;
        float *sdst = const_cast<float *>(isv ? (pinned ? p.pvs : p.svs) : (pinned ? p.pks : p.sks));
#pragma unroll
        for (int e = 0; e < E; ++e) {
            int qv = __float2int_rn(__fmul_rn(h[e], iv));
            qv = qv < -127 ? -127 : (qv > 127 ? 127 : qv);
            dst[lane + 32 * e] = (int8_t)qv;
        }
        if (lane == 0) sdst[row] = sc;
    }
}

// The same for one warp that owns a whole query (the warp-per-query decode,
// R <= 2): every unit at once -- all parts loaded together, the three norms'
// sums and the two quantisers' maxima reduced side by side -- so that the
// prologue costs about one load round trip rather than one per unit.
template <int HD, int R>
__device__ __forceinline__ void wpq_prologue(const AttnParams &p, int query, int kh, int pos, int s, float *qs,
                                             int lane) {
    constexpr int E = HD / 32, half = HD / 2;
    const int P = p.qkv_parts;
    const long long ps = p.qkv_pstride;
    const size_t qo = ((size_t)query * p.heads + kh * R) * HD, ko = ((size_t)query * p.kvheads + kh) * HD;
    float q[R][E], k[E], v[E], g[R][E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int d = lane + 32 * e;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            q[r][e] = eng::part_sum(p.qkv_q + qo + r * HD + d, P, ps);
            g[r][e] = p.qkv_g ? eng::part_sum(p.qkv_g + qo + r * HD + d, P, ps) : 0.f;
        }
        k[e] = eng::part_sum(p.qkv_k + ko + d, P, ps);
        v[e] = eng::part_sum(p.qkv_v + ko + d, P, ps);
    }
    // RMS norms (1 + w) of the query heads and of K
    float ss[R + 1];
#pragma unroll
    for (int r = 0; r <= R; ++r) {
        ss[r] = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const float x = r < R ? q[r][e] : k[e];
            ss[r] = fmaf(x, x, ss[r]);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int r = 0; r <= R; ++r) ss[r] += __shfl_xor_sync(kFull, ss[r], o);
#pragma unroll
    for (int r = 0; r <= R; ++r) {
        const float inv = eng::rms_inv(ss[r], HD);
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const int d = lane + 32 * e;
            if (r < R) q[r][e] = __fmul_rn(__fmul_rn(q[r][e], inv), __fadd_rn(1.f, p.q_norm[d]));
            else k[e] = __fmul_rn(__fmul_rn(k[e], inv), __fadd_rn(1.f, p.k_norm[d]));
        }
    }
    // rotary embedding at the token's position: pairs (j, j + HD / 2) in one lane
    const bool tab = p.rope_cos && pos < p.rope_len;
#pragma unroll
    for (int e = 0; e < E / 2; ++e) {
        const int j = lane + 32 * e;
        float co, si;
        if (tab) {
            co = p.rope_cos[(size_t)pos * half + j];
            si = p.rope_sin[(size_t)pos * half + j];
        } else {
            const float ang = __fdiv_rn((float)pos, p.rope_div[j]);
            co = cosf(ang);
            si = sinf(ang);
        }
#pragma unroll
        for (int r = 0; r <= R; ++r) {
            float &x0 = r < R ? q[r][e] : k[e];
            float &x1 = r < R ? q[r][e + E / 2] : k[e + E / 2];
            const float a = x0, c = x1;
            x0 = __fsub_rn(__fmul_rn(a, co), __fmul_rn(c, si));
            x1 = __fadd_rn(__fmul_rn(c, co), __fmul_rn(a, si));
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int e = 0; e < E; ++e) qs[r * HD + lane + 32 * e] = q[r][e];
    if (p.qkv_g)
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int e = 0; e < E; ++e) const_cast<float *>(p.gate)[qo + r * HD + lane + 32 * e] = g[r][e];
    // K and V of the token quantised into its cache row
    float mk = 0.f, mv = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        mk = fmaxf(mk, fabsf(k[e]));
        mv = fmaxf(mv, fabsf(v[e]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mk = fmaxf(mk, __shfl_xor_sync(kFull, mk, o));
        mv = fmaxf(mv, __shfl_xor_sync(kFull, mv, o));
    }
    const bool pinned = pos < p.prefix;
    const size_t row = pinned ? (size_t)kh * p.prefix + pos
                              : ((size_t)s * p.kvheads + kh) * p.cs +
                                    (p.window ? (pos - p.prefix) % p.window : pos - p.prefix);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const float mx = t ? mv : mk;
        const float sc = mx > 0.f ? __fdiv_rn(mx, 127.f) : 1.f;
        const float iv = mx > 0.f ? __fdiv_rn(127.f, mx) : 0.f;
        int8_t *dst = const_cast<int8_t *>(t ? (pinned ? p.pv : p.sv) : (pinned ? p.pk : p.sk)) + row * HD;
        float *sdst = const_cast<float *>(t ? (pinned ? p.pvs : p.svs) : (pinned ? p.pks : p.sks));
#pragma unroll
        for (int e = 0; e < E; ++e) {
            int qv = __float2int_rn(__fmul_rn(t ? v[e] : k[e], iv));
            qv = qv < -127 ? -127 : (qv > 127 ? 127 : qv);
            dst[lane + 32 * e] = (int8_t)qv;
        }
        if (lane == 0) sdst[row] = sc;
    }
}

template <int HD>
struct StreamGeo {
    static constexpr int NW = 4;                    // warps per CTA
    static constexpr int DL = HD / 4;               // dimensions per lane
    static constexpr int U = DL / 16;               // 16-byte pieces per lane and row
    static constexpr int CH = HD <= 64 ? 4 : 2;     // steps (of 8 slots) per chunk
    static constexpr int NCH = 2;                   // chunks in a warp's ring
    static constexpr int STEP = 2 * 32 * 16 * U + 64;   // K pieces, V pieces, 8 x (k scale, v scale)
    static constexpr int CHUNK = CH * STEP;
    static constexpr int RING = NCH * CHUNK;        // bytes per warp
};

// WPQ (warp per query): each warp takes one whole (query, KV head) pair (no
// split, no cross-warp combine, no block barrier) and the CTA's four warps four
// queries -- the short-context decode case, where per-CTA work is small.
// FQ: decode with the new token's projections as K parts (AttnParams::qkv_*;
// a separate instantiation, so that the plain kernels keep their code).
template <int HD, int R, bool WPQ, bool FQ>
__global__ void __launch_bounds__(128, 4) attn_stream_kernel(const AttnParams p) {
    pdl_enter();
    using Geo = StreamGeo<HD>;
    constexpr int NW = Geo::NW, DL = Geo::DL, U = Geo::U, WL = DL / 4, CH = Geo::CH, NCH = Geo::NCH;
    constexpr bool QREG = R * DL <= 32;   // query slice in registers
    static_assert(!WPQ || QREG, "warp-per-query needs the query slice in registers");
    extern __shared__ __align__(16) uint8_t ring_raw[];   // [NW][Geo::RING] from a 128-byte boundary (stream_smem)
    uint8_t *ring_all = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(ring_raw) + 127) & ~uintptr_t(127));
    __shared__ __align__(16) float qs[WPQ ? 4 : R * HD];
    __shared__ float wm[WPQ ? 1 : NW][R], wl[WPQ ? 1 : NW][R];
    __shared__ float wacc[WPQ ? 1 : NW][R][WPQ ? 1 : HD];

    const int warp = threadIdx.x >> 5;
    const int split = WPQ ? 0 : blockIdx.x, kh = blockIdx.y;
    const int query = WPQ ? blockIdx.z * NW + warp : blockIdx.z;
    if (WPQ && query >= p.queries) return;
    const int entry = query / p.tokens, t = query % p.tokens;
    const int s = p.session[entry];
    const int chunk_start = p.position[entry];
    const int pos = chunk_start + t;
    const int lane = threadIdx.x & 31, j = lane >> 2, c = lane & 3;
    uint8_t *ring = ring_all + warp * Geo::RING;

    const int prefix_count = p.window ? min(p.prefix, pos + 1) : 0;
    const int start = p.window ? max(p.prefix, pos - p.window + 1) : 0;
    const int len = prefix_count + max(0, pos - start + 1);
    const int per = (len + p.splits - 1) / p.splits;
    const int i0 = split * per, i1 = min(len, i0 + per);
    // this warp's share of the split, in whole steps of 8 slots (all of it with WPQ)
    const int steps = (max(0, i1 - i0) + 7) / 8, wsteps = WPQ ? steps : (steps + NW - 1) / NW;
    const int w0 = i0 + (WPQ ? 0 : warp) * wsteps * 8, w1 = min(i1, w0 + wsteps * 8);
    const int nchunks = w1 > w0 ? (w1 - w0 + 8 * CH - 1) / (8 * CH) : 0;

    // copies of chunk ch into its ring slot: lane (j, c) brings its own K and V
    // pieces of slot j of each step; lane c = 0 of each slot brings the scales
    auto issue = [&](int ch) {
        if (ch < nchunks) {
            uint8_t *dst = ring + (ch % NCH) * Geo::CHUNK;
            const int ib = w0 + ch * CH * 8 + j;   // this lane's slot of the chunk's first step
            const RowPtr r0 = ib < w1 ? visible_ptr(p, s, kh, ib, prefix_count, start, entry, chunk_start) : RowPtr{};
#pragma unroll
            for (int st = 0; st < CH; ++st) {
                const int i = ib + 8 * st;
                if (i < w1) {
                    RowPtr r = r0;
                    if (8 * st < r0.run) {   // same array, 8 rows further on
                        r.k += (size_t)8 * st * HD;
                        r.v += (size_t)8 * st * HD;
                        r.ks += 8 * st;
                        r.vs += 8 * st;
                    } else {
                        r = visible_ptr(p, s, kh, i, prefix_count, start, entry, chunk_start);
                    }
                    uint8_t *sd = dst + st * Geo::STEP;
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        cp_async<16>(sd + (lane * U + u) * 16, r.k + c * DL + 16 * u);
                        cp_async<16>(sd + 32 * 16 * U + (lane * U + u) * 16, r.v + c * DL + 16 * u);
                    }
                    if (c == 0) cp_async<4>(sd + 2 * 32 * 16 * U + 8 * j, r.ks);
                    if (c == 1) cp_async<4>(sd + 2 * 32 * 16 * U + 8 * j + 4, r.vs);
                }
            }
        }
        cp_async_commit();   // one group per chunk, empty ones included
    };

    // with the new token's projections as parts, this CTA may first store the
    // token's K/V: a warp issues its first chunks ahead of that only where they
    // end before the token's slot (the last visible one)
    constexpr bool fused = FQ;
    const bool early = !fused || w1 < len || w0 + (NCH - 1) * CH * 8 <= len - 1;
    if (early)
#pragma unroll
        for (int ch = 0; ch < NCH - 1; ++ch) issue(ch);
    // one warp per query: the warp's own prologue, its query heads staged in the
    // ring slot that the first issued chunks leave free
    float *const qw = reinterpret_cast<float *>(ring + (NCH - 1) * Geo::CHUNK);
    if constexpr (WPQ) {
        static_assert(R * HD * 4 <= Geo::CHUNK, "query heads fit a ring chunk");
        if (fused) {
            wpq_prologue<HD, R>(p, query, kh, pos, s, qw, lane);
            __threadfence_block();   // the token's K/V rows and gate before this warp's reads of them
            __syncwarp();
        }
    } else {
        if (fused) {
            qkv_prologue<HD, R, NW>(p, query, kh, pos, s, i0 < len && i1 == len, qs, warp, lane);
            __threadfence_block();   // the token's K/V rows before any warp's copies of them
        } else {
            for (int idx = threadIdx.x; idx < R * HD; idx += blockDim.x)
                qs[idx] = p.q[((size_t)query * p.heads + kh * R) * HD + idx];
        }
        __syncthreads();
    }
    if (!early)
#pragma unroll
        for (int ch = 0; ch < NCH - 1; ++ch) issue(ch);
    float2 qr[QREG ? R : 1][QREG ? DL / 2 : 1];
    if (QREG) {
        const float *qsrc = WPQ ? (fused ? qw : p.q + ((size_t)query * p.heads + kh * R) * HD) : qs;
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int e = 0; e < DL / 2; ++e)
                qr[r][e] = *reinterpret_cast<const float2 *>(qsrc + r * HD + c * DL + 2 * e);
        if (WPQ && fused) __syncwarp();   // every lane has read qw before the ring slot is refilled
    }

    const float inv_sqrt = p.inv_sqrt_hd;
    float m[R], l[R];
    float2 acc[R][DL / 2];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        m[r] = -INFINITY;
        l[r] = 0.f;
#pragma unroll
        for (int e = 0; e < DL / 2; ++e) acc[r][e] = make_float2(0.f, 0.f);
    }

    for (int ch = 0; ch < nchunks; ++ch) {
        issue(ch + NCH - 1);
        cp_async_wait<NCH - 1>();   // chunk ch has landed (for this lane) ...
        __syncwarp();               // ... and for every lane of the warp
        const uint8_t *src = ring + (ch % NCH) * Geo::CHUNK;
        bool valid[CH];
        float sc[CH][R];
#pragma unroll
        for (int st = 0; st < CH; ++st) {
            valid[st] = w0 + (ch * CH + st) * 8 + j < w1;
            const uint8_t *sd = src + st * Geo::STEP;
            const float ks = *reinterpret_cast<const float *>(sd + 2 * 32 * 16 * U + 8 * j);
            float2 dot[R];
#pragma unroll
            for (int r = 0; r < R; ++r) dot[r] = make_float2(0.f, 0.f);
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint4 kw = *reinterpret_cast<const uint4 *>(sd + (lane * U + u) * 16);
                const uint32_t words[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) {
                    float2 lo, hi;
                    i8x4_pairs(words[wi], lo, hi);
                    const int e = (u * 4 + wi) * 2;   // pair index within the lane's DL dims
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        float2 q0, q1;
                        if (QREG) {
                            q0 = qr[r][e];
                            q1 = qr[r][e + 1];
                        } else {
                            const float4 qv = *reinterpret_cast<const float4 *>(qs + r * HD + c * DL + 2 * e);
                            q0 = make_float2(qv.x, qv.y);
                            q1 = make_float2(qv.z, qv.w);
                        }
                        dot[r] = ffma2(lo, q0, dot[r]);
                        dot[r] = ffma2(hi, q1, dot[r]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
                float d = dot[r].x + dot[r].y;
                d += __shfl_xor_sync(kFull, d, 1);
                d += __shfl_xor_sync(kFull, d, 2);
                sc[st][r] = valid[st] ? __fmul_rn(__fmul_rn(d, ks), inv_sqrt) : -INFINITY;
            }
        }
        // running max, weights
        float wgt[CH][R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            float mx = sc[0][r];
#pragma unroll
            for (int st = 1; st < CH; ++st) mx = fmaxf(mx, sc[st][r]);
            mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 16));
            const float mn = fmaxf(m[r], mx);
            const float corr = m[r] == -INFINITY ? 0.f : __expf(m[r] - mn);
            m[r] = mn;
            float ps = 0.f;
#pragma unroll
            for (int st = 0; st < CH; ++st) {
                const float vs = *reinterpret_cast<const float *>(src + st * Geo::STEP + 2 * 32 * 16 * U + 8 * j + 4);
                const float pr = valid[st] ? __expf(sc[st][r] - mn) : 0.f;
                ps += pr;
                wgt[st][r] = valid[st] ? pr * vs : 0.f;   // the value scale folded into the weight
            }
            l[r] = l[r] * corr + (c == 0 ? ps : 0.f);   // one lane of each slot counts it
            const float2 c2 = make_float2(corr, corr);
#pragma unroll
            for (int e = 0; e < DL / 2; ++e) acc[r][e] = fmul2(acc[r][e], c2);
        }
        // values
#pragma unroll
        for (int st = 0; st < CH; ++st) {
            const uint8_t *sd = src + st * Geo::STEP + 32 * 16 * U;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint4 vw = *reinterpret_cast<const uint4 *>(sd + (lane * U + u) * 16);
                const uint32_t words[4] = {vw.x, vw.y, vw.z, vw.w};
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) {
                    float2 lo, hi;
                    i8x4_pairs(words[wi], lo, hi);
                    const int e = (u * 4 + wi) * 2;
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const float2 w2 = make_float2(wgt[st][r], wgt[st][r]);
                        acc[r][e] = ffma2(lo, w2, acc[r][e]);
                        acc[r][e + 1] = ffma2(hi, w2, acc[r][e + 1]);
                    }
                }
            }
        }
        __syncwarp();   // every lane is done with this ring slot before it is refilled
    }
    cp_async_wait<0>();
    // reduce over the warp's 8 slot lanes (same c), then over the CTA's warps
#pragma unroll
    for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            l[r] += __shfl_xor_sync(kFull, l[r], o);
#pragma unroll
            for (int e = 0; e < DL / 2; ++e) {
                acc[r][e].x += __shfl_xor_sync(kFull, acc[r][e].x, o);
                acc[r][e].y += __shfl_xor_sync(kFull, acc[r][e].y, o);
            }
        }
        if (WPQ) {
            // lanes 0-3 hold the whole sums for dimensions c * DL ..; the softmax
            // denominator was counted on the c == 0 lanes only, so lane 0 has it
            const float lt = __shfl_sync(kFull, l[r], 0);
            const float inv = lt > 0.f ? 1.f / lt : 0.f;
            const size_t o0 = ((size_t)query * p.heads + kh * R + r) * HD + c * DL;
#pragma unroll
            for (int e = 0; e < DL / 2; ++e) {
                acc[r][e].x = gated(p, o0 + 2 * e, acc[r][e].x * inv);
                acc[r][e].y = gated(p, o0 + 2 * e + 1, acc[r][e].y * inv);
                if (j == 0) {
                    p.out[o0 + 2 * e] = acc[r][e].x;
                    p.out[o0 + 2 * e + 1] = acc[r][e].y;
                }
            }
            continue;
        }
        if (lane == 0) {
            wm[warp][r] = m[r];
            wl[warp][r] = l[r];
        }
        if (j == 0)
#pragma unroll
            for (int e = 0; e < DL / 2; ++e) *reinterpret_cast<float2 *>(&wacc[warp][r][c * DL + 2 * e]) = acc[r][e];
    }
    if constexpr (WPQ) {
        if (p.hilo) {
            // the out projection's input rotation (CQ::transform over the R * HD
            // outputs of this KV head: element r * HD + c * DL + i) and bf16
            // split, with the Walsh-Hadamard stages in order h = 1, 2, 4, ...:
            // i bits in registers, c bits across lanes 0-3, r bits in registers
            float v[R][DL];
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int e = 0; e < DL / 2; ++e) {
                    v[r][2 * e] = acc[r][e].x;
                    v[r][2 * e + 1] = acc[r][e].y;
                }
#pragma unroll
            for (int h = 1; h < DL; h *= 2)
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int i = 0; i < DL; ++i)
                        if (!(i & h)) {
                            const float a = v[r][i], b = v[r][i + h];
                            v[r][i] = __fadd_rn(a, b);
                            v[r][i + h] = __fsub_rn(a, b);
                        }
#pragma unroll
            for (int m = 1; m < 4; m *= 2) {
                const bool upper = c & m;
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int i = 0; i < DL; ++i) {
                        const float o = __shfl_xor_sync(kFull, v[r][i], m);
                        v[r][i] = upper ? __fsub_rn(o, v[r][i]) : __fadd_rn(v[r][i], o);
                    }
            }
#pragma unroll
            for (int h = 1; h < R; h *= 2)
#pragma unroll
                for (int r = 0; r < R; ++r)
                    if (!(r & h))
#pragma unroll
                        for (int i = 0; i < DL; ++i) {
                            const float a = v[r][i], b = v[r + h][i];
                            v[r][i] = __fadd_rn(a, b);
                            v[r + h][i] = __fsub_rn(a, b);
                        }
            if (j == 0) {
                const size_t row = (size_t)query * p.hilo_ld + (size_t)kh * R * HD + c * DL;
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int i = 0; i < DL; ++i) {
                        const float x = __fmul_rn(v[r][i], p.rot_scale);
                        const __nv_bfloat16 hv = __float2bfloat16_rn(x);
                        p.hilo[row + r * HD + i] = __bfloat16_as_ushort(hv);
                        p.hilo[p.hilo_lo + row + r * HD + i] =
                            __bfloat16_as_ushort(__float2bfloat16_rn(__fsub_rn(x, __bfloat162float(hv))));
                    }
            }
        }
        return;
    }
    __syncthreads();
    if constexpr (R * HD % 32 == 0 && R * HD <= 32 * NW) {
        if (p.splits == 1 && p.hilo) {
            // one output a thread: merge the warps, gate and store it, then the
            // out projection's input rotation (CQ::transform over the R * HD
            // outputs of this KV head, stages h = 1, 2, 4, ...: shuffles below
            // 32, shared memory above) and bf16 split, as attn_combine_rot_kernel
            constexpr int n = R * HD;
            __shared__ float xs[2][n];
            const int t = threadIdx.x, r = t / HD, d = t % HD;
            float v = 0.f;
            if (t < n) {
                float mm = -INFINITY;
                for (int w = 0; w < NW; ++w) mm = fmaxf(mm, wm[w][r]);
                float ll = 0.f, aa = 0.f;
                for (int w = 0; w < NW; ++w) {
                    if (wm[w][r] == -INFINITY) continue;
                    const float f = __expf(wm[w][r] - mm);
                    ll += wl[w][r] * f;
                    aa += wacc[w][r][d] * f;
                }
                const size_t oi = ((size_t)query * p.heads + kh * R + r) * HD + d;
                v = gated(p, oi, ll > 0.f ? aa / ll : 0.f);
                p.out[oi] = v;
#pragma unroll
                for (int h = 1; h < 32 && h < n; h *= 2) {   // whole warps (n is a multiple of 32)
                    const float o = __shfl_xor_sync(kFull, v, h);
                    v = (t & h) ? __fsub_rn(o, v) : __fadd_rn(v, o);
                }
            }
            int buf = 0;
#pragma unroll
            for (int h = 32; h < n; h *= 2) {
                if (t < n) xs[buf][t] = v;
                __syncthreads();
                if (t < n) {
                    const float o = xs[buf][t ^ h];
                    v = (t & h) ? __fsub_rn(o, v) : __fadd_rn(v, o);
                }
                buf ^= 1;
            }
            if (t < n) {
                const float x = __fmul_rn(v, p.rot_scale);
                const size_t i = (size_t)query * p.hilo_ld + (size_t)kh * n + t;
                const __nv_bfloat16 hv = __float2bfloat16_rn(x);
                p.hilo[i] = __bfloat16_as_ushort(hv);
                p.hilo[p.hilo_lo + i] = __bfloat16_as_ushort(__float2bfloat16_rn(__fsub_rn(x, __bfloat162float(hv))));
            }
            return;
        }
    }
    for (int idx = threadIdx.x; idx < R * HD; idx += blockDim.x) {
        const int r = idx / HD, d = idx % HD;
        float mm = -INFINITY;
        for (int w = 0; w < NW; ++w) mm = fmaxf(mm, wm[w][r]);
        float ll = 0.f, aa = 0.f;
        for (int w = 0; w < NW; ++w) {
            if (wm[w][r] == -INFINITY) continue;
            const float f = __expf(wm[w][r] - mm);
            ll += wl[w][r] * f;
            aa += wacc[w][r][d] * f;
        }
        const int h = kh * R + r;
        if (p.splits == 1) {
            const size_t oi = ((size_t)query * p.heads + h) * HD + d;
            p.out[oi] = gated(p, oi, ll > 0.f ? aa / ll : 0.f);
        } else {
            const size_t prow = ((size_t)query * p.heads + h) * p.splits + split;
            p.part_acc[prow * HD + d] = aa;
            if (d == 0) {
                p.part_m[prow] = mm;
                p.part_l[prow] = ll;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Prefill with query tiles: one CTA per (entry, KV head, tile of TQ = 128 / R
// queries), one thread per (query, head) row holding its query in registers.
// Blocks of 32 positions -- the union of the tile's visible sets -- are read
// once into shared memory as floats (with their scales) and used by every query
// of the tile; per block each row computes its 32 scores (causally masked),
// updates its running max once, and accumulates (p * v_scale) * v.
constexpr int kPBK = 32;

// Memory row of absolute position `position` of (session s, KV head kh) for a
// query of entry `entry` whose chunk starts at chunk_start.
__device__ __forceinline__ RowPtr position_ptr(const AttnParams &p, int s, int kh, int position, int entry,
                                               int chunk_start) {
    size_t row;
    RowPtr r;
    if (p.stage_k && position >= chunk_start) {
        row = (size_t)kh * p.stage_rows + (size_t)entry * p.tokens + (position - chunk_start);
        r.k = p.stage_k; r.v = p.stage_v; r.ks = p.stage_ks; r.vs = p.stage_vs;
    } else if (position < p.prefix) {
        row = (size_t)kh * p.prefix + position;
        r.k = p.pk; r.v = p.pv; r.ks = p.pks; r.vs = p.pvs;
    } else {
        const int slot = p.window ? (position - p.prefix) % p.window : position - p.prefix;
        row = ((size_t)s * p.kvheads + kh) * p.cs + slot;
        r.k = p.sk; r.v = p.sv; r.ks = p.sks; r.vs = p.svs;
    }
    r.k += row * p.hd;
    r.v += row * p.hd;
    r.ks += row;
    r.vs += row;
    r.run = 0;
    return r;
}

template <int HD, int R>
__global__ void __launch_bounds__(128) attn_prefill_tile_kernel(const AttnParams p) {
    pdl_enter();
    constexpr int TQ = 128 / R;
    __shared__ __align__(16) float ks_f[kPBK][HD], vs_f[kPBK][HD];
    __shared__ float kscale[kPBK], vscale[kPBK];
    __shared__ int kpos[kPBK];

    const int tile = blockIdx.x, kh = blockIdx.y, entry = blockIdx.z;
    const int s = p.session[entry], chunk_start = p.position[entry];
    const int tid = threadIdx.x, r = tid % R, i = tid / R;
    const int t = tile * TQ + i;
    const bool active = t < p.tokens;
    const int pos = chunk_start + min(t, p.tokens - 1);
    const int h = kh * R + r;
    // visible set of this row: sinks [0, prefix_count) and [start, pos]
    const int prefix_count = p.window ? min(p.prefix, pos + 1) : 0;
    const int start = p.window ? max(p.prefix, pos - p.window + 1) : 0;
    // the tile's union: its last query has the largest position and the latest
    // start; its first query the earliest start
    const int t_last = min(p.tokens - 1, tile * TQ + TQ - 1), t_first = tile * TQ;
    const int pos_hi = chunk_start + t_last, pos_lo = chunk_start + t_first;
    const int sinks = p.window ? min(p.prefix, pos_hi + 1) : 0;
    const int ustart = p.window ? max(p.prefix, pos_lo - p.window + 1) : 0;
    const int nsink = sinks, nrange = max(0, pos_hi - max(ustart, nsink) + 1);
    const int range0 = max(ustart, nsink);
    const int total = nsink + nrange;   // union positions: [0, nsink) then range0 ...

    float q[HD];
    const float *qp = p.q + ((size_t)(entry * p.tokens + min(t, p.tokens - 1)) * p.heads + h) * HD;
#pragma unroll
    for (int d = 0; d < HD; d += 4) {
        const float4 v = *reinterpret_cast<const float4 *>(qp + d);
        q[d] = v.x; q[d + 1] = v.y; q[d + 2] = v.z; q[d + 3] = v.w;
    }
    float acc[HD];
#pragma unroll
    for (int d = 0; d < HD; ++d) acc[d] = 0.f;
    float m = -INFINITY, l = 0.f;
    const float inv_sqrt = p.inv_sqrt_hd;

    for (int b0 = 0; b0 < total; b0 += kPBK) {
        const int nb = min(kPBK, total - b0);
        __syncthreads();   // the previous block is no longer read
        // 128 threads: row j = tid / 4 of the block, 16 dims (HD = 64) or 32 (HD = 128) each
        {
            const int j = tid >> 2, part = tid & 3;
            if (j < nb) {
                const int u = b0 + j;
                const int position = u < nsink ? u : range0 + (u - nsink);
                const RowPtr rp = position_ptr(p, s, kh, position, entry, chunk_start);
                constexpr int PER = HD / 4;
#pragma unroll
                for (int c = 0; c < PER; c += 16) {
                    const uint4 kw = *reinterpret_cast<const uint4 *>(rp.k + part * PER + c);
                    const uint4 vw = *reinterpret_cast<const uint4 *>(rp.v + part * PER + c);
                    const uint32_t kwords[4] = {kw.x, kw.y, kw.z, kw.w}, vwords[4] = {vw.x, vw.y, vw.z, vw.w};
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        float2 lo, hi;
                        i8x4_pairs(kwords[w], lo, hi);
                        float *kd = &ks_f[j][part * PER + c + 4 * w];
                        kd[0] = lo.x; kd[1] = lo.y; kd[2] = hi.x; kd[3] = hi.y;
                        i8x4_pairs(vwords[w], lo, hi);
                        float *vd = &vs_f[j][part * PER + c + 4 * w];
                        vd[0] = lo.x; vd[1] = lo.y; vd[2] = hi.x; vd[3] = hi.y;
                    }
                }
                if (part == 0) {
                    kscale[j] = *rp.ks;
                    vscale[j] = *rp.vs;
                    kpos[j] = position;
                }
            }
        }
        __syncthreads();
        if (!active) continue;
        // sub-chunks of 8 keys (a rolled loop: the unrolled body stays small
        // enough for the instruction cache); one max update and rescale each
#pragma unroll 1
        for (int j0 = 0; j0 < nb; j0 += 8) {
            float sc[8];
            float mx = -INFINITY;
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                const int j = j0 + jj;
                float v = -INFINITY;
                if (j < nb) {
                    const int position = kpos[j];
                    const bool vis = position <= pos && (position < prefix_count || position >= start);
                    if (vis) {
                        float d0 = 0.f, d1 = 0.f;
#pragma unroll
                        for (int d = 0; d < HD; d += 4) {
                            const float4 kv = *reinterpret_cast<const float4 *>(&ks_f[j][d]);
                            d0 = fmaf(q[d], kv.x, d0);
                            d1 = fmaf(q[d + 1], kv.y, d1);
                            d0 = fmaf(q[d + 2], kv.z, d0);
                            d1 = fmaf(q[d + 3], kv.w, d1);
                        }
                        v = __fmul_rn(__fmul_rn(d0 + d1, kscale[j]), inv_sqrt);
                    }
                }
                sc[jj] = v;
                mx = fmaxf(mx, v);
            }
            if (mx == -INFINITY) continue;   // nothing of these keys is visible to this row
            const float mn = fmaxf(m, mx);
            const float corr = m == -INFINITY ? 0.f : __expf(m - mn);
            m = mn;
            l *= corr;
#pragma unroll
            for (int d = 0; d < HD; ++d) acc[d] *= corr;
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                if (sc[jj] == -INFINITY) continue;
                const int j = j0 + jj;
                const float pr = __expf(sc[jj] - mn);
                l += pr;
                const float w = pr * vscale[j];
#pragma unroll
                for (int d = 0; d < HD; d += 4) {
                    const float4 vv = *reinterpret_cast<const float4 *>(&vs_f[j][d]);
                    acc[d] = fmaf(w, vv.x, acc[d]);
                    acc[d + 1] = fmaf(w, vv.y, acc[d + 1]);
                    acc[d + 2] = fmaf(w, vv.z, acc[d + 2]);
                    acc[d + 3] = fmaf(w, vv.w, acc[d + 3]);
                }
            }
        }
    }
    if (active) {
        const size_t o0 = ((size_t)(entry * p.tokens + t) * p.heads + h) * HD;
        float *op = p.out + o0;
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
        for (int d = 0; d < HD; d += 4)
            *reinterpret_cast<float4 *>(op + d) =
                make_float4(gated(p, o0 + d, acc[d] * inv), gated(p, o0 + d + 1, acc[d + 1] * inv),
                            gated(p, o0 + d + 2, acc[d + 2] * inv), gated(p, o0 + d + 3, acc[d + 3] * inv));
    }
}

template <int HD>
bool launch_prefill_tile(const AttnParams &p, int entries, int R, cudaStream_t st) {
    const int tq = 128 / R;
    const dim3 grid((p.tokens + tq - 1) / tq, p.kvheads, entries);
    switch (R) {
        case 1: NB_CUDA_TRY(launch_pdl(attn_prefill_tile_kernel<HD, 1>, grid, 128, 0, st, p)); return true;
        case 2: NB_CUDA_TRY(launch_pdl(attn_prefill_tile_kernel<HD, 2>, grid, 128, 0, st, p)); return true;
        case 4: NB_CUDA_TRY(launch_pdl(attn_prefill_tile_kernel<HD, 4>, grid, 128, 0, st, p)); return true;
        default: return false;
    }
}

// Dynamic shared memory of attn_stream_kernel<HD, ...>: the warps' copy rings.
template <int HD>
constexpr size_t stream_smem() { return (size_t)StreamGeo<HD>::NW * StreamGeo<HD>::RING + 128; }

template <typename K>
bool launch_ring_kernel(K kernel, size_t smem, dim3 grid, cudaStream_t st, const AttnParams &p) {
    if (smem > 48 * 1024)   // (every launch: the kernels share K, so a per-type flag would not do)
        NB_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    NB_CUDA_TRY(launch_pdl(kernel, grid, 128, smem, st, p));
    return true;
}

template <int HD, bool WPQ, bool FQ>
bool launch_stream_fq(const AttnParams &p, dim3 grid, int R, cudaStream_t st) {
    constexpr size_t smem = stream_smem<HD>();
    switch (R) {
        case 1: return launch_ring_kernel(attn_stream_kernel<HD, 1, WPQ, FQ>, smem, grid, st, p);
        case 2:
            if constexpr (!WPQ || 2 * HD / 4 <= 32)
                return launch_ring_kernel(attn_stream_kernel<HD, 2, WPQ, FQ>, smem, grid, st, p);
            return false;
        case 4:
            if constexpr (HD <= 64 && !WPQ) return launch_ring_kernel(attn_stream_kernel<HD, 4, false, FQ>, smem, grid, st, p);
            return false;
        default: return false;
    }
}
template <int HD, bool WPQ>
bool launch_stream(const AttnParams &p, dim3 grid, int R, cudaStream_t st) {
    return p.qkv_q ? launch_stream_fq<HD, WPQ, true>(p, grid, R, st) : launch_stream_fq<HD, WPQ, false>(p, grid, R, st);
}

// Merge the split partials of each (query, head).
__global__ void attn_combine_kernel(const AttnParams p, int hd) {
    pdl_enter();
    const int qh = blockIdx.x;   // query * heads + h
    const float *pm = p.part_m + (size_t)qh * p.splits, *pl = p.part_l + (size_t)qh * p.splits;
    float mm = -INFINITY;
    for (int j = 0; j < p.splits; ++j) mm = fmaxf(mm, pm[j]);
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float ll = 0.f, aa = 0.f;
        for (int j = 0; j < p.splits; ++j) {
            if (pm[j] == -INFINITY) continue;
            const float f = expf(pm[j] - mm);
            ll += pl[j] * f;
            aa += p.part_acc[((size_t)qh * p.splits + j) * hd + d] * f;
        }
        p.out[(size_t)qh * hd + d] = gated(p, (size_t)qh * hd + d, ll > 0.f ? aa / ll : 0.f);
    }
}

// The split combine for one (query, KV head) with the out projection's input
// rotation: thread t = r * hd + d combines head kh * R + r, dimension d as
// attn_combine_kernel does, then the R * hd outputs are rotated (stages
// h < 32 across lanes, the rest through shared memory, in order) and split.
__global__ void attn_combine_rot_kernel(const AttnParams p, int hd) {
    pdl_enter();
    extern __shared__ float xs[];   // [2][R * hd]
    const int R = p.heads / p.kvheads, n = R * hd;
    const int t = threadIdx.x;
    const int query = blockIdx.x / p.kvheads, kh = blockIdx.x % p.kvheads;
    const int r = t / hd, d = t % hd;
    const int qh = query * p.heads + kh * R + r;
    const float *pm = p.part_m + (size_t)qh * p.splits, *pl = p.part_l + (size_t)qh * p.splits;
    float mm = -INFINITY;
    for (int j = 0; j < p.splits; ++j) mm = fmaxf(mm, pm[j]);
    float ll = 0.f, aa = 0.f;
    for (int j = 0; j < p.splits; ++j) {
        if (pm[j] == -INFINITY) continue;
        const float f = expf(pm[j] - mm);
        ll += pl[j] * f;
        aa += p.part_acc[((size_t)qh * p.splits + j) * hd + d] * f;
    }
    float v = gated(p, (size_t)qh * hd + d, ll > 0.f ? aa / ll : 0.f);
    p.out[(size_t)qh * hd + d] = v;
    int h = 1;
    for (; h < 32 && h < n; h *= 2) {
        const float o = __shfl_xor_sync(kFull, v, h);
        v = (t & h) ? __fsub_rn(o, v) : __fadd_rn(v, o);
    }
    int buf = 0;
    for (; h < n; h *= 2) {
        xs[buf * n + t] = v;
        __syncthreads();
        const float o = xs[buf * n + (t ^ h)];
        v = (t & h) ? __fsub_rn(o, v) : __fadd_rn(v, o);
        buf ^= 1;
    }
    const float x = __fmul_rn(v, p.rot_scale);
    const size_t i = (size_t)query * p.hilo_ld + (size_t)kh * n + t;
    const __nv_bfloat16 hv = __float2bfloat16_rn(x);
    p.hilo[i] = __bfloat16_as_ushort(hv);
    p.hilo[p.hilo_lo + i] = __bfloat16_as_ushort(__float2bfloat16_rn(__fsub_rn(x, __bfloat162float(hv))));
}

}  // namespace

bool launch_kv_quantize(const float *k, const float *v, int tokens, int kvheads, int hd, int8_t *ko, int8_t *vo,
                        float *ks, float *vs, const KVDest &dest, cudaStream_t st) {
    if (tokens <= 0) return true;
    const long long warps = (long long)tokens * kvheads;
    NB_CUDA_TRY(launch_pdl(kv_quantize_kernel, (unsigned)((warps * 32 + 255) / 256), 256, 0, st, k, v, tokens, kvheads, hd, ko, vo, ks, vs,
                                                                             dest));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_kv_store_f32(const float *k, const float *v, int tokens, int kvheads, int hd, float *ko, float *vo,
                         const KVDest &dest, cudaStream_t st) {
    if (tokens <= 0) return true;
    const long long warps = (long long)tokens * kvheads;
    NB_CUDA_TRY(launch_pdl(kv_store_f32_kernel, (unsigned)((warps * 32 + 255) / 256), 256, 0, st, k, v, tokens, kvheads, hd, ko, vo, dest));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

// (query, KV head) pairs from which decode runs one warp per pair: 1024 CTAs
// of four warps, several waves on 148 SMs.
constexpr long long kWpqMinPairs = 2048;

int attention_splits(int max_len, int queries_x_kv, int sms) {
    // split the context only while the (query, KV head) pairs leave SMs idle
    // (fewer than two CTAs an SM), down to 128 slots a split.  Measured at
    // config 5's 128 and 256 sessions (512 / 1024 pairs, ~300 slots): the
    // unsplit kernel, which also needs no combine launch, beats two splits
    // (0.600 vs 0.686 ms a decode step at 128 sessions).
    int splits = 1;
    while (splits < 32 && (long long)queries_x_kv * splits < 2LL * sms && max_len / (splits * 2) >= 128) splits *= 2;
    return splits;
}

// The split combine, rotating for the out projection where p.hilo asks for it.
bool launch_combine(const AttnParams &p, int queries, cudaStream_t st, bool *rot_done) {
    const int n = p.heads / p.kvheads * p.hd;
    if (p.hilo && n % 32 == 0 && n <= 1024) {
        NB_CUDA_TRY(launch_pdl(attn_combine_rot_kernel, queries * p.kvheads, n, 2 * n * sizeof(float), st, p, p.hd));
        if (rot_done) *rot_done = true;
    } else {
        NB_CUDA_TRY(launch_pdl(attn_combine_kernel, queries * p.heads, 64, 0, st, p, p.hd));
    }
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

namespace {
// INT8 decode runs one warp per (query, KV head) pair (attn_stream_kernel<.., true>).
bool decode_wpq(const AttnParams &p, int queries) {
    const int R = p.heads / p.kvheads;
    return p.splits == 1 && ((p.hd == 64 && R <= 2) || (p.hd == 128 && R <= 1)) &&
           (long long)queries * p.kvheads >= kWpqMinPairs;
}
}  // namespace

bool attention_fuses_qkv(const AttnParams &p, int queries, int sms) {
    if (p.f32 || p.tokens != 1 || p.stage_k || p.heads % p.kvheads) return false;
    // the warp-per-query form while its CTAs (four queries each, four CTAs an SM)
    // fit one wave: measured at config 5, 512 sessions 1.152 vs 1.25 ms a step
    // with the projections' epilogue instead; 1024 sessions (1.7 waves, the
    // prologue paid twice) 2.128 vs 1.997 ms
    if (decode_wpq(p, queries)) return (long long)p.kvheads * ((queries + 3) / 4) <= 4LL * sms;
    const int R = p.heads / p.kvheads;
    return (p.hd == 64 && (R == 1 || R == 2 || R == 4)) || (p.hd == 128 && (R == 1 || R == 2));
}

bool launch_attention(const AttnParams &p_in, int queries, cudaStream_t st, bool *rot_done) {
    if (rot_done) *rot_done = false;
    if (queries <= 0) return true;
    AttnParams p = p_in;
    if (p.tokens != 1) p.hilo = nullptr;   // decode only
    if (p.heads % p.kvheads || p.heads / p.kvheads > kMaxQueryGroup) {
        set_error("attention supports up to 8 query heads per KV head");
        return false;
    }
    if (p.qkv_q && !attention_fuses_qkv(p, queries, 1 << 20)) {
        set_error("attention: the new token's projections as parts need the unsplit-or-split INT8 decode kernel");
        return false;
    }
    dim3 grid(p.splits, p.kvheads, queries);
    const int R = p.heads / p.kvheads;
    if (p.f32) {
        switch (p.hd) {
            case 32: NB_CUDA_TRY(launch_pdl(attn_split_kernel<32, true, float>, grid, 128, 0, st, p)); break;
            case 64: NB_CUDA_TRY(launch_pdl(attn_split_kernel<64, true, float>, grid, 128, 0, st, p)); break;
            case 128: NB_CUDA_TRY(launch_pdl(attn_split_kernel<128, true, float>, grid, 128, 0, st, p)); break;
            default:
                if (p.hd <= 32) NB_CUDA_TRY(launch_pdl(attn_split_kernel<32, false, float>, grid, 128, 0, st, p));
                else if (p.hd <= 64) NB_CUDA_TRY(launch_pdl(attn_split_kernel<64, false, float>, grid, 128, 0, st, p));
                else if (p.hd <= 128) NB_CUDA_TRY(launch_pdl(attn_split_kernel<128, false, float>, grid, 128, 0, st, p));
                else {
                    set_error("head_dim above 128 is not supported by the GPU build");
                    return false;
                }
        }
        NB_CUDA_TRY(cudaGetLastError());
        if (p.splits > 1) return launch_combine(p, queries, st, rot_done);
        return true;
    }
    // prefill chunks of 16+ tokens: query tiles share every K/V read
    if (p.tokens >= 16 && p.hd == 64 && R <= 4 && queries % p.tokens == 0) {
        if (!launch_prefill_tile<64>(p, queries / p.tokens, R, st)) return false;
        NB_CUDA_TRY(cudaGetLastError());
        return true;
    }
    bool streamed = false;
    // one warp per query where the context needs no split, the query fits the
    // registers and the queries alone fill the machine; with fewer, the CTA's
    // warps share each query's slots
    const bool wpq = decode_wpq(p, queries);
    AttnParams pw = p;
    pw.queries = queries;
    // the warp-per-query epilogue rotates one KV head's 2 x 64 outputs
    if (!(wpq && p.hd == 64 && R == 2)) pw.hilo = nullptr;
    // the unsplit multi-warp stream kernel rotates up to 128 outputs of a KV head
    const int nkv = R * p.hd;
    const bool stream_rot = p.hilo && p.splits == 1 && !wpq && nkv % 32 == 0 && nkv <= 128;
    if (p.splits == 1 && !stream_rot) p.hilo = nullptr;
    const dim3 wgrid(1, p.kvheads, (queries + 3) / 4);
    if (wpq && p.hd == 64) {
        streamed = launch_stream<64, true>(pw, wgrid, R, st);
        if (streamed && pw.hilo && rot_done) *rot_done = true;
    }
    else if (wpq && p.hd == 128) streamed = launch_stream<128, true>(pw, wgrid, R, st);
    // the streaming kernel where its per-lane state fits in registers
    else if (p.hd == 64 && R <= 4) streamed = launch_stream<64, false>(p, grid, R, st);
    else if (p.hd == 128 && R <= 2) streamed = launch_stream<128, false>(p, grid, R, st);
    if (streamed && stream_rot && rot_done) *rot_done = true;
    if (!streamed) p.hilo = p.splits > 1 ? p.hilo : nullptr;
    if (!streamed) switch (p.hd) {
        case 32: NB_CUDA_TRY(launch_pdl(attn_split_kernel<32, true, int8_t>, grid, 128, 0, st, p)); break;
        case 64: NB_CUDA_TRY(launch_pdl(attn_split_kernel<64, true, int8_t>, grid, 128, 0, st, p)); break;
        case 128: NB_CUDA_TRY(launch_pdl(attn_split_kernel<128, true, int8_t>, grid, 128, 0, st, p)); break;
        default:
            if (p.hd <= 32) NB_CUDA_TRY(launch_pdl(attn_split_kernel<32, false, int8_t>, grid, 128, 0, st, p));
            else if (p.hd <= 64) NB_CUDA_TRY(launch_pdl(attn_split_kernel<64, false, int8_t>, grid, 128, 0, st, p));
            else if (p.hd <= 128) NB_CUDA_TRY(launch_pdl(attn_split_kernel<128, false, int8_t>, grid, 128, 0, st, p));
            else {
                set_error("head_dim above 128 is not supported by the GPU build");
                return false;
            }
    }
    NB_CUDA_TRY(cudaGetLastError());
    if (p.splits > 1) return launch_combine(p, queries, st, rot_done);
    return true;
}

}  // namespace nb200
