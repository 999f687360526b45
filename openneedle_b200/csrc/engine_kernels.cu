// Support kernels of the Needle-2 forward (see engine.cuh).  Each follows the
// cited operation of needle2/csrc/engine.cpp in FP32 with the same operation
// order where one thread owns an element; reductions over a row (RMS sums,
// dot products) run as warp/block trees, a different association within FP32
// rounding.  The x86 reference build has no FMA contraction, so the
// elementwise formulas here use explicit round-to-nearest multiply/add.
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "pdl.cuh"
#include "engine.cuh"
#include "engine_math.cuh"
#include "kv_pool.cuh"
#include "qkvg_epilogue.cuh"

namespace nb200 {
namespace eng {
namespace {

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

// Sum over the block (blockDim.x a multiple of 32, at most 1024); every thread
// gets the result.  `sh` holds 33 floats.
__device__ float block_sum(float v, float *sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = lane < nw ? sh[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) sh[32] = t;
    }
    __syncthreads();
    return sh[32];
}

// ------------------------------------------------------------------ kernels

__global__ void embed_lanes_kernel(const float *__restrict__ rows, int lanes, int D, float scale,
                                   float *__restrict__ x) {
    pdl_enter();
    const int r = blockIdx.x;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        const float v = __fmul_rn(rows[(size_t)r * D + d], scale);
        for (int n = 0; n < lanes; ++n) x[((size_t)r * lanes + n) * D + d] = v;
    }
}

__global__ void gather_dense_kernel(const float *__restrict__ w, const int64_t *__restrict__ ids, int cols,
                                    float *__restrict__ out) {
    pdl_enter();
    const int r = blockIdx.x;
    const float *src = w + (size_t)ids[r] * cols;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) out[(size_t)r * cols + c] = src[c];
}

__global__ void rms_kernel(const float *__restrict__ x, int ldx, int n, const float *__restrict__ scale,
                           float *__restrict__ y, int ldy) {
    pdl_enter();
    __shared__ float sh[33];
    const int r = blockIdx.x;
    const float *xr = x + (size_t)r * ldx;
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s = fmaf(xr[i], xr[i], s);
    const float inv = rms_inv(block_sum(s, sh), n);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = __fmul_rn(xr[i], inv);
        y[(size_t)r * ldy + i] = scale ? __fmul_rn(v, __fadd_rn(1.f, scale[i])) : v;
    }
}

struct DenseSegs {
    DenseSeg s[3];
    int n;
};

// One warp per matrix row, eight input rows per CTA.
__global__ void __launch_bounds__(256) dense_rows_kernel(const DenseSegs segs, const float *__restrict__ in, int ldin,
                                                         int R, int cols) {
    pdl_enter();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int j = blockIdx.x * 8 + warp;
    int si = 0;
    while (si < segs.n && j >= segs.s[si].rows) j -= segs.s[si++].rows;
    if (si >= segs.n) return;
    const DenseSeg &sg = segs.s[si];
    const float *w = sg.w + (size_t)(sg.first + j) * cols;
    const int r0 = blockIdx.y * 8;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int k = lane; k < cols; k += 32) {
        const float wv = __ldg(w + k);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (r0 + i < R) acc[i] = fmaf(wv, __ldg(in + (size_t)(r0 + i) * ldin + k), acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float v = warp_sum(acc[i]);
        if (lane == 0 && r0 + i < R) sg.out[(size_t)(r0 + i) * sg.ldo + j] = v;
    }
}

__global__ void __launch_bounds__(256) mhc_pre_kernel(const MhcLayer L, const float *__restrict__ raw, int ldraw,
                                                      const float *__restrict__ x, float *__restrict__ hpost,
                                                      float *__restrict__ u, float *__restrict__ bx,
                                                      float *__restrict__ z) {
    pdl_enter();
    extern __shared__ float smem[];
    float *bxs = smem;                 // [D]
    __shared__ float hpre[kMaxLanes];
    __shared__ float sh[33];
    const int r = blockIdx.x, N = L.lanes, D = L.D;
    const float *rr = raw + (size_t)r * ldraw;
    if (threadIdx.x < N) {
        const int n = threadIdx.x;
        const bool own = n == L.layer % N;
        // engine.cpp:983-984: sigmoid(a * h + b + (own lane ? 4 : -4)), 2 * sigmoid(a * h + b + (own ? 0 : -4))
        hpre[n] = sigm(__fadd_rn(__fadd_rn(__fmul_rn(L.a_pre, rr[n]), L.b_pre[n]), own ? 4.f : -4.f));
        hpost[(size_t)r * N + n] =
            __fmul_rn(2.f, sigm(__fadd_rn(__fadd_rn(__fmul_rn(L.a_post, rr[N + n]), L.b_post[n]), own ? 0.f : -4.f)));
    }
    __syncthreads();
    const float *xr = x + (size_t)r * N * D;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float sum = 0.f;
        for (int n = 0; n < N; ++n) sum = __fadd_rn(sum, __fmul_rn(hpre[n], xr[(size_t)n * D + d]));
        u[(size_t)r * D + d] = sum;
        bxs[d] = sum;
    }
    if (L.ek) {
        // engine.cpp:987-990: alpha = sigmoid(rms(u) . rms(ek) / sqrt(D)); bx += alpha * ev
        const float *ek = L.ek + (size_t)r * L.ld_site, *ev = L.ev + (size_t)r * L.ld_site;
        float su = 0.f, se = 0.f;
        for (int d = threadIdx.x; d < D; d += blockDim.x) {
            su = fmaf(bxs[d], bxs[d], su);
            se = fmaf(ek[d], ek[d], se);
        }
        const float iu = rms_inv(block_sum(su, sh), D), ie = rms_inv(block_sum(se, sh), D);
        float dot = 0.f;
        for (int d = threadIdx.x; d < D; d += blockDim.x) dot = fmaf(__fmul_rn(bxs[d], iu), __fmul_rn(ek[d], ie), dot);
        const float alpha = sigm(__fdiv_rn(block_sum(dot, sh), sqrtf((float)D)));
        for (int d = threadIdx.x; d < D; d += blockDim.x) bxs[d] = __fadd_rn(bxs[d], __fmul_rn(alpha, ev[d]));
    }
    __syncthreads();
    float sb = 0.f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) sb = fmaf(bxs[d], bxs[d], sb);
    const float ib = rms_inv(block_sum(sb, sh), D);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        bx[(size_t)r * D + d] = bxs[d];
        z[(size_t)r * D + d] = __fmul_rn(__fmul_rn(bxs[d], ib), __fadd_rn(1.f, L.norm_in[d]));
    }
}

__device__ float warp_sinkhorn(float a, int n, int lane);

// Fused mHC routing of SB rows per CTA (engine.cpp:980-992): the lanes' RMS
// (nx, staged in shared memory), the 2N + N^2 FP32 projections of nx (each
// CTA streams the layer's projection rows once for its SB rows), the gates,
// u, the engram mixing and z = rms(bx) * (1 + norm_in).  Needs N * D % 128 == 0.
template <int SB>
__global__ void __launch_bounds__(256) mhc_route_kernel(const MhcLayer L, const float *__restrict__ phi_pre,
                                                        const float *__restrict__ phi_post,
                                                        const float *__restrict__ phi_res,
                                                        const float *__restrict__ x, int R, float *__restrict__ raw,
                                                        int ldraw, float *__restrict__ hpost, float *__restrict__ u,
                                                        float *__restrict__ bx, float *__restrict__ z) {
    pdl_enter();
    extern __shared__ float smem[];
    const int N = L.lanes, D = L.D, ND = N * D;
    float *nx = smem;                              // [SB][ND]
    __shared__ float raws[SB][3 * kMaxLanes + kMaxLanes * kMaxLanes];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int r0 = blockIdx.x * SB;
    // 1. nx = rms(x) over the N lanes (engine.cpp:980)
    for (int s = warp; s < SB; s += nw) {
        const int r = r0 + s;
        if (r >= R) continue;
        const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)r * ND);
        float ss = 0.f;
        for (int k = lane; k < ND / 4; k += 32) {
            const float4 v = xr[k];
            ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
        }
        const float inv = rms_inv(warp_sum(ss), ND);
        float4 *dst = reinterpret_cast<float4 *>(nx + (size_t)s * ND);
        for (int k = lane; k < ND / 4; k += 32) {
            const float4 v = xr[k];
            dst[k] = make_float4(__fmul_rn(v.x, inv), __fmul_rn(v.y, inv), __fmul_rn(v.z, inv), __fmul_rn(v.w, inv));
        }
    }
    __syncthreads();
    // 2. raw[s][j] = phi_j . nx[s] for the layer's 2N + N^2 projection rows (engine.cpp:529-559)
    const int rows = 2 * N + N * N;
    for (int j = warp; j < rows; j += nw) {
        const float *w = j < N ? phi_pre + (size_t)(L.layer * N + j) * ND
                       : j < 2 * N ? phi_post + (size_t)(L.layer * N + j - N) * ND
                                   : phi_res + (size_t)(L.layer * N * N + j - 2 * N) * ND;
        float acc[SB];
#pragma unroll
        for (int s = 0; s < SB; ++s) acc[s] = 0.f;
        for (int k = lane; k < ND / 4; k += 32) {
            const float4 wv = __ldg(reinterpret_cast<const float4 *>(w) + k);
#pragma unroll
            for (int s = 0; s < SB; ++s) {
                const float4 v = reinterpret_cast<const float4 *>(nx + (size_t)s * ND)[k];
                acc[s] = fmaf(wv.x, v.x, fmaf(wv.y, v.y, fmaf(wv.z, v.z, fmaf(wv.w, v.w, acc[s]))));
            }
        }
#pragma unroll
        for (int s = 0; s < SB; ++s) {
            const float t = warp_sum(acc[s]);
            if (lane == 0) raws[s][j] = t;
        }
    }
    __syncthreads();
    // 3. per row: gates, u = sum_n hpre[n] x[n], engram mixing, z (engine.cpp:982-992)
    for (int s = warp; s < SB; s += nw) {
        const int r = r0 + s;
        if (r >= R) continue;
        for (int j = lane; j < 2 * N; j += 32) raw[(size_t)r * ldraw + j] = raws[s][j];
        {
            // engine.cpp:1033-1034: hres = sinkhorn(res * a_res + b_res), stored in place of res
            const int nn = N * N;
            const float hr = lane < nn ? __fadd_rn(__fmul_rn(raws[s][2 * N + lane], L.a_res), L.b_res[lane]) : 0.f;
            const float hres = warp_sinkhorn(hr, N, lane);
            if (lane < nn) raw[(size_t)r * ldraw + 2 * N + lane] = hres;
        }
        float hpre = 0.f;
        if (lane < N) {
            const bool own = lane == L.layer % N;
            hpre = sigm(__fadd_rn(__fadd_rn(__fmul_rn(L.a_pre, raws[s][lane]), L.b_pre[lane]), own ? 4.f : -4.f));
            hpost[(size_t)r * N + lane] = __fmul_rn(
                2.f, sigm(__fadd_rn(__fadd_rn(__fmul_rn(L.a_post, raws[s][N + lane]), L.b_post[lane]), own ? 0.f : -4.f)));
        }
        float *bxs = nx + (size_t)s * ND;          // this row's nx is no longer needed: bx lives there
        const float *xr = x + (size_t)r * ND;
        for (int d = lane; d < D; d += 32) {
            float sum = 0.f;
            for (int n = 0; n < N; ++n)
                sum = __fadd_rn(sum, __fmul_rn(__shfl_sync(kFull, hpre, n), xr[(size_t)n * D + d]));
            u[(size_t)r * D + d] = sum;
            bxs[d] = sum;
        }
        if (L.ek) {
            const float *ek = L.ek + (size_t)r * L.ld_site, *ev = L.ev + (size_t)r * L.ld_site;
            float su = 0.f, se = 0.f;
            for (int d = lane; d < D; d += 32) {
                su = fmaf(bxs[d], bxs[d], su);
                se = fmaf(ek[d], ek[d], se);
            }
            const float iu = rms_inv(warp_sum(su), D), ie = rms_inv(warp_sum(se), D);
            float dot = 0.f;
            for (int d = lane; d < D; d += 32) dot = fmaf(__fmul_rn(bxs[d], iu), __fmul_rn(ek[d], ie), dot);
            const float alpha = sigm(__fdiv_rn(warp_sum(dot), sqrtf((float)D)));
            for (int d = lane; d < D; d += 32) bxs[d] = __fadd_rn(bxs[d], __fmul_rn(alpha, ev[d]));
        }
        float sb = 0.f;
        for (int d = lane; d < D; d += 32) sb = fmaf(bxs[d], bxs[d], sb);
        const float ib = rms_inv(warp_sum(sb), D);
        for (int d = lane; d < D; d += 32) {
            bx[(size_t)r * D + d] = bxs[d];
            z[(size_t)r * D + d] = __fmul_rn(__fmul_rn(bxs[d], ib), __fadd_rn(1.f, L.norm_in[d]));
        }
    }
}

// One warp per head: RMS with (1 + norm), then RoPE on the half-split pairs.
__global__ void qk_norm_rope_kernel(float *__restrict__ q, float *__restrict__ k, int heads, int kvheads, int hd,
                                    const float *__restrict__ q_norm, const float *__restrict__ k_norm,
                                    const int *__restrict__ pos, const float *__restrict__ divisor) {
    pdl_enter();
    extern __shared__ float buf[];   // [warps][hd]
    const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const float fpos = (float)pos[r];
    for (int h = warp; h < heads + kvheads; h += nw) {
        const bool isq = h < heads;
        float *v = isq ? q + ((size_t)r * heads + h) * hd : k + ((size_t)r * kvheads + (h - heads)) * hd;
        const float *nrm = isq ? q_norm : k_norm;
        float *b = buf + warp * hd;
        float s = 0.f;
        for (int i = lane; i < hd; i += 32) s = fmaf(v[i], v[i], s);
        const float inv = rms_inv(warp_sum(s), hd);
        for (int i = lane; i < hd; i += 32) b[i] = __fmul_rn(__fmul_rn(v[i], inv), __fadd_rn(1.f, nrm[i]));
        __syncwarp();
        const int half = hd / 2;
        for (int j = lane; j < half; j += 32) {
            const float ang = __fdiv_rn(fpos, divisor[j]);
            const float co = cosf(ang), si = sinf(ang);
            const float a = b[j], c = b[j + half];
            v[j] = __fsub_rn(__fmul_rn(a, co), __fmul_rn(c, si));
            v[j + half] = __fadd_rn(__fmul_rn(c, co), __fmul_rn(a, si));
        }
        __syncwarp();
    }
}

// qk_norm_rope_kernel followed, for one token per row, by the KV store of the
// row's K (after RoPE) and V: INT8 by the reference's rule (engine.cpp:1005-1021,
// scale max/127 or 1, values rint(x * (127 / max)) clamped to +-127, as
// kv_quantize_kernel) or FP32 as is, into the row of target.dest.
__global__ void qk_rope_store_kernel(float *__restrict__ q, float *__restrict__ k, float *__restrict__ v, int heads,
                                     int kvheads, int hd, const float *__restrict__ q_norm,
                                     const float *__restrict__ k_norm, const int *__restrict__ pos,
                                     const float *__restrict__ divisor, const KVStoreTarget t,
                                     const float *__restrict__ cos_t, const float *__restrict__ sin_t, int table_len,
                                     const QkvgParts src) {
    pdl_enter();
    extern __shared__ float buf[];   // [warps][hd]
    const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const float fpos = (float)pos[r];
    const KVDest &d = t.dest;
    const int units = heads + 2 * kvheads + (src.q ? heads : 0);   // q, k, v heads (and gate heads)
    for (int h = warp; h < units; h += nw) {
        if (h >= heads + 2 * kvheads) {   // a gate head: its parts added
            const size_t o = ((size_t)r * heads + (h - heads - 2 * kvheads)) * hd;
            for (int i = lane; i < hd; i += 32) src.gate[o + i] = part_sum(src.g + o + i, src.parts, src.pstride);
            continue;
        }
        const bool isv = h >= heads + kvheads;
        const bool isq = h < heads;
        const int kh = isq ? 0 : isv ? h - heads - kvheads : h - heads;
        const size_t off = isq ? ((size_t)r * heads + h) * hd : ((size_t)r * kvheads + kh) * hd;
        float *vp = (isq ? q : isv ? v : k) + off;
        if (src.q) {
            const float *sp = (isq ? src.q : isv ? src.v : src.k) + off;
            for (int i = lane; i < hd; i += 32) vp[i] = part_sum(sp + i, src.parts, src.pstride);
            __syncwarp();
        }
        if (!isv) {
            const float *nrm = isq ? q_norm : k_norm;
            float *b = buf + warp * hd;
            float s = 0.f;
            for (int i = lane; i < hd; i += 32) s = fmaf(vp[i], vp[i], s);
            const float inv = rms_inv(warp_sum(s), hd);
            for (int i = lane; i < hd; i += 32) b[i] = __fmul_rn(__fmul_rn(vp[i], inv), __fadd_rn(1.f, nrm[i]));
            __syncwarp();
            const int half = hd / 2;
            const bool tab = cos_t && pos[r] < table_len;   // the per-position table, where it covers
            for (int j = lane; j < half; j += 32) {
                float co, si;
                if (tab) {
                    co = cos_t[(size_t)pos[r] * half + j];
                    si = sin_t[(size_t)pos[r] * half + j];
                } else {
                    const float ang = __fdiv_rn(fpos, divisor[j]);
                    co = cosf(ang);
                    si = sinf(ang);
                }
                const float a = b[j], c = b[j + half];
                vp[j] = __fsub_rn(__fmul_rn(a, co), __fmul_rn(c, si));
                vp[j + half] = __fadd_rn(__fmul_rn(c, co), __fmul_rn(a, si));
            }
            __syncwarp();
            if (isq) continue;
        }
        // store this row's K (roped) or V head
        const int s = d.session[r], p = d.position[r];
        size_t row;
        bool pinned = p < d.prefix;
        if (pinned) {
            row = (size_t)kh * d.prefix + p;
        } else {
            const int slot = d.window ? (p - d.prefix) % d.window : p - d.prefix;
            row = ((size_t)s * kvheads + kh) * d.rows + slot;
        }
        if (t.fp32) {
            float *dst = isv ? (pinned ? d.pvf : t.vf) : (pinned ? d.pkf : t.kf);
            for (int i = lane; i < hd; i += 32) dst[row * hd + i] = vp[i];
            continue;
        }
        float mx = 0.f;
        for (int i = lane; i < hd; i += 32) mx = fmaxf(mx, fabsf(vp[i]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
        const float sc = mx > 0.f ? __fdiv_rn(mx, 127.f) : 1.f;
        const float iv = mx > 0.f ? __fdiv_rn(127.f, mx) : 0.f;
        int8_t *dst = isv ? (pinned ? d.pv : t.v8) : (pinned ? d.pk : t.k8);
        float *sdst = isv ? (pinned ? d.pvs : t.vs) : (pinned ? d.pks : t.ks);
        for (int i = lane; i < hd; i += 32) {
            const int qv = __float2int_rn(__fmul_rn(vp[i], iv));
            dst[row * hd + i] = (int8_t)(qv < -127 ? -127 : (qv > 127 ? 127 : qv));
        }
        if (lane == 0) sdst[row] = sc;
    }
}

__global__ void gate_kernel(float *__restrict__ att, const float *__restrict__ gate, long long n) {
    pdl_enter();
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        att[i] = __fmul_rn(att[i], sigm(gate[i]));
}

// Sinkhorn of engine.cpp:151-180 (the generic loops), on one thread.
__device__ void sinkhorn(float *a, int n) {
    float maximum = a[0], minimum = a[0];
    for (int i = 1; i < n * n; ++i) {
        maximum = fmaxf(maximum, a[i]);
        minimum = fminf(minimum, a[i]);
    }
    if (!isfinite(maximum) || __fsub_rn(maximum, minimum) > 60.f) {
        for (int it = 0; it < 20; ++it) {
            for (int i = 0; i < n; ++i) {
                float m = -INFINITY;
                for (int j = 0; j < n; ++j) m = fmaxf(m, a[i * n + j]);
                float sum = 0.f;
                for (int j = 0; j < n; ++j) sum = __fadd_rn(sum, expf(__fsub_rn(a[i * n + j], m)));
                const float lse = __fadd_rn(m, logf(sum));
                for (int j = 0; j < n; ++j) a[i * n + j] = __fsub_rn(a[i * n + j], lse);
            }
            for (int j = 0; j < n; ++j) {
                float m = -INFINITY;
                for (int i = 0; i < n; ++i) m = fmaxf(m, a[i * n + j]);
                float sum = 0.f;
                for (int i = 0; i < n; ++i) sum = __fadd_rn(sum, expf(__fsub_rn(a[i * n + j], m)));
                const float lse = __fadd_rn(m, logf(sum));
                for (int i = 0; i < n; ++i) a[i * n + j] = __fsub_rn(a[i * n + j], lse);
            }
        }
        for (int i = 0; i < n * n; ++i) a[i] = expf(a[i]);
        return;
    }
    for (int i = 0; i < n * n; ++i) a[i] = expf(__fsub_rn(a[i], maximum));
    for (int it = 0; it < 20; ++it) {
        for (int i = 0; i < n; ++i) {
            float sum = 0.f;
            for (int j = 0; j < n; ++j) sum = __fadd_rn(sum, a[i * n + j]);
            const float inv = __fdiv_rn(1.f, sum);
            for (int j = 0; j < n; ++j) a[i * n + j] = __fmul_rn(a[i * n + j], inv);
        }
        for (int j = 0; j < n; ++j) {
            float sum = 0.f;
            for (int i = 0; i < n; ++i) sum = __fadd_rn(sum, a[i * n + j]);
            const float inv = __fdiv_rn(1.f, sum);
            for (int i = 0; i < n; ++i) a[i * n + j] = __fmul_rn(a[i * n + j], inv);
        }
    }
}

// In-place normalised Walsh-Hadamard transform of v[n] in shared memory with
// the reference's radix-2 stage order (needle2/csrc/cq.cpp:30-46).
__device__ void block_fwht(float *v, int n) {
    for (int h = 1; h < n; h *= 2) {
        __syncthreads();
        for (int idx = threadIdx.x; idx < n / 2; idx += blockDim.x) {
            const int base = (idx / h) * 2 * h, j = idx % h;
            const float a = v[base + j], b = v[base + j + h];
            v[base + j] = __fadd_rn(a, b);
            v[base + j + h] = __fsub_rn(a, b);
        }
    }
    __syncthreads();
    const float scale = __fdiv_rn(1.f, sqrtf((float)n));
    for (int i = threadIdx.x; i < n; i += blockDim.x) v[i] = __fmul_rn(v[i], scale);
    __syncthreads();
}

__global__ void __launch_bounds__(256) mhc_post_kernel(const PostLayer L, const float *__restrict__ proj,
                                                       const float *__restrict__ raw, int ldraw,
                                                       const float *__restrict__ hpost, const float *__restrict__ u,
                                                       const float *__restrict__ bx, float *__restrict__ x,
                                                       float *__restrict__ hidden, int ldh) {
    pdl_enter();
    extern __shared__ float smem[];
    float *bxs = smem;             // [D]
    float *mlp = smem + L.D;       // [hada]
    __shared__ float hres[kMaxLanes * kMaxLanes];
    __shared__ float hp[kMaxLanes];
    __shared__ float sh[33];
    const int r = blockIdx.x, N = L.lanes, D = L.D, H = L.hada;
    const float *pr = proj + (size_t)r * D;
    // engine.cpp:1025-1026: proj = rms(proj) * (1 + post_norm); bx += sigmoid(attn_gate) * proj
    float sp = 0.f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) sp = fmaf(pr[d], pr[d], sp);
    const float ip = rms_inv(block_sum(sp, sh), D);
    const float ag = sigm(L.attn_gate[0]);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        const float pv = __fmul_rn(__fmul_rn(pr[d], ip), __fadd_rn(1.f, L.post_norm[d]));
        bxs[d] = __fadd_rn(bx[(size_t)r * D + d], __fmul_rn(ag, pv));
    }
    if (threadIdx.x < N * N) {
        // engine.cpp:1033: hres = res * a_res + b_res (or the routing kernel's finished hres)
        const int ij = threadIdx.x;
        const float rv = raw[(size_t)r * ldraw + 2 * N + ij];
        hres[ij] = L.hres_ready ? rv : __fadd_rn(__fmul_rn(rv, L.a_res), L.b_res[ij]);
    }
    if (threadIdx.x < N) hp[threadIdx.x] = hpost[(size_t)r * N + threadIdx.x];
    __syncthreads();
    // engine.cpp:1027-1031: Hadamard MLP on rms(bx) * (1 + pre_hada)
    float sb = 0.f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) sb = fmaf(bxs[d], bxs[d], sb);
    const float ib = rms_inv(block_sum(sb, sh), D);
    for (int d = threadIdx.x; d < H; d += blockDim.x)
        mlp[d] = d < D ? __fmul_rn(__fmul_rn(__fmul_rn(bxs[d], ib), __fadd_rn(1.f, L.pre_hada[d])), L.d1[d]) : 0.f;
    block_fwht(mlp, H);
    for (int d = threadIdx.x; d < H; d += blockDim.x) {
        const float a = __fmul_rn(mlp[d], L.d2[d]);
        mlp[d] = __fmul_rn(a, sigm(a));
    }
    block_fwht(mlp, H);
    if (threadIdx.x == 0 && !L.hres_ready) sinkhorn(hres, N);
    for (int d = threadIdx.x; d < D; d += blockDim.x)
        bxs[d] = __fsub_rn(__fadd_rn(bxs[d], __fmul_rn(L.d3[d], mlp[d])), u[(size_t)r * D + d]);
    __syncthreads();
    // engine.cpp:1035-1037: x[n] = hpost[n] * bx + sum_j hres[n][j] * x[j]; hidden = lane mean
    float *xr = x + (size_t)r * N * D;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float xs[kMaxLanes], nv[kMaxLanes];
        for (int n = 0; n < N; ++n) xs[n] = xr[(size_t)n * D + d];
        float mean = 0.f;
        for (int n = 0; n < N; ++n) {
            float val = __fmul_rn(hp[n], bxs[d]);
            for (int j = 0; j < N; ++j) val = __fadd_rn(val, __fmul_rn(hres[n * N + j], xs[j]));
            nv[n] = val;
            mean = __fadd_rn(mean, val);
        }
        for (int n = 0; n < N; ++n) xr[(size_t)n * D + d] = nv[n];
        if (hidden) hidden[(size_t)r * ldh + d] = __fdiv_rn(mean, (float)N);
    }
}

// ---- warp-per-row post-attention mixing (hada = 32 * E) ---------------------
//
// Lane l holds elements [l*E, (l+1)*E) of the row's D- and hada-vectors in
// registers.  The Walsh-Hadamard stages h < E pair elements within a lane,
// the stages h >= E pair lane l with lane l ^ (h / E) (same element slot):
// every butterfly is the reference's a + b, a - b on the same pair
// (needle2/csrc/cq.cpp:30-46), so the transform is bit-identical to it.

template <int E>
__device__ __forceinline__ void warp_fwht_regs(float (&v)[E], int lane, float scale) {
#pragma unroll
    for (int h = 1; h < E; h *= 2) {
#pragma unroll
        for (int i = 0; i < E; ++i)
            if (!(i & h)) {
                const float a = v[i], b = v[i + h];
                v[i] = __fadd_rn(a, b);
                v[i + h] = __fsub_rn(a, b);
            }
    }
#pragma unroll
    for (int m = 1; m < 32; m *= 2) {
        const bool upper = lane & m;
#pragma unroll
        for (int i = 0; i < E; ++i) {
            const float o = __shfl_xor_sync(kFull, v[i], m);
            v[i] = upper ? __fsub_rn(o, v[i]) : __fadd_rn(v[i], o);
        }
    }
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = __fmul_rn(v[i], scale);
}

// Sinkhorn of engine.cpp:151-180 on an n x n matrix (n <= 8) held one element
// per lane (lanes n*n .. 31 hold nothing useful); sums in the reference's
// sequential order, broadcast by shuffles.
__device__ float warp_sinkhorn(float a, int n, int lane) {
    const int nn = n * n;
    const bool mine = lane < nn;
    const int i = lane / n, j = lane % n;
    float mx = mine ? a : -INFINITY, mn = mine ? a : INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
        mn = fminf(mn, __shfl_xor_sync(kFull, mn, o));
    }
    if (!isfinite(mx) || __fsub_rn(mx, mn) > 60.f) {
        for (int it = 0; it < 20; ++it) {
            for (int pass = 0; pass < 2; ++pass) {   // rows, then columns
                float m = -INFINITY;
                for (int t = 0; t < n; ++t) {
                    const int src = pass == 0 ? i * n + t : t * n + j;
                    m = fmaxf(m, __shfl_sync(kFull, a, src & 31));
                }
                float sum = 0.f;
                for (int t = 0; t < n; ++t) {
                    const int src = pass == 0 ? i * n + t : t * n + j;
                    sum = __fadd_rn(sum, expf(__fsub_rn(__shfl_sync(kFull, a, src & 31), m)));
                }
                a = __fsub_rn(a, __fadd_rn(m, logf(sum)));
            }
        }
        return expf(a);
    }
    a = expf(__fsub_rn(a, mx));
    for (int it = 0; it < 20; ++it) {
        for (int pass = 0; pass < 2; ++pass) {
            float sum = 0.f;
            for (int t = 0; t < n; ++t) sum = __fadd_rn(sum, __shfl_sync(kFull, a, (pass == 0 ? i * n + t : t * n + j) & 31));
            a = __fmul_rn(a, __fdiv_rn(1.f, sum));
        }
    }
    return a;
}

template <int E, int N>
__global__ void __launch_bounds__(128) mhc_post_warp_kernel(const PostLayer L, const float *__restrict__ proj,
                                                            const float *__restrict__ raw, int ldraw,
                                                            const float *__restrict__ hpost,
                                                            const float *__restrict__ u, const float *__restrict__ bx,
                                                            float *__restrict__ x, int R, float *__restrict__ hidden,
                                                            int ldh) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= R) return;
    const int D = L.D;
    const int base = lane * E;
    // engine.cpp:1025-1026: proj = rms(proj) * (1 + post_norm); bx += sigmoid(attn_gate) * proj
    float pv[E], b[E];
    float sp = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) {
        const int d = base + i;
        pv[i] = d < D ? proj[(size_t)r * D + d] : 0.f;
        sp = fmaf(pv[i], pv[i], sp);
    }
    const float ip = rms_inv(warp_sum(sp), D);
    const float ag = sigm(L.attn_gate[0]);
    float sb = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) {
        const int d = base + i;
        if (d < D) {
            const float t = __fmul_rn(__fmul_rn(pv[i], ip), __fadd_rn(1.f, L.post_norm[d]));
            b[i] = __fadd_rn(bx[(size_t)r * D + d], __fmul_rn(ag, t));
        } else {
            b[i] = 0.f;
        }
        sb = fmaf(b[i], b[i], sb);
    }
    // engine.cpp:1027-1031: Hadamard MLP on rms(bx) * (1 + pre_hada)
    const float ib = rms_inv(warp_sum(sb), D);
    float mlp[E];
#pragma unroll
    for (int i = 0; i < E; ++i) {
        const int d = base + i;
        mlp[i] = d < D ? __fmul_rn(__fmul_rn(__fmul_rn(b[i], ib), __fadd_rn(1.f, L.pre_hada[d])), L.d1[d]) : 0.f;
    }
    const float scale = __fdiv_rn(1.f, sqrtf((float)L.hada));
    warp_fwht_regs<E>(mlp, lane, scale);
#pragma unroll
    for (int i = 0; i < E; ++i) {
        const float a = __fmul_rn(mlp[i], L.d2[base + i]);
        mlp[i] = __fmul_rn(a, sigm(a));
    }
    warp_fwht_regs<E>(mlp, lane, scale);
#pragma unroll
    for (int i = 0; i < E; ++i) {
        const int d = base + i;
        if (d < D) b[i] = __fsub_rn(__fadd_rn(b[i], __fmul_rn(L.d3[d], mlp[i])), u[(size_t)r * D + d]);
    }
    // engine.cpp:1033-1034: hres = sinkhorn(res * a_res + b_res)
    constexpr int nn = N * N;
    float hres;
    if (L.hres_ready) {
        hres = lane < nn ? raw[(size_t)r * ldraw + 2 * N + lane] : 0.f;   // made by the routing kernel
    } else {
        const float hr = lane < nn ? __fadd_rn(__fmul_rn(raw[(size_t)r * ldraw + 2 * N + lane], L.a_res), L.b_res[lane])
                                   : 0.f;
        hres = warp_sinkhorn(hr, N, lane);
    }
    float hres_all[nn];
    float hp[N];
#pragma unroll
    for (int t = 0; t < nn; ++t) hres_all[t] = __shfl_sync(kFull, hres, t);
#pragma unroll
    for (int n = 0; n < N; ++n) hp[n] = hpost[(size_t)r * N + n];
    // engine.cpp:1035-1037: x[n] = hpost[n] * bx + sum_j hres[n][j] * x[j]; hidden = lane mean
    float *xr = x + (size_t)r * N * D;
#pragma unroll
    for (int i = 0; i < E; ++i) {
        const int d = base + i;
        if (d >= D) continue;
        float xs[N];
#pragma unroll
        for (int n = 0; n < N; ++n) xs[n] = xr[(size_t)n * D + d];
        float mean = 0.f;
#pragma unroll
        for (int n = 0; n < N; ++n) {
            float val = __fmul_rn(hp[n], b[i]);
#pragma unroll
            for (int j = 0; j < N; ++j) val = __fadd_rn(val, __fmul_rn(hres_all[n * N + j], xs[j]));
            xr[(size_t)n * D + d] = val;
            mean = __fadd_rn(mean, val);
        }
        if (hidden) hidden[(size_t)r * ldh + d] = __fdiv_rn(mean, (float)N);
    }
}

__global__ void final_norm_kernel(const float *__restrict__ x, int lanes, int D, const float *__restrict__ fnorm,
                                  float *__restrict__ z) {
    pdl_enter();
    extern __shared__ float zs[];
    __shared__ float sh[33];
    const int r = blockIdx.x;
    const float *xr = x + (size_t)r * lanes * D;
    float s = 0.f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float sum = 0.f;
        for (int n = 0; n < lanes; ++n) sum = __fadd_rn(sum, xr[(size_t)n * D + d]);
        const float m = __fdiv_rn(sum, (float)lanes);
        zs[d] = m;
        s = fmaf(m, m, s);
    }
    const float inv = rms_inv(block_sum(s, sh), D);
    for (int d = threadIdx.x; d < D; d += blockDim.x)
        z[(size_t)r * D + d] = __fmul_rn(__fmul_rn(zs[d], inv), __fadd_rn(1.f, fnorm[d]));
}

__device__ __forceinline__ int engram_token(const EngramHash &h, int e, int p) {
    if (h.chunk && p >= h.chunk_start[e]) return h.chunk[(size_t)e * h.T + (p - h.chunk_start[e])];
    return h.ring[(size_t)e * h.hist_cap + ((p % h.hist_cap) + h.hist_cap) % h.hist_cap];
}

__global__ void engram_ids_kernel(const EngramHash h, const int *__restrict__ pos, int R, int64_t *__restrict__ ids,
                                  uint8_t *__restrict__ valid) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)R * h.tables) return;
    const int r = (int)(i / h.tables), t = (int)(i % h.tables);
    const int e = r / h.T, p = pos[r];
    const int per_order = h.tables / h.num_orders;
    const int order = h.orders[t / per_order];
    // engine.cpp:763: n-grams reaching before the sequence, or across an evicted window, are zero
    const bool ok = !(p + 1 < order || (h.window && order - 1 >= h.window && p - order + 1 >= h.prefix));
    uint32_t acc = 0x9e3779b9u * (uint32_t)(t + 1);
    if (ok) {
        for (int j = 0; j < order; ++j) acc = (acc ^ (uint32_t)engram_token(h, e, p - j)) * 0x01000193u;
        acc ^= acc >> 15;
    }
    ids[i] = (int64_t)t * h.slots + (ok ? (int64_t)(acc % (uint32_t)h.slots) : 0);
    valid[i] = ok ? 1 : 0;
}

__global__ void engram_mask_kernel(float *__restrict__ e, const uint8_t *__restrict__ valid, int subdim) {
    pdl_enter();
    const long long rt = blockIdx.x;   // row * tables + table
    if (valid[rt]) return;
    for (int c = threadIdx.x; c < subdim; c += blockDim.x) e[rt * subdim + c] = 0.f;
}

__global__ void engram_conv_kernel(const EngramConv c, const int *__restrict__ pos, float *__restrict__ ev, int ldev) {
    pdl_enter();
    const int r = blockIdx.x, e = r / c.T, p = pos[r], cs = c.chunk_start[e];
    for (int d = threadIdx.x; d < c.D; d += blockDim.x) {
        float sum = 0.f;
        for (int tap = 0; tap < c.taps; ++tap) {
            const int past = p - tap * c.dilation;
            if (past >= 0 && (!c.window || tap * c.dilation < c.window || past < c.prefix)) {
                const float v = past >= cs ? c.chunk_raw[((size_t)e * c.T + (past - cs)) * c.ld_chunk + d]
                                           : c.ring[(size_t)e * c.ld_ring_s + (size_t)(past % c.engring) * c.D + d];
                sum = __fadd_rn(sum, __fmul_rn(c.taps_w[(size_t)tap * c.D + d], v));
            }
        }
        ev[(size_t)r * ldev + d] = sum;
    }
}

__global__ void engram_ring_store_kernel(float *__restrict__ ring, size_t ld_ring_s, const float *__restrict__ raw,
                                         int ld_chunk, const int *__restrict__ chunk_start, int T, int keep,
                                         int engring, int D) {
    pdl_enter();
    const int e = blockIdx.x, j = blockIdx.y;
    const int t = T - keep + j, position = chunk_start[e] + t;
    float *dst = ring + (size_t)e * ld_ring_s + (size_t)(position % engring) * D;
    const float *src = raw + ((size_t)e * T + t) * ld_chunk;
    for (int d = threadIdx.x; d < D; d += blockDim.x) dst[d] = src[d];
}

__global__ void history_store_kernel(int *__restrict__ ring, int cap, const int *__restrict__ tokens, int T,
                                     const int *__restrict__ chunk_start, int keep, int entries) {
    pdl_enter();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= entries * keep) return;
    const int e = i / keep, t = T - keep + i % keep;
    const int position = chunk_start[e] + t;
    ring[(size_t)e * cap + position % cap] = tokens[(size_t)e * T + t];
}

__global__ void row_positions_kernel(const int *__restrict__ base, int entries, int T, int *__restrict__ sess,
                                     int *__restrict__ pos) {
    pdl_enter();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= entries * T) return;
    if (sess) sess[r] = r / T;
    pos[r] = base[r / T] + r % T;
}

__global__ void advance_kernel(int *base, int n, int delta) {
    pdl_enter();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) base[i] += delta;
}

__global__ void copy_tokens_kernel(const int *__restrict__ src, int n, int *__restrict__ dst, int ld) {
    pdl_enter();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[(size_t)i * ld] = src[i];
}

__global__ void widen_ids_kernel(const int *__restrict__ src, int64_t *__restrict__ dst, int n) {
    pdl_enter();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = src[i];
}

__device__ __forceinline__ unsigned index_at(const uint8_t *p, int i, int bits) {
    const int bit = i * bits, byte = bit >> 3, shift = bit & 7;
    unsigned word = p[byte];
    if (shift + bits > 8) word |= (unsigned)p[byte + 1] << 8;
    return (word >> shift) & ((1u << bits) - 1u);
}

struct Lut {
    float v[16];
};
struct Ctab {
    uint32_t w[4];
};

// One warp per candidate row (FP32 mode).
__global__ void candidates_f32_kernel(const uint8_t *__restrict__ packed, const uint16_t *__restrict__ norms,
                                      int rowbytes, int groups, int group, int storage_bits, const Lut lut,
                                      const float *__restrict__ rot, const int *__restrict__ cand, int n,
                                      float *__restrict__ out) {
    pdl_enter();
    const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (i >= n) return;
    const int row = cand[i];
    const uint8_t *p = packed + (size_t)row * rowbytes;
    float sum = 0.f;
    for (int g = 0; g < groups; ++g) {
        float gs = 0.f;
        for (int k = lane; k < group; k += 32) {
            const int e = g * group + k;
            gs = fmaf(lut.v[index_at(p, e, storage_bits)], rot[e], gs);
        }
        gs = warp_sum(gs);
        sum = __fadd_rn(sum, __fmul_rn(gs, half_bits_to_float(norms[(size_t)row * groups + g])));
    }
    if (lane == 0) out[i] = sum;
}

// One warp per candidate row (int8 mode): exact int32 group dots and the SDOT
// epilogue y = sum_g (float(d) * (half(norm) * cs)) * xs[g] in group order
// (needle2/csrc/sdot.cpp:142-149).
__global__ void candidates_i8_kernel(const uint8_t *__restrict__ packed, const uint16_t *__restrict__ norms,
                                     int rowbytes, int groups, int group, int bits, const Ctab ctab, float cs,
                                     const int8_t *__restrict__ q, const float *__restrict__ xs,
                                     const int *__restrict__ cand, int n, float *__restrict__ out) {
    pdl_enter();
    const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (i >= n) return;
    int8_t cent[16];
    memcpy(cent, ctab.w, 16);
    const int row = cand[i];
    const uint8_t *p = packed + (size_t)row * rowbytes;
    float value = 0.f;
    for (int g = 0; g < groups; ++g) {
        int acc = 0;
        for (int k = lane; k < group; k += 32) {
            const int e = g * group + k;
            const int d = bits == 2 ? ((k & ~15) | ((k & 1) ? 8 + ((k & 15) >> 1) : ((k & 15) >> 1))) : k;
            acc += (int)cent[index_at(p, e, bits)] * (int)q[(size_t)g * group + d];
        }
        acc = warp_sum_int(acc);
        const float ns = __fmul_rn(half_bits_to_float(norms[(size_t)row * groups + g]), cs);
        value = __fadd_rn(value, __fmul_rn(__fmul_rn(__int2float_rn(acc), ns), xs[g]));
    }
    if (lane == 0) out[i] = value;
}

inline unsigned blocks_for(long long n, int threads) { return (unsigned)((n + threads - 1) / threads); }

}  // namespace

bool launch_embed_lanes(const float *rows, int R, int lanes, int D, float scale, float *x, cudaStream_t st) {
    if (R <= 0) return true;
    NB_CUDA_TRY(launch_pdl(embed_lanes_kernel, R, 256, 0, st, rows, lanes, D, scale, x));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_gather_dense(const float *w, const int64_t *ids, int R, int cols, float *out, cudaStream_t st) {
    if (R <= 0) return true;
    NB_CUDA_TRY(launch_pdl(gather_dense_kernel, R, 256, 0, st, w, ids, cols, out));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_rms(const float *x, int ldx, int R, int n, const float *scale, float *y, int ldy, cudaStream_t st) {
    if (R <= 0) return true;
    NB_CUDA_TRY(launch_pdl(rms_kernel, R, 256, 0, st, x, ldx, n, scale, y, ldy));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_dense_rows(const DenseSeg *segs, int nseg, const float *in, int ldin, int R, int cols, cudaStream_t st) {
    if (R <= 0 || nseg <= 0) return true;
    if (nseg > 3) { set_error("at most three dense slices per launch"); return false; }
    DenseSegs s{};
    int rows = 0;
    for (int i = 0; i < nseg; ++i) {
        s.s[i] = segs[i];
        rows += segs[i].rows;
    }
    s.n = nseg;
    const dim3 grid((rows + 7) / 8, (R + 7) / 8);
    NB_CUDA_TRY(launch_pdl(dense_rows_kernel, grid, 256, 0, st, s, in, ldin, R, cols));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_mhc_pre(const MhcLayer &L, const float *raw, int ldraw, const float *x, int R, float *hpost, float *u,
                    float *bx, float *z, cudaStream_t st) {
    if (R <= 0) return true;
    NB_CUDA_TRY(launch_pdl(mhc_pre_kernel, R, 256, sizeof(float) * L.D, st, L, raw, ldraw, x, hpost, u, bx, z));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_mhc_route(const MhcLayer &L, const float *phi_pre, const float *phi_post, const float *phi_res,
                      const float *x, int R, float *raw, int ldraw, float *hpost, float *u, float *bx, float *z,
                      int sms, cudaStream_t st) {
    if (R <= 0) return true;
    const int ND = L.lanes * L.D;
    if (ND % 128 || L.lanes > kMaxLanes) return false;
    // rows per CTA: as many as keep about one CTA per SM busy, at most 8
    int sb = 8;
    while (sb > 1 && (R + sb - 1) / sb < sms - sms / 8) sb /= 2;
    const size_t smem = sizeof(float) * (size_t)sb * ND;
    if (smem > 200 * 1024) return false;
    const unsigned grid = (unsigned)((R + sb - 1) / sb);
    int dev = 0;   // the shared-memory limit is a per-device attribute
    NB_CUDA_TRY(cudaGetDevice(&dev));
#define NB_ROUTE(SB)                                                                                               \
    {                                                                                                              \
        static bool configured[64] = {};                                                                           \
        if (dev < 0 || dev >= 64 || !configured[dev]) {                                                           \
            NB_CUDA_TRY(cudaFuncSetAttribute(mhc_route_kernel<SB>, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                             200 * 1024));                                                         \
            if (dev >= 0 && dev < 64) configured[dev] = true;                                                      \
        }                                                                                                          \
        NB_CUDA_TRY(launch_pdl(mhc_route_kernel<SB>, grid, 256, smem, st, L, phi_pre, phi_post, phi_res, x, R, raw, ldraw, hpost, u,   \
                                                      bx, z));                                                      \
    }
    switch (sb) {
        case 8: NB_ROUTE(8) break;
        case 4: NB_ROUTE(4) break;
        case 2: NB_ROUTE(2) break;
        default: NB_ROUTE(1) break;
    }
#undef NB_ROUTE
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_qk_norm_rope(float *q, float *k, int R, int heads, int kvheads, int hd, const float *q_norm,
                         const float *k_norm, const int *pos, const float *divisor, cudaStream_t st) {
    if (R <= 0) return true;
    const int warps = std::min(heads + kvheads, 16);
    NB_CUDA_TRY(launch_pdl(qk_norm_rope_kernel, R, 32 * warps, sizeof(float) * warps * hd, st, q, k, heads, kvheads, hd, q_norm, k_norm,
                                                                         pos, divisor));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_qk_rope_store(float *q, float *k, float *v, int R, int heads, int kvheads, int hd,
                          const float *q_norm, const float *k_norm, const int *pos, const float *divisor,
                          const KVStoreTarget &t, cudaStream_t st, const float *cos_t, const float *sin_t,
                          int table_len, const QkvgParts *src) {
    if (R <= 0) return true;
    const QkvgParts parts = src ? *src : QkvgParts{};
    if (parts.q && (parts.parts < 1 || parts.parts > kMaxKParts || !parts.k || !parts.v || !parts.g || !parts.gate)) {
        set_error("q/k/v/gate parts: bad arguments");
        return false;
    }
    const int warps = std::min(heads + 2 * kvheads + (parts.q ? heads : 0), 32);
    NB_CUDA_TRY(launch_pdl(qk_rope_store_kernel, R, 32 * warps, sizeof(float) * warps * hd, st, q, k, v, heads, kvheads, hd, q_norm,
                           k_norm, pos, divisor, t, cos_t, sin_t, table_len, parts));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

__global__ void sum_parts_kernel(const float *__restrict__ part, int parts, long long pstride, long long n,
                                 float *__restrict__ out) {
    pdl_enter();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = part_sum(part + i, parts, pstride);
}

bool launch_sum_parts(const float *part, int parts, long long pstride, long long n, float *out, cudaStream_t st) {
    if (n <= 0) return true;
    if (parts < 1 || parts > kMaxKParts) {
        set_error("sum of parts: bad part count");
        return false;
    }
    NB_CUDA_TRY(launch_pdl(sum_parts_kernel, std::min<unsigned>(blocks_for(n, 256), 4096), 256, 0, st, part, parts, pstride, n, out));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_gate(float *att, const float *gate, int R, int A, cudaStream_t st) {
    const long long n = (long long)R * A;
    if (n <= 0) return true;
    NB_CUDA_TRY(launch_pdl(gate_kernel, std::min<unsigned>(blocks_for(n, 256), 4096), 256, 0, st, att, gate, n));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_mhc_post(const PostLayer &L, const float *proj, const float *raw, int ldraw, const float *hpost,
                     const float *u, float *bx, float *x, int R, float *hidden, int ldh, cudaStream_t st) {
    if (R <= 0) return true;
    // warp per row where the Hadamard width is 32 * E and the lane count N are supported
    const unsigned grid = (unsigned)((R + 3) / 4);
#define NB_POST(E, N)                                                                                     \
    NB_CUDA_TRY(launch_pdl(mhc_post_warp_kernel<E, N>, grid, 128, 0, st, L, proj, raw, ldraw, hpost, u, bx, x, R, hidden, ldh)); \
    break;
#define NB_POST_LANES(E)                    \
    switch (L.lanes) {                      \
        case 1: NB_POST(E, 1)               \
        case 2: NB_POST(E, 2)               \
        case 4: NB_POST(E, 4)               \
        default: goto block_kernel;         \
    }                                       \
    break;
    switch (L.hada) {
        case 128: NB_POST_LANES(4)
        case 256: NB_POST_LANES(8)
        case 512: NB_POST_LANES(16)
        case 1024: NB_POST_LANES(32)
        default: goto block_kernel;
    }
#undef NB_POST_LANES
#undef NB_POST
    NB_CUDA_TRY(cudaGetLastError());
    return true;
block_kernel:
    NB_CUDA_TRY(launch_pdl(mhc_post_kernel, R, 256, sizeof(float) * (L.D + L.hada), st, L, proj, raw, ldraw, hpost, u, bx, x, hidden,
                                                                     ldh));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_final_norm(const float *x, int R, int lanes, int D, const float *final_norm, float *z, cudaStream_t st) {
    if (R <= 0) return true;
    NB_CUDA_TRY(launch_pdl(final_norm_kernel, R, 256, sizeof(float) * D, st, x, lanes, D, final_norm, z));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_engram_ids(const EngramHash &h, const int *sess, const int *pos, int R, int64_t *ids, uint8_t *valid,
                       cudaStream_t st) {
    (void)sess;
    const long long n = (long long)R * h.tables;
    if (n <= 0) return true;
    NB_CUDA_TRY(launch_pdl(engram_ids_kernel, blocks_for(n, 128), 128, 0, st, h, pos, R, ids, valid));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_engram_mask(float *e, const uint8_t *valid, int R, int tables, int subdim, cudaStream_t st) {
    const long long n = (long long)R * tables;
    if (n <= 0) return true;
    NB_CUDA_TRY(launch_pdl(engram_mask_kernel, (unsigned)n, 128, 0, st, e, valid, subdim));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_engram_conv(const EngramConv &c, const int *sess, const int *pos, int R, float *ev, int ldev,
                        cudaStream_t st) {
    (void)sess;
    if (R <= 0) return true;
    NB_CUDA_TRY(launch_pdl(engram_conv_kernel, R, 256, 0, st, c, pos, ev, ldev));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_engram_ring_store(float *ring, size_t ld_ring_s, const float *chunk_raw, int ld_chunk, int S_count,
                              const int *sess_of_entry, const int *chunk_start, int T, int engring, int D,
                              cudaStream_t st) {
    (void)sess_of_entry;
    const int keep = std::min(T, engring);
    if (S_count <= 0 || keep <= 0) return true;
    NB_CUDA_TRY(launch_pdl(engram_ring_store_kernel, dim3(S_count, keep), 256, 0, st, ring, ld_ring_s, chunk_raw, ld_chunk, chunk_start, T,
                                                                  keep, engring, D));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_history_store(int *ring, int cap, const int *tokens, int T, const int *sess, const int *chunk_start,
                          int entries, cudaStream_t st) {
    (void)sess;
    const int keep = std::min(T, cap);
    if (entries <= 0 || keep <= 0) return true;
    NB_CUDA_TRY(launch_pdl(history_store_kernel, blocks_for((long long)entries * keep, 128), 128, 0, st, ring, cap, tokens, T, chunk_start,
                                                                                    keep, entries));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_candidates_f32(const uint8_t *packed, const uint16_t *norms, int rowbytes, int groups, int group,
                           int storage_bits, const float lut_in[16], const float *rot, const int *cand, int n,
                           float *out, cudaStream_t st) {
    if (n <= 0) return true;
    Lut lut;
    for (int i = 0; i < 16; ++i) lut.v[i] = lut_in[i];
    NB_CUDA_TRY(launch_pdl(candidates_f32_kernel, blocks_for((long long)n * 32, 256), 256, 0, st, packed, norms, rowbytes, groups, group,
                                                                             storage_bits, lut, rot, cand, n, out));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_candidates_i8(const uint8_t *packed, const uint16_t *norms, int rowbytes, int groups, int group, int bits,
                          const uint32_t ctab_in[4], float cs, const int8_t *q, const float *xs, const int *cand,
                          int n, float *out, cudaStream_t st) {
    if (n <= 0) return true;
    Ctab ctab;
    for (int i = 0; i < 4; ++i) ctab.w[i] = ctab_in[i];
    NB_CUDA_TRY(launch_pdl(candidates_i8_kernel, blocks_for((long long)n * 32, 256), 256, 0, st, packed, norms, rowbytes, groups, group,
                                                                            bits, ctab, cs, q, xs, cand, n, out));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_row_positions(const int *base, int entries, int T, int *sess_out, int *pos_out, cudaStream_t st) {
    const long long n = (long long)entries * T;
    if (n <= 0) return true;
    NB_CUDA_TRY(launch_pdl(row_positions_kernel, blocks_for(n, 256), 256, 0, st, base, entries, T, sess_out, pos_out));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_advance(int *base, int n, int delta, cudaStream_t st) {
    if (n <= 0) return true;
    NB_CUDA_TRY(launch_pdl(advance_kernel, blocks_for(n, 256), 256, 0, st, base, n, delta));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_widen_ids(const int *src, int64_t *dst, int n, cudaStream_t st) {
    if (n <= 0) return true;
    NB_CUDA_TRY(launch_pdl(widen_ids_kernel, blocks_for(n, 256), 256, 0, st, src, dst, n));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

bool launch_copy_tokens(const int *src, int n, int *dst, int ld_dst, cudaStream_t st) {
    if (n <= 0) return true;
    NB_CUDA_TRY(launch_pdl(copy_tokens_kernel, blocks_for(n, 256), 256, 0, st, src, n, dst, ld_dst));
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

}  // namespace eng

namespace {
__global__ void rope_table_kernel(const float *__restrict__ divisor, int half, int positions, float *cos_t,
                                  float *sin_t) {
    const long long n = (long long)positions * half;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int p = (int)(i / half), j = (int)(i % half);
        const float ang = __fdiv_rn((float)p, divisor[j]);
        cos_t[i] = cosf(ang);
        sin_t[i] = sinf(ang);
    }
}
}  // namespace

bool launch_rope_table(const float *divisor, int half, int positions, float *cos_t, float *sin_t, cudaStream_t st) {
    const long long n = (long long)positions * half;
    if (n <= 0) return true;
    rope_table_kernel<<<(unsigned)std::min<long long>((n + 255) / 256, 4096), 256, 0, st>>>(divisor, half, positions,
                                                                                          cos_t, sin_t);
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

}  // namespace nb200
