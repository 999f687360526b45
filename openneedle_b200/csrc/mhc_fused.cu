// Layer-boundary kernel of the decode/prefill forward: the post-attention part
// of layer l (attention-output norm and gate, Hadamard MLP, Sinkhorn lane
// mixing; needle2/csrc/engine.cpp:1025-1037) followed by the mHC routing of
// layer l + 1 (lane RMS, the 2N + N^2 projections, gates, u, engram mixing, z;
// engine.cpp:980-992), or by the final norm after the last layer
// (engine.cpp:1039-1040).  Each CTA owns SB whole rows, so the lane state
// never leaves the CTA between the two halves, and every phase runs on all of
// the CTA's threads: thread t of the 256 compute threads owns elements
// [tP, tP + P) of each D-wide vector (P = Hadamard width / 256).  A ninth warp
// runs the Sinkhorn normalisation of the new mixing matrices while the others
// finish the row.  Elementwise formulas keep the reference's operation order
// with explicit round-to-nearest operations (the x86 reference has no FMA
// contraction); sums over a row run as trees, a different association within
// FP32 rounding; the Walsh-Hadamard stages run in the reference's order
// (h = 1, 2, 4, ...), so each butterfly matches it.
#include <math.h>
#include <stdint.h>

#include <cuda_bf16.h>

#include "common.cuh"
#include "engine.cuh"
#include "engine_math.cuh"
#include "pdl.cuh"
#include "sm100_async.cuh"

namespace nb200 {
namespace eng {
namespace {

constexpr int kComputeThreads = 256;
constexpr int kMixThreads = kComputeThreads + 32;   // + the Sinkhorn warp
constexpr int kMaxProj = 3 * kMaxLanes + kMaxLanes * kMaxLanes;

// Barrier of the 8 compute warps only (the Sinkhorn warp never joins it).
__device__ __forceinline__ void bar_compute() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// The one barrier of all nine warps: the Sinkhorn warp's matrices are in
// shared memory.
__device__ __forceinline__ void bar_mix() { asm volatile("bar.sync 2, 288;" ::: "memory"); }

// Exchange area of the compute warps: two alternating halves, each large
// enough for one D-wide vector per row.  Every exchange writes one half,
// passes one barrier and reads it back, and consecutive exchanges alternate
// halves, so a half is rewritten only after every thread has passed the
// barrier that follows its last read.
template <int SB, int P>
struct Xchg {
    float *base;
    int par = 0;
    __device__ float *next() {
        float *b = base + par * (SB * kComputeThreads * P);
        par ^= 1;
        return b;
    }
};

// Sums of M values over the 256 compute threads; every thread gets them.
// Warp trees, then the 8 warp partials added in warp order.
template <int M, int SB, int P>
__device__ __forceinline__ void cta_sums(float (&v)[M], Xchg<SB, P> &x) {
    static_assert(M * 8 <= SB * kComputeThreads * P, "exchange area too small");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float *b = x.next();
#pragma unroll
    for (int m = 0; m < M; ++m) v[m] = warp_sum(v[m]);
    if (lane == 0) {
#pragma unroll
        for (int m = 0; m < M; ++m) b[warp * M + m] = v[m];
    }
    bar_compute();
#pragma unroll
    for (int m = 0; m < M; ++m) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) t += b[w * M + m];
        v[m] = t;
    }
}

// Normalised Walsh-Hadamard transform of every `len`-element block (len a
// power of two, P <= len <= 256 P) of each row's vector, P elements per thread:
// stages h < P in registers, h < 32 P across lanes, the rest across warps
// through the exchange area; then every element times `scale`.
template <int SB, int P>
__device__ __forceinline__ void cta_fwht(float (&v)[SB][P], int len, float scale, Xchg<SB, P> &x) {
    const int t = threadIdx.x, lane = t & 31;
#pragma unroll
    for (int h = 1; h < P; h *= 2) {
        if (h >= len) break;
#pragma unroll
        for (int s = 0; s < SB; ++s)
#pragma unroll
            for (int i = 0; i < P; ++i)
                if (!(i & h)) {
                    const float a = v[s][i], b = v[s][i + h];
                    v[s][i] = __fadd_rn(a, b);
                    v[s][i + h] = __fsub_rn(a, b);
                }
    }
#pragma unroll
    for (int m = 1; m < 32; m *= 2) {
        if (m * P >= len) break;
        const bool upper = lane & m;
#pragma unroll
        for (int s = 0; s < SB; ++s)
#pragma unroll
            for (int i = 0; i < P; ++i) {
                const float o = __shfl_xor_sync(kFull, v[s][i], m);
                v[s][i] = upper ? __fsub_rn(o, v[s][i]) : __fadd_rn(v[s][i], o);
            }
    }
    for (int m = 32; m * P < len; m *= 2) {
        float *b = x.next();
#pragma unroll
        for (int s = 0; s < SB; ++s)
#pragma unroll
            for (int i = 0; i < P; ++i) b[(s * kComputeThreads + t) * P + i] = v[s][i];
        bar_compute();
        const bool upper = t & m;
        const int pt = t ^ m;
#pragma unroll
        for (int s = 0; s < SB; ++s)
#pragma unroll
            for (int i = 0; i < P; ++i) {
                const float o = b[(s * kComputeThreads + pt) * P + i];
                v[s][i] = upper ? __fsub_rn(o, v[s][i]) : __fadd_rn(v[s][i], o);
            }
    }
#pragma unroll
    for (int s = 0; s < SB; ++s)
#pragma unroll
        for (int i = 0; i < P; ++i) v[s][i] = __fmul_rn(v[s][i], scale);
}

// Sinkhorn of engine.cpp:151-180 on an N x N matrix held one element per lane
// by the N * N lanes from `base` (lane base + i N + j holds element (i, j));
// every row and column sum runs in the reference's sequential order over
// values fetched by shuffles, and 1 / sum is the correctly rounded reciprocal,
// the same value as the reference's division.  All 32 lanes take part.
template <int N>
__device__ float lanes_sinkhorn(float a, int base, int lane) {
    const int e = lane - base, i = e / N, j = e % N;
    const bool mine = e >= 0 && e < N * N;
    float mx = mine ? a : -INFINITY, mn = mine ? a : INFINITY;
#pragma unroll
    for (int t = 0; t < N * N; ++t) {
        const float v = __shfl_sync(kFull, a, (base + t) & 31);
        mx = fmaxf(mx, v);
        mn = fminf(mn, v);
    }
    if (!isfinite(mx) || __fsub_rn(mx, mn) > 60.f) {
        for (int it = 0; it < 20; ++it) {
#pragma unroll
            for (int pass = 0; pass < 2; ++pass) {
                float v[N];
#pragma unroll
                for (int t = 0; t < N; ++t)
                    v[t] = __shfl_sync(kFull, a, (base + (pass == 0 ? i * N + t : t * N + j)) & 31);
                float m = -INFINITY;
#pragma unroll
                for (int t = 0; t < N; ++t) m = fmaxf(m, v[t]);
                float sum = 0.f;
#pragma unroll
                for (int t = 0; t < N; ++t) sum = __fadd_rn(sum, expf(__fsub_rn(v[t], m)));
                a = __fsub_rn(a, __fadd_rn(m, logf(sum)));
            }
        }
        return expf(a);
    }
    a = expf(__fsub_rn(a, mx));
    for (int it = 0; it < 20; ++it) {
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
            float v[N];
#pragma unroll
            for (int t = 0; t < N; ++t)
                v[t] = __shfl_sync(kFull, a, (base + (pass == 0 ? i * N + t : t * N + j)) & 31);
            float sum = 0.f;
#pragma unroll
            for (int t = 0; t < N; ++t) sum = __fadd_rn(sum, v[t]);
            a = __fmul_rn(a, __frcp_rn(sum));
        }
    }
    return a;
}

// P contiguous floats at p (P = 1, 2 or 4; p aligned to P floats).
template <int P>
__device__ __forceinline__ void load_p(float (&v)[P], const float *p) {
    if constexpr (P == 4) {
        const float4 t = *reinterpret_cast<const float4 *>(p);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else if constexpr (P == 2) {
        const float2 t = *reinterpret_cast<const float2 *>(p);
        v[0] = t.x; v[1] = t.y;
    } else {
        v[0] = *p;
    }
}
template <int P>
__device__ __forceinline__ void store_p(float *p, const float (&v)[P]) {
    if constexpr (P == 4) {
        *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else if constexpr (P == 2) {
        *reinterpret_cast<float2 *>(p) = make_float2(v[0], v[1]);
    } else {
        *p = v[0];
    }
}

template <int P, int N, int SB, bool STAGED>
__global__ void __launch_bounds__(kMixThreads, STAGED ? 1 : 2) mhc_mix_kernel(const MixArgs a, int R) {
    constexpr int NN = N * N, NPROJ = 2 * N + N * N;
    extern __shared__ __align__(16) float smem_raw[];   // from a 128-byte boundary (launch_mhc_mix adds 128)
    float *smem = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    __shared__ float raws[SB][kMaxProj];
    __shared__ float hres_s[SB][NN], hp_s[SB][N];
    __shared__ __align__(8) uint64_t phibar;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int D = a.D, ND = N * D;
    const int r0 = blockIdx.x * SB;
    float *phis = smem + 2 * SB * kComputeThreads * P;   // [NPROJ][ND] when a.phi_smem
    auto phi_row = [&](int layer, int j) -> const float * {
        return j < N ? a.phi_pre + (size_t)(layer * N + j) * ND
             : j < 2 * N ? a.phi_post + (size_t)(layer * N + j - N) * ND
                         : a.phi_res + (size_t)(layer * N * N + j - 2 * N) * ND;
    };
    if (STAGED && a.phi_smem && a.has_route && t == 0) {
        // the routed layer's projection rows do not depend on earlier kernels:
        // bulk-copy them into shared memory before waiting for those kernels
        mbar_init(&phibar, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(&phibar, (uint32_t)(NPROJ * ND * sizeof(float)));
        for (int j = 0; j < NPROJ; ++j)
            bulk_g2s(phis + (size_t)j * ND, phi_row(a.route.layer, j), (uint32_t)(ND * sizeof(float)), &phibar);
    }
    pdl_enter();

    if (warp == 8) {
        // Sinkhorn warp: layer l's residual mixing matrices from the raw
        // projections the routing left in raw (engine.cpp:1033-1034), while the
        // compute warps run the attention-output norm and the Hadamard MLP
        if (!a.has_post) return;
        constexpr int PER = 32 / NN;   // matrices per pass of the warp
        for (int s0 = 0; s0 < SB; s0 += PER) {
            const int s = s0 + lane / NN, k = lane % NN;
            const bool live = s < SB && r0 + s < R;
            const float hr = live ? __fadd_rn(__fmul_rn(a.raw[(size_t)(r0 + s) * a.ldraw + 2 * N + k], a.post.a_res),
                                              a.post.b_res[k])
                                  : 0.f;
            const float h = lanes_sinkhorn<N>(hr, (lane / NN) * NN, lane);
            if (s < SB && lane / NN < PER) hres_s[s][k] = h;
        }
        bar_mix();
        return;
    }

    Xchg<SB, P> xc{smem};
    const int d0 = t * P;
    const bool dv = d0 < D;
    bool rv[SB];
#pragma unroll
    for (int s = 0; s < SB; ++s) rv[s] = r0 + s < R;

    // the thread's elements of the lane state
    float xv[SB][N][P];
#pragma unroll
    for (int s = 0; s < SB; ++s)
#pragma unroll
        for (int n = 0; n < N; ++n) {
            if (rv[s] && dv) load_p<P>(xv[s][n], a.x + ((size_t)(r0 + s) * N + n) * D + d0);
            else
#pragma unroll
                for (int i = 0; i < P; ++i) xv[s][n][i] = 0.f;
        }

    float zout[SB][P];   // route: z; final: the lane means
    if (a.has_post) {
        const PostLayer &L = a.post;
        if (t < SB * N) {
            const int s = t / N, n = t % N;
            hp_s[s][n] = r0 + s < R ? a.hpost[(size_t)(r0 + s) * N + n] : 0.f;
        }
        float pv[SB][P], bb[SB][P], uv[SB][P];
#pragma unroll
        for (int s = 0; s < SB; ++s) {
            const size_t o = (size_t)(r0 + s) * D + d0;
            if (rv[s] && dv) {
                load_p<P>(pv[s], a.proj + o);
                // the out projection's K-split parts, added in order
                float pp[kMaxKParts - 1][P];
#pragma unroll
                for (int k = 1; k < kMaxKParts; ++k)
                    if (k < a.proj_parts) load_p<P>(pp[k - 1], a.proj + k * a.proj_pstride + o);
#pragma unroll
                for (int k = 1; k < kMaxKParts; ++k)
                    if (k < a.proj_parts)
#pragma unroll
                        for (int i = 0; i < P; ++i) pv[s][i] += pp[k - 1][i];
                load_p<P>(bb[s], a.bx + o);
                load_p<P>(uv[s], a.u + o);
            } else {
#pragma unroll
                for (int i = 0; i < P; ++i) pv[s][i] = bb[s][i] = uv[s][i] = 0.f;
            }
        }
        float pn[P], ph[P], w1[P], w2[P], w3[P];
#pragma unroll
        for (int i = 0; i < P; ++i) {
            const int d = d0 + i;
            pn[i] = dv ? L.post_norm[d] : 0.f;
            ph[i] = dv ? L.pre_hada[d] : 0.f;
            w1[i] = dv ? L.d1[d] : 0.f;
            w2[i] = L.d2[d];
            w3[i] = dv ? L.d3[d] : 0.f;
        }
        // engine.cpp:1025-1026: proj = rms(proj) * (1 + post_norm); bx += sigmoid(attn_gate) * proj
        float sp[SB];
#pragma unroll
        for (int s = 0; s < SB; ++s) {
            sp[s] = 0.f;
#pragma unroll
            for (int i = 0; i < P; ++i) sp[s] = fmaf(pv[s][i], pv[s][i], sp[s]);
        }
        cta_sums<SB>(sp, xc);   // also publishes hp_s
        const float ag = sigm(L.attn_gate[0]);
        float sb[SB];
#pragma unroll
        for (int s = 0; s < SB; ++s) {
            const float ip = rms_inv(sp[s], D);
            sb[s] = 0.f;
#pragma unroll
            for (int i = 0; i < P; ++i) {
                if (dv) {
                    const float tt = __fmul_rn(__fmul_rn(pv[s][i], ip), __fadd_rn(1.f, pn[i]));
                    bb[s][i] = __fadd_rn(bb[s][i], __fmul_rn(ag, tt));
                }
                sb[s] = fmaf(bb[s][i], bb[s][i], sb[s]);
            }
        }
        cta_sums<SB>(sb, xc);
        // engine.cpp:1027-1031: Hadamard MLP on rms(bx) * (1 + pre_hada)
        float mlp[SB][P];
#pragma unroll
        for (int s = 0; s < SB; ++s) {
            const float ib = rms_inv(sb[s], D);
#pragma unroll
            for (int i = 0; i < P; ++i)
                mlp[s][i] = dv ? __fmul_rn(__fmul_rn(__fmul_rn(bb[s][i], ib), __fadd_rn(1.f, ph[i])), w1[i]) : 0.f;
        }
        const float hs = __fdiv_rn(1.f, sqrtf((float)L.hada));
        cta_fwht<SB, P>(mlp, L.hada, hs, xc);
#pragma unroll
        for (int s = 0; s < SB; ++s)
#pragma unroll
            for (int i = 0; i < P; ++i) {
                const float v = __fmul_rn(mlp[s][i], w2[i]);
                mlp[s][i] = __fmul_rn(v, sigm(v));
            }
        cta_fwht<SB, P>(mlp, L.hada, hs, xc);
        bar_mix();   // hres_s from the Sinkhorn warp
        // engine.cpp:1033-1037: x[n] = hpost[n] * bx + sum_j hres[n][j] * x[j]; hidden = lane mean
#pragma unroll
        for (int s = 0; s < SB; ++s) {
            const int r = r0 + s;
#pragma unroll
            for (int i = 0; i < P; ++i) {
                const float b = dv ? __fsub_rn(__fadd_rn(bb[s][i], __fmul_rn(w3[i], mlp[s][i])), uv[s][i]) : 0.f;
                float xs[N];
#pragma unroll
                for (int n = 0; n < N; ++n) xs[n] = xv[s][n][i];
                float mean = 0.f;
#pragma unroll
                for (int n = 0; n < N; ++n) {
                    float val = __fmul_rn(hp_s[s][n], b);
#pragma unroll
                    for (int j = 0; j < N; ++j) val = __fadd_rn(val, __fmul_rn(hres_s[s][n * N + j], xs[j]));
                    xv[s][n][i] = dv ? val : 0.f;
                    mean = __fadd_rn(mean, val);
                }
                zout[s][i] = __fdiv_rn(mean, (float)N);
                if (a.hidden && rv[s] && dv) a.hidden[(size_t)r * a.ldh + d0 + i] = zout[s][i];
            }
            if (rv[s] && dv)
#pragma unroll
                for (int n = 0; n < N; ++n) store_p<P>(a.x + ((size_t)r * N + n) * D + d0, xv[s][n]);
        }
    }

    if (a.final_norm) {
        // engine.cpp:1039-1040: z = rms(lane mean) * (1 + final_norm)
        float sq[SB];
#pragma unroll
        for (int s = 0; s < SB; ++s) {
            sq[s] = 0.f;
#pragma unroll
            for (int i = 0; i < P; ++i) sq[s] = fmaf(zout[s][i], zout[s][i], sq[s]);
        }
        cta_sums<SB>(sq, xc);
#pragma unroll
        for (int s = 0; s < SB; ++s) {
            const float inv = rms_inv(sq[s], D);
            if (!(rv[s] && dv)) continue;
            float o[P];
#pragma unroll
            for (int i = 0; i < P; ++i) o[i] = __fmul_rn(__fmul_rn(zout[s][i], inv), __fadd_rn(1.f, a.fnorm[d0 + i]));
            store_p<P>(a.zf + (size_t)(r0 + s) * D + d0, o);
        }
    }


    if (!a.has_route) return;
    const MhcLayer &L = a.route;
    // engram key/value rows and the input norm, loaded ahead of the reductions
    float ekv[SB][P], evv[SB][P], ni[P];
#pragma unroll
    for (int i = 0; i < P; ++i) ni[i] = dv ? L.norm_in[d0 + i] : 0.f;
#pragma unroll
    for (int s = 0; s < SB; ++s) {
        if (L.ek && rv[s] && dv) {
            load_p<P>(ekv[s], L.ek + (size_t)(r0 + s) * L.ld_site + d0);
            load_p<P>(evv[s], L.ev + (size_t)(r0 + s) * L.ld_site + d0);
        } else {
#pragma unroll
            for (int i = 0; i < P; ++i) ekv[s][i] = evv[s][i] = 0.f;
        }
    }
    // engine.cpp:980: nx = rms(x) over the N lanes
    float ss[SB];
#pragma unroll
    for (int s = 0; s < SB; ++s) {
        ss[s] = 0.f;
#pragma unroll
        for (int n = 0; n < N; ++n)
#pragma unroll
            for (int i = 0; i < P; ++i) ss[s] = fmaf(xv[s][n][i], xv[s][n][i], ss[s]);
    }
    cta_sums<SB>(ss, xc);
    float nxv[SB][N][P];
#pragma unroll
    for (int s = 0; s < SB; ++s) {
        const float inv = rms_inv(ss[s], ND);
#pragma unroll
        for (int n = 0; n < N; ++n)
#pragma unroll
            for (int i = 0; i < P; ++i) nxv[s][n][i] = __fmul_rn(xv[s][n][i], inv);
    }
    // engine.cpp:529-559: raw[s][j] = phi_j . nx[s]; each thread its N x P
    // elements of every projection row, then a tree over the CTA
    if constexpr (STAGED) {
        // each thread its N x P elements of every staged projection row, then a
        // tree over the CTA
        bool staged = a.phi_smem != 0;
        if (staged && !mbar_wait(&phibar, 0)) staged = false;   // (bounded) fall back to global reads
        float *b = xc.next();   // [8 warps][SB * NPROJ]
        constexpr int JC = 8;   // projection rows per pass (bounds the partials' registers)
#pragma unroll
        for (int j0 = 0; j0 < NPROJ; j0 += JC) {
            float part[SB][JC];
#pragma unroll
            for (int jj = 0; jj < JC; ++jj) {
                const int j = j0 + jj;
#pragma unroll
                for (int s = 0; s < SB; ++s) part[s][jj] = 0.f;
                if (j >= NPROJ || !dv) continue;
                const float *w = staged ? phis + (size_t)j * ND : phi_row(L.layer, j);
#pragma unroll
                for (int n = 0; n < N; ++n) {
                    float wv[P];
                    load_p<P>(wv, w + n * D + d0);
#pragma unroll
                    for (int s = 0; s < SB; ++s)
#pragma unroll
                        for (int i = 0; i < P; ++i) part[s][jj] = fmaf(wv[i], nxv[s][n][i], part[s][jj]);
                }
            }
#pragma unroll
            for (int s = 0; s < SB; ++s)
#pragma unroll
                for (int jj = 0; jj < JC; ++jj) {
                    if (j0 + jj >= NPROJ) continue;
                    const float v = warp_sum(part[s][jj]);
                    if (lane == 0) b[warp * SB * NPROJ + s * NPROJ + j0 + jj] = v;
                }
        }
        bar_compute();
        if (t < SB * NPROJ) {
            float v = 0.f;
#pragma unroll
            for (int w8 = 0; w8 < 8; ++w8) v += b[w8 * SB * NPROJ + t];
            raws[t / NPROJ][t % NPROJ] = v;
        }
        bar_compute();
    } else {
        // many CTAs per SM: nx through shared memory, one warp per projection
        // row streaming it from global memory (16 float4 loads in flight a lane)
        float *nx = phis;   // [SB][ND]
#pragma unroll
        for (int s = 0; s < SB; ++s)
#pragma unroll
            for (int n = 0; n < N; ++n)
                if (dv) store_p<P>(nx + (size_t)s * ND + n * D + d0, nxv[s][n]);
        bar_compute();
        constexpr int CMAX = N * P * 2;   // float4 chunks per lane at D = 256 P
        const int chunks = ND / 4;
        for (int j = warp; j < NPROJ; j += 8) {
            const float *w = phi_row(L.layer, j);
            float4 wv[CMAX];
#pragma unroll
            for (int c = 0; c < CMAX; ++c) {
                const int k = c * 32 + lane;
                wv[c] = k < chunks ? __ldg(reinterpret_cast<const float4 *>(w) + k) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int s = 0; s < SB; ++s) {
                float acc = 0.f;
#pragma unroll
                for (int c = 0; c < CMAX; ++c) {
                    const int k = c * 32 + lane;
                    if (k < chunks) {
                        const float4 v = reinterpret_cast<const float4 *>(nx + (size_t)s * ND)[k];
                        acc = fmaf(wv[c].x, v.x, fmaf(wv[c].y, v.y, fmaf(wv[c].z, v.z, fmaf(wv[c].w, v.w, acc))));
                    }
                }
                acc = warp_sum(acc);
                if (lane == 0) raws[s][j] = acc;
            }
        }
        bar_compute();
    }
    // engine.cpp:982-986: gates; u = sum_n hpre[n] x[n]
    float hpre[SB][N];
#pragma unroll
    for (int s = 0; s < SB; ++s)
#pragma unroll
        for (int n = 0; n < N; ++n) {
            const bool own = n == L.layer % N;
            hpre[s][n] = sigm(__fadd_rn(__fadd_rn(__fmul_rn(L.a_pre, raws[s][n]), L.b_pre[n]), own ? 4.f : -4.f));
        }
    if (t < SB * NPROJ) {
        // the raw projections, the residual part included: the next layer
        // boundary normalises it (its Sinkhorn warp)
        const int s = t / NPROJ, j = t % NPROJ, r = r0 + s;
        if (r < R) {
            a.raw[(size_t)r * a.ldraw + j] = raws[s][j];
            if (j >= N && j < 2 * N) {
                const int n = j - N;
                const bool own = n == L.layer % N;
                a.hpost[(size_t)r * N + n] = __fmul_rn(
                    2.f, sigm(__fadd_rn(__fadd_rn(__fmul_rn(L.a_post, raws[s][j]), L.b_post[n]), own ? 0.f : -4.f)));
            }
        }
    }
    float bxv[SB][P];
    float su[2 * SB];
#pragma unroll
    for (int s = 0; s < SB; ++s) {
        su[2 * s] = su[2 * s + 1] = 0.f;
#pragma unroll
        for (int i = 0; i < P; ++i) {
            float sum = 0.f;
#pragma unroll
            for (int n = 0; n < N; ++n) sum = __fadd_rn(sum, __fmul_rn(hpre[s][n], xv[s][n][i]));
            bxv[s][i] = sum;
            su[2 * s] = fmaf(sum, sum, su[2 * s]);
            su[2 * s + 1] = fmaf(ekv[s][i], ekv[s][i], su[2 * s + 1]);
        }
        if (rv[s] && dv) store_p<P>(a.u + (size_t)(r0 + s) * D + d0, bxv[s]);
    }
    if (L.ek) {
        // engine.cpp:987-990: bx += sigmoid(rms(bx) . rms(ek) / sqrt(D)) * ev
        cta_sums<2 * SB>(su, xc);
        float dot[SB];
#pragma unroll
        for (int s = 0; s < SB; ++s) {
            const float iu = rms_inv(su[2 * s], D), ie = rms_inv(su[2 * s + 1], D);
            dot[s] = 0.f;
#pragma unroll
            for (int i = 0; i < P; ++i) dot[s] = fmaf(__fmul_rn(bxv[s][i], iu), __fmul_rn(ekv[s][i], ie), dot[s]);
        }
        cta_sums<SB>(dot, xc);
#pragma unroll
        for (int s = 0; s < SB; ++s) {
            const float alpha = sigm(__fdiv_rn(dot[s], sqrtf((float)D)));
#pragma unroll
            for (int i = 0; i < P; ++i) bxv[s][i] = __fadd_rn(bxv[s][i], __fmul_rn(alpha, evv[s][i]));
        }
    }
    // engine.cpp:991-992: z = rms(bx) * (1 + norm_in)
    float sz[SB];
#pragma unroll
    for (int s = 0; s < SB; ++s) {
        sz[s] = 0.f;
#pragma unroll
        for (int i = 0; i < P; ++i) sz[s] = fmaf(bxv[s][i], bxv[s][i], sz[s]);
    }
    cta_sums<SB>(sz, xc);
#pragma unroll
    for (int s = 0; s < SB; ++s) {
        const float ib = rms_inv(sz[s], D);
#pragma unroll
        for (int i = 0; i < P; ++i) zout[s][i] = dv ? __fmul_rn(__fmul_rn(bxv[s][i], ib), __fadd_rn(1.f, ni[i])) : 0.f;
        if (rv[s] && dv) {
            const size_t o = (size_t)(r0 + s) * D + d0;
            store_p<P>(a.bx + o, bxv[s]);
            store_p<P>(a.z + o, zout[s]);
        }
    }
    if (a.zhl) {
        // the projections' input rotation (CQ::transform, group-wise) and bf16 hi/lo split
        cta_fwht<SB, P>(zout, a.group, a.rot_scale, xc);
#pragma unroll
        for (int s = 0; s < SB; ++s) {
            if (!(rv[s] && dv)) continue;
            const size_t o = (size_t)(r0 + s) * D + d0;
#pragma unroll
            for (int i = 0; i < P; ++i) {
                const __nv_bfloat16 h = __float2bfloat16_rn(zout[s][i]);
                a.zhl[o + i] = __bfloat16_as_ushort(h);
                a.zhl[a.lo_off + o + i] = __bfloat16_as_ushort(__float2bfloat16_rn(__fsub_rn(zout[s][i], __bfloat162float(h))));
            }
        }
    }
}

}  // namespace

bool mhc_mix_supported(int D, int lanes, int hada) {
    return lanes == 4 && (hada == 256 || hada == 512) && D <= hada && D % 32 == 0 && D > 0;
}

bool launch_mhc_mix(const MixArgs &a, int R, int sms, cudaStream_t st) {
    if (R <= 0) return true;
    if (!mhc_mix_supported(a.D, a.lanes, a.hada)) return false;
    if (a.has_post && (a.post.hada != a.hada || a.post.hres_ready)) return false;
    if (a.zhl && (a.group < 2 || a.group > a.hada || a.D % a.group || (a.group & (a.group - 1)))) return false;
    const int P = a.hada / 256, N = 4;
    // Up to one row per SM: one CTA per SM with the routing projections (24
    // rows of N * D floats) staged whole in shared memory.  More rows: two
    // rows a CTA, two CTAs per SM, the projections streamed from global
    // memory (measured faster there than fewer, longer CTAs).
    const bool staged = R <= sms;
    const int sb = staged ? 1 : 2;
    const unsigned grid = (unsigned)((R + sb - 1) / sb);
    MixArgs args = a;
    const size_t phi_bytes = sizeof(float) * (size_t)(2 * N + N * N) * N * a.D;
    size_t smem = sizeof(float) * 2 * (size_t)sb * kComputeThreads * P;
    args.phi_smem = staged && a.has_route && smem + phi_bytes <= 220 * 1024 ? 1 : 0;
    smem += args.phi_smem ? phi_bytes : sizeof(float) * (size_t)sb * N * a.D;   // (else nx of the rows)
    smem += 128;                                                                // base alignment
    // the shared-memory limit is a per-device attribute of each instantiation
    int dev = 0;
    NB_CUDA_TRY(cudaGetDevice(&dev));
#define NB_MIX(PP, SBB, ST)                                                                                      \
    {                                                                                                          \
        auto kernel = mhc_mix_kernel<PP, 4, SBB, ST>;                                                          \
        static bool configured[64] = {};                                                                       \
        if (dev < 0 || dev >= 64 || !configured[dev]) {                                                       \
            NB_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024)); \
            if (dev >= 0 && dev < 64) configured[dev] = true;                                                  \
        }                                                                                                      \
        NB_CUDA_TRY(launch_pdl(kernel, grid, kMixThreads, smem, st, args, R));                                  \
    }
    if (P == 1) {
        if (staged) NB_MIX(1, 1, true) else NB_MIX(1, 2, false)
    } else {
        if (staged) NB_MIX(2, 1, true) else NB_MIX(2, 2, false)
    }
#undef NB_MIX
    NB_CUDA_TRY(cudaGetLastError());
    return true;
}

}  // namespace eng
}  // namespace nb200
