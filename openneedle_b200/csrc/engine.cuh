// Support kernels of the Needle-2 forward on the GPU (engine_kernels.cu): the
// operations of needle2/csrc/engine.cpp around the CQ matmuls and the INT8/FP32
// KV attention, batched over rows (one row = one session's token).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace nb200 {
namespace eng {

constexpr int kMaxLanes = 8;      // mHC lanes
constexpr int kMaxSites = 4;      // engram sites (the ABI's sites[4])
constexpr int kMaxOrders = 4;     // engram n-gram orders (orders[4])
constexpr int kMaxDim = 4096;     // d_model and hada
constexpr int kMaxHeadDim = 128;

// x[r][n][d] = rows[r][d] * scale for every lane n (engine.cpp:973-974).
bool launch_embed_lanes(const float *rows, int R, int lanes, int D, float scale, float *x, cudaStream_t st);
// Dense FP32 rows gathered by index: out[r][c] = w[ids[r] * cols + c].
bool launch_gather_dense(const float *w, const int64_t *ids, int R, int cols, float *out, cudaStream_t st);
// y[r] = rms(x[r][0..n)) (engine.cpp:181-184) with optional (1 + scale).
bool launch_rms(const float *x, int ldx, int R, int n, const float *scale, float *y, int ldy, cudaStream_t st);

// One dense FP32 matrix slice: out[r][j * ldo_step] ... see launch_dense_rows.
struct DenseSeg {
    const float *w;   // [rows_total][cols]
    int first, rows;  // rows [first, first + rows)
    float *out;       // out[r * ldo + j] for row j of the slice
    int ldo;
};
// out_s[r][j] = sum_k w_s[(first_s + j) * cols + k] * in[r * ldin + k] for the
// given slices (engine.cpp:529-559 mHC projections, 526 dense linear).
bool launch_dense_rows(const DenseSeg *segs, int nseg, const float *in, int ldin, int R, int cols, cudaStream_t st);

// Layer constants of the mHC routing and the layer's engram site.
struct MhcLayer {
    int layer, lanes, D;
    float a_pre, a_post, a_res;   // mhc_a_*[layer]
    const float *b_pre;           // [lanes] (mhc_b_pre row of the layer), device
    const float *b_post;          // [lanes]
    const float *b_res;           // [lanes * lanes]
    const float *norm_in;         // [D]
    const float *ek, *ev;         // engram key/value of this layer's site [R][ld_site] or null
    int ld_site;
};
// Pre-attention part of a layer (engine.cpp:983-992): hpre/hpost gates from the
// raw projections (raw[r] = pre[lanes], post[lanes], res[lanes^2]), u = sum_n
// hpre[n] x[n], engram mixing, z = rms(bx) * (1 + norm_in).  Writes hpost, u,
// bx, z.
bool launch_mhc_pre(const MhcLayer &L, const float *raw, int ldraw, const float *x, int R, float *hpost, float *u,
                    float *bx, float *z, cudaStream_t st);

// The same as launch_rms + launch_dense_rows (the three projections) +
// launch_mhc_pre in one kernel, which also replaces raw's residual part by
// the Sinkhorn-normalised mixing matrix (PostLayer::hres_ready); false
// (nothing launched) where the geometry does not fit it (lanes * D % 128 !=
// 0), and the caller takes that path.
bool launch_mhc_route(const MhcLayer &L, const float *phi_pre, const float *phi_post, const float *phi_res,
                      const float *x, int R, float *raw, int ldraw, float *hpost, float *u, float *bx, float *z,
                      int sms, cudaStream_t st);

// q/k RMS with (1 + norm) per head, then rotary embedding at each row's
// position (engine.cpp:994-1000); positions pos[r] (device), divisor[HD/2] =
// rope_theta^(2j/HD).
bool launch_qk_norm_rope(float *q, float *k, int R, int heads, int kvheads, int hd, const float *q_norm,
                         const float *k_norm, const int *pos, const float *divisor, cudaStream_t st);

}  // namespace eng
struct KVStoreTarget;
namespace eng {
// launch_qk_norm_rope, then the KV store of the row's token (one token per
// row; the positions are the rows' positions) into target.  cos_t / sin_t
// (optional, [table_len][hd / 2]): cosf / sinf of position / divisor, read
// instead of evaluated for positions the table covers (the same values).
// src (optional): q, k, v and gate as K-split partial outputs of the
// projections (qkvg_part of each at src.* + p * pstride, p < parts), added in
// order into q, k, v and src.gate before the norm.
struct QkvgParts {
    const float *q, *k, *v, *g;
    float *gate;
    int parts;
    long long pstride;
};
bool launch_qk_rope_store(float *q, float *k, float *v, int R, int heads, int kvheads, int hd,
                          const float *q_norm, const float *k_norm, const int *pos, const float *divisor,
                          const KVStoreTarget &target, cudaStream_t st, const float *cos_t = nullptr,
                          const float *sin_t = nullptr, int table_len = 0, const QkvgParts *src = nullptr);
// out[i] = sum over p < parts of part[i + p * pstride], in order (i < n).
bool launch_sum_parts(const float *part, int parts, long long pstride, long long n, float *out, cudaStream_t st);

// att *= sigmoid(gate) (engine.cpp:1023).
bool launch_gate(float *att, const float *gate, int R, int A, cudaStream_t st);

struct PostLayer {
    int layer, lanes, D, hada;
    int hres_ready;                // raw's residual part already holds sinkhorn(res * a_res + b_res)
    float a_res;
    const float *b_res;            // [lanes * lanes]
    const float *post_norm, *attn_gate, *pre_hada, *d1, *d2, *d3;
};
// Post-attention part (engine.cpp:1025-1037): attention output norm and gate,
// Hadamard MLP, Sinkhorn mixing of the lanes.  Updates x in place; writes the
// lanes' mean into hidden[r] when hidden is not null.
bool launch_mhc_post(const PostLayer &L, const float *proj, const float *raw, int ldraw, const float *hpost,
                     const float *u, float *bx, float *x, int R, float *hidden, int ldh, cudaStream_t st);

// One launch at a layer boundary: the post-attention part of layer post.layer
// (has_post; launch_mhc_post), then the routing of layer route.layer
// (has_route; launch_mhc_route, with the Sinkhorn-normalised residual matrix
// written into raw) or the final norm (final_norm; launch_final_norm).  Each
// CTA owns whole rows, so the lane state stays on chip between the halves.
struct MixArgs {
    int D, lanes, hada;
    int has_post, has_route, final_norm;
    PostLayer post;                 // has_post (hres_ready must be 1)
    MhcLayer route;                 // has_route
    const float *phi_pre, *phi_post, *phi_res;   // the routing projections of every layer
    const float *proj;              // post: out-projection output [R][D]
    int proj_parts;                 // post: proj as K-split parts (proj + p * proj_pstride; 0 or 1: one)
    long long proj_pstride;
    float *raw;                     // post reads layer l's mixing matrix; route writes layer l + 1's values
    int ldraw;
    float *hpost, *u, *bx;          // post reads layer l's; route writes layer l + 1's
    float *x;                       // [R][lanes][D] lane state, updated in place
    float *z;                       // route: z [R][D]
    float *hidden;                  // post: lane means [R][ldh] (optional)
    int ldh;
    const float *fnorm;             // final: final_norm weights
    float *zf;                      // final: [R][D]
    uint16_t *zhl;                  // route (optional): z rotated per group and split to bf16, hi [R][D] then lo
    long long lo_off;               // at zhl + lo_off
    int group;                      // rotation group (a power of two dividing D)
    float rot_scale;                // 1 / sqrt(group)
    int phi_smem;                   // set by launch_mhc_mix: projections staged in shared memory
};
// Whether launch_mhc_mix takes this geometry (4 lanes, Hadamard width 256 or
// 512, D a multiple of 32 up to that width).
bool mhc_mix_supported(int D, int lanes, int hada);
bool launch_mhc_mix(const MixArgs &a, int R, int sms, cudaStream_t st);

// z[r] = rms(mean over lanes of x[r]) * (1 + final_norm) (engine.cpp:1039-1040).
bool launch_final_norm(const float *x, int R, int lanes, int D, const float *final_norm, float *z, cudaStream_t st);

// Engram rows (engine.cpp:755-768): for every row r (position pos[r] of session
// sess[r]) and table t, the hashed row id t * slots + h % slots of the
// n-gram ending at pos, and whether that n-gram is valid.  Tokens come from
// the chunk (positions >= chunk_start[sess]) or the session's history ring.
struct EngramHash {
    int tables, slots, num_orders, orders[kMaxOrders], window, prefix, hist_cap;
    const int *ring;          // [S][hist_cap]
    const int *chunk;         // [S][T] tokens of the current call, or null
    int T;
    const int *chunk_start;   // [S] position of chunk[s][0]
};
bool launch_engram_ids(const EngramHash &h, const int *sess, const int *pos, int R, int64_t *ids, uint8_t *valid,
                       cudaStream_t st);
// e[r][t * subdim ...] = 0 where the n-gram is invalid.
bool launch_engram_mask(float *e, const uint8_t *valid, int R, int tables, int subdim, cudaStream_t st);
// Dilated causal convolution of the raw engram values (engine.cpp:772-781):
// ev[r][d] = sum_tap taps[tap][d] * raw(pos[r] - tap * dilation)[d] over the
// visible taps; raw values of positions in the current call come from
// chunk_raw[sess][pos - chunk_start], older ones from the ring [S][engring][D].
struct EngramConv {
    int D, taps, dilation, engring, window, prefix, T;
    const float *taps_w;         // [taps][D]
    const float *ring;           // [S][engring][D] of this site (ld_ring_s between sessions)
    size_t ld_ring_s;
    const float *chunk_raw;      // [S][T][D] of this site (ld_chunk rows)
    int ld_chunk;
    const int *chunk_start;      // [S]
};
bool launch_engram_conv(const EngramConv &c, const int *sess, const int *pos, int R, float *ev, int ldev,
                        cudaStream_t st);
// Store the last min(T, engring) raw values of each session's chunk into its ring.
bool launch_engram_ring_store(float *ring, size_t ld_ring_s, const float *chunk_raw, int ld_chunk, int S_count,
                              const int *sess_of_entry, const int *chunk_start, int T, int engring, int D,
                              cudaStream_t st);

// History ring update: ring[sess[e]][(chunk_start[e] + t) % cap] = tokens[e][t]
// for the last min(T, cap) tokens of every entry.
bool launch_history_store(int *ring, int cap, const int *tokens, int T, const int *sess, const int *chunk_start,
                          int entries, cudaStream_t st);

// Candidate projections (engine.cpp:1307-1349): FP32 mode logits[i] = CQ row
// cand[i] . rot (rot = the rotated input, per group FP32 sums times the group
// norm); int8 mode exact int32 group dots and the SDOT epilogue.
bool launch_candidates_f32(const uint8_t *packed, const uint16_t *norms, int rowbytes, int groups, int group,
                           int storage_bits, const float lut[16], const float *rot, const int *cand, int n,
                           float *out, cudaStream_t st);
bool launch_candidates_i8(const uint8_t *packed, const uint16_t *norms, int rowbytes, int groups, int group, int bits,
                          const uint32_t ctab[4], float cs, const int8_t *q, const float *xs, const int *cand, int n,
                          float *out, cudaStream_t st);

// Per-row positions: pos[r] = base[sess(r)] + r % T, sess(r) = r / T.
bool launch_row_positions(const int *base, int entries, int T, int *sess_out, int *pos_out, cudaStream_t st);
// base[i] += delta.
bool launch_advance(int *base, int n, int delta, cudaStream_t st);
// dst[i] = src[i] as int64 (token ids as row ids).
bool launch_widen_ids(const int *src, int64_t *dst, int n, cudaStream_t st);
// Greedy tokens of logits rows -> dst[i * ld_dst] (argmax of needle2_b200_argmax_device).
bool launch_copy_tokens(const int *src, int n, int *dst, int ld_dst, cudaStream_t st);

}  // namespace eng
}  // namespace nb200
