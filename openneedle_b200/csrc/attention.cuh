// INT8 (and FP32) KV-cache attention launchers (see attention.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace nb200 {

constexpr int kMaxQueryGroup = 8;  // query heads per KV head

// Where the store kernels write token t.
struct KVDest {
    enum Mode { kLinear = 0, kRing = 1 } mode;
    int rows;              // kLinear: rows per KV head; kRing: slots per session and head (Cs)
    int prefix, window;    // kRing: positions < prefix go to the pinned prefix rows [KV][prefix];
                           // others to slot window ? (pos-prefix) % window : pos-prefix
    int tokens_per_entry;  // kRing: token t belongs to entry t / tokens_per_entry ...
    int min_t;             // ... and is skipped when t % tokens_per_entry < min_t
    const int *session;    // kRing, device [entries]
    const int *position;   // kRing, device [entries]: position of the entry's first token
    // kRing: the pinned prefix rows (int8 + scales, or FP32), for positions < prefix
    int8_t *pk, *pv;
    float *pks, *pvs;
    float *pkf, *pvf;
};

struct AttnParams {
    int heads, kvheads, hd, prefix, window, cs, splits, tokens;
    int queries;                      // entries * tokens (set by launch_attention)
    int f32;                          // 1: FP32 cache (the *f pointers), 0: INT8 cache
    float inv_sqrt_hd;
    const int8_t *pk, *pv;            // shared prefix [KV][P][HD]
    const float *pks, *pvs;           // [KV][P]
    const int8_t *sk, *sv;            // sessions [S][KV][Cs][HD]
    const float *sks, *svs;           // [S][KV][Cs]
    const int8_t *stage_k, *stage_v;  // prefill chunk [KV][stage_rows][HD] or null
    const float *stage_ks, *stage_vs;
    const float *pkf, *pvf, *skf, *svf, *stage_kf, *stage_vf;   // FP32 cache, same layouts
    int stage_rows;
    const int *session, *position;    // per entry (device): session, position of its first query
    const float *q;                   // [queries][heads][HD], queries = entries * tokens
    float *out;                       // [queries][heads][HD]
    const float *gate;                // null, or [queries][heads][HD]: out is written as out * sigmoid(gate)
    float *part_m, *part_l, *part_acc; // split partials (splits > 1)
    // null, or the operands of the out projection's tensor-core GEMM: out of
    // each query, rotated per group of heads / kvheads heads (one KV head's
    // query heads, the CQ group of the out projection) and split into bf16
    // hi [queries][hilo_ld] and lo (at hilo + hilo_lo)
    uint16_t *hilo;
    long long hilo_lo;
    int hilo_ld;
    float rot_scale;
    // null, or decode (tokens == 1, INT8 cache, attention_fuses_qkv) with the
    // new token's projections as K-split parts: q and gate [queries][heads][HD]
    // and k, v [queries][kvheads][HD] (part k at + k * qkv_pstride).  Each CTA
    // (or warp, one per query) adds, norms and ropes its query heads; the one
    // whose slots include the token's own stores the token's K and V before it
    // reads its slots, and writes its heads' gate sums to `gate` (then required).
    const float *qkv_q, *qkv_k, *qkv_v, *qkv_g;
    int qkv_parts;
    long long qkv_pstride;
    const float *q_norm, *k_norm;     // [HD]: RMS-norm weights (applied as 1 + w)
    const float *rope_cos, *rope_sin; // [rope_len][HD / 2] or null: cos / sin of position / rope_div[j]
    const float *rope_div;            // [HD / 2]
    int rope_len;
};

// The new token's projections handed to the decode attention (AttnParams::qkv_*).
struct QkvParts {
    const float *q, *k, *v, *gate;    // part 0 of each
    int parts;
    long long pstride;
    const float *q_norm, *k_norm, *rope_cos, *rope_sin, *rope_div;
    int rope_len;
};

// Request for AttnParams::hilo (see there); group must equal heads / kvheads * hd.
struct AttnRot {
    uint16_t *hilo;
    long long lo_off;
    int ld, group;
    float scale;
};

// INT8: quantise (engine.cpp:1005-1021) and store k/v [tokens][kvheads*hd].
bool launch_kv_quantize(const float *k, const float *v, int tokens, int kvheads, int hd, int8_t *ko, int8_t *vo,
                        float *ks, float *vs, const KVDest &dest, cudaStream_t st);
// FP32: store k/v unchanged (engine.cpp:1002-1004) in the same row layout.
bool launch_kv_store_f32(const float *k, const float *v, int tokens, int kvheads, int hd, float *ko, float *vo,
                         const KVDest &dest, cudaStream_t st);
int attention_splits(int max_len, int queries_x_kv, int sms);
// Whether launch_attention(p, queries) on `sms` SMs should take the new
// token's projections as parts (AttnParams::qkv_*; p.splits set): its decode
// kernel can, and measured faster than the projections' own epilogue.
bool attention_fuses_qkv(const AttnParams &p, int queries, int sms);
// rot_done (optional): whether p.hilo was written (the decode forms write it;
// the others leave it to the caller and launch as if it were null).
bool launch_attention(const AttnParams &p, int queries, cudaStream_t st, bool *rot_done = nullptr);

}  // namespace nb200
