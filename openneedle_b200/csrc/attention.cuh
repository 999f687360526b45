// INT8 KV-cache attention launchers (see attention.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace nb200 {

constexpr int kMaxGroup = 8;  // query heads per KV head

// Where kv_quantize_kernel writes token t.
struct KVDest {
    enum Mode { kLinear = 0, kRing = 1 } mode;
    int rows;              // kLinear: rows per KV head; kRing: slots per session and head (Cs)
    int prefix, window;    // kRing: slot = window ? (pos-prefix) % window : pos-prefix
    int tokens_per_entry;  // kRing: token t belongs to entry t / tokens_per_entry ...
    int min_t;             // ... and is skipped when t % tokens_per_entry < min_t
    const int *session;    // kRing, device [entries]
    const int *position;   // kRing, device [entries]: position of the entry's first token
};

struct AttnParams {
    int heads, kvheads, hd, prefix, window, cs, splits, tokens;
    float inv_sqrt_hd;
    const int8_t *pk, *pv;            // shared prefix [KV][P][HD]
    const float *pks, *pvs;           // [KV][P]
    const int8_t *sk, *sv;            // sessions [S][KV][Cs][HD]
    const float *sks, *svs;           // [S][KV][Cs]
    const int8_t *stage_k, *stage_v;  // prefill chunk [KV][stage_rows][HD] or null
    const float *stage_ks, *stage_vs;
    int stage_rows;
    const int *session, *position;    // per entry (device): session, position of its first query
    const float *q;                   // [queries][heads][HD], queries = entries * tokens
    float *out;                       // [queries][heads][HD]
    float *part_m, *part_l, *part_acc; // split partials (splits > 1)
};

bool launch_kv_quantize(const float *k, const float *v, int tokens, int kvheads, int hd, int8_t *ko, int8_t *vo,
                        float *ks, float *vs, const KVDest &dest, cudaStream_t st);
int attention_splits(int max_len, int queries_x_kv, int sms);
bool launch_attention(const AttnParams &p, int queries, cudaStream_t st);

}  // namespace nb200
