// KV cache of one layer for many sequences with one pinned prefix (see
// kv_abi.cu): the storage and attention calls that the C ABI's KV pool and the
// engine share.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "attention.cuh"

namespace nb200 {

struct KVPool;

// sessions sequences of one layer; heads/kvheads/head_dim as the model;
// positions [0, prefix) are the pinned prefix (one copy shared by every
// session), the others take window slots (window > 0) or max_seq - prefix
// linear slots per session, exactly as Engine::cache_slot maps them
// (needle2/csrc/engine.cpp:500).  fp32 selects the FP32 cache instead of INT8.
KVPool *kv_pool_new(int sessions, int heads, int kvheads, int head_dim, int max_seq, int window, int prefix, bool fp32);
void kv_pool_delete(KVPool *kv);
size_t kv_pool_bytes(const KVPool *kv);
int kv_pool_device(const KVPool *kv);

// Longest visible set of `count` entries whose `tokens` queries start at pos[i]
// (sinks plus the window, or everything up to the position).
int kv_max_visible(int prefix, int window, const int *pos_host, int count, int tokens);

// One call over `count` entries (device arrays ids[count], pos[count]: the
// session and the position of the entry's first token), `tokens` consecutive
// tokens each; q/out [count*tokens][heads*head_dim], k/v [count*tokens][kvheads*head_dim].
//   kStore:  store k/v at their positions (prefix positions into the pinned rows)
//   kDecode: tokens = 1: store, then attend
//   kPrefill: the chunk's own k/v staged, every token attends causally over
//             older slots plus the chunk (store-then-attend order of
//             engine.cpp:1170-1210), then the chunk is stored
//   kQuery:  attend only
// max_visible bounds the entries' visible sets (kv_max_visible).
enum KVOp { kStore = 0, kDecode = 1, kPrefill = 2, kQuery = 3 };
// gate (optional, same layout as out): out is written as out * sigmoid(gate),
// the engine's attention output gate (engine.cpp:1023).
// rot (optional, kQuery): also write out rotated and split for the out
// projection's GEMM (AttnRot); *rot_done tells whether it was.
// qkv (optional, kQuery with tokens = 1 where kv_pool_fuses_qkv): the new
// token's projections as K-split parts (QkvParts); the attention kernel norms
// and ropes q and stores the token's K/V itself (q, k and v above are
// ignored), and writes the gate's sum to `gate` (required with qkv->gate).
bool kv_pool_run(KVPool *kv, KVOp op, const int *ids, const int *pos, int count, int tokens, int max_visible,
                 const float *q, const float *k, const float *v, float *out, cudaStream_t st,
                 const float *gate = nullptr, const AttnRot *rot = nullptr, bool *rot_done = nullptr,
                 const QkvParts *qkv = nullptr);
// Whether kQuery over `count` one-token entries runs the decode kernel that
// takes QkvParts.
bool kv_pool_fuses_qkv(KVPool *kv, int count, int max_visible);

// Where kStore puts one token per entry (ids/pos device arrays): the ring
// destination with this pool's arrays, for kernels that store K/V themselves
// (the engine's fused RoPE + store) before a kQuery call attends.
struct KVStoreTarget {
    KVDest dest;
    int8_t *k8, *v8;       // INT8 cache rows [S][KV][Cs][HD] and their scales
    float *ks, *vs;
    float *kf, *vf;        // FP32 cache rows
    int fp32, kvheads, hd;
};
KVStoreTarget kv_pool_target(KVPool *kv, const int *ids, const int *pos);

}  // namespace nb200
