// C ABI of the batched INT8 KV cache and its attention (additive to the
// reference ABI; the reference serves one sequence per Engine and snapshots a
// prefix per instance, needle2/csrc/engine.cpp:192-199,450-499).  Here one
// read-only prefix is stored once on the device and shared by every session;
// a session's state is the prefix plus its own suffix slots, so "restore to
// prefix" is simply continuing from position P.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/needle2_b200.h"
#include "attention.cuh"
#include "common.cuh"
#include "cq_gemv.cuh"
#include "kv_pool.cuh"

namespace nb200 {
namespace {

template <typename T>
struct Buf {
    T *ptr = nullptr;
    size_t cap = 0;
    bool reserve(size_t n) {
        if (n <= cap) return true;
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        cap = 0;
        cudaError_t e = cudaMalloc(&ptr, sizeof(T) * std::max<size_t>(n, 1));
        if (e != cudaSuccess) {
            set_error(std::string("device allocation failed: ") + cudaGetErrorString(e));
            ptr = nullptr;
            return false;
        }
        cap = n;
        return true;
    }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        cap = 0;
    }
};

}  // namespace

struct KVPool {
    int sessions, heads, kvheads, hd, max_seq, window, prefix, cs, device = 0, sms = 148;
    bool fp32 = false;
    bool prefix_set = false;
    cudaStream_t stream = nullptr;
    Buf<int8_t> pk, pv, sk, sv, stk, stv;
    Buf<float> pks, pvs, sks, svs, stks, stvs, pm, pl, pacc, hq, hk, hv, hout;
    Buf<float> pkf, pvf, skf, svf, stkf, stvf;   // FP32 cache
    Buf<int> ids, pos;
    ~KVPool() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        for (auto *b : {&pk, &pv, &sk, &sv, &stk, &stv}) b->release();
        for (auto *b : {&pks, &pvs, &sks, &svs, &stks, &stvs, &pm, &pl, &pacc, &hq, &hk, &hv, &hout}) b->release();
        for (auto *b : {&pkf, &pvf, &skf, &svf, &stkf, &stvf}) b->release();
        ids.release();
        pos.release();
        if (stream) cudaStreamDestroy(stream);
    }
    int capacity() const { return window ? window + prefix : max_seq; }
};

namespace {

// Host-side checks of one call's sessions and positions (tokens per entry).
bool validate(const KVPool &kv, const int *session_ids, const int *positions, int count, int tokens,
              bool query_only = false) {
    if (count < 0 || tokens < 1) { set_error("invalid count"); return false; }
    std::vector<char> seen(kv.sessions, 0);
    for (int i = 0; i < count; ++i) {
        const int s = session_ids[i], p = positions[i];
        if (s < 0 || s >= kv.sessions) { set_error("session id outside the pool"); return false; }
        if (seen[s]) { set_error("a session appears twice in one call"); return false; }
        seen[s] = 1;
        if (p < (query_only ? 0 : kv.prefix)) {
            set_error(query_only ? "negative position" : "position lies inside the shared prefix");
            return false;
        }
        if (kv.prefix && !kv.prefix_set) { set_error("shared prefix not set"); return false; }
        if (!kv.window && (long long)p + tokens > kv.max_seq) { set_error("maximum context reached"); return false; }
        if (kv.window && (long long)p + tokens > 0x7fffffffLL) { set_error("position overflow"); return false; }
    }
    return true;
}

AttnParams base_params(KVPool &kv) {
    AttnParams p{};
    p.heads = kv.heads; p.kvheads = kv.kvheads; p.hd = kv.hd; p.prefix = kv.prefix; p.window = kv.window;
    p.cs = kv.cs;
    p.inv_sqrt_hd = 1 / std::sqrt((float)kv.hd);   // the reference's 1/sqrt(float(HD))
    p.f32 = kv.fp32 ? 1 : 0;
    p.pk = kv.pk.ptr; p.pv = kv.pv.ptr; p.pks = kv.pks.ptr; p.pvs = kv.pvs.ptr;
    p.sk = kv.sk.ptr; p.sv = kv.sv.ptr; p.sks = kv.sks.ptr; p.svs = kv.svs.ptr;
    p.pkf = kv.pkf.ptr; p.pvf = kv.pvf.ptr; p.skf = kv.skf.ptr; p.svf = kv.svf.ptr;
    return p;
}

// Session ids and positions of up to kIndexArgMax entries travel as a kernel
// argument, which the launch copies from the host arrays as it is enqueued:
// no staging copy of pageable memory (which a stream capture cannot record)
// and no pinned buffer whose reuse would have to wait for the stream.
constexpr int kIndexArgMax = 1024;
struct IndexArgs {
    int count;
    int ids[kIndexArgMax];
    int pos[kIndexArgMax];
};

__global__ void index_upload_kernel(const __grid_constant__ IndexArgs a, int *ids, int *pos) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.count; i += gridDim.x * blockDim.x) {
        ids[i] = a.ids[i];
        pos[i] = a.pos[i];
    }
}

bool upload_index(KVPool &kv, const int *session_ids, const int *positions, int count, cudaStream_t st) {
    if (!kv.ids.reserve(count) || !kv.pos.reserve(count)) return false;
    if (count <= kIndexArgMax) {
        IndexArgs a;
        a.count = count;
        std::memcpy(a.ids, session_ids, sizeof(int) * count);
        std::memcpy(a.pos, positions, sizeof(int) * count);
        index_upload_kernel<<<1, 256, 0, st>>>(a, kv.ids.ptr, kv.pos.ptr);
        NB_CUDA_TRY(cudaGetLastError());
        return true;
    }
    NB_CUDA_TRY(cudaMemcpyAsync(kv.ids.ptr, session_ids, sizeof(int) * count, cudaMemcpyHostToDevice, st));
    NB_CUDA_TRY(cudaMemcpyAsync(kv.pos.ptr, positions, sizeof(int) * count, cudaMemcpyHostToDevice, st));
    return true;
}

KVDest ring_dest(KVPool &kv, const int *ids, const int *pos, int tokens, int min_t) {
    KVDest d{};
    d.mode = KVDest::kRing;
    d.rows = kv.cs;
    d.prefix = kv.prefix;
    d.window = kv.window;
    d.tokens_per_entry = tokens;
    d.min_t = min_t;
    d.session = ids;
    d.position = pos;
    d.pk = kv.pk.ptr; d.pv = kv.pv.ptr; d.pks = kv.pks.ptr; d.pvs = kv.pvs.ptr;
    d.pkf = kv.pkf.ptr; d.pvf = kv.pvf.ptr;
    return d;
}

bool store_ring(KVPool &kv, const int *ids, const int *pos, const float *k, const float *v, int count, int tokens,
                int min_t, cudaStream_t st) {
    const KVDest d = ring_dest(kv, ids, pos, tokens, min_t);
    if (kv.fp32)
        return launch_kv_store_f32(k, v, count * tokens, kv.kvheads, kv.hd, kv.skf.ptr, kv.svf.ptr, d, st);
    return launch_kv_quantize(k, v, count * tokens, kv.kvheads, kv.hd, kv.sk.ptr, kv.sv.ptr, kv.sks.ptr, kv.svs.ptr, d,
                              st);
}

// Attention of `count` entries x `tokens` queries; staging holds the entries'
// own new K/V when `staged` (prefill).
bool attend(KVPool &kv, const int *ids, const int *pos, int count, int tokens, int max_len, const float *q, float *out,
            bool staged, cudaStream_t st, const float *gate = nullptr, const AttnRot *rot = nullptr,
            bool *rot_done = nullptr, const QkvParts *qkv = nullptr) {
    AttnParams p = base_params(kv);
    p.gate = gate;
    if (qkv) {
        p.qkv_q = qkv->q; p.qkv_k = qkv->k; p.qkv_v = qkv->v; p.qkv_g = qkv->gate;
        p.qkv_parts = qkv->parts;
        p.qkv_pstride = qkv->pstride;
        p.q_norm = qkv->q_norm; p.k_norm = qkv->k_norm;
        p.rope_cos = qkv->rope_cos; p.rope_sin = qkv->rope_sin; p.rope_div = qkv->rope_div;
        p.rope_len = qkv->rope_len;
        q = nullptr;
    }
    if (rot && rot->group == kv.heads / kv.kvheads * kv.hd) {
        p.hilo = rot->hilo;
        p.hilo_lo = rot->lo_off;
        p.hilo_ld = rot->ld;
        p.rot_scale = rot->scale;
    }
    p.tokens = tokens;
    p.session = ids;
    p.position = pos;
    p.q = q;
    p.out = out;
    if (staged) {
        p.stage_k = kv.stk.ptr; p.stage_v = kv.stv.ptr; p.stage_ks = kv.stks.ptr; p.stage_vs = kv.stvs.ptr;
        p.stage_kf = kv.stkf.ptr; p.stage_vf = kv.stvf.ptr;
        p.stage_rows = count * tokens;
    }
    const int queries = count * tokens;
    p.splits = attention_splits(max_len, queries * kv.kvheads, kv.sms);
    if (p.splits > 1) {
        const size_t rows = (size_t)queries * kv.heads * p.splits;
        if (!kv.pm.reserve(rows) || !kv.pl.reserve(rows) || !kv.pacc.reserve(rows * kv.hd)) return false;
        p.part_m = kv.pm.ptr; p.part_l = kv.pl.ptr; p.part_acc = kv.pacc.ptr;
    }
    return launch_attention(p, queries, st, rot_done);
}

// The chunk's own K/V in the staging layout [KV][rows][HD] (quantised for INT8).
bool stage(KVPool &kv, const float *k, const float *v, int rows, cudaStream_t st) {
    const size_t n = (size_t)kv.kvheads * rows;
    KVDest d{};
    d.mode = KVDest::kLinear;
    d.rows = rows;
    if (kv.fp32) {
        if (!kv.stkf.reserve(n * kv.hd) || !kv.stvf.reserve(n * kv.hd)) return false;
        // the FP32 staging rows are still written by the ring store's kernel, in linear mode
        return launch_kv_store_f32(k, v, rows, kv.kvheads, kv.hd, kv.stkf.ptr, kv.stvf.ptr, d, st);
    }
    if (!kv.stk.reserve(n * kv.hd) || !kv.stv.reserve(n * kv.hd) || !kv.stks.reserve(n) || !kv.stvs.reserve(n))
        return false;
    return launch_kv_quantize(k, v, rows, kv.kvheads, kv.hd, kv.stk.ptr, kv.stv.ptr, kv.stks.ptr, kv.stvs.ptr, d, st);
}

KVPool *pool(void *h) { return static_cast<KVPool *>(h); }

}  // namespace

// ---- the pool calls shared by the C ABI below and the engine --------------

KVPool *kv_pool_new(int sessions, int heads, int kvheads, int head_dim, int max_seq, int window, int prefix,
                    bool fp32) {
    if (sessions < 1 || heads < 1 || kvheads < 1 || head_dim < 1 || max_seq < 1 || window < 0 || prefix < 0) {
        set_error("invalid KV geometry");
        return nullptr;
    }
    if (heads % kvheads || heads / kvheads > kMaxQueryGroup) {
        set_error("heads must be a multiple of kvheads with at most 8 query heads per KV head");
        return nullptr;
    }
    if (head_dim > 128) { set_error("head_dim above 128 is not supported by the GPU build"); return nullptr; }
    if (prefix > max_seq) { set_error("prefix_len must lie between 0 and max_seq"); return nullptr; }
    auto *kv = new (std::nothrow) KVPool();
    if (!kv) { set_error("out of host memory"); return nullptr; }
    kv->sessions = sessions; kv->heads = heads; kv->kvheads = kvheads; kv->hd = head_dim; kv->max_seq = max_seq;
    kv->window = window; kv->prefix = prefix; kv->fp32 = fp32;
    kv->cs = window ? window : max_seq - prefix;
    cudaGetDevice(&kv->device);
    cudaDeviceGetAttribute(&kv->sms, cudaDevAttrMultiProcessorCount, kv->device);
    const size_t prow = (size_t)kvheads * prefix, srow = (size_t)sessions * kvheads * kv->cs;
    bool ok = cudaStreamCreateWithFlags(&kv->stream, cudaStreamNonBlocking) == cudaSuccess;
    if (fp32) {
        ok = ok && kv->pkf.reserve(prow * head_dim) && kv->pvf.reserve(prow * head_dim);
        ok = ok && kv->skf.reserve(srow * head_dim) && kv->svf.reserve(srow * head_dim);
    } else {
        ok = ok && kv->pk.reserve(prow * head_dim) && kv->pv.reserve(prow * head_dim) && kv->pks.reserve(prow) &&
             kv->pvs.reserve(prow);
        ok = ok && kv->sk.reserve(srow * head_dim) && kv->sv.reserve(srow * head_dim) && kv->sks.reserve(srow) &&
             kv->svs.reserve(srow);
    }
    if (!ok) {
        if (last_error()[0] == 0) set_error("KV pool creation failed");
        delete kv;
        return nullptr;
    }
    return kv;
}

void kv_pool_delete(KVPool *kv) { delete kv; }

size_t kv_pool_bytes(const KVPool *kv) {
    if (!kv) return 0;
    const size_t rows = (size_t)kv->kvheads * kv->prefix + (size_t)kv->sessions * kv->kvheads * kv->cs;
    return kv->fp32 ? rows * 2 * sizeof(float) * kv->hd : rows * (2 * (size_t)kv->hd + 2 * sizeof(float));
}

int kv_pool_device(const KVPool *kv) { return kv->device; }

bool kv_pool_fuses_qkv(KVPool *kv, int count, int max_visible) {
    if (!kv || count <= 0) return false;
    AttnParams p = base_params(*kv);
    p.tokens = 1;
    p.splits = attention_splits(max_visible, count * kv->kvheads, kv->sms);
    return attention_fuses_qkv(p, count, kv->sms);
}

KVStoreTarget kv_pool_target(KVPool *kv, const int *ids, const int *pos) {
    KVStoreTarget t{};
    t.dest = ring_dest(*kv, ids, pos, 1, 0);
    t.k8 = kv->sk.ptr; t.v8 = kv->sv.ptr; t.ks = kv->sks.ptr; t.vs = kv->svs.ptr;
    t.kf = kv->skf.ptr; t.vf = kv->svf.ptr;
    t.fp32 = kv->fp32 ? 1 : 0;
    t.kvheads = kv->kvheads;
    t.hd = kv->hd;
    return t;
}

int kv_max_visible(int prefix, int window, const int *positions, int count, int tokens) {
    int best = 1;
    for (int i = 0; i < count; ++i) {
        const int pos = positions[i] + tokens - 1;
        const int pc = window ? std::min(prefix, pos + 1) : 0;
        const int start = window ? std::max(prefix, pos - window + 1) : 0;
        best = std::max(best, pc + std::max(0, pos - start + 1));
    }
    return best;
}

bool kv_pool_run(KVPool *kv, KVOp op, const int *ids, const int *pos, int count, int tokens, int max_visible,
                 const float *q, const float *k, const float *v, float *out, cudaStream_t st, const float *gate,
                 const AttnRot *rot, bool *rot_done, const QkvParts *qkv) {
    if (rot_done) *rot_done = false;
    if (count <= 0) return true;
    if (qkv && (op != kQuery || tokens != 1 || qkv->parts < 1 || qkv->parts > kMaxKParts || !qkv->q || !qkv->k ||
                !qkv->v || !qkv->q_norm || !qkv->k_norm || !qkv->rope_div || (qkv->gate && !gate))) {
        set_error("KV pool: projections as parts need a one-token query with every operand");
        return false;
    }
    switch (op) {
        case kStore: return store_ring(*kv, ids, pos, k, v, count, tokens, 0, st);
        case kQuery:
            return attend(*kv, ids, pos, count, tokens, max_visible, q, out, false, st, gate, rot, rot_done, qkv);
        case kDecode:
            if (tokens != 1) { set_error("decode takes one token per entry"); return false; }
            return store_ring(*kv, ids, pos, k, v, count, 1, 0, st) &&
                   attend(*kv, ids, pos, count, 1, max_visible, q, out, false, st, gate);
        case kPrefill: {
            if (!stage(*kv, k, v, count * tokens, st)) return false;
            if (!attend(*kv, ids, pos, count, tokens, max_visible, q, out, true, st, gate)) return false;
            // write the slots after attending; with a window only the last `window`
            // tokens of the chunk outside the pinned prefix survive (earlier ones
            // would be overwritten anyway)
            const int min_t = kv->window && tokens > kv->window ? tokens - kv->window : 0;
            return store_ring(*kv, ids, pos, k, v, count, tokens, min_t, st);
        }
    }
    return false;
}

}  // namespace nb200

using nb200::KVPool;

extern "C" {

void *needle2_kv_create(int sessions, int heads, int kvheads, int head_dim, int max_seq, int window, int prefix_len) {
    nb200::clear_error();
    return nb200::kv_pool_new(sessions, heads, kvheads, head_dim, max_seq, window, prefix_len, false);
}

void needle2_kv_destroy(void *h) { nb200::kv_pool_delete(nb200::pool(h)); }

size_t needle2_kv_storage_bytes(void *h) { return nb200::kv_pool_bytes(nb200::pool(h)); }

int needle2_kv_set_prefix_device(void *h, const float *k, const float *v, void *stream) {
    nb200::clear_error();
    KVPool *kv = nb200::pool(h);
    if (!kv) { nb200::set_error("null KV pool"); return -1; }
    if (cudaSetDevice(kv->device) != cudaSuccess) { nb200::set_error("cudaSetDevice failed"); return -1; }
    nb200::KVDest d{};
    d.mode = nb200::KVDest::kLinear;
    d.rows = kv->prefix;
    if (!nb200::launch_kv_quantize(k, v, kv->prefix, kv->kvheads, kv->hd, kv->pk.ptr, kv->pv.ptr, kv->pks.ptr,
                                   kv->pvs.ptr, d, static_cast<cudaStream_t>(stream)))
        return -1;
    kv->prefix_set = true;
    return 0;
}

int needle2_kv_set_prefix(void *h, const float *k, const float *v) {
    nb200::clear_error();
    KVPool *kv = nb200::pool(h);
    if (!kv) { nb200::set_error("null KV pool"); return -1; }
    if (cudaSetDevice(kv->device) != cudaSuccess) { nb200::set_error("cudaSetDevice failed"); return -1; }
    const size_t n = (size_t)kv->prefix * kv->kvheads * kv->hd;
    if (!n) { kv->prefix_set = true; return 0; }
    if (!kv->hk.reserve(n) || !kv->hv.reserve(n)) return -1;
    cudaStream_t st = kv->stream;
    if (cudaMemcpyAsync(kv->hk.ptr, k, 4 * n, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(kv->hv.ptr, v, 4 * n, cudaMemcpyHostToDevice, st) != cudaSuccess) {
        nb200::set_error("prefix upload failed");
        return -1;
    }
    if (needle2_kv_set_prefix_device(h, kv->hk.ptr, kv->hv.ptr, st)) return -1;
    if (cudaStreamSynchronize(st) != cudaSuccess) { nb200::set_error("prefix store failed"); return -1; }
    return 0;
}

// mode: 0 = store only, 1 = store then attend (decode), 2 = attend only.
static int decode_device(void *h, const int *session_ids, const int *positions, const float *q, const float *k,
                         const float *v, float *out, int count, void *stream, int mode) {
    nb200::clear_error();
    KVPool *kv = nb200::pool(h);
    if (!kv) { nb200::set_error("null KV pool"); return -1; }
    if (count == 0) return 0;
    if (!nb200::validate(*kv, session_ids, positions, count, 1, mode == 2)) return -1;
    if (cudaSetDevice(kv->device) != cudaSuccess) { nb200::set_error("cudaSetDevice failed"); return -1; }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (!nb200::upload_index(*kv, session_ids, positions, count, st)) return -1;
    const nb200::KVOp op = mode == 0 ? nb200::kStore : mode == 1 ? nb200::kDecode : nb200::kQuery;
    const int len = nb200::kv_max_visible(kv->prefix, kv->window, positions, count, 1);
    return nb200::kv_pool_run(kv, op, kv->ids.ptr, kv->pos.ptr, count, 1, len, q, k, v, out, st) ? 0 : -1;
}

int needle2_attention_decode_device(void *h, const int *session_ids, const int *positions, const float *q,
                                    const float *k, const float *v, float *out, int count, void *stream) {
    return decode_device(h, session_ids, positions, q, k, v, out, count, stream, 1);
}
int needle2_kv_store_device(void *h, const int *session_ids, const int *positions, const float *k, const float *v,
                            int count, void *stream) {
    return decode_device(h, session_ids, positions, nullptr, k, v, nullptr, count, stream, 0);
}
int needle2_attention_query_device(void *h, const int *session_ids, const int *positions, const float *q, float *out,
                                   int count, void *stream) {
    return decode_device(h, session_ids, positions, q, nullptr, nullptr, out, count, stream, 2);
}

int needle2_attention_prefill_device(void *h, const int *session_ids, const int *start_positions, int tokens,
                                     const float *q, const float *k, const float *v, float *out, int count,
                                     void *stream) {
    nb200::clear_error();
    KVPool *kv = nb200::pool(h);
    if (!kv) { nb200::set_error("null KV pool"); return -1; }
    if (count == 0) return 0;
    if (!nb200::validate(*kv, session_ids, start_positions, count, tokens)) return -1;
    if (cudaSetDevice(kv->device) != cudaSuccess) { nb200::set_error("cudaSetDevice failed"); return -1; }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (!nb200::upload_index(*kv, session_ids, start_positions, count, st)) return -1;
    const int len = nb200::kv_max_visible(kv->prefix, kv->window, start_positions, count, tokens);
    return nb200::kv_pool_run(kv, nb200::kPrefill, kv->ids.ptr, kv->pos.ptr, count, tokens, len, q, k, v, out, st)
               ? 0
               : -1;
}

// Host-pointer forms: copy in, run on the pool's stream, copy out, synchronise.
static int host_call(void *h, const int *ids, const int *pos, const float *q, const float *k, const float *v,
                     float *out, int count, int tokens, int mode) {
    nb200::clear_error();
    KVPool *kv = nb200::pool(h);
    if (!kv) { nb200::set_error("null KV pool"); return -1; }
    if (count <= 0) return count == 0 ? 0 : -1;
    if (cudaSetDevice(kv->device) != cudaSuccess) { nb200::set_error("cudaSetDevice failed"); return -1; }
    const size_t nq = (size_t)count * tokens * kv->heads * kv->hd, nk = (size_t)count * tokens * kv->kvheads * kv->hd;
    cudaStream_t st = kv->stream;
    if ((q && !kv->hq.reserve(nq)) || (k && !kv->hk.reserve(nk)) || (v && !kv->hv.reserve(nk)) ||
        (out && !kv->hout.reserve(nq)))
        return -1;
    cudaError_t e = cudaSuccess;
    if (q) e = cudaMemcpyAsync(kv->hq.ptr, q, 4 * nq, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && k) e = cudaMemcpyAsync(kv->hk.ptr, k, 4 * nk, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && v) e = cudaMemcpyAsync(kv->hv.ptr, v, 4 * nk, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) { nb200::set_error(std::string("upload: ") + cudaGetErrorString(e)); return -1; }
    int rc;
    if (mode == 3)
        rc = needle2_attention_prefill_device(h, ids, pos, tokens, kv->hq.ptr, kv->hk.ptr, kv->hv.ptr, kv->hout.ptr,
                                              count, st);
    else
        rc = decode_device(h, ids, pos, q ? kv->hq.ptr : nullptr, k ? kv->hk.ptr : nullptr,
                           v ? kv->hv.ptr : nullptr, out ? kv->hout.ptr : nullptr, count, st, mode);
    if (rc) return rc;
    if (out) e = cudaMemcpyAsync(out, kv->hout.ptr, 4 * nq, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) { nb200::set_error(std::string("attention: ") + cudaGetErrorString(e)); return -1; }
    return 0;
}

int needle2_attention_decode(void *h, const int *session_ids, const int *positions, const float *q, const float *k,
                             const float *v, float *out, int count) {
    return host_call(h, session_ids, positions, q, k, v, out, count, 1, 1);
}
int needle2_kv_store(void *h, const int *session_ids, const int *positions, const float *k, const float *v,
                     int count) {
    return host_call(h, session_ids, positions, nullptr, k, v, nullptr, count, 1, 0);
}
int needle2_attention_query(void *h, const int *session_ids, const int *positions, const float *q, float *out,
                            int count) {
    return host_call(h, session_ids, positions, q, nullptr, nullptr, out, count, 1, 2);
}
int needle2_attention_prefill(void *h, const int *session_ids, const int *start_positions, int tokens, const float *q,
                              const float *k, const float *v, float *out, int count) {
    if (tokens < 1) { nb200::set_error("tokens must be positive"); return -1; }
    return host_call(h, session_ids, start_positions, q, k, v, out, count, tokens, 3);
}

// One session's cache in the reference layout (needle2/csrc/engine.cpp:376-449):
// keys/values [capacity][kvheads*hd], scales [capacity][kvheads],
// capacity = window ? window + prefix : max_seq; slot s < prefix is the
// shared prefix, the rest the session's own slots.
int needle2_kv_export(void *h, int session, int8_t *keys, int8_t *values, float *k_scales, float *v_scales) {
    nb200::clear_error();
    KVPool *kv = nb200::pool(h);
    if (!kv || session < 0 || session >= kv->sessions) { nb200::set_error("invalid pool or session"); return -1; }
    if (cudaSetDevice(kv->device) != cudaSuccess || cudaStreamSynchronize(kv->stream) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        nb200::set_error("device sync failed");
        return -1;
    }
    const int KV = kv->kvheads, HD = kv->hd, P = kv->prefix, C = kv->cs;
    std::vector<int8_t> pk((size_t)KV * P * HD), pv(pk.size()), sk((size_t)KV * C * HD), sv(sk.size());
    std::vector<float> pks((size_t)KV * P), pvs(pks.size()), sks((size_t)KV * C), svs(sks.size());
    const size_t soff = (size_t)session * KV * C;
    cudaError_t e = cudaSuccess;
    if (P) {
        e = cudaMemcpy(pk.data(), kv->pk.ptr, pk.size(), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(pv.data(), kv->pv.ptr, pv.size(), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(pks.data(), kv->pks.ptr, 4 * pks.size(), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(pvs.data(), kv->pvs.ptr, 4 * pvs.size(), cudaMemcpyDeviceToHost);
    }
    if (e == cudaSuccess && C) {
        e = cudaMemcpy(sk.data(), kv->sk.ptr + soff * HD, sk.size(), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(sv.data(), kv->sv.ptr + soff * HD, sv.size(), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(sks.data(), kv->sks.ptr + soff, 4 * sks.size(), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(svs.data(), kv->svs.ptr + soff, 4 * svs.size(), cudaMemcpyDeviceToHost);
    }
    if (e != cudaSuccess) { nb200::set_error(std::string("export: ") + cudaGetErrorString(e)); return -1; }
    const int cap = kv->capacity();
    for (int slot = 0; slot < cap; ++slot) {
        for (int kh = 0; kh < KV; ++kh) {
            const bool pre = slot < P;
            const size_t src = pre ? (size_t)kh * P + slot : (size_t)kh * C + (slot - P);
            const size_t dst = (size_t)slot * KV + kh;
            if (pre || slot - P < C) {
                for (int d = 0; d < HD; ++d) {
                    keys[dst * HD + d] = pre ? pk[src * HD + d] : sk[src * HD + d];
                    values[dst * HD + d] = pre ? pv[src * HD + d] : sv[src * HD + d];
                }
                k_scales[dst] = pre ? pks[src] : sks[src];
                v_scales[dst] = pre ? pvs[src] : svs[src];
            }
        }
    }
    return 0;
}

}  // extern "C"
