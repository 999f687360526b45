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

struct KVPool {
    int sessions, heads, kvheads, hd, max_seq, window, prefix, cs, device = 0, sms = 148;
    bool prefix_set = false;
    cudaStream_t stream = nullptr;
    Buf<int8_t> pk, pv, sk, sv, stk, stv;
    Buf<float> pks, pvs, sks, svs, stks, stvs, pm, pl, pacc, hq, hk, hv, hout;
    Buf<int> ids, pos;
    ~KVPool() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        for (auto *b : {&pk, &pv, &sk, &sv, &stk, &stv}) b->release();
        for (auto *b : {&pks, &pvs, &sks, &svs, &stks, &stvs, &pm, &pl, &pacc, &hq, &hk, &hv, &hout}) b->release();
        ids.release();
        pos.release();
        if (stream) cudaStreamDestroy(stream);
    }
    int capacity() const { return window ? window + prefix : max_seq; }
};

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
    p.pk = kv.pk.ptr; p.pv = kv.pv.ptr; p.pks = kv.pks.ptr; p.pvs = kv.pvs.ptr;
    p.sk = kv.sk.ptr; p.sv = kv.sv.ptr; p.sks = kv.sks.ptr; p.svs = kv.svs.ptr;
    return p;
}

int max_visible(const KVPool &kv, const int *positions, int count, int tokens) {
    int best = 1;
    for (int i = 0; i < count; ++i) {
        const int pos = positions[i] + tokens - 1;
        const int pc = kv.window ? std::min(kv.prefix, pos + 1) : 0;
        const int start = kv.window ? std::max(kv.prefix, pos - kv.window + 1) : 0;
        best = std::max(best, pc + std::max(0, pos - start + 1));
    }
    return best;
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

bool store_ring(KVPool &kv, const float *k, const float *v, int count, int tokens, int min_t, cudaStream_t st) {
    KVDest d{};
    d.mode = KVDest::kRing;
    d.rows = kv.cs;
    d.prefix = kv.prefix;
    d.window = kv.window;
    d.tokens_per_entry = tokens;
    d.min_t = min_t;
    d.session = kv.ids.ptr;
    d.position = kv.pos.ptr;
    return launch_kv_quantize(k, v, count * tokens, kv.kvheads, kv.hd, kv.sk.ptr, kv.sv.ptr, kv.sks.ptr, kv.svs.ptr, d,
                              st);
}

// Attention of `count` entries x `tokens` queries; staging holds the entries'
// own new K/V when tokens > 1 (prefill).
bool attend(KVPool &kv, const int *positions, int count, int tokens, const float *q, float *out, bool staged,
            cudaStream_t st) {
    AttnParams p = base_params(kv);
    p.tokens = tokens;
    p.session = kv.ids.ptr;
    p.position = kv.pos.ptr;
    p.q = q;
    p.out = out;
    if (staged) {
        p.stage_k = kv.stk.ptr; p.stage_v = kv.stv.ptr; p.stage_ks = kv.stks.ptr; p.stage_vs = kv.stvs.ptr;
        p.stage_rows = count * tokens;
    }
    const int queries = count * tokens;
    p.splits = attention_splits(max_visible(kv, positions, count, tokens), queries * kv.kvheads, kv.sms);
    if (p.splits > 1) {
        const size_t rows = (size_t)queries * kv.heads * p.splits;
        if (!kv.pm.reserve(rows) || !kv.pl.reserve(rows) || !kv.pacc.reserve(rows * kv.hd)) return false;
        p.part_m = kv.pm.ptr; p.part_l = kv.pl.ptr; p.part_acc = kv.pacc.ptr;
    }
    return launch_attention(p, queries, st);
}

bool stage(KVPool &kv, const float *k, const float *v, int rows, cudaStream_t st) {
    const size_t n = (size_t)kv.kvheads * rows;
    if (!kv.stk.reserve(n * kv.hd) || !kv.stv.reserve(n * kv.hd) || !kv.stks.reserve(n) || !kv.stvs.reserve(n))
        return false;
    KVDest d{};
    d.mode = KVDest::kLinear;
    d.rows = rows;
    return launch_kv_quantize(k, v, rows, kv.kvheads, kv.hd, kv.stk.ptr, kv.stv.ptr, kv.stks.ptr, kv.stvs.ptr, d, st);
}

KVPool *pool(void *h) { return static_cast<KVPool *>(h); }

}  // namespace
}  // namespace nb200

using nb200::KVPool;

extern "C" {

void *needle2_kv_create(int sessions, int heads, int kvheads, int head_dim, int max_seq, int window, int prefix_len) {
    nb200::clear_error();
    if (sessions < 1 || heads < 1 || kvheads < 1 || head_dim < 1 || max_seq < 1 || window < 0 || prefix_len < 0) {
        nb200::set_error("invalid KV geometry");
        return nullptr;
    }
    if (heads % kvheads || heads / kvheads > nb200::kMaxGroup) {
        nb200::set_error("heads must be a multiple of kvheads with at most 8 query heads per KV head");
        return nullptr;
    }
    if (head_dim > 128) { nb200::set_error("head_dim above 128 is not supported by the GPU build"); return nullptr; }
    if (prefix_len > max_seq) { nb200::set_error("prefix_len must lie between 0 and max_seq"); return nullptr; }
    auto *kv = new (std::nothrow) KVPool();
    if (!kv) { nb200::set_error("out of host memory"); return nullptr; }
    kv->sessions = sessions; kv->heads = heads; kv->kvheads = kvheads; kv->hd = head_dim; kv->max_seq = max_seq;
    kv->window = window; kv->prefix = prefix_len;
    kv->cs = window ? window : max_seq - prefix_len;
    cudaGetDevice(&kv->device);
    cudaDeviceGetAttribute(&kv->sms, cudaDevAttrMultiProcessorCount, kv->device);
    const size_t prow = (size_t)kvheads * prefix_len, srow = (size_t)sessions * kvheads * kv->cs;
    bool ok = cudaStreamCreateWithFlags(&kv->stream, cudaStreamNonBlocking) == cudaSuccess;
    ok = ok && kv->pk.reserve(prow * head_dim) && kv->pv.reserve(prow * head_dim) && kv->pks.reserve(prow) &&
         kv->pvs.reserve(prow);
    ok = ok && kv->sk.reserve(srow * head_dim) && kv->sv.reserve(srow * head_dim) && kv->sks.reserve(srow) &&
         kv->svs.reserve(srow);
    if (!ok) {
        if (nb200::last_error()[0] == 0) nb200::set_error("KV pool creation failed");
        delete kv;
        return nullptr;
    }
    return kv;
}

void needle2_kv_destroy(void *h) { delete nb200::pool(h); }

size_t needle2_kv_storage_bytes(void *h) {
    KVPool *kv = nb200::pool(h);
    if (!kv) return 0;
    const size_t prow = (size_t)kv->kvheads * kv->prefix, srow = (size_t)kv->sessions * kv->kvheads * kv->cs;
    return (prow + srow) * (2 * (size_t)kv->hd + 2 * sizeof(float));
}

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
    if (mode != 2 && !nb200::store_ring(*kv, k, v, count, 1, 0, st)) return -1;
    if (mode != 0 && !nb200::attend(*kv, positions, count, 1, q, out, false, st)) return -1;
    return 0;
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
    if (!nb200::stage(*kv, k, v, count * tokens, st)) return -1;
    if (!nb200::attend(*kv, start_positions, count, tokens, q, out, true, st)) return -1;
    // write the ring after attending; with a window only the last `window`
    // tokens of the chunk survive (earlier ones would be overwritten anyway)
    const int min_t = kv->window && tokens > kv->window ? tokens - kv->window : 0;
    if (!nb200::store_ring(*kv, k, v, count, tokens, min_t, st)) return -1;
    return 0;
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
