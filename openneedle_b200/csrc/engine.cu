// The Needle-2 forward on the GPU behind the reference's engine ABI
// (needle2/csrc/engine.cpp:1499-1548) and a batch extension for many
// sequences in lockstep.
//
// A Model holds the weights: the caller's CQ handles (device-resident, made
// by needle2_cq_create), their int8 twins once SDOT is enabled, and device
// copies of every FP32 tensor.  A State holds S sequences: per layer one KV
// pool (INT8 or FP32; a pinned prefix shared by all sequences plus per-
// sequence slots, Engine::cache_slot's mapping), the token-history ring and
// the engram value rings.  One forward pass runs T tokens of each of E
// sequences as R = E*T rows: engrams, embedding, then per layer the mHC
// routing, fused Q/K/V/gate projection, QK norm + RoPE, store-then-attend,
// gate, out projection and the Hadamard MLP/Sinkhorn mixing, then the final
// norm and LM head (engine.cpp:968-1044 for a step, 1045-1301 for prefill,
// whose chunked order gives the same values).  Every kernel is this
// library's: CQ matmuls (cq_*), attention (attention.cu), the rest
// (engine_kernels.cu).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/needle2_b200.h"
#include "common.cuh"
#include "cq_gemv.cuh"
#include "cq_handle.cuh"
#include "cq_kernels.cuh"
#include "engine.cuh"
#include "kv_pool.cuh"
#include "pdl.cuh"
#include "qkvg_epilogue.cuh"

namespace nb200 {
namespace {

thread_local std::string g_engine_error;

struct Failure : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// Turns a failed library call into an exception carrying its message.
void check(bool ok, const char *what) {
    if (!ok) {
        const char *msg = last_error();
        throw Failure(std::string(what) + (msg && *msg ? std::string(": ") + msg : std::string()));
    }
}
void cuda_check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) throw Failure(std::string(what) + ": " + cudaGetErrorString(e));
}

template <typename T>
struct DevBuf {
    T *ptr = nullptr;
    size_t cap = 0;
    void reserve(size_t n) {
        if (n <= cap) return;
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        cap = 0;
        cuda_check(cudaMalloc(&ptr, sizeof(T) * std::max<size_t>(n, 1)), "device allocation");
        cap = n;
    }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        cap = 0;
    }
    ~DevBuf() { release(); }
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
};

// One tensor of the model.
struct Tensor {
    void *cq = nullptr;      // FP32-mode CQ handle (caller's)
    void *sdot = nullptr;    // int8 twin (owned), once SDOT is enabled
    float *dense = nullptr;  // device copy of FP32 data
    std::vector<float> host; // small FP32 tensors also kept on the host (scalars read by the host)
    int rows = 0, cols = 0;
};

struct Model {
    needle2_engine_config c{};
    int abits = 0, device = 0, lookup = -1, sms = 148;
    bool sdot = false;
    std::vector<Tensor> t;
    float *rope_divisor = nullptr;   // [head_dim / 2]
    float *rope_cos = nullptr, *rope_sin = nullptr;   // [rope_len][head_dim / 2], position / divisor
    int rope_len = 0;
    cudaStream_t stream = nullptr;
    int count() const { return (int)t.size(); }
    int mh() const { return 1 + 14 * c.layers; }
    int site_base(int s) const { return mh() + 9 + 4 * s; }
    int final_norm() const { return mh() + 9 + 4 * c.num_sites; }
    int A() const { return c.heads * c.head_dim; }
    int K() const { return c.kvheads * c.head_dim; }
    int engring() const { return (c.taps - 1) * c.dilation + 1; }
    int hist_cap() const {
        int mo = 1;
        for (int i = 0; i < c.num_orders; ++i) mo = std::max(mo, c.orders[i]);
        return c.num_sites ? engring() + mo - 1 : 1;
    }
    ~Model() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        for (auto &x : t) {
            if (x.sdot) needle2_sdot_destroy(x.sdot);
            if (x.dense) cudaFree(x.dense);
        }
        if (rope_divisor) cudaFree(rope_divisor);
        if (rope_cos) cudaFree(rope_cos);
        if (rope_sin) cudaFree(rope_sin);
        if (stream) cudaStreamDestroy(stream);
    }
    // The handle a matmul of tensor i runs on: the int8 twin in SDOT mode.
    void *handle(int i) const { return sdot && t[i].sdot ? t[i].sdot : t[i].cq; }
};

// Scratch of one forward pass, grown to the largest row count seen.
struct Scratch {
    DevBuf<float> x, nx, raw, hpost, u, bx, z, q, k, v, gate, att, proj, e, ek, ev, rawv, zf, logits, hidden;
    DevBuf<uint16_t> zhl;   // z rotated and split into the QKVG GEMM's bf16 operands
    DevBuf<uint16_t> ahl;   // the attention output rotated and split for the out projection
    DevBuf<float> part;     // K-split partial outputs of the decode projections (q/k/v/gate, then out)
    DevBuf<int64_t> ids;
    DevBuf<uint8_t> valid;
    DevBuf<int> rsess, rpos, tokens, argmax;
};

// Stages of a forward pass timed by the profiler (needle2_batch_profile).
constexpr int kStages = 8;

struct State {
    Model *m = nullptr;
    int S = 1, prefix = 0;
    bool int8 = false;
    std::vector<KVPool *> kv;
    std::vector<int> pos;            // per sequence, host mirror of base
    DevBuf<int> base, iota, hist;    // base[S], iota[S] = 0..S-1, hist[S][hist_cap]
    DevBuf<float> engring;           // [S][sites][engring][D]
    // prefix snapshot (single sequence): history + engram rings at position == prefix
    DevBuf<int> hist_snap;
    DevBuf<float> eng_snap;
    bool snapshot = false;
    int snap_position = 0, snap_capacity = 0;
    Scratch s;
    // stage timers: an event at every stage boundary of each forward pass while enabled
    struct Prof {
        bool on = false;
        std::vector<cudaEvent_t> events;
        std::vector<int> tags;   // stage that starts at events[i] (-1: a pass ends)
        size_t used = 0;
        double ms[kStages] = {};
    } prof;
    // CUDA graph of one decode step (needle2_batch_decode_greedy_device)
    cudaStream_t capture = nullptr;
    cudaGraphExec_t step_graph = nullptr;
    bool graphs = true;
    int step_kernels = 0;   // kernel nodes of the last captured step
    ~State() {
        if (m) cudaSetDevice(m->device);
        if (step_graph || capture) cudaDeviceSynchronize();
        if (step_graph) cudaGraphExecDestroy(step_graph);
        if (capture) cudaStreamDestroy(capture);
        for (auto *p : kv) kv_pool_delete(p);
        for (auto e : prof.events) cudaEventDestroy(e);
    }
    int capacity() const { return m->c.window ? m->c.window + prefix : m->c.max_seq; }
    size_t engring_stride() const { return (size_t)std::max(1, m->c.num_sites) * m->engring() * m->c.dim; }
};

struct Engine {
    std::unique_ptr<Model> model;
    std::unique_ptr<State> state;
    DevBuf<float> zlast;   // the last step's final-normed hidden (project_candidates' input)
    bool zlast_valid = false, zlast_quantised = false;
};

struct Batch {
    Engine *engine = nullptr;
    std::unique_ptr<State> state;
};

// ------------------------------------------------------------- validation

void validate_config(const needle2_engine_config &c) {
    if (c.vocab <= 0 || c.dim <= 0 || c.heads <= 0 || c.kvheads <= 0 || c.layers <= 0 || c.head_dim <= 0 ||
        c.max_seq <= 0 || c.hada <= 0 || c.lanes <= 0 || c.window < 0)
        throw Failure("invalid engine geometry");
    if (c.heads % c.kvheads || c.heads / c.kvheads > 8)
        throw Failure("heads must be a multiple of kvheads with at most 8 query heads per KV head");
    if (c.head_dim % 2 || c.head_dim > eng::kMaxHeadDim) throw Failure("head_dim must be even and at most 128");
    if (c.dim > eng::kMaxDim || c.hada > eng::kMaxDim || c.hada < c.dim || (c.hada & (c.hada - 1)))
        throw Failure("hada must be a power of two >= dim, both at most 4096");
    if (c.lanes > eng::kMaxLanes) throw Failure("at most 8 mHC lanes");
    if (c.num_sites < 0 || c.num_sites > 4 || c.num_orders < 0 || c.num_orders > 4) throw Failure("invalid engram counts");
    if (c.taps < 1 || c.dilation < 1) throw Failure("invalid Engram ring size");
    if (c.num_sites) {
        if (c.num_orders < 1 || c.tables < 1 || c.tables % c.num_orders || c.slots < 1 || c.subdim < 1 ||
            (long long)c.tables * c.subdim != c.dim)
            throw Failure("inconsistent engram geometry");
        for (int i = 0; i < c.num_orders; ++i)
            if (c.orders[i] < 1) throw Failure("engram orders must be positive");
        for (int s = 0; s < c.num_sites; ++s)
            if (c.sites[s] < 0 || c.sites[s] >= c.layers) throw Failure("engram site outside the layers");
    }
    if (!(c.rope_theta > 0) || !std::isfinite(c.rope_theta)) throw Failure("rope_theta must be finite and positive");
}

// Expected (rows, cols) of tensor i and whether it is a matrix that may be CQ.
struct Shape {
    int rows, cols;
    bool matrix;
};
std::vector<Shape> canonical_shapes(const needle2_engine_config &c) {
    const int D = c.dim, N = c.lanes, L = c.layers, A = c.heads * c.head_dim, K = c.kvheads * c.head_dim;
    std::vector<Shape> s;
    s.push_back({c.vocab, D, true});
    for (int l = 0; l < L; ++l) {
        s.push_back({1, D, false});                  // norm_in
        s.push_back({A, D, true});                   // q_proj
        s.push_back({K, D, true});                   // k_proj
        s.push_back({K, D, true});                   // v_proj
        s.push_back({1, c.head_dim, false});         // q_norm
        s.push_back({1, c.head_dim, false});         // k_norm
        s.push_back({A, D, true});                   // gate_proj
        s.push_back({D, A, true});                   // out_proj
        s.push_back({1, D, false});                  // post_norm
        s.push_back({1, 1, false});                  // attn_gate
        s.push_back({1, D, false});                  // pre_hada
        for (int j = 0; j < 3; ++j) s.push_back({1, c.hada, false});   // d1, d2, d3
    }
    for (int j = 0; j < 3; ++j) s.push_back({1, L, false});             // mhc_a_*
    s.push_back({L, N, false});                                        // mhc_b_pre
    s.push_back({L, N, false});                                        // mhc_b_post
    s.push_back({L, N * N, false});                                    // mhc_b_res
    s.push_back({L * N, N * D, false});                                // mhc_phi_pre
    s.push_back({L * N, N * D, false});                                // mhc_phi_post
    s.push_back({L * N * N, N * D, false});                            // mhc_phi_res
    for (int i = 0; i < c.num_sites; ++i) {
        s.push_back({c.tables * c.slots, c.subdim, true});              // tables
        s.push_back({D, c.tables * c.subdim, true});                    // key_proj
        s.push_back({D, c.tables * c.subdim, true});                    // value_proj
        s.push_back({c.taps, D, false});                                // taps
    }
    s.push_back({1, D, false});                                        // final_norm
    return s;
}

Model *build_model(const needle2_engine_config &c, const needle2_tensor_desc *td, int count, int abits) {
    validate_config(c);
    if (abits != 0 && abits != 8 && (abits < 2 || abits > 16)) throw Failure("activation_bits must be 0 or 8");
    const auto shapes = canonical_shapes(c);
    if (count != (int)shapes.size())
        throw Failure("expected " + std::to_string(shapes.size()) + " tensors, got " + std::to_string(count));
    auto m = std::make_unique<Model>();
    m->c = c;
    m->abits = abits;
    cuda_check(cudaGetDevice(&m->device), "cudaGetDevice");
    cuda_check(cudaDeviceGetAttribute(&m->sms, cudaDevAttrMultiProcessorCount, m->device), "SM count");
    cuda_check(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking), "stream");
    m->t.resize(count);
    const int mh = 1 + 14 * c.layers;
    for (int i = 0; i < count; ++i) {
        const Shape &sh = shapes[i];
        Tensor &t = m->t[i];
        t.rows = sh.rows;
        t.cols = sh.cols;
        const long long elems = (long long)sh.rows * sh.cols;
        if (td[i].cq) {
            const bool mhc_phi = i >= mh + 6 && i <= mh + 8;
            if (!sh.matrix || mhc_phi)
                throw Failure("tensor " + std::to_string(i) + ": CQ is only supported for projection matrices here");
            if (handle_is_sdot(td[i].cq)) throw Failure("tensor " + std::to_string(i) + ": expected an FP32 CQ handle");
            const CQDevice *w = handle_matrix(td[i].cq);
            if (w->out != sh.rows || w->in != sh.cols)
                throw Failure("tensor " + std::to_string(i) + ": CQ shape " + std::to_string(w->out) + "x" +
                              std::to_string(w->in) + " does not match " + std::to_string(sh.rows) + "x" +
                              std::to_string(sh.cols));
            if (handle_device(td[i].cq) != m->device) throw Failure("CQ handle lives on another device");
            t.cq = td[i].cq;
        } else {
            if (!td[i].data) throw Failure("tensor " + std::to_string(i) + ": neither CQ handle nor data");
            if ((long long)td[i].rows * td[i].cols != elems)
                throw Failure("tensor " + std::to_string(i) + ": " + std::to_string(td[i].rows) + "x" +
                              std::to_string(td[i].cols) + " elements do not match the geometry");
            cuda_check(cudaMalloc(&t.dense, sizeof(float) * std::max<long long>(elems, 1)), "tensor allocation");
            cuda_check(cudaMemcpy(t.dense, td[i].data, sizeof(float) * elems, cudaMemcpyHostToDevice), "tensor upload");
            if (!sh.matrix && elems <= (1 << 16)) t.host.assign(td[i].data, td[i].data + elems);
        }
    }
    // RoPE divisors theta^(2j/HD), as the reference computes them in float (engine.cpp:401)
    std::vector<float> div(c.head_dim / 2);
    for (int j = 0; j < c.head_dim / 2; ++j) div[j] = std::pow(c.rope_theta, float(2 * j) / c.head_dim);
    cuda_check(cudaMalloc(&m->rope_divisor, sizeof(float) * std::max<size_t>(div.size(), 1)), "rope");
    cuda_check(cudaMemcpy(m->rope_divisor, div.data(), sizeof(float) * div.size(), cudaMemcpyHostToDevice), "rope");
    // cos / sin of every position below max_seq_len (the decode GEMM epilogue reads them)
    if (c.head_dim == 64 && c.max_seq > 0) {
        m->rope_len = c.max_seq;
        const size_t n = (size_t)m->rope_len * (c.head_dim / 2);
        cuda_check(cudaMalloc(&m->rope_cos, sizeof(float) * n), "rope table");
        cuda_check(cudaMalloc(&m->rope_sin, sizeof(float) * n), "rope table");
        check(launch_rope_table(m->rope_divisor, c.head_dim / 2, m->rope_len, m->rope_cos, m->rope_sin, m->stream),
              "rope table");
        cuda_check(cudaStreamSynchronize(m->stream), "rope table");
    }
    return m.release();
}

// ----------------------------------------------------------------- state

void rebuild_pools(State &st) {
    const auto &c = st.m->c;
    for (auto *p : st.kv) kv_pool_delete(p);
    st.kv.assign(c.layers, nullptr);
    for (int l = 0; l < c.layers; ++l) {
        st.kv[l] = kv_pool_new(st.S, c.heads, c.kvheads, c.head_dim, c.max_seq, c.window, st.prefix, !st.int8);
        check(st.kv[l] != nullptr, "KV cache allocation");
    }
}

State *new_state(Model *m, int sessions, int prefix, bool int8) {
    auto st = std::make_unique<State>();
    st->m = m;
    st->S = sessions;
    st->prefix = prefix;
    st->int8 = int8;
    st->pos.assign(sessions, 0);
    st->base.reserve(sessions);
    st->iota.reserve(sessions);
    st->hist.reserve((size_t)sessions * m->hist_cap());
    st->engring.reserve((size_t)sessions * st->engring_stride());
    std::vector<int> iota(sessions);
    for (int i = 0; i < sessions; ++i) iota[i] = i;
    cuda_check(cudaMemcpy(st->iota.ptr, iota.data(), sizeof(int) * sessions, cudaMemcpyHostToDevice), "state");
    cuda_check(cudaMemset(st->base.ptr, 0, sizeof(int) * sessions), "state");
    cuda_check(cudaMemset(st->hist.ptr, 0, sizeof(int) * st->hist.cap), "state");
    cuda_check(cudaMemset(st->engring.ptr, 0, sizeof(float) * st->engring.cap), "state");
    rebuild_pools(*st);
    return st.release();
}

// Engine::reset (engine.cpp:433-449): position 0, history cleared, the pinned
// prefix length set; the KV pools are laid out again when it changes.
void reset_state(State &st, int prefix, bool force_pools) {
    const Model &m = *st.m;
    cuda_check(cudaStreamSynchronize(m.stream), "sync");
    st.snapshot = false;
    if (prefix != st.prefix || force_pools) {
        st.prefix = prefix;
        rebuild_pools(st);
    }
    std::fill(st.pos.begin(), st.pos.end(), 0);
    cuda_check(cudaMemsetAsync(st.base.ptr, 0, sizeof(int) * st.S, m.stream), "reset");
    cuda_check(cudaMemsetAsync(st.hist.ptr, 0, sizeof(int) * st.hist.cap, m.stream), "reset");
    cuda_check(cudaMemsetAsync(st.engring.ptr, 0, sizeof(float) * st.engring.cap, m.stream), "reset");
}

// ----------------------------------------------------------------- matmuls

// y[R][rows] = tensor i (rows x cols) applied to x[R][cols].
void linear(const Model &m, int i, const float *x, int R, float *y, cudaStream_t st) {
    const Tensor &t = m.t[i];
    if (t.cq) {
        void *h = m.handle(i);
        const int rc = handle_is_sdot(h) ? needle2_sdot_linear_device(h, x, y, R, st)
                                         : needle2_cq_linear_device(h, x, y, R, st);
        check(rc == 0, "CQ linear");
        return;
    }
    eng::DenseSeg seg{t.dense, 0, t.rows, y, t.rows};
    check(eng::launch_dense_rows(&seg, 1, x, t.cols, R, t.cols, st), "dense linear");
}

// Q, K, V and gate from one input (the fused projections of engine.cpp:560-606).
void projections(const Model &m, int ti, const float *x, int R, float *q, float *k, float *v, float *g,
                 cudaStream_t st) {
    const int ids[4] = {ti + 1, ti + 2, ti + 3, ti + 6};
    float *outs[4] = {q, k, v, g};
    bool all_cq = true;
    for (int j = 0; j < 4; ++j) all_cq = all_cq && m.t[ids[j]].cq;
    if (all_cq) {
        void *hs[4];
        for (int j = 0; j < 4; ++j) hs[j] = m.handle(ids[j]);
        const bool i8 = handle_is_sdot(hs[0]);
        bool same = true;
        for (int j = 1; j < 4; ++j) same = same && handle_is_sdot(hs[j]) == i8;
        if (same) {
            check(needle2_cq_linear_many_device(hs, 4, x, outs, R, i8 ? 1 : 0, st) == 0, "QKVG projections");
            return;
        }
    }
    for (int j = 0; j < 4; ++j) linear(m, ids[j], x, R, outs[j], st);
}

// Rows ids[R] of tensor i (CQ::row dequantisation or FP32 copy) into y[R][cols].
void gather_rows(const Model &m, int i, const int64_t *ids, int R, float *y, cudaStream_t st) {
    const Tensor &t = m.t[i];
    if (t.cq) {
        check(launch_rows(*handle_matrix(t.cq), ids, R, y, st), "CQ rows");
        return;
    }
    check(eng::launch_gather_dense(t.dense, ids, R, t.cols, y, st), "dense rows");
}

void aq(const Model &m, float *x, int rows, int dim, cudaStream_t st) {
    if (m.abits) check(launch_activation_quant(x, rows, dim, m.abits, st), "activation quantiser");
}

// ----------------------------------------------------------------- forward

struct Outputs {
    bool all_logits = false;   // logits of every row, else of each entry's last token
    bool logits = false;
    float *logits_dev = nullptr;   // [rows][vocab] (caller's device buffer) or the scratch
    int *argmax_dev = nullptr;     // greedy token of each logits row
    bool hidden = false;           // per-layer lane means of the last row
    bool keep_z = false;           // final-normed last row kept for candidate projections
    int max_visible = 0;           // bound on the visible set (0: from the current positions)
};

// Records a profiler event where `stage` begins (-1: the pass ends).
void mark(State &st, int stage, cudaStream_t stream) {
    auto &p = st.prof;
    if (!p.on) return;
    if (p.used == p.events.size()) {
        cudaEvent_t e;
        cuda_check(cudaEventCreate(&e), "profiler event");
        p.events.push_back(e);
        p.tags.push_back(-1);
    }
    cuda_check(cudaEventRecord(p.events[p.used], stream), "profiler event");
    p.tags[p.used++] = stage;
}

// Folds the recorded events into per-stage totals (synchronises).
void collect(State &st) {
    auto &p = st.prof;
    if (!p.used) return;
    cuda_check(cudaEventSynchronize(p.events[p.used - 1]), "profiler");
    for (size_t i = 0; i + 1 < p.used; ++i) {
        if (p.tags[i] < 0) continue;
        float ms = 0.f;
        cuda_check(cudaEventElapsedTime(&ms, p.events[i], p.events[i + 1]), "profiler");
        p.ms[p.tags[i]] += ms;
    }
    p.used = 0;
}

// Engram keys/values of R = E*T rows (engine.cpp:755-783) into s.ek / s.ev
// ([site][R][D]), and the engram value rings updated with this call's raw
// values.  Row positions must be in s.rpos; tokens of the call are tokens[E][T].
void engram_stage(State &st, int E, int T, const int *tokens, cudaStream_t stream) {
    const Model &m = *st.m;
    const auto &c = m.c;
    const int R = E * T, D = c.dim;
    Scratch &s = st.s;
    if (c.num_sites) {
        s.ids.reserve((size_t)R * c.tables);
        s.valid.reserve((size_t)R * c.tables);
        s.e.reserve((size_t)R * D);
        s.ek.reserve((size_t)c.num_sites * R * D);
        s.ev.reserve((size_t)c.num_sites * R * D);
        s.rawv.reserve((size_t)R * D);
        eng::EngramHash h{};
        h.tables = c.tables; h.slots = c.slots; h.num_orders = c.num_orders;
        for (int i = 0; i < 4; ++i) h.orders[i] = c.orders[i];
        h.window = c.window; h.prefix = st.prefix; h.hist_cap = m.hist_cap();
        h.ring = st.hist.ptr; h.chunk = tokens; h.T = T; h.chunk_start = st.base.ptr;
        check(eng::launch_engram_ids(h, s.rsess.ptr, s.rpos.ptr, R, s.ids.ptr, s.valid.ptr, stream), "engram ids");
        const int er = m.engring();
        for (int site = 0; site < c.num_sites; ++site) {
            const int ti = m.site_base(site);
            gather_rows(m, ti, s.ids.ptr, R * c.tables, s.e.ptr, stream);
            check(eng::launch_engram_mask(s.e.ptr, s.valid.ptr, R, c.tables, c.subdim, stream), "engram mask");
            aq(m, s.e.ptr, R, D, stream);
            float *ek = s.ek.ptr + (size_t)site * R * D, *ev = s.ev.ptr + (size_t)site * R * D;
            if (m.t[ti + 1].cq && m.t[ti + 2].cq && handle_is_sdot(m.handle(ti + 1)) == handle_is_sdot(m.handle(ti + 2))) {
                void *hs[2] = {m.handle(ti + 1), m.handle(ti + 2)};
                float *ys[2] = {ek, s.rawv.ptr};
                check(needle2_cq_linear_many_device(hs, 2, s.e.ptr, ys, R, handle_is_sdot(hs[0]) ? 1 : 0, stream) == 0,
                      "engram projections");
            } else {
                linear(m, ti + 1, s.e.ptr, R, ek, stream);
                linear(m, ti + 2, s.e.ptr, R, s.rawv.ptr, stream);
            }
            float *ring = st.engring.ptr + (size_t)site * er * D;
            eng::EngramConv cv{};
            cv.D = D; cv.taps = c.taps; cv.dilation = c.dilation; cv.engring = er; cv.window = c.window;
            cv.prefix = st.prefix; cv.T = T; cv.taps_w = m.t[ti + 3].dense; cv.ring = ring;
            cv.ld_ring_s = st.engring_stride(); cv.chunk_raw = s.rawv.ptr; cv.ld_chunk = D; cv.chunk_start = st.base.ptr;
            check(eng::launch_engram_conv(cv, s.rsess.ptr, s.rpos.ptr, R, ev, D, stream), "engram conv");
            check(eng::launch_engram_ring_store(ring, st.engring_stride(), s.rawv.ptr, D, E, nullptr, st.base.ptr, T, er,
                                                D, stream),
                  "engram ring");
        }
    }
}

// T tokens (device tokens[E][T]) for sequences 0..E-1 from their current positions.
void forward(State &st, int E, int T, const int *tokens, const Outputs &o, float *zlast, cudaStream_t stream) {
    const Model &m = *st.m;
    const auto &c = m.c;
    const int R = E * T, D = c.dim, N = c.lanes, A = m.A(), K = m.K(), V = c.vocab;
    const int ldraw = 2 * N + N * N;
    Scratch &s = st.s;
    s.x.reserve((size_t)R * N * D);
    s.nx.reserve((size_t)R * N * D);
    s.raw.reserve((size_t)R * ldraw);
    s.hpost.reserve((size_t)R * N);
    s.u.reserve((size_t)R * D);
    s.bx.reserve((size_t)R * D);
    s.z.reserve((size_t)R * D);
    s.q.reserve((size_t)R * A);
    s.gate.reserve((size_t)R * A);
    s.att.reserve((size_t)R * A);
    s.k.reserve((size_t)R * K);
    s.v.reserve((size_t)R * K);
    s.proj.reserve((size_t)R * D);
    s.rsess.reserve(R);
    s.rpos.reserve(R);
    check(eng::launch_row_positions(st.base.ptr, E, T, s.rsess.ptr, s.rpos.ptr, stream), "positions");
    int max_visible = o.max_visible;
    if (max_visible <= 0) {
        std::vector<int> first(st.pos.begin(), st.pos.begin() + E);
        max_visible = kv_max_visible(st.prefix, c.window, first.data(), E, T);
    }

    // engrams (engine.cpp:755-783), all sites, before the history ring takes this call's tokens
    if (st.prof.on && st.prof.used > 4096) collect(st);
    mark(st, 0, stream);
    engram_stage(st, E, T, tokens, stream);
    check(eng::launch_history_store(st.hist.ptr, m.hist_cap(), tokens, T, nullptr, st.base.ptr, E, stream), "history");

    // embedding rows * sqrt(D) into every lane (engine.cpp:973-974)
    s.ids.reserve(R);
    s.e.reserve((size_t)R * D);
    check(eng::launch_widen_ids(tokens, s.ids.ptr, R, stream), "token ids");
    gather_rows(m, 0, s.ids.ptr, R, s.e.ptr, stream);
    check(eng::launch_embed_lanes(s.e.ptr, R, N, D, std::sqrt(float(D)), s.x.ptr, stream), "embedding");

    if (o.hidden) s.hidden.reserve((size_t)R * c.layers * D);
    const int mh = m.mh();
    // Layer boundaries run as one kernel (post-attention part of layer l, then
    // the routing of layer l + 1 or the final norm) where the geometry allows.
    const bool mix = eng::mhc_mix_supported(D, N, c.hada);
    const bool every = o.all_logits;
    const int rows = every ? R : E;
    const bool want_z = o.logits || o.keep_z;
    const bool mix_final = mix && want_z && (every || T == 1);
    auto route_layer = [&](int l) {
        eng::MhcLayer ml{};
        const int ti = 1 + 14 * l;
        ml.layer = l; ml.lanes = N; ml.D = D;
        ml.a_pre = m.t[mh].host[l]; ml.a_post = m.t[mh + 1].host[l]; ml.a_res = m.t[mh + 2].host[l];
        ml.b_pre = m.t[mh + 3].dense + (size_t)l * N;
        ml.b_post = m.t[mh + 4].dense + (size_t)l * N;
        ml.b_res = m.t[mh + 5].dense + (size_t)l * N * N;
        ml.norm_in = m.t[ti].dense;
        for (int site = 0; site < c.num_sites; ++site)
            if (c.sites[site] == l) {
                ml.ek = s.ek.ptr + (size_t)site * R * D;
                ml.ev = s.ev.ptr + (size_t)site * R * D;
                ml.ld_site = D;
            }
        return ml;
    };
    auto post_layer = [&](int l, int routed) {
        const int ti = 1 + 14 * l;
        eng::PostLayer pl{};
        pl.layer = l; pl.lanes = N; pl.D = D; pl.hada = c.hada; pl.a_res = m.t[mh + 2].host[l];
        pl.b_res = m.t[mh + 5].dense + (size_t)l * N * N;
        pl.hres_ready = routed;
        pl.post_norm = m.t[ti + 8].dense; pl.attn_gate = m.t[ti + 9].dense; pl.pre_hada = m.t[ti + 10].dense;
        pl.d1 = m.t[ti + 11].dense; pl.d2 = m.t[ti + 12].dense; pl.d3 = m.t[ti + 13].dense;
        return pl;
    };
    // the routed z of each layer is also written rotated and split into the
    // QKVG GEMM's bf16 operands when that GEMM takes them
    auto qkvg_handles = [&](int l, void **hs) {
        const int ti = 1 + 14 * l;
        const int ids[4] = {ti + 1, ti + 2, ti + 3, ti + 6};
        for (int j = 0; j < 4; ++j) {
            if (!m.t[ids[j]].cq) return false;
            hs[j] = m.handle(ids[j]);
        }
        return true;
    };
    auto zhl_for = [&](int l, eng::MixArgs &a) {
        void *hs[4];
        int G = 0;
        float sc = 0.f;
        a.zhl = nullptr;
        if (m.abits || !qkvg_handles(l, hs) || !handle_hilo_gemm(hs, 4, R, &G, &sc) || D % G) return false;
        s.zhl.reserve(2 * (size_t)R * D);
        a.zhl = s.zhl.ptr; a.lo_off = (long long)R * D; a.group = G; a.rot_scale = sc;
        return true;
    };
    auto mix_args = [&]() {
        eng::MixArgs a{};
        a.D = D; a.lanes = N; a.hada = c.hada;
        a.phi_pre = m.t[mh + 6].dense; a.phi_post = m.t[mh + 7].dense; a.phi_res = m.t[mh + 8].dense;
        a.proj = s.proj.ptr; a.raw = s.raw.ptr; a.ldraw = ldraw; a.hpost = s.hpost.ptr; a.u = s.u.ptr;
        a.bx = s.bx.ptr; a.x = s.x.ptr; a.z = s.z.ptr;
        return a;
    };
    // routed: layer l's routing already ran (in the previous layer's boundary kernel);
    // hres_norm: raw's residual part holds the Sinkhorn-normalised matrix (the
    // routing kernel's output) rather than the raw projections
    bool routed = false, hres_norm = false, zhl_ready = false, final_done = false;
    for (int l = 0; l < c.layers; ++l) {
        const int ti = 1 + 14 * l;
        if (!routed) {
            mark(st, 1, stream);
            const eng::MhcLayer ml = route_layer(l);
            bool done = false;
            if (mix) {
                eng::MixArgs a = mix_args();
                a.has_route = 1; a.route = ml;
                zhl_ready = zhl_for(l, a);
                done = eng::launch_mhc_mix(a, R, m.sms, stream);
                check(done || last_error()[0] == 0, "mHC routing");
                zhl_ready = zhl_ready && done;
                hres_norm = false;
            }
            if (!done) {
                zhl_ready = false;
                done = eng::launch_mhc_route(ml, m.t[mh + 6].dense, m.t[mh + 7].dense, m.t[mh + 8].dense, s.x.ptr, R,
                                             s.raw.ptr, ldraw, s.hpost.ptr, s.u.ptr, s.bx.ptr, s.z.ptr, m.sms, stream);
                check(done || last_error()[0] == 0, "mHC routing");
                hres_norm = done;
            }
            if (!done) {
                check(eng::launch_rms(s.x.ptr, N * D, R, N * D, nullptr, s.nx.ptr, N * D, stream), "lane rms");
                eng::DenseSeg segs[3] = {{m.t[mh + 6].dense, l * N, N, s.raw.ptr, ldraw},
                                         {m.t[mh + 7].dense, l * N, N, s.raw.ptr + N, ldraw},
                                         {m.t[mh + 8].dense, l * N * N, N * N, s.raw.ptr + 2 * N, ldraw}};
                check(eng::launch_dense_rows(segs, 3, s.nx.ptr, N * D, R, N * D, stream), "mHC projections");
                check(eng::launch_mhc_pre(ml, s.raw.ptr, ldraw, s.x.ptr, R, s.hpost.ptr, s.u.ptr, s.bx.ptr, s.z.ptr,
                                          stream),
                      "mHC routing");
            }
            routed = true;
        }
        aq(m, s.z.ptr, R, D, stream);
        mark(st, 2, stream);
        void *hs[4];
        bool roped = false;   // norm, RoPE and the KV store done by the projections' epilogue
        // decode whose attention kernel can take the projections as parts (then it
        // norms and ropes q and stores the token's K/V itself)
        const bool attn_qkv = T == 1 && kv_pool_fuses_qkv(st.kv[l], E, max_visible);
        eng::QkvgParts qkvg_src{};   // the projections' outputs as K parts (q null: in q, k, v, gate)
        if (zhl_ready && qkvg_handles(l, hs)) {
            float *outs[4] = {s.q.ptr, s.k.ptr, s.v.ptr, s.gate.ptr};
            QkvgEpilogue epi{};
            // where attention cannot take the projections as parts; measured: the fused epilogue pays
            // off from four 128-row tiles on (1024 rows: 0.07 ms a step saved against the separate
            // kernel); with fewer tiles its per-thread work outlasts the separate kernel
            if (T == 1 && m.rope_cos && R >= 512 && !attn_qkv) {
                epi.active = 1;
                epi.heads = c.heads; epi.kvheads = c.kvheads; epi.hd = c.head_dim;
                epi.q_norm = m.t[ti + 4].dense; epi.k_norm = m.t[ti + 5].dense;
                epi.cos_t = m.rope_cos; epi.sin_t = m.rope_sin; epi.table_len = m.rope_len;
                epi.divisor = m.rope_divisor; epi.pos = s.rpos.ptr;
                epi.kv = kv_pool_target(st.kv[l], st.iota.ptr, st.base.ptr);
            }
            // decode without the fused epilogue: the projections may split K into parts,
            // written side by side into s.part, which the RoPE/KV-store kernel adds
            const int qn = c.heads * c.head_dim, kn = c.kvheads * c.head_dim;
            int qparts = 0;
            KParts kp{};
            if (T == 1 && !epi.active && handle_matrix(hs[0])->out == qn && handle_matrix(hs[1])->out == kn &&
                handle_matrix(hs[2])->out == kn && handle_matrix(hs[3])->out == qn) {
                const long long span = (long long)R * 2 * (qn + kn);
                s.part.reserve((size_t)kMaxKParts * span);
                float *b = s.part.ptr;
                outs[0] = b; outs[1] = b + (size_t)R * qn; outs[2] = b + (size_t)R * (qn + kn);
                outs[3] = b + (size_t)R * (qn + 2 * kn);
                kp = KParts{kMaxKParts, span, &qparts};
                qkvg_src = eng::QkvgParts{outs[0], outs[1], outs[2], outs[3], s.gate.ptr, 1, span};
            }
            check(handle_many_hilo(hs, 4, s.zhl.ptr, outs, R, stream, epi.active ? &epi : nullptr, &roped,
                                   kp.max_parts ? &kp : nullptr),
                  "QKVG projections");
            qkvg_src.parts = qparts;
        } else {
            projections(m, ti, s.z.ptr, R, s.q.ptr, s.k.ptr, s.v.ptr, s.gate.ptr, stream);
        }
        mark(st, 3, stream);
        // decode with the projections as parts and a kernel that takes them:
        // attention itself norms and ropes q and stores the token's K/V
        QkvParts qkv{};
        const bool qkv_fused = !roped && attn_qkv && qkvg_src.q;
        if (qkv_fused)
            qkv = QkvParts{qkvg_src.q, qkvg_src.k, qkvg_src.v, qkvg_src.g, qkvg_src.parts, qkvg_src.pstride,
                           m.t[ti + 4].dense, m.t[ti + 5].dense, m.rope_cos, m.rope_sin, m.rope_divisor, m.rope_len};
        if (roped || qkv_fused) {
            // q/k normed and roped, the token's K/V stored (or attention does it): attention follows
        } else if (T == 1) {
            // decode: the new token's K/V stored as RoPE finishes, then attention alone
            check(eng::launch_qk_rope_store(s.q.ptr, s.k.ptr, s.v.ptr, R, c.heads, c.kvheads, c.head_dim,
                                            m.t[ti + 4].dense, m.t[ti + 5].dense, s.rpos.ptr, m.rope_divisor,
                                            kv_pool_target(st.kv[l], st.iota.ptr, st.base.ptr), stream, m.rope_cos,
                                            m.rope_sin, m.rope_len, qkvg_src.q ? &qkvg_src : nullptr),
                  "q/k norm, RoPE and KV store");
        } else {
            check(eng::launch_qk_norm_rope(s.q.ptr, s.k.ptr, R, c.heads, c.kvheads, c.head_dim, m.t[ti + 4].dense,
                                           m.t[ti + 5].dense, s.rpos.ptr, m.rope_divisor, stream),
                  "q/k norm and RoPE");
        }
        mark(st, 4, stream);
        // attention with the output gate applied as it is written (engine.cpp:1022-1023)
        // at decode the attention kernels also write their output rotated and split
        // into the out projection's GEMM operands, when that GEMM takes them
        AttnRot rot{};
        void *oh = nullptr;
        bool want_rot = false, rotated = false;
        if (T == 1 && !m.abits && m.t[ti + 7].cq) {
            oh = m.handle(ti + 7);
            int G = 0;
            float sc = 0.f;
            if (handle_hilo_gemm(&oh, 1, R, &G, &sc)) {
                s.ahl.reserve(2 * (size_t)R * A);
                rot = AttnRot{s.ahl.ptr, (long long)R * A, A, G, sc};
                want_rot = true;
            }
        }
        check(kv_pool_run(st.kv[l], T == 1 ? kQuery : kPrefill, st.iota.ptr, st.base.ptr, E, T, max_visible, s.q.ptr,
                          s.k.ptr, s.v.ptr, s.att.ptr, stream, s.gate.ptr, want_rot ? &rot : nullptr, &rotated,
                          qkv_fused ? &qkv : nullptr),
              "attention");
        mark(st, 5, stream);
        // the out projection's K parts, when the layer-boundary kernel adds them
        const float *proj_src = s.proj.ptr;
        int proj_parts = 1;
        if (rotated) {
            float *ys[1] = {s.proj.ptr};
            KParts kp{};
            if (mix && !hres_norm) {
                s.part.reserve((size_t)kMaxKParts * R * D);
                ys[0] = s.part.ptr;
                kp = KParts{kMaxKParts, (long long)R * D, &proj_parts};
            }
            check(handle_many_hilo(&oh, 1, s.ahl.ptr, ys, R, stream, nullptr, nullptr, kp.max_parts ? &kp : nullptr),
                  "out projection");
            proj_src = ys[0];
        } else {
            aq(m, s.att.ptr, R, A, stream);
            linear(m, ti + 7, s.att.ptr, R, s.proj.ptr, stream);
        }
        mark(st, 6, stream);
        float *hid = o.hidden ? s.hidden.ptr + (size_t)l * D : nullptr;
        const bool last = l + 1 == c.layers;
        bool fused = false;
        if (mix && !hres_norm) {
            eng::MixArgs a = mix_args();
            a.has_post = 1; a.post = post_layer(l, 0);   // the boundary kernel normalises the mixing matrix
            a.proj = proj_src; a.proj_parts = proj_parts; a.proj_pstride = (long long)R * D;
            a.hidden = hid; a.ldh = c.layers * D;
            if (!last) {
                a.has_route = 1; a.route = route_layer(l + 1);
                zhl_ready = zhl_for(l + 1, a);
            } else if (mix_final) {
                s.zf.reserve((size_t)R * D);
                a.final_norm = 1; a.fnorm = m.t[m.final_norm()].dense; a.zf = s.zf.ptr;
            }
            fused = eng::launch_mhc_mix(a, R, m.sms, stream);
            check(fused || last_error()[0] == 0, "mHC mixing");
            if (fused) final_done = last && a.final_norm;
            zhl_ready = zhl_ready && fused;
        }
        if (!fused) {
            zhl_ready = false;
            if (proj_src != s.proj.ptr)
                check(eng::launch_sum_parts(proj_src, proj_parts, (long long)R * D, (long long)R * D, s.proj.ptr, stream),
                      "out projection parts");
            check(eng::launch_mhc_post(post_layer(l, hres_norm ? 1 : 0), s.proj.ptr, s.raw.ptr, ldraw, s.hpost.ptr,
                                       s.u.ptr, s.bx.ptr, s.x.ptr, R, hid, c.layers * D, stream),
                  "mHC mixing");
        }
        routed = fused && !last;
        hres_norm = false;
    }

    // final norm (engine.cpp:1039-1041) on every row or each entry's last token
    mark(st, 7, stream);
    if (want_z) {
        s.zf.reserve((size_t)rows * D);
        if (final_done) {
            // made by the last layer's boundary kernel for every row (rows == R here)
        } else if (every || T == 1) {
            check(eng::launch_final_norm(s.x.ptr, rows, N, D, m.t[m.final_norm()].dense, s.zf.ptr, stream), "final norm");
        } else {
            for (int e = 0; e < E; ++e)
                check(eng::launch_final_norm(s.x.ptr + ((size_t)e * T + T - 1) * N * D, 1, N, D,
                                             m.t[m.final_norm()].dense, s.zf.ptr + (size_t)e * D, stream),
                      "final norm");
        }
        if (o.keep_z && zlast)
            cuda_check(cudaMemcpyAsync(zlast, s.zf.ptr + (size_t)(rows - 1) * D, sizeof(float) * D,
                                       cudaMemcpyDeviceToDevice, stream),
                       "z");
    }
    if (o.logits) {
        aq(m, s.zf.ptr, rows, D, stream);
        float *lg = o.logits_dev;
        if (!lg) {
            s.logits.reserve((size_t)rows * V);
            lg = s.logits.ptr;
        }
        linear(m, 0, s.zf.ptr, rows, lg, stream);
        if (o.argmax_dev) check(launch_argmax(lg, rows, V, V, o.argmax_dev, stream), "argmax");
    }
    check(eng::launch_advance(st.base.ptr, E, T, stream), "advance");
    mark(st, -1, stream);
    for (int e = 0; e < E; ++e) st.pos[e] += T;
}

// ------------------------------------------------------- engine operations

constexpr int kMaxChunkRows = 1 << 16;   // rows of one forward pass

void sync(const Model &m, cudaStream_t st) { cuda_check(cudaStreamSynchronize(st), "engine"); }

void upload_tokens(State &st, const int *host, int n, cudaStream_t stream) {
    st.s.tokens.reserve(n);
    cuda_check(cudaMemcpyAsync(st.s.tokens.ptr, host, sizeof(int) * n, cudaMemcpyHostToDevice, stream), "tokens");
}

void check_tokens(const Model &m, const int *tokens, long long n) {
    for (long long i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= m.c.vocab) throw Failure("token outside vocabulary");
}

void check_room(const State &st, int e, long long tokens) {
    if (!st.m->c.window && st.pos[e] + tokens > st.capacity()) throw Failure("maximum context reached");
}

// Engine::step (engine.cpp:968-1044) on the single sequence.
void engine_step(Engine &en, int token, float *logits, float *hidden, int *greedy = nullptr) {
    Model &m = *en.model;
    State &st = *en.state;
    if (token < 0 || token >= m.c.vocab) throw Failure("token outside vocabulary");
    check_room(st, 0, 1);
    cudaStream_t stream = m.stream;
    upload_tokens(st, &token, 1, stream);
    en.zlast.reserve(m.c.dim);
    Outputs o;
    o.logits = logits != nullptr || greedy != nullptr;
    o.hidden = hidden != nullptr;
    o.keep_z = true;
    if (greedy) {
        st.s.argmax.reserve(1);
        o.argmax_dev = st.s.argmax.ptr;
    }
    forward(st, 1, 1, st.s.tokens.ptr, o, en.zlast.ptr, stream);
    if (logits)
        cuda_check(cudaMemcpyAsync(logits, st.s.logits.ptr, sizeof(float) * m.c.vocab, cudaMemcpyDeviceToHost, stream),
                   "logits");
    if (hidden)
        cuda_check(cudaMemcpyAsync(hidden, st.s.hidden.ptr, sizeof(float) * m.c.layers * m.c.dim,
                                   cudaMemcpyDeviceToHost, stream),
                   "hidden");
    if (greedy) cuda_check(cudaMemcpyAsync(greedy, st.s.argmax.ptr, sizeof(int), cudaMemcpyDeviceToHost, stream), "token");
    sync(m, stream);
    en.zlast_valid = true;
    // step() quantises z in place before the LM head when it computes logits
    // (engine.cpp:1041); project_candidates quantises it once more
    en.zlast_quantised = o.logits;
}

// Engine::prefill (engine.cpp:1045-1301) on the single sequence.
void engine_prefill(Engine &en, const int *tokens, int n, bool last_only, float *logits, float *hidden) {
    Model &m = *en.model;
    State &st = *en.state;
    if (n <= 0) return;
    check_tokens(m, tokens, n);
    check_room(st, 0, n);
    cudaStream_t stream = m.stream;
    const int chunk = std::min(n, 512);
    for (int c0 = 0; c0 < n; c0 += chunk) {
        const int T = std::min(chunk, n - c0);
        const bool final_chunk = c0 + T == n;
        upload_tokens(st, tokens + c0, T, stream);
        Outputs o;
        o.logits = logits && (!last_only || final_chunk);
        o.all_logits = !last_only;
        o.hidden = hidden && final_chunk;
        forward(st, 1, T, st.s.tokens.ptr, o, nullptr, stream);
        if (o.logits) {
            const size_t rows = last_only ? 1 : (size_t)T;
            float *dst = last_only ? logits : logits + (size_t)c0 * m.c.vocab;
            cuda_check(cudaMemcpyAsync(dst, st.s.logits.ptr, sizeof(float) * rows * m.c.vocab, cudaMemcpyDeviceToHost,
                                       stream),
                       "logits");
        }
        if (o.hidden)
            cuda_check(cudaMemcpyAsync(hidden, st.s.hidden.ptr + (size_t)(T - 1) * m.c.layers * m.c.dim,
                                       sizeof(float) * m.c.layers * m.c.dim, cudaMemcpyDeviceToHost, stream),
                       "hidden");
        sync(m, stream);
    }
}

void validate_candidates(const Model &m, const int *cand, int n) {
    if (!cand || n <= 0) throw Failure("candidates must be nonempty");
    for (int i = 0; i < n; ++i)
        if (cand[i] < 0 || cand[i] >= m.c.vocab) throw Failure("candidate outside vocabulary");
}

// Engine::project_candidates (engine.cpp:1307-1349): the last step's final
// hidden state against the LM-head rows of the candidates.
void engine_project(Engine &en, const int *cand, int n, float *out) {
    Model &m = *en.model;
    State &st = *en.state;
    validate_candidates(m, cand, n);
    if (!out) return;
    if (!en.zlast_valid) throw Failure("no step has produced a hidden state to project");
    cudaStream_t stream = m.stream;
    const int D = m.c.dim;
    Scratch &s = st.s;
    s.zf.reserve(D);
    s.tokens.reserve(n);
    s.logits.reserve(n);
    cuda_check(cudaMemcpyAsync(s.zf.ptr, en.zlast.ptr, sizeof(float) * D, cudaMemcpyDeviceToDevice, stream), "z");
    for (int i = 0; i < (en.zlast_quantised ? 2 : 1); ++i) aq(m, s.zf.ptr, 1, D, stream);
    cuda_check(cudaMemcpyAsync(s.tokens.ptr, cand, sizeof(int) * n, cudaMemcpyHostToDevice, stream), "candidates");
    const Tensor &t = m.t[0];
    if (t.cq) {
        void *h = m.handle(0);
        const CQDevice &w = *handle_matrix(h);
        if (handle_is_sdot(h)) {
            const int8_t *q = nullptr;
            const float *xs = nullptr;
            check(handle_prepare(h, s.zf.ptr, 1, nullptr, &q, &xs, stream), "candidate input");
            check(eng::launch_candidates_i8(w.packed, w.norms, w.rowbytes, w.groups, w.group, w.bits, w.ctab,
                                            w.centroid_scale, q, xs, s.tokens.ptr, n, s.logits.ptr, stream),
                  "candidate projection");
        } else {
            const float *rot = nullptr;
            check(handle_prepare(h, s.zf.ptr, 1, &rot, nullptr, nullptr, stream), "candidate input");
            check(eng::launch_candidates_f32(w.packed, w.norms, w.rowbytes, w.groups, w.group, w.storage_bits, w.lut,
                                             rot, s.tokens.ptr, n, s.logits.ptr, stream),
                  "candidate projection");
        }
    } else {
        s.ids.reserve(n);
        s.e.reserve((size_t)n * D);
        check(eng::launch_widen_ids(s.tokens.ptr, s.ids.ptr, n, stream), "candidate ids");
        check(eng::launch_gather_dense(t.dense, s.ids.ptr, n, D, s.e.ptr, stream), "candidate rows");
        eng::DenseSeg seg{s.e.ptr, 0, n, s.logits.ptr, n};
        check(eng::launch_dense_rows(&seg, 1, s.zf.ptr, D, 1, D, stream), "candidate projection");
    }
    cuda_check(cudaMemcpyAsync(out, s.logits.ptr, sizeof(float) * n, cudaMemcpyDeviceToHost, stream), "candidates");
    sync(m, stream);
}

// Engine::decode_loop (engine.cpp:1360-1497): greedy decoding with optional
// DFA states, each step's greedy choice made on the GPU (only the chosen
// token crosses to the host).
int engine_decode_loop(Engine &en, int first, int max_new, const needle2_dfa_state_desc *dfa, int *out, int *count_out) {
    Model &m = *en.model;
    const auto &c = m.c;
    if (max_new <= 0) {
        if (count_out) *count_out = 0;
        return 0;
    }
    if (first < 0 || first >= c.vocab) throw Failure("token outside vocabulary");
    if (dfa) {
        if (dfa->num_states <= 0 || dfa->initial_state < 0 || dfa->initial_state >= dfa->num_states ||
            !dfa->state_types || !dfa->fallback_next_states || !dfa->candidate_offsets)
            throw Failure("invalid DFA states");
        for (int tok : {dfa->eos_id, dfa->stop_id, dfa->tool_start_id, dfa->tool_end_id})
            if (tok < 0 || tok >= c.vocab) throw Failure("DFA token outside vocabulary");
        if (dfa->candidate_offsets[0] != 0) throw Failure("invalid DFA offsets");
        for (int st = 0; st < dfa->num_states; ++st) {
            const int type = dfa->state_types[st], fb = dfa->fallback_next_states[st];
            const int b = dfa->candidate_offsets[st], e = dfa->candidate_offsets[st + 1];
            if ((type != 0 && type != 1 && type != 4) || fb < -1 || fb >= dfa->num_states || b < 0 || e < b)
                throw Failure("invalid DFA state");
            if (type == 1 && b == e) throw Failure("DFA state has no candidates");
            if (e > b) {
                if (!dfa->candidate_tokens || !dfa->next_states) throw Failure("missing DFA transitions");
                validate_candidates(m, dfa->candidate_tokens + b, e - b);
            }
            for (int i = b; i < e; ++i)
                if (dfa->next_states[i] < 0 || dfa->next_states[i] >= dfa->num_states)
                    throw Failure("invalid DFA transition");
        }
    }
    const int eos = dfa ? dfa->eos_id : 1, stop = dfa ? dfa->stop_id : 5;
    out[0] = first;
    int count = 1, cur = first;
    if (first == eos || first == stop) {
        if (count_out) *count_out = count;
        return 0;
    }
    int state = 0;
    if (dfa) {
        state = dfa->initial_state;
        bool matched = false;
        for (int i = dfa->candidate_offsets[state]; i < dfa->candidate_offsets[state + 1]; ++i)
            if (dfa->candidate_tokens[i] == first) {
                state = dfa->next_states[i];
                matched = true;
                break;
            }
        if (!matched) {
            if (dfa->state_types[state] != 0) throw Failure("first token rejected by DFA");
            if (dfa->fallback_next_states[state] >= 0) state = dfa->fallback_next_states[state];
        }
    }
    std::vector<float> cand_logits;
    while (count < max_new) {
        if (dfa && dfa->state_types[state] == 4) break;
        int next = -1;
        if (!dfa || dfa->state_types[state] == 0) {
            engine_step(en, cur, nullptr, nullptr, &next);
            if (dfa) {
                bool matched = false;
                for (int i = dfa->candidate_offsets[state]; i < dfa->candidate_offsets[state + 1]; ++i)
                    if (dfa->candidate_tokens[i] == next) {
                        state = dfa->next_states[i];
                        matched = true;
                        break;
                    }
                if (!matched && dfa->fallback_next_states[state] >= 0) state = dfa->fallback_next_states[state];
            }
        } else {
            const int b = dfa->candidate_offsets[state], n = dfa->candidate_offsets[state + 1] - b;
            if (n == 1) {
                next = dfa->candidate_tokens[b];
                engine_step(en, cur, nullptr, nullptr);
                state = dfa->next_states[b];
            } else {
                const int *cands = dfa->candidate_tokens + b;
                cand_logits.resize(n);
                engine_step(en, cur, nullptr, nullptr);
                engine_project(en, cands, n, cand_logits.data());
                int best = 0;
                float mv = cand_logits[0];
                for (int i = 1; i < n; ++i)
                    if (cand_logits[i] > mv) {
                        mv = cand_logits[i];
                        best = i;
                    }
                next = cands[best];
                state = dfa->next_states[b + best];
            }
        }
        out[count++] = next;
        cur = next;
        if (next == eos || next == stop || (dfa && dfa->state_types[state] == 4)) break;
    }
    if (count_out) *count_out = count;
    return 0;
}

// Engine::import_state (engine.cpp:784-815): a prompt's K/V computed elsewhere
// (the reference's PyTorch prefill), its token history, and the engram value
// ring recomputed for the last positions.
void engine_import(Engine &en, int pos, int prefix, const int *ids, const int *positions, int count, const float *k,
                   const float *v) {
    Model &m = *en.model;
    State &st = *en.state;
    const auto &c = m.c;
    if (pos < 0 || prefix < 0 || prefix > c.max_seq || count < 0) throw Failure("invalid import geometry");
    if (!c.window && pos > c.max_seq) throw Failure("maximum context reached");
    check_tokens(m, ids, pos);
    reset_state(st, prefix, false);
    cudaStream_t stream = m.stream;
    const int cap = m.hist_cap();
    std::vector<int> ring(cap, 0);
    for (int i = std::max(0, pos - cap); i < pos; ++i) ring[i % cap] = ids[i];
    cuda_check(cudaMemcpyAsync(st.hist.ptr, ring.data(), sizeof(int) * cap, cudaMemcpyHostToDevice, stream), "history");
    if (count > 0) {
        for (int t = 0; t < count; ++t)
            if (positions[t] < 0 || (!c.window && positions[t] >= c.max_seq)) throw Failure("import position outside the cache");
        const int K = m.K();
        Scratch &s = st.s;
        s.rsess.reserve(count);
        s.rpos.reserve(count);
        s.q.reserve((size_t)count * K);
        s.k.reserve((size_t)count * K);
        std::vector<int> zeros(count, 0);
        cuda_check(cudaMemcpyAsync(s.rsess.ptr, zeros.data(), sizeof(int) * count, cudaMemcpyHostToDevice, stream), "ids");
        cuda_check(cudaMemcpyAsync(s.rpos.ptr, positions, sizeof(int) * count, cudaMemcpyHostToDevice, stream), "positions");
        for (int l = 0; l < c.layers; ++l) {
            cuda_check(cudaMemcpyAsync(s.q.ptr, k + (size_t)l * count * K, sizeof(float) * count * K,
                                       cudaMemcpyHostToDevice, stream),
                       "keys");
            cuda_check(cudaMemcpyAsync(s.k.ptr, v + (size_t)l * count * K, sizeof(float) * count * K,
                                       cudaMemcpyHostToDevice, stream),
                       "values");
            check(kv_pool_run(st.kv[l], kStore, s.rsess.ptr, s.rpos.ptr, count, 1, 1, nullptr, s.q.ptr, s.k.ptr, nullptr,
                              stream),
                  "KV import");
            sync(m, stream);   // the next layer reuses the staging buffers
        }
    }
    // raw engram values of positions [max(0, pos - engring), pos)
    const int q0 = std::max(0, pos - m.engring());
    if (c.num_sites && pos > q0) {
        const int T = pos - q0;
        cuda_check(cudaMemcpyAsync(st.base.ptr, &q0, sizeof(int), cudaMemcpyHostToDevice, stream), "base");
        upload_tokens(st, ids + q0, T, stream);
        st.s.rsess.reserve(T);
        st.s.rpos.reserve(T);
        check(eng::launch_row_positions(st.base.ptr, 1, T, st.s.rsess.ptr, st.s.rpos.ptr, stream), "positions");
        engram_stage(st, 1, T, st.s.tokens.ptr, stream);
    }
    st.pos[0] = pos;
    cuda_check(cudaMemcpyAsync(st.base.ptr, &pos, sizeof(int), cudaMemcpyHostToDevice, stream), "base");
    sync(m, stream);
    en.zlast_valid = false;
}

void engine_cache_prefix(Engine &en) {
    State &st = *en.state;
    const Model &m = *en.model;
    if (st.pos[0] <= 0 || st.pos[0] != st.prefix) throw Failure("prefix snapshot requires position == prefix_len > 0");
    st.hist_snap.reserve(st.hist.cap);
    st.eng_snap.reserve(st.engring.cap);
    cuda_check(cudaMemcpyAsync(st.hist_snap.ptr, st.hist.ptr, sizeof(int) * st.hist.cap, cudaMemcpyDeviceToDevice,
                               m.stream),
               "snapshot");
    cuda_check(cudaMemcpyAsync(st.eng_snap.ptr, st.engring.ptr, sizeof(float) * st.engring.cap,
                               cudaMemcpyDeviceToDevice, m.stream),
               "snapshot");
    sync(m, m.stream);
    // the prefix's K/V live in the pinned prefix rows, which later positions never overwrite
    st.snapshot = true;
    st.snap_position = st.pos[0];
    st.snap_capacity = st.capacity();
}

int engine_reset_to_prefix(Engine &en) {
    State &st = *en.state;
    const Model &m = *en.model;
    if (!st.snapshot) throw Failure("no cached prefix; call cache_prefix() after consuming the complete prefix");
    if (st.prefix != st.snap_position || st.capacity() != st.snap_capacity)
        throw Failure("cached prefix geometry no longer matches the current state");
    cuda_check(cudaMemcpyAsync(st.hist.ptr, st.hist_snap.ptr, sizeof(int) * st.hist.cap, cudaMemcpyDeviceToDevice,
                               m.stream),
               "restore");
    cuda_check(cudaMemcpyAsync(st.engring.ptr, st.eng_snap.ptr, sizeof(float) * st.engring.cap,
                               cudaMemcpyDeviceToDevice, m.stream),
               "restore");
    st.pos[0] = st.snap_position;
    cuda_check(cudaMemcpyAsync(st.base.ptr, &st.pos[0], sizeof(int), cudaMemcpyHostToDevice, m.stream), "restore");
    sync(m, m.stream);
    en.zlast_valid = false;
    return st.pos[0];
}

size_t state_kv_bytes(const State &st) {
    size_t b = 0;
    for (auto *p : st.kv) b += kv_pool_bytes(p);
    return b;
}

// ----------------------------------------------------------- batch operations

// Copies sequence 0's history and engram rings to every sequence and sets all
// positions to sequence 0's.
__global__ void broadcast_state_kernel(int *hist, int hist_n, float *eng, size_t eng_n, int *base, int S) {
    pdl_enter();
    const int s = blockIdx.x + 1;
    if (s >= S) return;
    for (int i = threadIdx.x; i < hist_n; i += blockDim.x) hist[(size_t)s * hist_n + i] = hist[i];
    for (size_t i = threadIdx.x; i < eng_n; i += blockDim.x) eng[(size_t)s * eng_n + i] = eng[i];
    if (threadIdx.x == 0) base[s] = base[0];
}

void batch_set_prefix(Batch &b, const int *tokens) {
    State &st = *b.state;
    const Model &m = *st.m;
    const int P = st.prefix;
    if (P <= 0) throw Failure("the batch was created without a prefix");
    if (st.pos[0] != 0) throw Failure("the prefix must be set before any other call");
    check_tokens(m, tokens, P);
    cudaStream_t stream = m.stream;
    for (int c0 = 0; c0 < P; c0 += 512) {
        const int T = std::min(512, P - c0);
        upload_tokens(st, tokens + c0, T, stream);
        forward(st, 1, T, st.s.tokens.ptr, Outputs{}, nullptr, stream);
    }
    if (st.S > 1) {
        cuda_check(launch_pdl(broadcast_state_kernel, st.S - 1, 256, 0, stream, st.hist.ptr, m.hist_cap(), st.engring.ptr,
                                                             st.engring_stride(), st.base.ptr, st.S), "kernel launch");
        cuda_check(cudaGetLastError(), "prefix broadcast");
    }
    std::fill(st.pos.begin(), st.pos.end(), P);
    sync(m, stream);
}

void batch_prefill(Batch &b, const int *tokens, int n, float *logits, int *next) {
    State &st = *b.state;
    const Model &m = *st.m;
    const int S = st.S, V = m.c.vocab;
    if (n <= 0) throw Failure("prefill needs at least one token per session");
    check_tokens(m, tokens, (long long)S * n);
    for (int e = 0; e < S; ++e) check_room(st, e, n);
    cudaStream_t stream = m.stream;
    const int chunk = std::max(1, std::min(n, kMaxChunkRows / S));
    for (int c0 = 0; c0 < n; c0 += chunk) {
        const int T = std::min(chunk, n - c0);
        const bool final_chunk = c0 + T == n;
        st.s.tokens.reserve((size_t)S * T);
        cuda_check(cudaMemcpy2DAsync(st.s.tokens.ptr, sizeof(int) * T, tokens + c0, sizeof(int) * n, sizeof(int) * T, S,
                                     cudaMemcpyHostToDevice, stream),
                   "tokens");
        Outputs o;
        o.logits = final_chunk && (logits || next);
        if (o.logits && next) {
            st.s.argmax.reserve(S);
            o.argmax_dev = st.s.argmax.ptr;
        }
        forward(st, S, T, st.s.tokens.ptr, o, nullptr, stream);
        if (o.logits && logits)
            cuda_check(cudaMemcpyAsync(logits, st.s.logits.ptr, sizeof(float) * S * V, cudaMemcpyDeviceToHost, stream),
                       "logits");
        if (o.logits && next)
            cuda_check(cudaMemcpyAsync(next, st.s.argmax.ptr, sizeof(int) * S, cudaMemcpyDeviceToHost, stream), "tokens");
    }
    sync(m, stream);
}

void batch_step(Batch &b, const int *tokens, float *logits, int *next) {
    State &st = *b.state;
    const Model &m = *st.m;
    const int S = st.S, V = m.c.vocab;
    check_tokens(m, tokens, S);
    for (int e = 0; e < S; ++e) check_room(st, e, 1);
    cudaStream_t stream = m.stream;
    upload_tokens(st, tokens, S, stream);
    Outputs o;
    o.logits = logits || next;
    if (next) {
        st.s.argmax.reserve(S);
        o.argmax_dev = st.s.argmax.ptr;
    }
    forward(st, S, 1, st.s.tokens.ptr, o, nullptr, stream);
    if (logits)
        cuda_check(cudaMemcpyAsync(logits, st.s.logits.ptr, sizeof(float) * S * V, cudaMemcpyDeviceToHost, stream),
                   "logits");
    if (next) cuda_check(cudaMemcpyAsync(next, st.s.argmax.ptr, sizeof(int) * S, cudaMemcpyDeviceToHost, stream), "tokens");
    sync(m, stream);
}

// out[s][counter] = nxt[s]; cur[s] = nxt[s] (the step's greedy tokens become the next inputs).
__global__ void commit_tokens_kernel(const int *__restrict__ nxt, int *__restrict__ cur, int S,
                                     int *__restrict__ out, int steps, const int *__restrict__ counter) {
    pdl_enter();
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    const int c = *counter;
    if (s < S) {
        out[(size_t)s * steps + c] = nxt[s];
        cur[s] = nxt[s];
    }
}

// One greedy decode step of every sequence: forward on cur, greedy tokens
// committed to out's column *counter and to cur.
void decode_step(State &st, int *cur, int *nxt, int *out, int steps, int *counter, int max_visible,
                 cudaStream_t stream) {
    Outputs o;
    o.logits = true;
    o.argmax_dev = nxt;
    o.max_visible = max_visible;
    forward(st, st.S, 1, cur, o, nullptr, stream);
    cuda_check(launch_pdl(commit_tokens_kernel, (st.S + 255) / 256, 256, 0, stream, nxt, cur, st.S, out, steps, counter), "kernel launch");
    cuda_check(cudaGetLastError(), "tokens");
    check(eng::launch_advance(counter, 1, 1, stream), "step counter");
}

// `steps` greedy steps on device buffers: first[S] in, out[S][steps] the
// generated tokens, enqueued on `stream`.  The first step runs launch by
// launch (it also sizes every buffer); the others replay a CUDA graph of one
// step captured on a private stream, with the attention split chosen for the
// longest context of the run (each kernel reads the true positions from the
// device, so only the work division is fixed).
void batch_decode_device(Batch &b, const int *first, int steps, int *out, cudaStream_t stream) {
    State &st = *b.state;
    const Model &m = *st.m;
    const int S = st.S;
    if (steps <= 0) return;
    for (int e = 0; e < S; ++e) check_room(st, e, steps);
    if (st.step_graph) {
        cuda_check(cudaDeviceSynchronize(), "graph");
        cudaGraphExecDestroy(st.step_graph);
        st.step_graph = nullptr;
    }
    st.s.argmax.reserve(2 * (size_t)S + 1);
    int *cur = st.s.argmax.ptr, *nxt = st.s.argmax.ptr + S, *counter = st.s.argmax.ptr + 2 * S;
    cuda_check(cudaMemcpyAsync(cur, first, sizeof(int) * S, cudaMemcpyDeviceToDevice, stream), "tokens");
    cuda_check(cudaMemsetAsync(counter, 0, sizeof(int), stream), "step counter");
    int max_visible = 1;
    {
        std::vector<int> last(st.pos.begin(), st.pos.end());
        for (int &p : last) p += steps - 1;
        max_visible = kv_max_visible(st.prefix, m.c.window, last.data(), S, 1);
    }
    const std::vector<int> start = st.pos;
    decode_step(st, cur, nxt, out, steps, counter, max_visible, stream);
    int done = 1;
    if (steps > 2 && st.graphs && !st.prof.on) {
        if (!st.capture) cuda_check(cudaStreamCreateWithFlags(&st.capture, cudaStreamNonBlocking), "capture stream");
        cudaEvent_t ready;
        cuda_check(cudaEventCreateWithFlags(&ready, cudaEventDisableTiming), "event");
        cuda_check(cudaEventRecord(ready, stream), "event");
        cuda_check(cudaStreamWaitEvent(st.capture, ready, 0), "event");
        cudaEventDestroy(ready);
        cudaGraph_t graph = nullptr;
        bool captured = false;
        if (cudaStreamBeginCapture(st.capture, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            try {
                decode_step(st, cur, nxt, out, steps, counter, max_visible, st.capture);
            } catch (const std::exception &) {
            }
            captured = cudaStreamEndCapture(st.capture, &graph) == cudaSuccess && graph &&
                       cudaGraphInstantiate(&st.step_graph, graph, 0) == cudaSuccess;
            if (captured) {
                // kernels of one step (the launch count a step replays)
                size_t n = 0;
                cudaGraphGetNodes(graph, nullptr, &n);
                std::vector<cudaGraphNode_t> nodes(n);
                cudaGraphGetNodes(graph, nodes.data(), &n);
                st.step_kernels = 0;
                for (auto nd : nodes) {
                    cudaGraphNodeType t;
                    if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++st.step_kernels;
                }
            }
            if (graph) cudaGraphDestroy(graph);
        }
        cudaGetLastError();   // a refused capture leaves its error behind; the steps then run eagerly
        st.pos = start;
        for (int &p : st.pos) p += 1;
        if (captured) {
            for (; done < steps; ++done) cuda_check(cudaGraphLaunch(st.step_graph, stream), "graph launch");
            for (int &p : st.pos) p += steps - 1;
        } else if (st.step_graph) {
            cudaGraphExecDestroy(st.step_graph);
            st.step_graph = nullptr;
        }
    }
    for (; done < steps; ++done) decode_step(st, cur, nxt, out, steps, counter, max_visible, stream);
}

template <typename F>
int guarded(F &&f) {
    try {
        g_engine_error.clear();
        clear_error();
        f();
        return 0;
    } catch (const std::exception &e) {
        g_engine_error = e.what();
        set_error(e.what());
        return -1;
    }
}

Engine *as_engine(void *p) {
    if (!p) throw Failure("null engine");
    return static_cast<Engine *>(p);
}
Batch *as_batch(void *p) {
    if (!p) throw Failure("null batch");
    return static_cast<Batch *>(p);
}

}  // namespace
}  // namespace nb200

using nb200::Batch;
using nb200::Engine;

extern "C" {

void *needle2_engine_create(const needle2_engine_config *config, const needle2_tensor_desc *tensors, int count,
                            int threads, int activation_bits) {
    (void)threads;
    Engine *out = nullptr;
    const int rc = nb200::guarded([&] {
        if (!config || (!tensors && count)) throw nb200::Failure("null config or tensors");
        auto en = std::make_unique<Engine>();
        en->model.reset(nb200::build_model(*config, tensors, count, activation_bits));
        en->state.reset(nb200::new_state(en->model.get(), 1, 0, false));
        out = en.release();
    });
    return rc ? nullptr : out;
}

void needle2_engine_destroy(void *p) { delete static_cast<Engine *>(p); }

void needle2_engine_set_lookup(void *p, int mode) {
    nb200::guarded([&] { nb200::as_engine(p)->model->lookup = mode; });
}

int needle2_engine_set_sdot(void *p) {
    return nb200::guarded([&] {
        Engine *en = nb200::as_engine(p);
        nb200::Model &m = *en->model;
        nb200::cuda_check(cudaSetDevice(m.device), "cudaSetDevice");
        for (auto &t : m.t) {
            if (!t.cq || t.sdot) continue;
            const nb200::CQDevice &w = *nb200::handle_matrix(t.cq);
            if ((w.bits == 2 || w.bits == 4) && w.group >= 64) {
                t.sdot = nb200::handle_make_sdot(t.cq);
                nb200::check(t.sdot != nullptr, "int8 matrix");
            }
        }
        m.sdot = true;
    });
}

void needle2_engine_reset(void *p, int prefix) {
    nb200::guarded([&] {
        Engine *en = nb200::as_engine(p);
        if (prefix < 0 || prefix > en->model->c.max_seq) throw nb200::Failure("prefix_len must lie between 0 and max_seq");
        nb200::reset_state(*en->state, prefix, false);
        en->zlast_valid = false;
    });
}

int needle2_engine_cache_prefix(void *p) {
    return nb200::guarded([&] { nb200::engine_cache_prefix(*nb200::as_engine(p)); });
}

int needle2_engine_reset_to_prefix(void *p) {
    int pos = -1;
    const int rc = nb200::guarded([&] { pos = nb200::engine_reset_to_prefix(*nb200::as_engine(p)); });
    return rc ? -1 : pos;
}

int needle2_engine_step(void *p, int token, float *logits, float *hidden) {
    return nb200::guarded([&] { nb200::engine_step(*nb200::as_engine(p), token, logits, hidden); });
}

int needle2_engine_prefill(void *p, const int *tokens, int num_tokens, int last_only, float *logits, float *hidden) {
    return nb200::guarded(
        [&] { nb200::engine_prefill(*nb200::as_engine(p), tokens, num_tokens, last_only != 0, logits, hidden); });
}

int needle2_engine_step_candidates(void *p, int token, const int *candidates, int num_candidates,
                                   float *candidate_logits, float *hidden) {
    return nb200::guarded([&] {
        Engine &en = *nb200::as_engine(p);
        nb200::validate_candidates(*en.model, candidates, num_candidates);
        nb200::engine_step(en, token, nullptr, hidden);
        if (candidate_logits) nb200::engine_project(en, candidates, num_candidates, candidate_logits);
    });
}

int needle2_engine_project_candidates(void *p, const int *candidates, int num_candidates, float *candidate_logits) {
    return nb200::guarded(
        [&] { nb200::engine_project(*nb200::as_engine(p), candidates, num_candidates, candidate_logits); });
}

int needle2_engine_decode_loop(void *p, int first_token, int max_new_tokens, const needle2_dfa_state_desc *dfa,
                               int *output_tokens, int *out_generated_count) {
    return nb200::guarded([&] {
        nb200::engine_decode_loop(*nb200::as_engine(p), first_token, max_new_tokens, dfa, output_tokens,
                                  out_generated_count);
    });
}

int needle2_engine_import(void *p, int position, int prefix_len, const int *ids, const int *positions, int count,
                          const float *k, const float *v) {
    return nb200::guarded(
        [&] { nb200::engine_import(*nb200::as_engine(p), position, prefix_len, ids, positions, count, k, v); });
}

int needle2_engine_set_int8_kv(void *p, int enable) {
    return nb200::guarded([&] {
        Engine *en = nb200::as_engine(p);
        en->state->int8 = enable != 0;
        nb200::reset_state(*en->state, en->state->prefix, true);
        en->zlast_valid = false;
    });
}

size_t needle2_engine_kv_storage_bytes(void *p) {
    return p ? nb200::state_kv_bytes(*static_cast<Engine *>(p)->state) : 0;
}

const char *needle2_engine_error(void) { return nb200::g_engine_error.c_str(); }

int needle2_engine_vocab(void *p) { return p ? static_cast<Engine *>(p)->model->c.vocab : -1; }

void *needle2_batch_create(void *engine, int sessions, int prefix_len) {
    Batch *out = nullptr;
    const int rc = nb200::guarded([&] {
        Engine *en = nb200::as_engine(engine);
        if (sessions < 1) throw nb200::Failure("sessions must be positive");
        if (prefix_len < 0 || prefix_len > en->model->c.max_seq)
            throw nb200::Failure("prefix_len must lie between 0 and max_seq");
        nb200::cuda_check(cudaSetDevice(en->model->device), "cudaSetDevice");
        auto b = std::make_unique<Batch>();
        b->engine = en;
        b->state.reset(nb200::new_state(en->model.get(), sessions, prefix_len, en->state->int8));
        out = b.release();
    });
    return rc ? nullptr : out;
}

void needle2_batch_destroy(void *b) { delete static_cast<Batch *>(b); }

size_t needle2_batch_kv_storage_bytes(void *b) {
    return b ? nb200::state_kv_bytes(*static_cast<Batch *>(b)->state) : 0;
}

int needle2_batch_set_prefix(void *b, const int *tokens) {
    return nb200::guarded([&] { nb200::batch_set_prefix(*nb200::as_batch(b), tokens); });
}

int needle2_batch_prefill(void *b, const int *tokens, int n, float *logits, int *next) {
    return nb200::guarded([&] { nb200::batch_prefill(*nb200::as_batch(b), tokens, n, logits, next); });
}

int needle2_batch_step(void *b, const int *tokens, float *logits, int *next) {
    return nb200::guarded([&] { nb200::batch_step(*nb200::as_batch(b), tokens, logits, next); });
}

int needle2_batch_decode_greedy(void *b, const int *first, int steps, int *out) {
    return nb200::guarded([&] {
        Batch &bt = *nb200::as_batch(b);
        nb200::State &st = *bt.state;
        const nb200::Model &m = *st.m;
        const int S = st.S;
        nb200::check_tokens(m, first, S);
        if (steps <= 0) return;
        nb200::DevBuf<int> f, o;
        f.reserve(S);
        o.reserve((size_t)S * steps);
        nb200::cuda_check(cudaMemcpyAsync(f.ptr, first, sizeof(int) * S, cudaMemcpyHostToDevice, m.stream), "tokens");
        nb200::batch_decode_device(bt, f.ptr, steps, o.ptr, m.stream);
        nb200::cuda_check(cudaMemcpyAsync(out, o.ptr, sizeof(int) * S * steps, cudaMemcpyDeviceToHost, m.stream),
                          "tokens");
        nb200::sync(m, m.stream);
    });
}

int needle2_batch_decode_greedy_device(void *b, const int *first, int steps, int *out, void *stream) {
    return nb200::guarded([&] {
        nb200::batch_decode_device(*nb200::as_batch(b), first, steps, out, static_cast<cudaStream_t>(stream));
    });
}

int needle2_batch_profile(void *b, int enable) {
    return nb200::guarded([&] {
        nb200::State &st = *nb200::as_batch(b)->state;
        nb200::collect(st);
        st.prof.on = enable != 0;
        for (double &v : st.prof.ms) v = 0.0;
    });
}

int needle2_batch_profile_read(void *b, double *ms, int n) {
    return nb200::guarded([&] {
        nb200::State &st = *nb200::as_batch(b)->state;
        nb200::collect(st);
        for (int i = 0; i < n && i < nb200::kStages; ++i) ms[i] = st.prof.ms[i];
        for (double &v : st.prof.ms) v = 0.0;
    });
}

int needle2_batch_step_kernels(void *b) {
    int n = -1;
    nb200::guarded([&] { n = nb200::as_batch(b)->state->step_kernels; });
    return n;
}

int needle2_batch_set_graphs(void *b, int enable) {
    return nb200::guarded([&] { nb200::as_batch(b)->state->graphs = enable != 0; });
}

int needle2_batch_positions(void *b, int *positions) {
    return nb200::guarded([&] {
        const nb200::State &st = *nb200::as_batch(b)->state;
        std::copy(st.pos.begin(), st.pos.end(), positions);
    });
}

}  // extern "C"
