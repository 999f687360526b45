// REFERENCE SHIM — test infrastructure only.
//
// Compiles OpenNeedle's own CPU sources unchanged, where they lie (the Makefile
// passes their directory with -I), and exports the internals that its public
// C ABI does not: the SDOT activation quantiser and per-group int32 dots
// (SdotCQ is refused by the public ABI on x86, needle2/csrc/sdot.cpp:351-354,
// although its portable branches compute the same integers), the INT8 KV
// import/quantise rule and single-layer attention of Engine.  The library also
// carries the reference's public needle2_* C ABI, because cq.cpp defines it.
//
// Used only by tests/ (to pin the oracle restatement) and by bench.py's
// reference arm (to time the reference's CPU path).  Output: oracle/_ref/.
#include "cq.cpp"

extern "C" {

// SdotCQ::prepare (needle2/csrc/sdot.cpp:47-103). q_out receives the
// reference's permuted bit-plane order, rows x padded; scales rows x groups.
void ref_sdot_prepare(const uint8_t *p, const uint16_t *n, int out, int in, int bits, int group,
                      const float *cb, const float *x, int rows, int8_t *q_out, float *scales_out) {
    SdotCQ s(p, n, out, in, bits, group, cb);
    Prepared prep;
    for (int m = 0; m < rows; ++m) {
        s.prepare(x + size_t(m) * in, prep);
        std::copy(prep.q.begin(), prep.q.end(), q_out + size_t(m) * s.padded);
        std::copy(prep.scales.begin(), prep.scales.end(), scales_out + size_t(m) * s.groups);
    }
}

// SdotCQ centroid table and scale (needle2/csrc/sdot.cpp:35-45).
void ref_sdot_centroids(const uint8_t *p, const uint16_t *n, int out, int in, int bits, int group,
                        const float *cb, int8_t *centroids16, float *centroid_scale, float *norm_scales) {
    SdotCQ s(p, n, out, in, bits, group, cb);
    std::copy(s.centroids, s.centroids + 16, centroids16);
    *centroid_scale = s.centroid_scale;
    std::copy(s.norm_scales.begin(), s.norm_scales.end(), norm_scales);
}

// SdotCQ::dot_group for every (row of x, output row, group):
// partials[m][r][g] (needle2/csrc/sdot.cpp:108-137).
void ref_sdot_partials(const uint8_t *p, const uint16_t *n, int out, int in, int bits, int group,
                       const float *cb, const float *x, int rows, int32_t *partials) {
    SdotCQ s(p, n, out, in, bits, group, cb);
    Prepared prep;
    for (int m = 0; m < rows; ++m) {
        s.prepare(x + size_t(m) * in, prep);
        for (int r = 0; r < out; ++r)
            for (int g = 0; g < s.groups; ++g)
                partials[(size_t(m) * out + r) * s.groups + g] =
                    s.dot_group(p + size_t(r) * s.rowbytes + size_t(g) * group * bits / 8, prep.q.data() + size_t(g) * group);
    }
}

// SdotCQ::linear per row of x with OpenMP row threads (needle2/csrc/sdot.cpp:338-346,356-359).
void ref_sdot_linear(const uint8_t *p, const uint16_t *n, int out, int in, int bits, int group,
                     const float *cb, const float *x, float *y, int rows, int threads) {
    SdotCQ s(p, n, out, in, bits, group, cb);
    Prepared prep;
    for (int m = 0; m < rows; ++m) {
        s.prepare(x + size_t(m) * in, prep);
        s.multiply(prep, y + size_t(m) * out, threads);
    }
}

// Persistent SdotCQ for timing the reference's int8 path (prepare + multiply
// per activation row, needle2/csrc/sdot.cpp:346,356-359).
void *ref_sdot_new(const uint8_t *p, const uint16_t *n, int out, int in, int bits, int group, const float *cb) {
    return new SdotCQ(p, n, out, in, bits, group, cb);
}
void ref_sdot_run(void *h, const float *x, float *y, int rows, int threads) {
    auto *s = static_cast<SdotCQ *>(h);
    Prepared prep;
    for (int m = 0; m < rows; ++m) {
        s->prepare(x + size_t(m) * s->columns, prep);
        s->multiply(prep, y + size_t(m) * s->rows, threads);
    }
}
void ref_sdot_free(void *h) { delete static_cast<SdotCQ *>(h); }

// A single-layer Engine with INT8 KV and no weights: enough for the KV import
// rule and compute_attention.
static Engine *attention_engine(int heads, int kvheads, int head_dim, int max_seq, int window, int prefix) {
    EngineConfig c{};
    c.vocab = 1; c.dim = heads * head_dim; c.heads = heads; c.kvheads = kvheads; c.layers = 1;
    c.head_dim = head_dim; c.max_seq = max_seq; c.hada = 1; c.lanes = 1; c.window = window;
    c.taps = 1; c.dilation = 1; c.rope_theta = 10000.0f;
    auto *e = new Engine(c, nullptr, 0, 1, 0);
    e->int8_kv_enabled = true;
    e->reset(prefix);
    return e;
}

// Engine::import_state's INT8 quantise-store (needle2/csrc/engine.cpp:784-815):
// k, v are [count][kvheads*head_dim] for `positions`; outputs are the cache
// arrays [capacity][...] (capacity = window ? window + prefix : max_seq).
int ref_kv_import(int heads, int kvheads, int head_dim, int max_seq, int window, int prefix,
                  const int *positions, int count, const float *k, const float *v, int8_t *keys_i8,
                  int8_t *values_i8, float *k_scales, float *v_scales) {
    Engine *e = attention_engine(heads, kvheads, head_dim, max_seq, window, prefix);
    std::vector<int> ids(size_t(positions[count - 1] + 1), 0);
    e->import_state(positions[count - 1] + 1, prefix, ids.data(), positions, count, k, v);
    int cap = e->capacity;
    std::copy(e->keys_i8.begin(), e->keys_i8.end(), keys_i8);
    std::copy(e->values_i8.begin(), e->values_i8.end(), values_i8);
    std::copy(e->k_scales.begin(), e->k_scales.end(), k_scales);
    std::copy(e->v_scales.begin(), e->v_scales.end(), v_scales);
    delete e;
    return cap;
}

// Engine::compute_attention for one query position over a given INT8 cache
// (needle2/csrc/engine.cpp:898-967).  Cache arrays as returned by ref_kv_import.
void ref_attention_i8(int heads, int kvheads, int head_dim, int max_seq, int window, int prefix,
                      const int8_t *keys_i8, const int8_t *values_i8, const float *k_scales,
                      const float *v_scales, int pos_cur, const float *q, float *out) {
    Engine *e = attention_engine(heads, kvheads, head_dim, max_seq, window, prefix);
    std::copy(keys_i8, keys_i8 + e->keys_i8.size(), e->keys_i8.begin());
    std::copy(values_i8, values_i8 + e->values_i8.size(), e->values_i8.begin());
    std::copy(k_scales, k_scales + e->k_scales.size(), e->k_scales.begin());
    std::copy(v_scales, v_scales + e->v_scales.size(), e->v_scales.begin());
    e->compute_attention(0, pos_cur, q, out);
    delete e;
}

}  // extern "C"

extern "C" {

// Engine::configure_sdot (needle2/csrc/engine.cpp:424-432) without its ARM64
// DotProd gate: the portable SdotCQ branches compute the same integers on
// x86, so the reference engine's SDOT arithmetic can serve as the oracle here.
int ref_engine_force_sdot(void *p) {
    auto *e = static_cast<Engine *>(p);
    for (size_t i = 0; i < e->t.size(); ++i)
        if (e->t[i].cq) {
            auto *q = static_cast<CQ *>(e->t[i].cq);
            if ((q->bits == 2 || q->bits == 4) && q->group >= 64 && q->group <= 131072)
                e->sdot[i] = std::make_unique<SdotCQ>(q->packed, q->norms, q->out, q->in, q->bits, q->group,
                                                      q->cb.data());
        }
    e->sdot_enabled = true;
    return 0;
}

}  // extern "C"
