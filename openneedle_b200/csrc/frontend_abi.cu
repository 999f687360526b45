// The frontend symbols of the reference's native library (needle2/csrc/
// frontend.h:15-35), so that needle2/frontend.py binds this library unchanged.
//
// The tokenizer and the tool-schema grammar compiler are host text processing,
// outside the GPU hot path: their entry points forward to the reference's own
// native library, loaded from NEEDLE2_FRONTEND_LIBRARY (a library built from
// the reference's sources).  needle2_engine_decode_compiled
// (frontend.cpp:1057-1079) is this library's own: the greedy first token of the
// prefill logits (first maximum wins, NaN refused), then this library's
// needle2_engine_decode_loop with the grammar's token automaton, which the
// reference library hands out through needle2_grammar_dfa.
#include <dlfcn.h>
#include <stddef.h>

#include <cmath>
#include <cstdlib>
#include <mutex>
#include <string>

#include "../../include/needle2_b200.h"

namespace {

thread_local std::string g_frontend_error;   // errors raised here (the reference keeps its own)

void *frontend_library(std::string *why) {
    static std::once_flag once;
    static void *handle = nullptr;
    static std::string failure;
    std::call_once(once, [] {
        const char *path = std::getenv("NEEDLE2_FRONTEND_LIBRARY");
        if (!path || !*path) {
            failure = "the tokenizer and grammar compiler come from the reference's native library: set "
                      "NEEDLE2_FRONTEND_LIBRARY to its path";
            return;
        }
        handle = dlopen(path, RTLD_NOW | RTLD_LOCAL);
        if (!handle) {
            const char *e = dlerror();
            failure = std::string("cannot load NEEDLE2_FRONTEND_LIBRARY: ") + (e ? e : path);
        }
    });
    if (!handle && why) *why = failure;
    return handle;
}

// The reference's entry point `name`, or null with g_frontend_error set.
template <typename Fn>
Fn frontend_symbol(const char *name) {
    std::string why;
    void *h = frontend_library(&why);
    if (!h) {
        g_frontend_error = why;
        return nullptr;
    }
    void *f = dlsym(h, name);
    if (!f) {
        g_frontend_error = std::string("the frontend library lacks ") + name;
        return nullptr;
    }
    g_frontend_error.clear();
    return reinterpret_cast<Fn>(f);
}

}  // namespace

extern "C" {

const char *needle2_frontend_error(void) {
    if (!g_frontend_error.empty()) return g_frontend_error.c_str();
    std::string why;
    void *h = frontend_library(&why);
    if (!h) return "";
    auto f = reinterpret_cast<const char *(*)()>(dlsym(h, "needle2_frontend_error"));
    return f ? f() : "";
}

void *needle2_tokenizer_create(const unsigned char *blob, size_t size) {
    auto f = frontend_symbol<void *(*)(const unsigned char *, size_t)>("needle2_tokenizer_create");
    return f ? f(blob, size) : nullptr;
}

void needle2_tokenizer_free(void *tokenizer) {
    auto f = frontend_symbol<void (*)(void *)>("needle2_tokenizer_free");
    if (f) f(tokenizer);
}

int needle2_tokenizer_encode(void *tokenizer, const char *text, size_t size, int dummy, int *out, int capacity) {
    auto f = frontend_symbol<int (*)(void *, const char *, size_t, int, int *, int)>("needle2_tokenizer_encode");
    return f ? f(tokenizer, text, size, dummy, out, capacity) : -1;
}

int needle2_tokenizer_decode(void *tokenizer, const int *ids, int count, char *out, int capacity) {
    auto f = frontend_symbol<int (*)(void *, const int *, int, char *, int)>("needle2_tokenizer_decode");
    return f ? f(tokenizer, ids, count, out, capacity) : -1;
}

void *needle2_grammar_compile(void *tokenizer, const char *tools, size_t size) {
    auto f = frontend_symbol<void *(*)(void *, const char *, size_t)>("needle2_grammar_compile");
    return f ? f(tokenizer, tools, size) : nullptr;
}

void needle2_grammar_free(void *grammar) {
    auto f = frontend_symbol<void (*)(void *)>("needle2_grammar_free");
    if (f) f(grammar);
}

const needle2_dfa_state_desc *needle2_grammar_dfa(void *grammar) {
    auto f = frontend_symbol<const needle2_dfa_state_desc *(*)(void *)>("needle2_grammar_dfa");
    return f ? f(grammar) : nullptr;
}

int needle2_engine_decode_compiled(void *engine, const float *logits, int vocab, int limit, void *grammar,
                                   int *out, int *count) {
    g_frontend_error.clear();
    if (!engine || !logits || !out || !count || limit < 0 || vocab != needle2_engine_vocab(engine)) {
        g_frontend_error = "invalid compiled decode arguments";
        return -1;
    }
    const needle2_dfa_state_desc *dfa = nullptr;
    if (grammar) {
        dfa = needle2_grammar_dfa(grammar);
        if (!dfa) {
            if (g_frontend_error.empty()) g_frontend_error = "grammar has no token automaton";
            return -1;
        }
    }
    int best = 0;
    for (int i = 0; i < vocab; ++i) {
        if (std::isnan(logits[i])) {
            g_frontend_error = "NaN logits are not supported";
            return -1;
        }
        if (logits[i] > logits[best]) best = i;
    }
    if (needle2_engine_decode_loop(engine, best, limit, dfa, out, count) != 0) {
        g_frontend_error = needle2_engine_error();
        return -1;
    }
    return 0;
}

}  // extern "C"
