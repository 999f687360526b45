/*
 * needle2_b200 — C ABI of the B200 build of OpenNeedle's quantized hot path.
 *
 * libneedle2_b200.so is a drop-in for the library that needle2/native.py
 * loads (NEEDLE2_NATIVE_LIBRARY=<path>): the first block of entry points has
 * the reference's names, argument meaning and ownership rules; everything
 * after it is additive.  Plain C types only; host pointers unless a name ends
 * in _device.
 *
 * Ownership: the GPU build copies packed weights, norms and the codebook to
 * device memory at create time and owns those copies; host inputs are only
 * read during the call (the reference borrows them for the handle's life).
 * Errors: create functions return NULL; int functions return -1; in both cases,
 * and after any failed void call, needle2_b200_error() holds the message
 * (thread-local).  Calls on one handle must be serialised.
 */
#ifndef NEEDLE2_B200_H
#define NEEDLE2_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- reference-compatible CQ matrix ABI --------------------------------- */

/* Replaces needle2_native_features, needle2/csrc/cq.cpp:343-349. */
const char *needle2_native_features(void);

/* Replaces needle2_cq_create, needle2/csrc/cq.cpp:350-352.  bits in {2,3,4} or
 * 5 (signed ternary crumbs, 3 centroids); group a power of two in [8, 16384]. */
void *needle2_cq_create(const uint8_t *packed, const uint16_t *norms_fp16, int out, int in, int bits, int group,
                        const float *codebook);
/* Replaces needle2_cq_destroy, needle2/csrc/cq.cpp:353. */
void needle2_cq_destroy(void *handle);
/* Replaces needle2_cq_linear, needle2/csrc/cq.cpp:354-356: y[batch][out] =
 * CQ(x[batch][in]) in FP32 mode.  `threads` is accepted and unused. */
void needle2_cq_linear(void *handle, const float *x, float *y, int batch, int threads);
/* Replaces needle2_cq_linear_lookup, needle2/csrc/cq.cpp:357-359.  The lookup
 * table modes are CPU reassociations of the same FP32 sums; every mode runs
 * the FP32 kernel here. */
void needle2_cq_linear_lookup(void *handle, const float *x, float *y, int batch, int threads, int mode);
/* Replaces needle2_cq_linear_many, needle2/csrc/cq.cpp:360-366: one input row
 * against `count` matrices sharing its rotation. */
void needle2_cq_linear_many(void *const *handles, int count, const float *x, float *const *ys, int threads,
                            int mode);
/* Replaces needle2_cq_rows, needle2/csrc/cq.cpp:367-370: dequantised rows. */
void needle2_cq_rows(void *handle, const int64_t *ids, float *y, int count);

/* ---- reference-compatible SDOT (int8) ABI ------------------------------- */

/* Replaces needle2_sdot_supported, needle2/csrc/sdot.cpp:350: 1 on this build. */
int needle2_sdot_supported(void);
/* Replaces needle2_sdot_create, needle2/csrc/sdot.cpp:351-354: CQ2/CQ4,
 * group in [64, 16384]; NULL otherwise. */
void *needle2_sdot_create(const uint8_t *packed, const uint16_t *norms_fp16, int out, int in, int bits, int group,
                          const float *codebook);
/* Replaces needle2_sdot_destroy, needle2/csrc/sdot.cpp:355. */
void needle2_sdot_destroy(void *handle);
/* Replaces needle2_sdot_linear, needle2/csrc/sdot.cpp:356-359. */
void needle2_sdot_linear(void *handle, const float *x, float *y, int batch, int threads);

/* ---- additive: error channel, device pointers, debug exports ------------ */

/* Message of the last failure on this thread ("" if none). */
const char *needle2_b200_error(void);

/* Int-returning forms of needle2_cq_linear / needle2_sdot_linear (0 or -1). */
int needle2_cq_linear_checked(void *handle, const float *x, float *y, int batch);
int needle2_sdot_linear_checked(void *handle, const float *x, float *y, int batch);

/* Same computations on device pointers, enqueued on `stream` (a cudaStream_t,
 * NULL for the legacy default stream); no host synchronisation.  The handle's
 * device scratch is reused across calls, so calls on one handle must not run
 * concurrently on different streams. */
int needle2_cq_linear_device(void *handle, const float *x, float *y, int batch, void *stream);
int needle2_sdot_linear_device(void *handle, const float *x, float *y, int batch, void *stream);

/* No counterpart in the reference.  needle2_sdot_linear_device without any
 * device allocation, for callers that may not allocate while they run (a
 * serving loop on memory reserved up front, code that must avoid the
 * device-wide synchronisation of cudaMalloc/cudaFree).  Its activation scratch
 * is one fixed array pair per device inside this library: batch * padded input
 * width must be <= 1048576 and batch * groups <= 16384, larger batches fail
 * with -1 and a message.  The scratch needs no initial contents.  All calls on
 * a device share it, so two calls whose kernels may overlap (different streams,
 * or different threads without ordering) race: serialise them.  The first call
 * on a device looks up the scratch address; make one call outside any stream
 * capture before capturing.  The address is looked up again whenever the
 * device's context has changed (after cudaDeviceReset, for instance).  It
 * always runs the int8 GEMV kernel, never the tensor-core GEMM that
 * needle2_sdot_linear_device uses from 64 activation rows on, so
 * prefill-sized batches are slower here than there (same results). */
int needle2_sdot_linear_device_noalloc(void *handle, const float *x, float *y, int batch, void *stream);

/* Several matrices against one activation batch: ys[i][batch][out_i].  Matrices
 * with the same input geometry and codebook share one prepared activation and
 * run as one fused launch (the fused projections of needle2/csrc/engine.cpp:560-606);
 * others run one after another.  `sdot` selects the int8 mode (all handles
 * must be of that kind).  Host pointers / device pointers respectively. */
int needle2_cq_linear_many_checked(void *const *handles, int count, const float *x, float *const *ys, int batch,
                                   int sdot);
int needle2_cq_linear_many_device(void *const *handles, int count, const float *x, float *const *ys, int batch,
                                  int sdot, void *stream);
/* Fused multiply only, from the activations last prepared on handles[0]
 * (needle2_cq_prepare_device / needle2_sdot_prepare_device); the matrices must
 * be able to share a launch. */
int needle2_cq_multiply_many_device(void *const *handles, int count, float *const *ys, int batch, int sdot,
                                    void *stream);

/* Two-phase device form: prepare rotates (FP32 mode) or rotates and quantises
 * (SDOT mode) x[batch][in] into the handle's device scratch; multiply then
 * writes y[batch][out] from it.  Split as SdotCQ::prepare / SdotCQ::multiply,
 * needle2/csrc/sdot.cpp:47-103,338-345.  multiply's batch must not exceed the
 * last prepare's. */
int needle2_cq_prepare_device(void *handle, const float *x, int batch, void *stream);
int needle2_cq_multiply_device(void *handle, float *y, int batch, void *stream);
int needle2_sdot_prepare_device(void *handle, const float *x, int batch, void *stream);
int needle2_sdot_multiply_device(void *handle, float *y, int batch, void *stream);

/* N-sharded matrices (no counterpart in the reference, which runs on one host):
 * multiply from the last prepare into ndst (1..8) device buffers at once, y[b][o]
 * going to dsts[i][b * ldy + o] (ldy >= out).  With dsts[i] = this shard's
 * column range of every rank's full [batch][N] output, the all-gather of an
 * N-sharded GEMM happens in the GEMM's epilogue (peer stores over NVLink;
 * batches of 64 rows and more with group 128), or as one copy per buffer
 * otherwise.  The caller orders the ranks' calls before reading (a barrier). */
int needle2_sdot_multiply_gather_device(void *handle, float *const *dsts, int ndst, int ldy, int batch,
                                        void *stream);

/* CUDA IPC between the processes of one node: export a device pointer as a
 * 64-byte handle plus its offset inside its allocation; import gives this
 * process a pointer to the same bytes (peer access enabled); close releases
 * an imported pointer. */
int needle2_b200_ipc_export(const void *ptr, void *handle64, unsigned long long *offset);
int needle2_b200_ipc_import(const void *handle64, unsigned long long offset, void **ptr);
int needle2_b200_ipc_close(void *ptr);

/* The decode loop's greedy token of each row of logits[rows][ld] (vocab <= ld
 * entries used): out[r] = the first index of the row's maximum, NaNs never
 * chosen, 0 when the row's first logit is NaN -- the reference's scan
 * (best = 0, then any strictly greater logit), Engine::decode_loop,
 * needle2/csrc/engine.cpp:1434-1442 and the candidate scan 1472-1479.
 * Device pointers on a stream. */
int needle2_b200_argmax_device(const float *logits, int rows, int vocab, int ld, int *out, void *stream);

/* The engine's fake activation quantiser for activation_bits = bits, in place
 * on x[rows][dim], each row separately: a = max|x|, unchanged when a is 0,
 * otherwise x = clamp(round_half_even(x / (a / m)), -m - 1, m) * (a / m) with
 * m = 2^(bits-1) - 1.  Replaces activation_quant, needle2/csrc/engine.cpp:185-191
 * (applied before the QKVG, out_proj, engram and LM-head matmuls,
 * engine.cpp:769,992,1024,1041).  bits 0 leaves x unchanged.  Device pointer on
 * a stream / host pointer (synchronous). */
int needle2_b200_activation_quant_device(float *x, int rows, int dim, int bits, void *stream);
int needle2_b200_activation_quant(float *x, int rows, int dim, int bits);

/* SDOT internals the reference never exports (its per-group int32 dots stay
 * inside SdotCQ::row, needle2/csrc/sdot.cpp:142-149): partials[batch][out][groups]
 * int32, q[batch][padded] int8 in natural element order, scales[batch][groups];
 * any output pointer may be NULL.  Host pointers. */
int needle2_sdot_debug(void *handle, const float *x, int batch, float *y, int32_t *partials, int8_t *q,
                       float *scales);

/* 1 if a kernel's bounded wait on an asynchronous copy ran out since the last
 * call (the kernel then abandons its work instead of spinning); 0 otherwise,
 * -1 if the flag could not be read.  Reading clears it. */
int needle2_b200_device_fault(void);

/* Geometry of a handle: out, in, bits, group, padded, groups. */
int needle2_cq_geometry(void *handle, int *geometry6);

/* Which kernel runs FP32-mode GEMVs of up to 8 activation rows, process-wide:
 * 0 automatic (one activation row: the product-table cluster kernel; up to 4
 * rows: the row-per-lane kernel; where their shared-memory tables fit, the
 * slot-per-lane kernel otherwise), 1 always the slot-per-lane kernel, 2 the
 * row-per-lane kernel without the product table.  All compute CQ::linear's
 * sums in FP32 (association differs; results agree within FP32 rounding); the
 * switch exists for tests and measurements.  Returns the previous setting, or
 * -1 for an unknown kind. */
int needle2_b200_set_f32_gemv(int kind);

/* ---- additive: batched INT8 KV cache with a shared prefix ---------------- */
/*
 * The reference keeps one sequence per Engine and an optional per-instance
 * prefix snapshot (needle2/csrc/engine.cpp:192-199,376-499).  A KV pool holds
 * `sessions` sequences of one layer that share ONE read-only prefix of
 * `prefix_len` positions (the sinks of the reference's slot map) stored once on
 * the device; each session owns window (or max_seq - prefix_len) further slots
 * addressed as Engine::cache_slot does (engine.cpp:500).  Positions passed to
 * the calls are absolute and must be >= prefix_len.  Quantisation is the
 * reference's INT8 rule (engine.cpp:1005-1021); attention its
 * compute_attention (engine.cpp:898-967).  Calls on one pool must be
 * serialised; sessions within one call must be distinct.
 */
void *needle2_kv_create(int sessions, int heads, int kvheads, int head_dim, int max_seq, int window, int prefix_len);
void needle2_kv_destroy(void *kv);
size_t needle2_kv_storage_bytes(void *kv);
/* Quantise and store the shared prefix: k, v [prefix_len][kvheads*head_dim]. */
int needle2_kv_set_prefix(void *kv, const float *k, const float *v);
int needle2_kv_set_prefix_device(void *kv, const float *k, const float *v, void *stream);
/* Store one new token per listed session (k, v [count][kvheads*head_dim]). */
int needle2_kv_store(void *kv, const int *session_ids, const int *positions, const float *k, const float *v,
                     int count);
int needle2_kv_store_device(void *kv, const int *session_ids, const int *positions, const float *k, const float *v,
                            int count, void *stream);
/* Attention of one query per listed session at `positions` over the current
 * cache (q, out [count][heads*head_dim]); nothing is stored. */
int needle2_attention_query(void *kv, const int *session_ids, const int *positions, const float *q, float *out,
                            int count);
int needle2_attention_query_device(void *kv, const int *session_ids, const int *positions, const float *q, float *out,
                                   int count, void *stream);
/* Decode step: store each session's new K/V at its position, then attend. */
int needle2_attention_decode(void *kv, const int *session_ids, const int *positions, const float *q, const float *k,
                             const float *v, float *out, int count);
int needle2_attention_decode_device(void *kv, const int *session_ids, const int *positions, const float *q,
                                    const float *k, const float *v, float *out, int count, void *stream);
/* Prefill `tokens` new tokens per listed session starting at start_positions,
 * causal, with the reference's store-then-attend order per token
 * (engine.cpp:1170-1210).  q/out [count][tokens][heads*head_dim],
 * k/v [count][tokens][kvheads*head_dim]. */
int needle2_attention_prefill(void *kv, const int *session_ids, const int *start_positions, int tokens, const float *q,
                              const float *k, const float *v, float *out, int count);
int needle2_attention_prefill_device(void *kv, const int *session_ids, const int *start_positions, int tokens,
                                     const float *q, const float *k, const float *v, float *out, int count,
                                     void *stream);
/* One session's cache in the reference layout: keys/values [capacity][kvheads*head_dim]
 * int8, scales [capacity][kvheads], capacity = window ? window + prefix_len : max_seq. */
int needle2_kv_export(void *kv, int session, int8_t *keys, int8_t *values, float *k_scales, float *v_scales);

/* ---- reference-compatible engine ABI (whole Needle-2 forward on the GPU) -- */
/*
 * Layouts of needle2/csrc/engine.cpp:14-19 and :327-339 (bound from Python by
 * needle2/native.py:282-304).  Tensors come in the canonical order of
 * needle2/native.py:350-395: embedding; per layer norm_in, q_proj, k_proj,
 * v_proj, q_norm, k_norm, gate_proj, out_proj, post_norm, attn_gate, pre_hada,
 * d1, d2, d3; mhc_a_pre/post/res, mhc_b_pre/post/res, mhc_phi_pre/post/res;
 * per engram site tables, key_proj, value_proj, taps; final_norm.  A matrix is
 * either a CQ handle of this library (needle2_cq_create; `cq`) or host FP32
 * data (`data`, rows x cols, copied to the device at create time); the mHC
 * projections must be FP32 data, as the reference's NativeEngine passes them.
 */
typedef struct {
    void *cq;
    const float *data;
    int rows, cols;
} needle2_tensor_desc;

typedef struct {
    int vocab, dim, heads, kvheads, layers, head_dim, max_seq, hada, lanes, window;
    int slots, subdim, tables, taps, dilation, num_orders, orders[4], num_sites, sites[4];
    float rope_theta;
} needle2_engine_config;

typedef struct {
    int num_states, initial_state, eos_id, stop_id, tool_start_id, tool_end_id;
    const int *state_types, *fallback_next_states, *candidate_offsets, *candidate_tokens, *next_states;
} needle2_dfa_state_desc;

/* Replace needle2_engine_* of needle2/csrc/engine.cpp:1499-1548 with the same
 * arguments, return values and error convention (NULL / -1 and the thread-local
 * needle2_engine_error()).  One engine = one sequence, as in the reference;
 * calls on one engine must be serialised.  `threads` is accepted and unused. */
void *needle2_engine_create(const needle2_engine_config *config, const needle2_tensor_desc *tensors, int count,
                            int threads, int activation_bits);
void needle2_engine_destroy(void *engine);
void needle2_engine_set_lookup(void *engine, int mode);
int needle2_engine_set_sdot(void *engine);
void needle2_engine_reset(void *engine, int prefix_len);
int needle2_engine_cache_prefix(void *engine);
int needle2_engine_reset_to_prefix(void *engine);
int needle2_engine_step(void *engine, int token, float *logits, float *hidden);
int needle2_engine_prefill(void *engine, const int *tokens, int num_tokens, int last_only, float *logits,
                           float *hidden);
int needle2_engine_step_candidates(void *engine, int token, const int *candidates, int num_candidates,
                                   float *candidate_logits, float *hidden);
int needle2_engine_project_candidates(void *engine, const int *candidates, int num_candidates,
                                      float *candidate_logits);
int needle2_engine_decode_loop(void *engine, int first_token, int max_new_tokens, const needle2_dfa_state_desc *dfa,
                               int *output_tokens, int *out_generated_count);
int needle2_engine_import(void *engine, int position, int prefix_len, const int *ids, const int *positions,
                          int count, const float *k, const float *v);
int needle2_engine_set_int8_kv(void *engine, int enable);
size_t needle2_engine_kv_storage_bytes(void *engine);
const char *needle2_engine_error(void);

/* Vocabulary size of the engine's model (additive; -1 for a null engine). */
int needle2_engine_vocab(void *engine);

/* ---- frontend: needle2/csrc/frontend.h:15-35 ------------------------------
 * The tokenizer and grammar entry points forward to the reference's own
 * native library (built from its sources), loaded from the path in
 * NEEDLE2_FRONTEND_LIBRARY at the first call; without it they fail (NULL / -1)
 * with needle2_frontend_error() saying so.  needle2_engine_decode_compiled is
 * this library's: argmax of the prefill logits (first maximum, NaN refused),
 * then needle2_engine_decode_loop with the grammar's automaton
 * (frontend.cpp:1057-1079).  The grammar's vocabulary is not compared with the
 * engine's (the automaton carries none); candidate tokens are range-checked by
 * the decode loop. */
const char *needle2_frontend_error(void);
void *needle2_tokenizer_create(const unsigned char *blob, size_t size);
void needle2_tokenizer_free(void *tokenizer);
int needle2_tokenizer_encode(void *tokenizer, const char *text, size_t size, int dummy, int *output, int capacity);
int needle2_tokenizer_decode(void *tokenizer, const int *tokens, int count, char *output, int capacity);
void *needle2_grammar_compile(void *tokenizer, const char *tools_json, size_t size);
void needle2_grammar_free(void *grammar);
const needle2_dfa_state_desc *needle2_grammar_dfa(void *grammar);
int needle2_engine_decode_compiled(void *engine, const float *logits, int vocab, int limit, void *grammar,
                                   int *output, int *count);

/* ---- additive: many sequences of one engine's model, in lockstep --------- */
/*
 * The reference serves one unpadded sequence per Engine (needle2/native.py:307-314).
 * A batch holds `sessions` sequences that share the engine's weights (the
 * engine must outlive it) and one pinned prefix; every call advances all of
 * them by the same number of tokens, each through exactly the per-sequence
 * arithmetic of the engine (teacher-forced logits equal the engine's within
 * FP32 rounding).  The KV format (INT8 or FP32) and the matmul mode (FP32 or
 * SDOT) are the engine's at batch creation.
 */
void *needle2_batch_create(void *engine, int sessions, int prefix_len);
void needle2_batch_destroy(void *batch);
size_t needle2_batch_kv_storage_bytes(void *batch);
/* Run the shared prefix (prefix_len tokens) once; every session then continues
 * from position prefix_len with the prefix's KV, token history and engram state. */
int needle2_batch_set_prefix(void *batch, const int *tokens);
/* tokens[sessions][n] appended to every session; logits of each session's last
 * token into logits[sessions][vocab] and/or its greedy token into next[sessions]
 * (either may be NULL).  Host pointers; synchronous. */
int needle2_batch_prefill(void *batch, const int *tokens, int n, float *logits, int *next);
/* One token per session (teacher forcing): logits[sessions][vocab] and/or greedy next[sessions]. */
int needle2_batch_step(void *batch, const int *tokens, float *logits, int *next);
/* `steps` greedy steps from first[sessions]: out[sessions][steps] = the tokens
 * fed at each step (first, then each step's greedy choice); the sessions
 * advance by `steps` positions.  Host pointers; synchronous. */
int needle2_batch_decode_greedy(void *batch, const int *first, int steps, int *out);
/* The same on device pointers, enqueued on `stream` without host synchronisation.
 * From the second step on, the steps replay a CUDA graph of one step (unless
 * disabled with needle2_batch_set_graphs or while the profiler runs). */
int needle2_batch_decode_greedy_device(void *batch, const int *first, int steps, int *out, void *stream);
/* 1 (default): decode steps replay a captured CUDA graph; 0: launch by launch. */
int needle2_batch_set_graphs(void *batch, int enable);
/* Kernels in the last captured decode-step graph (0 before any capture). */
int needle2_batch_step_kernels(void *batch);
/* Current position of every session (host copy). */
int needle2_batch_positions(void *batch, int *positions);
/* Stage timers (CUDA events at every stage boundary of each forward pass, on
 * the pass's stream) while enabled; enabling or disabling clears the totals.
 * profile_read returns the milliseconds per stage since the last read and
 * clears them (synchronises): 0 engrams and embedding, 1 mHC routing (lane
 * RMS, projections, gates) where it runs on its own (the first layer, or
 * geometries without the fused layer boundary), 2 Q/K/V/gate projections,
 * 3 QK norm and RoPE, 4 KV store and attention, 5 out projection, 6 Hadamard
 * MLP and lane mixing, with the next layer's routing (or the final norm)
 * where the layer boundary is one kernel, 7 final norm (where separate), LM
 * head and greedy choice. */
int needle2_batch_profile(void *batch, int enable);
int needle2_batch_profile_read(void *batch, double *ms, int n);

#ifdef __cplusplus
}
#endif

#endif /* NEEDLE2_B200_H */
