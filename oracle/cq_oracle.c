/*
 * CPU ORACLE — test infrastructure only.
 *
 * A plain-C restatement of OpenNeedle's CPU arithmetic for the quantized hot
 * path, used as the checker for the CUDA kernels in openneedle_b200.  Only the
 * test suite, __graft_entry__.smoke() and bench.py's cpu_baseline leg load this
 * library.  Nothing in the product links or calls it.
 *
 * Every function follows the x86 (non-NEON) branch of the reference, which is
 * what the reference build executes on x86_64, in the same operation order, so
 * that this oracle is bit-identical to the reference compiled without FMA
 * contraction.  Parity is pinned by tests/test_oracle_pins.py: against golden
 * vectors produced by the reference itself (tests/golden/make_golden.py) and,
 * when the reference sources are present, against oracle/_ref built from them.
 *
 * Build: oracle/Makefile (gcc -O2 -std=c11 -ffp-contract=off).
 * Citations are paths inside the OpenNeedle project.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* IEEE binary16 -> binary32, exact.  Follows needle2/csrc/cq.cpp:14-28. */
float oracle_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exponent = (h >> 10) & 0x1fu;
    uint32_t mantissa = h & 0x3ffu;
    uint32_t bits;
    if (exponent == 0) {
        if (mantissa == 0) {
            bits = sign;
        } else {
            /* subnormal half: normalise the mantissa */
            int e = -14;
            while ((mantissa & 0x400u) == 0) { mantissa <<= 1; --e; }
            bits = sign | ((uint32_t)(e + 127) << 23) | ((mantissa & 0x3ffu) << 13);
        }
    } else if (exponent == 31) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else {
        bits = sign | ((exponent + 112u) << 23) | (mantissa << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Normalised radix-2 Walsh-Hadamard transform, butterfly strides 1,2,4,...,n/2,
 * then one multiply by 1/sqrtf(n).  Follows needle2/csrc/cq.cpp:30-46. */
void oracle_fwht(float *v, int n) {
    for (int h = 1; h < n; h *= 2) {
        for (int base = 0; base < n; base += 2 * h) {
            for (int j = 0; j < h; ++j) {
                float a = v[base + j], b = v[base + j + h];
                v[base + j] = a + b;
                v[base + j + h] = a - b;
            }
        }
    }
    float scale = 1.0f / sqrtf((float)n);
    for (int i = 0; i < n; ++i) v[i] *= scale;
}

/* Index i of an LSB-first bitstream of `bits`-wide fields.
 * Follows needle2/csrc/cq.cpp:48-53. */
unsigned oracle_index_at(const uint8_t *p, int i, int bits) {
    int bit = i * bits, byte = bit >> 3, shift = bit & 7;
    unsigned word = p[byte];
    if (shift + bits > 8) word |= (unsigned)p[byte + 1] << 8;
    return (word >> shift) & ((1u << bits) - 1u);
}

static int padded_of(int in, int group) { return (in + group - 1) / group * group; }
static int storage_bits_of(int bits) { return bits == 5 ? 2 : bits; }

/* Codebook value of element i of a packed group.  bits==5 is the signed
 * ternary crumb code (3 -> cb[0], 0 -> cb[1], 1 -> cb[2]).
 * Follows needle2/csrc/cq.cpp:71-74. */
static float cq_weight(const uint8_t *p, int i, int bits, const float *cb) {
    unsigned idx = oracle_index_at(p, i, storage_bits_of(bits));
    return bits == 5 ? cb[idx == 3 ? 0 : idx + 1] : cb[idx];
}

/* Zero-pad one activation row to `padded` and rotate each group.
 * Follows CQ::transform, needle2/csrc/cq.cpp:153-156. */
void oracle_cq_transform(const float *x, float *rot, int in, int group) {
    int padded = padded_of(in, group);
    memcpy(rot, x, sizeof(float) * (size_t)in);
    for (int i = in; i < padded; ++i) rot[i] = 0.0f;
    for (int g = 0; g < padded / group; ++g) oracle_fwht(rot + (size_t)g * group, group);
}

/* FP32 mode: y[b,r] = sum_g half(norm[r,g]) * sum_i cb[idx[r,g,i]] * rot[b,g,i],
 * each group summed sequentially from i=0, groups added in g order.
 * Follows CQ::linear / group_dot / dot_row, needle2/csrc/cq.cpp:75-109,157-197
 * (x86 path: group_dot_pair reduces to the same sequential sums). */
void oracle_cq_linear(const uint8_t *packed, const uint16_t *norms, int out, int in,
                      int bits, int group, const float *cb, const float *x, float *y,
                      int batch) {
    int padded = padded_of(in, group), groups = padded / group;
    int sbits = storage_bits_of(bits);
    size_t rowbytes = (size_t)padded * sbits / 8;
    float *rot = (float *)malloc(sizeof(float) * (size_t)padded * (size_t)(batch > 0 ? batch : 1));
    for (int b = 0; b < batch; ++b)
        oracle_cq_transform(x + (size_t)b * in, rot + (size_t)b * padded, in, group);
    for (int r = 0; r < out; ++r) {
        const uint8_t *p = packed + (size_t)r * rowbytes;
        const uint16_t *s = norms + (size_t)r * groups;
        for (int b = 0; b < batch; ++b) {
            const float *rb = rot + (size_t)b * padded;
            float sum = 0.0f;
            for (int g = 0; g < groups; ++g) {
                const uint8_t *pg = p + (size_t)g * group * sbits / 8;
                const float *xg = rb + (size_t)g * group;
                float gsum = 0.0f;
                for (int i = 0; i < group; ++i) gsum += cq_weight(pg, i, bits, cb) * xg[i];
                sum += gsum * oracle_half_to_float(s[g]);
            }
            y[(size_t)b * out + r] = sum;
        }
    }
    free(rot);
}

/* Dequantised rows: tmp = cb[idx]*half(norm), inverse-rotated per group, cropped.
 * Follows CQ::row, needle2/csrc/cq.cpp:276-284 and needle2_cq_rows :367-370. */
void oracle_cq_rows(const uint8_t *packed, const uint16_t *norms, int out, int in, int bits,
                    int group, const float *cb, const int64_t *ids, float *y, int count) {
    (void)out;
    int padded = padded_of(in, group), groups = padded / group;
    size_t rowbytes = (size_t)padded * storage_bits_of(bits) / 8;
    float *tmp = (float *)malloc(sizeof(float) * (size_t)padded);
    for (int c = 0; c < count; ++c) {
        int64_t r = ids[c];
        for (int g = 0; g < groups; ++g) {
            float norm = oracle_half_to_float(norms[(size_t)r * groups + g]);
            for (int i = 0; i < group; ++i)
                tmp[g * group + i] = cq_weight(packed + (size_t)r * rowbytes, g * group + i, bits, cb) * norm;
            oracle_fwht(tmp + (size_t)g * group, group);
        }
        memcpy(y + (size_t)c * in, tmp, sizeof(float) * (size_t)in);
    }
    free(tmp);
}

static float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* SDOT weight side: matrix-wide centroid scale max|cb|/127 (1 if zero),
 * int8 centroids round-half-even(cb/scale) clamped to +-127.
 * Follows SdotCQ::SdotCQ, needle2/csrc/sdot.cpp:35-45. */
void oracle_sdot_centroids(const float *cb, int bits, int8_t *centroids, float *centroid_scale) {
    float maximum = 0.0f;
    for (int i = 0; i < (1 << bits); ++i) {
        float a = fabsf(cb[i]);
        if (a > maximum) maximum = a;
    }
    float cs = maximum > 0 ? maximum / 127 : 1;
    for (int i = 0; i < 16; ++i) centroids[i] = 0;
    for (int i = 0; i < (1 << bits); ++i)
        centroids[i] = (int8_t)clampf(nearbyintf(cb[i] / cs), -127.0f, 127.0f);
    *centroid_scale = cs;
}

/* SDOT activation quantiser, per row and per group after the rotation:
 * scale = absmax/127 (1 when absmax is 0; absmax itself when absmax/127
 * underflows to 0), q = clamp(round-half-even(x/scale), -127, 127).
 * q is written in natural element order (the reference additionally permutes
 * it into bit planes for its NEON loads; the permutation is applied to both
 * factors of every product and does not change any integer sum).
 * Follows SdotCQ::prepare, needle2/csrc/sdot.cpp:47-103 (x86 branch :78-80). */
void oracle_sdot_prepare(const float *x, int rows, int in, int group, int8_t *q, float *scales) {
    int padded = padded_of(in, group), groups = padded / group;
    float *rot = (float *)malloc(sizeof(float) * (size_t)padded);
    for (int m = 0; m < rows; ++m) {
        oracle_cq_transform(x + (size_t)m * in, rot, in, group);
        for (int g = 0; g < groups; ++g) {
            const float *v = rot + (size_t)g * group;
            float absmax = 0.0f;
            for (int i = 0; i < group; ++i) {
                float a = fabsf(v[i]);
                absmax = a > absmax ? a : absmax;   /* std::max(absmax, a) */
            }
            float scale = absmax > 0 ? absmax / 127 : 1;
            if (!scale) scale = absmax;
            scales[(size_t)m * groups + g] = scale;
            int8_t *dst = q + (size_t)m * padded + (size_t)g * group;
            for (int i = 0; i < group; ++i)
                dst[i] = (int8_t)clampf(nearbyintf(v[i] / scale), -127.0f, 127.0f);
        }
    }
    free(rot);
}

/* Per-group int32 dots d[m,r,g] = sum_i centroid[idx[r,g,i]] * q[m,g,i].
 * Follows SdotCQ::dot_group, needle2/csrc/sdot.cpp:108-137. */
void oracle_sdot_partials(const uint8_t *packed, int out, int in, int bits, int group,
                          const int8_t *centroids, const int8_t *q, int rows, int32_t *partials) {
    int padded = padded_of(in, group), groups = padded / group;
    size_t rowbytes = (size_t)padded * bits / 8;
    for (int m = 0; m < rows; ++m)
        for (int r = 0; r < out; ++r)
            for (int g = 0; g < groups; ++g) {
                const uint8_t *p = packed + (size_t)r * rowbytes + (size_t)g * group * bits / 8;
                const int8_t *xg = q + (size_t)m * padded + (size_t)g * group;
                int32_t sum = 0;
                for (int i = 0; i < group; ++i)
                    sum += (int32_t)centroids[oracle_index_at(p, i, bits)] * (int32_t)xg[i];
                partials[((size_t)m * out + r) * groups + g] = sum;
            }
}

/* SDOT output: y[m,r] = sum over g, in g order, of
 * (float(d[m,r,g]) * (half(norm[r,g]) * centroid_scale)) * scale[m,g].
 * Follows SdotCQ::row, needle2/csrc/sdot.cpp:142-149 and :43-44. */
void oracle_sdot_linear(const uint8_t *packed, const uint16_t *norms, int out, int in, int bits,
                        int group, const float *cb, const float *x, float *y, int rows,
                        int32_t *partials_out, int8_t *q_out, float *scales_out) {
    int padded = padded_of(in, group), groups = padded / group;
    int8_t centroids[16];
    float cs;
    oracle_sdot_centroids(cb, bits, centroids, &cs);
    int8_t *q = q_out ? q_out : (int8_t *)malloc((size_t)rows * padded);
    float *scales = scales_out ? scales_out : (float *)malloc(sizeof(float) * (size_t)rows * groups);
    int32_t *d = partials_out ? partials_out
                              : (int32_t *)malloc(sizeof(int32_t) * (size_t)rows * out * groups);
    oracle_sdot_prepare(x, rows, in, group, q, scales);
    oracle_sdot_partials(packed, out, in, bits, group, centroids, q, rows, d);
    for (int m = 0; m < rows; ++m)
        for (int r = 0; r < out; ++r) {
            float value = 0.0f;
            for (int g = 0; g < groups; ++g) {
                float ns = oracle_half_to_float(norms[(size_t)r * groups + g]) * cs;
                value += (float)d[((size_t)m * out + r) * groups + g] * ns * scales[(size_t)m * groups + g];
            }
            y[(size_t)m * out + r] = value;
        }
    if (!q_out) free(q);
    if (!scales_out) free(scales);
    if (!partials_out) free(d);
}

/* Greedy token of one logits row: best = 0, then every later index whose
 * logit is strictly greater than the best so far (the first maximum wins; a NaN
 * is never greater, so NaNs after index 0 are skipped and a NaN at index 0
 * keeps 0).  Follows Engine::decode_loop, needle2/csrc/engine.cpp:1434-1442
 * (and the candidate scan, 1472-1479). */
int oracle_argmax(const float *x, int n) {
    int best = 0;
    float max_v = x[0];
    for (int i = 1; i < n; ++i) {
        if (x[i] > max_v) {
            max_v = x[i];
            best = i;
        }
    }
    return best;
}

/* A8 fake activation quantiser on one vector: a = max|x|; unchanged if 0;
 * x = clamp(round-half-even(x/(a/127)), -128, 127) * (a/127).
 * Follows activation_quant, needle2/csrc/engine.cpp:185-191. */
void oracle_activation_quant(float *x, int n, int bits) {
    if (!bits) return;
    float a = 0.0f;
    for (int i = 0; i < n; ++i) {
        float v = fabsf(x[i]);
        a = a > v ? a : v;
    }
    if (!a) return;
    int maxq = (1 << (bits - 1)) - 1;
    float scale = a / (float)maxq;
    for (int i = 0; i < n; ++i) {
        float r = nearbyintf(x[i] / scale);
        float lo = (float)(-maxq - 1), hi = (float)maxq;
        r = r < hi ? r : hi;      /* std::min(float(max), r) */
        r = lo > r ? lo : r;      /* std::max(float(-max-1), .) */
        x[i] = r * scale;
    }
}

/* INT8 KV store of one token: per KV head, scale = max|k|/127 (1 if 0),
 * k_i8 = clamp(round-half-even(k * (127/max)), -127, 127); the same for v.
 * Multiplies by the reciprocal (unlike the SDOT quantiser, which divides).
 * Follows Engine::step, needle2/csrc/engine.cpp:1005-1021. */
void oracle_kv_quantize(const float *k, const float *v, int kvheads, int head_dim,
                        int8_t *k_i8, int8_t *v_i8, float *k_scale, float *v_scale) {
    for (int kh = 0; kh < kvheads; ++kh) {
        const float *kp = k + (size_t)kh * head_dim, *vp = v + (size_t)kh * head_dim;
        float max_k = 0.0f, max_v = 0.0f;
        for (int d = 0; d < head_dim; ++d) {
            float a = fabsf(kp[d]), b = fabsf(vp[d]);
            max_k = max_k > a ? max_k : a;
            max_v = max_v > b ? max_v : b;
        }
        float scale_k = max_k > 0 ? max_k / 127.0f : 1.0f, scale_v = max_v > 0 ? max_v / 127.0f : 1.0f;
        float inv_k = max_k > 0 ? 127.0f / max_k : 0.0f, inv_v = max_v > 0 ? 127.0f / max_v : 0.0f;
        k_scale[kh] = scale_k;
        v_scale[kh] = scale_v;
        for (int d = 0; d < head_dim; ++d) {
            float a = nearbyintf(kp[d] * inv_k), b = nearbyintf(vp[d] * inv_v);
            a = 127.0f < a ? 127.0f : a; a = -127.0f > a ? -127.0f : a;
            b = 127.0f < b ? 127.0f : b; b = -127.0f > b ? -127.0f : b;
            k_i8[(size_t)kh * head_dim + d] = (int8_t)a;
            v_i8[(size_t)kh * head_dim + d] = (int8_t)b;
        }
    }
}

/* Ring slot of a position: sinks [0,prefix) are pinned, the rest cycles through
 * `window` slots; without a window the slot is the position.
 * Follows Engine::cache_slot, needle2/csrc/engine.cpp:500. */
int oracle_cache_slot(int pos, int prefix, int window) {
    return !window ? pos : pos < prefix ? pos : prefix + (pos - prefix) % window;
}

/* Visible slots of the query at pos_cur: sinks then the window, in that order.
 * Returns the count and writes the slots.  Follows compute_attention,
 * needle2/csrc/engine.cpp:898-911. */
int oracle_attention_slots(int pos_cur, int prefix, int window, int *slots) {
    int prefix_count = window ? (prefix < pos_cur + 1 ? prefix : pos_cur + 1) : 0;
    int start = window ? (prefix > pos_cur - window + 1 ? prefix : pos_cur - window + 1) : 0;
    int tail = pos_cur - start + 1;
    int length = prefix_count + (tail > 0 ? tail : 0);
    if (slots)
        for (int s = 0; s < length; ++s)
            slots[s] = oracle_cache_slot(s < prefix_count ? s : start + s - prefix_count, prefix, window);
    return length;
}

/* One query token's attention over an INT8 KV cache of one layer.
 * Cache layout as in the reference: keys_i8/values_i8 [capacity][kvheads][head_dim],
 * k_scales/v_scales [capacity][kvheads].  q and out are [heads][head_dim].
 * s = (sum_d q*float(k_i8)) * k_scale * (1/sqrtf(hd)); p = softmax(s) with
 * exp(s - max), sequential denominators and one multiply by 1/den;
 * out[d] = sum_s (p*v_scale) * float(v_i8[d]), sequential over s.
 * Follows compute_attention / accumulate_values / softmax_inplace,
 * needle2/csrc/engine.cpp:137-147, 816-897 (x86 tail loops), 898-967. */
void oracle_attention_i8(const int8_t *keys_i8, const int8_t *values_i8, const float *k_scales,
                         const float *v_scales, int heads, int kvheads, int head_dim, int pos_cur,
                         int prefix, int window, const float *q, float *out) {
    int K = kvheads * head_dim;
    int length = oracle_attention_slots(pos_cur, prefix, window, NULL);
    int *slots = (int *)malloc(sizeof(int) * (size_t)(length > 0 ? length : 1));
    float *scores = (float *)malloc(sizeof(float) * (size_t)(length > 0 ? length : 1));
    oracle_attention_slots(pos_cur, prefix, window, slots);
    float scale = 1 / sqrtf((float)head_dim);
    int group = heads / kvheads;
    for (int h = 0; h < heads; ++h) {
        int kh = h / group;
        const float *qh = q + (size_t)h * head_dim;
        float maximum = -INFINITY;
        for (int s = 0; s < length; ++s) {
            int slot = slots[s];
            const int8_t *kp = keys_i8 + (size_t)slot * K + (size_t)kh * head_dim;
            float sum = 0.0f;
            for (int d = 0; d < head_dim; ++d) sum += qh[d] * (float)kp[d];
            float sc = sum * k_scales[(size_t)slot * kvheads + kh];
            sc *= scale;
            scores[s] = sc;
            maximum = maximum > sc ? maximum : sc;   /* std::max(max0, s0[s]) */
        }
        float den = 0.0f;
        for (int s = 0; s < length; ++s) {
            scores[s] = expf(scores[s] - maximum);
            den += scores[s];
        }
        float inv = 1 / den;
        for (int s = 0; s < length; ++s) scores[s] *= inv;
        float *oh = out + (size_t)h * head_dim;
        for (int d = 0; d < head_dim; ++d) {
            float a = 0.0f;
            for (int s = 0; s < length; ++s) {
                int slot = slots[s];
                float prob = scores[s];
                prob *= v_scales[(size_t)slot * kvheads + kh];
                a += prob * (float)values_i8[(size_t)slot * K + (size_t)kh * head_dim + d];
            }
            oh[d] = a;
        }
    }
    free(slots);
    free(scores);
}

/* Causal prefill of `count` tokens at positions start_pos.. on top of a cache
 * that already holds positions < start_pos: each token stores its own K/V
 * first, then attends, before the next token can evict a window slot.
 * k, v are [count][kvheads][head_dim], q and out are [count][heads][head_dim].
 * Follows Engine::prefill, needle2/csrc/engine.cpp:1170-1210. */
void oracle_attention_prefill_i8(int8_t *keys_i8, int8_t *values_i8, float *k_scales,
                                 float *v_scales, int heads, int kvheads, int head_dim,
                                 int start_pos, int count, int prefix, int window,
                                 const float *q, const float *k, const float *v, float *out) {
    int K = kvheads * head_dim;
    for (int t = 0; t < count; ++t) {
        int pos = start_pos + t;
        int slot = oracle_cache_slot(pos, prefix, window);
        oracle_kv_quantize(k + (size_t)t * K, v + (size_t)t * K, kvheads, head_dim,
                           keys_i8 + (size_t)slot * K, values_i8 + (size_t)slot * K,
                           k_scales + (size_t)slot * kvheads, v_scales + (size_t)slot * kvheads);
        oracle_attention_i8(keys_i8, values_i8, k_scales, v_scales, heads, kvheads, head_dim, pos,
                            prefix, window, q + (size_t)t * heads * head_dim,
                            out + (size_t)t * heads * head_dim);
    }
}
