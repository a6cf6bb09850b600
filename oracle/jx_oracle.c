/*
 * jx_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of jxai's per-token attention step (RoPE, KV append,
 * grouped-query decode attention) used as the parity checker for the CUDA
 * library in jxai_b200/.  Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg load this file's shared object; the product library never
 * links, loads or calls it, and it is not a fallback for anything.
 *
 * Every function cites the reference source it restates (paths inside the
 * jacxishipping/jxai project).  Rounding is pinned explicitly instead of being
 * left to the compiler: the file is built with -ffp-contract=off and every
 * fused multiply-add that the reference's own build (-O3 -mavx2 -mfma, GNU
 * C++20, gcc 13) forms is written as fmaf().  The forms were established by
 * comparing against the reference's compiled apply_rope over 2.4M rotated
 * pairs, and tests/test_oracle_golden.py re-checks them bit for bit against
 * fixtures the reference build in oracle/_ref/ produced (tests/golden/).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define JXO_F32 0
#define JXO_BF16 1
#define JXO_F16T 2

/* ---- scalar conversions: src/quant.cpp:876-939 ------------------------- */

/* src/quant.cpp:876-904 (exact IEEE half -> float; F16C path is identical). */
float jxo_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t ex = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x03FFu;
    uint32_t fbits;
    if (ex == 0) {
        if (mant == 0) {
            fbits = sign;
        } else {
            int e = 1;
            while ((mant & 0x0400u) == 0) { mant <<= 1; e--; }
            mant &= 0x03FFu;
            fbits = sign | ((uint32_t)(e + (127 - 15)) << 23) | (mant << 13);
        }
    } else if (ex == 31) {
        fbits = sign | 0x7F800000u | (mant << 13);
    } else {
        fbits = sign | ((ex + (127 - 15)) << 23) | (mant << 13);
    }
    float out;
    memcpy(&out, &fbits, 4);
    return out;
}

/* src/quant.cpp:906-925: truncating float -> half (mant >> 13, no rounding;
 * exponent overflow, Inf and NaN all become +-Inf; tiny values flush to +-0). */
uint16_t jxo_fp32_to_fp16(float f) {
    uint32_t fbits;
    memcpy(&fbits, &f, 4);
    uint16_t sign = (uint16_t)((fbits >> 16) & 0x8000u);
    int32_t ex = (int32_t)((fbits >> 23) & 0xFFu) - 127 + 15;
    uint32_t mant = fbits & 0x007FFFFFu;
    if (ex <= 0) {
        if (ex < -10) return sign;
        mant |= 0x00800000u;
        uint32_t shift = (uint32_t)(14 - ex);
        return (uint16_t)(sign | (uint16_t)(mant >> shift));
    } else if (ex >= 31) {
        return (uint16_t)(sign | 0x7C00u);
    }
    return (uint16_t)(sign | (uint16_t)(ex << 10) | (uint16_t)(mant >> 13));
}

/* src/quant.cpp:927-932 */
float jxo_bf16_to_fp32(uint16_t b) {
    uint32_t fbits = (uint32_t)b << 16;
    float out;
    memcpy(&out, &fbits, 4);
    return out;
}

/* src/quant.cpp:934-939: round-to-nearest-even with no NaN special case
 * (uint32 wrap-around included). */
uint16_t jxo_fp32_to_bf16(float f) {
    uint32_t fbits;
    memcpy(&fbits, &f, 4);
    uint32_t rounding_bias = ((fbits >> 16) & 1u) + 0x7FFFu;
    return (uint16_t)((fbits + rounding_bias) >> 16);
}

static inline float load_elem(const void* base, size_t i, int dtype) {
    if (dtype == JXO_F32) return ((const float*)base)[i];
    uint16_t h = ((const uint16_t*)base)[i];
    return dtype == JXO_BF16 ? jxo_bf16_to_fp32(h) : jxo_fp16_to_fp32(h);
}

static inline void store_elem(void* base, size_t i, float x, int dtype) {
    if (dtype == JXO_F32) { ((float*)base)[i] = x; return; }
    ((uint16_t*)base)[i] = dtype == JXO_BF16 ? jxo_fp32_to_bf16(x) : jxo_fp32_to_fp16(x);
}

/* ---- RoPE: src/transformer.cpp:76-138 ----------------------------------- */

/* Angle table exactly as apply_rope computes it (transformer.cpp:83, 88-92 for
 * Neox, 113-116 for interleaved).  cs[2*j] = cos, cs[2*j+1] = sin for pair j. */
void jxo_rope_cos_sin(uint32_t head_dim, uint32_t rope_dim, uint32_t pos, float freq_base,
                      float yarn_scale, int is_neox, const float* rope_freqs, float* cs) {
    uint32_t rdim = head_dim < rope_dim ? head_dim : rope_dim;
    float ys = yarn_scale > 1e-4f ? yarn_scale : 1e-4f;
    float pos_scaled = (float)pos / ys;
    uint32_t half = rdim / 2;
    for (uint32_t j = 0; j < half; ++j) {
        float freq;
        if (is_neox) {
            freq = 1.0f / powf(freq_base, (2.0f * (float)j) / (float)rdim);
            if (rope_freqs) freq /= rope_freqs[j];
        } else {
            uint32_t d = 2 * j;
            freq = 1.0f / powf(freq_base, (float)d / (float)rdim);
        }
        float angle = pos_scaled * freq;
        cs[2 * j] = cosf(angle);
        cs[2 * j + 1] = sinf(angle);
    }
}

/* Rotation of one head.  Rounding forms of the reference build:
 *   Neox (transformer.cpp:95-96):        r0 = fma(a, c, -(b*s)),  r1 = fma(a, s, b*c)
 *   interleaved (transformer.cpp:122-123): r0 = a*c - b*s,          r1 = a*s + b*c
 * where (a, b) is the pair, c = cos, s = sin, every product rounded. */
static void rope_head(float* x, uint32_t rdim, int is_neox, const float* cs) {
    uint32_t half = rdim / 2;
    for (uint32_t j = 0; j < half; ++j) {
        float c = cs[2 * j], s = cs[2 * j + 1];
        uint32_t i0 = is_neox ? j : 2 * j;
        uint32_t i1 = is_neox ? j + half : 2 * j + 1;
        float a = x[i0], b = x[i1];
        if (is_neox) {
            float bs = b * s, bc = b * c;
            x[i0] = fmaf(a, c, -bs);
            x[i1] = fmaf(a, s, bc);
        } else {
            float ac = a * c, bs = b * s, as = a * s, bc = b * c;
            x[i0] = ac - bs;
            x[i1] = as + bc;
        }
    }
}

/* src/transformer.cpp:76-138 (apply_rope), same signature meaning. */
void jxo_apply_rope(float* q, float* k, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                    uint32_t rope_dim, uint32_t pos, float freq_base, float yarn_scale, int is_neox,
                    const float* rope_freqs) {
    uint32_t rdim = head_dim < rope_dim ? head_dim : rope_dim;
    float* cs = (float*)malloc(sizeof(float) * (rdim + 2));
    jxo_rope_cos_sin(head_dim, rope_dim, pos, freq_base, yarn_scale, is_neox, rope_freqs, cs);
    for (uint32_t h = 0; h < n_heads; ++h) rope_head(q + (size_t)h * head_dim, rdim, is_neox, cs);
    if (k)
        for (uint32_t h = 0; h < n_kv_heads; ++h) rope_head(k + (size_t)h * head_dim, rdim, is_neox, cs);
    free(cs);
}

/* ---- softmax: src/transformer.cpp:1901-1916 ----------------------------- */
void jxo_softmax(float* x, int64_t size) {
    if (size <= 0) return;
    float max_val = x[0];
    for (int64_t i = 1; i < size; ++i)
        if (x[i] > max_val) max_val = x[i];
    float sum = 0.0f;
    for (int64_t i = 0; i < size; ++i) {
        x[i] = expf(x[i] - max_val);
        sum += x[i];
    }
    float inv_sum = (sum > 0.0f) ? (1.0f / sum) : (1.0f / (float)size);
    for (int64_t i = 0; i < size; ++i) x[i] *= inv_sum;
}

/* ---- the attention block: src/transformer.cpp:2497-2566 ------------------
 *
 * One (sequence, layer) step.  k_layer / v_layer point at the cache of
 * layer `kv_source_layer` of this sequence: `capacity` rows of `row_stride`
 * elements (KVCacheSlot::k_cache[kv_layer], transformer.h:120-122, with the
 * element type chosen by `dtype`).  q (n_heads*head_dim), k and v (kv_dim =
 * n_kv_heads*head_dim) are the projected vectors; q and k are rotated in place
 * as the reference does.  attn_out receives n_heads*head_dim floats.
 *
 * Loop order and accumulation order follow the reference exactly:
 *   QK  (2539-2545): dot = fma(q[d], K[t,d], dot) over d ascending, then *scale
 *   cap (2549-2555): cap * tanhf(s * (1/cap)) when softcap > 0
 *   softmax (2556)
 *   PV  (2559-2565): out[d] = fma(p_t, V[t,d], out[d]) over t ascending.
 */
int jxo_append_attend(void* k_layer, void* v_layer, int dtype, uint32_t row_stride,
                      float* q, float* k, const float* v, float* attn_out,
                      uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, uint32_t rope_dim,
                      uint32_t pos, float rope_base, float yarn_scale, int is_neox,
                      const float* rope_freqs, int shares_kv, int is_swa, uint32_t sliding_window,
                      float scale, float softcap) {
    const uint32_t kv_dim = n_kv_heads * head_dim;
    jxo_apply_rope(q, k, n_heads, n_kv_heads, head_dim, rope_dim, pos, rope_base, yarn_scale,
                   is_neox, rope_freqs);
    if (!shares_kv) {
        for (uint32_t i = 0; i < kv_dim; ++i) {
            store_elem(k_layer, (size_t)pos * row_stride + i, k[i], dtype);
            store_elem(v_layer, (size_t)pos * row_stride + i, v[i], dtype);
        }
    }
    memset(attn_out, 0, sizeof(float) * (size_t)n_heads * head_dim);
    const uint32_t nkv = n_kv_heads ? n_kv_heads : 1;
    const uint32_t kv_mul = (n_heads / nkv) ? (n_heads / nkv) : 1;
    const uint32_t t_start = (is_swa && sliding_window > 0 && pos >= sliding_window)
                                 ? (pos - sliding_window + 1) : 0;
    const uint32_t win_len = pos - t_start + 1;
    int failed = 0;
#pragma omp parallel for if (n_heads >= 4 && pos >= 32) schedule(static)
    for (int h_i = 0; h_i < (int)n_heads; ++h_i) {
        const uint32_t h = (uint32_t)h_i;
        const float* qh = q + (size_t)h * head_dim;
        const uint32_t kvh = h / kv_mul;
        float* scores = (float*)malloc(sizeof(float) * win_len);
        if (!scores) { failed = 1; continue; }
        for (uint32_t t = t_start; t <= pos; ++t) {
            size_t base = (size_t)t * row_stride + (size_t)kvh * head_dim;
            float dot = 0.0f;
            for (uint32_t d = 0; d < head_dim; ++d)
                dot = fmaf(qh[d], load_elem(k_layer, base + d, dtype), dot);
            scores[t - t_start] = dot * scale;
        }
        if (softcap > 0.0f) {
            const float inv_cap = 1.0f / softcap;
            for (uint32_t s = 0; s < win_len; ++s) scores[s] = softcap * tanhf(scores[s] * inv_cap);
        }
        jxo_softmax(scores, win_len);
        float* oh = attn_out + (size_t)h * head_dim;
        for (uint32_t t = t_start; t <= pos; ++t) {
            size_t base = (size_t)t * row_stride + (size_t)kvh * head_dim;
            const float a = scores[t - t_start];
            for (uint32_t d = 0; d < head_dim; ++d)
                oh[d] = fmaf(a, load_elem(v_layer, base + d, dtype), oh[d]);
        }
        free(scores);
    }
    return failed ? -3 : 0;
}

/* ---- whole decode step over many (sequence, layer) pairs ------------------
 *
 * The loop forward_token runs once per token (transformer.cpp:2442, one layer
 * after another) generalised to several independent sequences, which the
 * reference serves one after another under engine_mtx_ (transformer.cpp:2361).
 * Cache layout: [seq][layer][capacity][row_stride] elements of `dtype`.
 * q/out: [seq][layer][q_stride] floats; k/v: [seq][layer][kv_stride] floats.
 * Inputs q and k are copied before rotation, so callers' buffers stay intact.
 * layer arrays (n_layers entries): head_dim is shared; rope_dim, rope_base,
 * is_swa, shares_kv and kv_source_layer are per layer.
 */
int jxo_step(void* k_cache, void* v_cache, int dtype, uint32_t capacity, uint32_t row_stride,
             uint32_t n_cache_layers, uint32_t n_seqs, const int32_t* pos,
             uint32_t n_layers, const uint32_t* rope_dim, const float* rope_base,
             const int32_t* is_swa, const int32_t* shares_kv, const uint32_t* kv_source_layer,
             const float* q, const float* k, const float* v, float* out,
             uint32_t q_stride, uint32_t kv_stride, uint32_t n_heads, uint32_t n_kv_heads,
             uint32_t head_dim, float scale, float softcap, uint32_t sliding_window,
             float yarn_scale, int is_neox, const float* rope_freqs) {
    const size_t esz = dtype == JXO_F32 ? 4 : 2;
    const size_t layer_elems = (size_t)capacity * row_stride;
    const uint32_t kv_dim = n_kv_heads * head_dim;
    float* qb = (float*)malloc(sizeof(float) * (size_t)n_heads * head_dim);
    float* kb = (float*)malloc(sizeof(float) * kv_dim);
    if (!qb || !kb) { free(qb); free(kb); return -3; }
    int rc = 0;
    for (uint32_t s = 0; s < n_seqs && rc == 0; ++s) {
        if (pos[s] < 0 || (uint32_t)pos[s] >= capacity) { rc = -5; break; }
        for (uint32_t l = 0; l < n_layers && rc == 0; ++l) {
            size_t io = (size_t)s * n_layers + l;
            memcpy(qb, q + io * q_stride, sizeof(float) * (size_t)n_heads * head_dim);
            memcpy(kb, k + io * kv_stride, sizeof(float) * kv_dim);
            uint32_t cl = kv_source_layer[l];
            size_t off = ((size_t)s * n_cache_layers + cl) * layer_elems * esz;
            rc = jxo_append_attend((char*)k_cache + off, (char*)v_cache + off, dtype, row_stride,
                                   qb, kb, v + io * kv_stride, out + io * q_stride, n_heads,
                                   n_kv_heads, head_dim, rope_dim[l], (uint32_t)pos[s],
                                   rope_base[l], yarn_scale, is_neox,
                                   is_swa[l] ? NULL : rope_freqs, shares_kv[l], is_swa[l],
                                   sliding_window, scale, softcap);
        }
    }
    free(qb);
    free(kb);
    return rc;
}

/* ---- KVCacheSlot::compact: src/transformer.cpp:41-66 ---------------------
 * Keeps the 4 sink rows and the last keep_recent rows of every layer of one
 * sequence's cache; returns the new sequence length (unchanged when
 * seq_pos <= 4 + keep_recent). */
uint32_t jxo_compact(void* k_seq, void* v_seq, int dtype, uint32_t n_layers, uint32_t capacity,
                     uint32_t row_stride, uint32_t seq_pos, uint32_t keep_recent) {
    const uint32_t sink_tokens = 4;
    if (seq_pos <= sink_tokens + keep_recent) return seq_pos;
    const size_t esz = dtype == JXO_F32 ? 4 : 2;
    uint32_t src_start = seq_pos - keep_recent;
    size_t layer_bytes = (size_t)capacity * row_stride * esz;
    size_t row_bytes = (size_t)row_stride * esz;
    for (uint32_t l = 0; l < n_layers; ++l) {
        memmove((char*)k_seq + l * layer_bytes + sink_tokens * row_bytes,
                (char*)k_seq + l * layer_bytes + src_start * row_bytes, keep_recent * row_bytes);
        memmove((char*)v_seq + l * layer_bytes + sink_tokens * row_bytes,
                (char*)v_seq + l * layer_bytes + src_start * row_bytes, keep_recent * row_bytes);
    }
    return sink_tokens + keep_recent;
}

int jxo_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
