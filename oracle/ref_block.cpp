// ref_block.cpp -- TEST INFRASTRUCTURE ONLY (reference-built oracle).
//
// Compiled by oracle/Makefile together with the reference's own sources
// (src/quant.cpp, src/transformer.cpp and the files they link against, built
// in place from the read-only reference tree with the reference's flags
// -std=gnu++20 -O3 -mavx2 -mfma -mf16c -fopenmp) into oracle/_ref/libjxref.so.
//
// The attention block of MoETransformerEngine::forward_token
// (src/transformer.cpp:2497-2566) is inline code, not a callable function, so
// jxr_append_attend() restates those lines with the reference's own
// expressions and calls the reference's compiled apply_rope, softmax,
// fp16/bf16 converters and KVCacheSlot.  Compiled with the same compiler and
// flags as the reference, it rounds as the reference's forward_token does.
// Only tests/ and bench.py's reference arm load this library.
#include "transformer.h"

#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#if defined(_OPENMP)
#include <omp.h>
#endif

using moe::MoETransformerEngine;

namespace {

enum { F32 = 0, BF16 = 1, F16T = 2 };

inline float load_elem(const void* base, size_t i, int dtype) {
    if (dtype == F32) return static_cast<const float*>(base)[i];
    const uint16_t h = static_cast<const uint16_t*>(base)[i];
    return dtype == BF16 ? moe::bf16_to_fp32(h) : moe::fp16_to_fp32(h);
}

inline void store_elem(void* base, size_t i, float x, int dtype) {
    if (dtype == F32) {
        static_cast<float*>(base)[i] = x;
        return;
    }
    static_cast<uint16_t*>(base)[i] = dtype == BF16 ? moe::fp32_to_bf16(x) : moe::fp32_to_fp16(x);
}

// src/transformer.cpp:2497-2566 with the KV element type made a parameter
// (F16T is the reference's native cache; F32 and BF16 are the storage
// variants the B200 library adds).
int append_attend(void* k_layer, void* v_layer, int dtype, uint32_t max_kv_dim, float* q, float* k,
                  const float* v, float* attn_out, uint32_t n_heads, uint32_t n_kv_heads,
                  uint32_t head_dim, uint32_t rope_dim, uint32_t pos, float rope_base,
                  float yarn_scale, bool is_neox, const float* rf_ptr, bool shares_kv,
                  bool is_swa, uint32_t sliding_window, float scale, float softcap) {
    const uint32_t kv_dim = n_kv_heads * head_dim;
    MoETransformerEngine::apply_rope(q, k, n_heads, n_kv_heads, head_dim, rope_dim, pos, rope_base,
                                     yarn_scale, is_neox, rf_ptr);
    if (!shares_kv) {
        for (uint32_t i = 0; i < kv_dim; ++i) {
            store_elem(k_layer, static_cast<size_t>(pos) * max_kv_dim + i, k[i], dtype);
            store_elem(v_layer, static_cast<size_t>(pos) * max_kv_dim + i, v[i], dtype);
        }
    }
    std::fill(attn_out, attn_out + static_cast<size_t>(n_heads) * head_dim, 0.0f);
    const uint32_t kv_mul = std::max(1u, n_heads / std::max(1u, n_kv_heads));
    const uint32_t t_start_win =
        (is_swa && sliding_window > 0 && pos >= sliding_window) ? (pos - sliding_window + 1) : 0;
#if defined(_OPENMP)
#pragma omp parallel for if (n_heads >= 4 && pos >= 32) schedule(static)
#endif
    for (int h_i = 0; h_i < static_cast<int>(n_heads); ++h_i) {
        const uint32_t h = static_cast<uint32_t>(h_i);
        const float* q_head = q + h * head_dim;
        const uint32_t kvh = h / kv_mul;
        const uint32_t win_len = pos - t_start_win + 1;
        std::vector<float> scores(win_len);
        for (uint32_t t = t_start_win; t <= pos; ++t) {
            const size_t base = static_cast<size_t>(t) * max_kv_dim + kvh * head_dim;
            float dot = 0.0f;
            for (uint32_t d = 0; d < head_dim; ++d) {
                dot += q_head[d] * load_elem(k_layer, base + d, dtype);
            }
            scores[t - t_start_win] = dot * scale;
        }
        if (softcap > 0.0f) {
            const float cap = softcap;
            const float inv_cap = 1.0f / cap;
            for (uint32_t s = 0; s < win_len; ++s) {
                scores[s] = cap * std::tanh(scores[s] * inv_cap);
            }
        }
        MoETransformerEngine::softmax(scores.data(), win_len);
        float* out_head = attn_out + h * head_dim;
        for (uint32_t t = t_start_win; t <= pos; ++t) {
            const size_t base = static_cast<size_t>(t) * max_kv_dim + kvh * head_dim;
            const float a = scores[t - t_start_win];
            for (uint32_t d = 0; d < head_dim; ++d) {
                out_head[d] += a * load_elem(v_layer, base + d, dtype);
            }
        }
    }
    return 0;
}

}  // namespace

extern "C" {

float jxr_fp16_to_fp32(uint16_t h) { return moe::fp16_to_fp32(h); }
uint16_t jxr_fp32_to_fp16(float f) { return moe::fp32_to_fp16(f); }
float jxr_bf16_to_fp32(uint16_t b) { return moe::bf16_to_fp32(b); }
uint16_t jxr_fp32_to_bf16(float f) { return moe::fp32_to_bf16(f); }

void jxr_apply_rope(float* q, float* k, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                    uint32_t rope_dim, uint32_t pos, float freq_base, float yarn_scale, int is_neox,
                    const float* rope_freqs) {
    MoETransformerEngine::apply_rope(q, k, n_heads, n_kv_heads, head_dim, rope_dim, pos, freq_base,
                                     yarn_scale, is_neox != 0, rope_freqs);
}

void jxr_softmax(float* x, int64_t size) { MoETransformerEngine::softmax(x, size); }

int jxr_append_attend(void* k_layer, void* v_layer, int dtype, uint32_t row_stride, float* q,
                      float* k, const float* v, float* attn_out, uint32_t n_heads,
                      uint32_t n_kv_heads, uint32_t head_dim, uint32_t rope_dim, uint32_t pos,
                      float rope_base, float yarn_scale, int is_neox, const float* rope_freqs,
                      int shares_kv, int is_swa, uint32_t sliding_window, float scale,
                      float softcap) {
    return append_attend(k_layer, v_layer, dtype, row_stride, q, k, v, attn_out, n_heads,
                         n_kv_heads, head_dim, rope_dim, pos, rope_base, yarn_scale, is_neox != 0,
                         rope_freqs, shares_kv != 0, is_swa != 0, sliding_window, scale, softcap);
}

// Whole step over n_seqs x n_layers; same argument meaning as jxo_step in
// oracle/jx_oracle.c.
int jxr_step(void* k_cache, void* v_cache, int dtype, uint32_t capacity, uint32_t row_stride,
             uint32_t n_cache_layers, uint32_t n_seqs, const int32_t* pos, uint32_t n_layers,
             const uint32_t* rope_dim, const float* rope_base, const int32_t* is_swa,
             const int32_t* shares_kv, const uint32_t* kv_source_layer, const float* q,
             const float* k, const float* v, float* out, uint32_t q_stride, uint32_t kv_stride,
             uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, float scale, float softcap,
             uint32_t sliding_window, float yarn_scale, int is_neox, const float* rope_freqs) {
    const size_t esz = dtype == F32 ? 4 : 2;
    const size_t layer_elems = static_cast<size_t>(capacity) * row_stride;
    const uint32_t kv_dim = n_kv_heads * head_dim;
    std::vector<float> qb(static_cast<size_t>(n_heads) * head_dim), kb(kv_dim);
    for (uint32_t s = 0; s < n_seqs; ++s) {
        if (pos[s] < 0 || static_cast<uint32_t>(pos[s]) >= capacity) return -5;
        for (uint32_t l = 0; l < n_layers; ++l) {
            const size_t io = static_cast<size_t>(s) * n_layers + l;
            std::memcpy(qb.data(), q + io * q_stride, sizeof(float) * qb.size());
            std::memcpy(kb.data(), k + io * kv_stride, sizeof(float) * kv_dim);
            const size_t off = (static_cast<size_t>(s) * n_cache_layers + kv_source_layer[l]) *
                               layer_elems * esz;
            append_attend(static_cast<char*>(k_cache) + off, static_cast<char*>(v_cache) + off,
                          dtype, row_stride, qb.data(), kb.data(), v + io * kv_stride,
                          out + io * q_stride, n_heads, n_kv_heads, head_dim, rope_dim[l],
                          static_cast<uint32_t>(pos[s]), rope_base[l], yarn_scale, is_neox != 0,
                          is_swa[l] ? nullptr : rope_freqs, shares_kv[l] != 0, is_swa[l] != 0,
                          sliding_window, scale, softcap);
        }
    }
    return 0;
}

// KVCacheSlot::compact (src/transformer.cpp:41-66) run on the reference's own
// struct.  k_seq/v_seq hold n_layers x capacity x kv_dim uint16 values (the
// reference stores fp16 bit patterns); they are copied in, compacted by the
// reference code, and copied back.  Returns the new seq_pos.
uint32_t jxr_compact_u16(uint16_t* k_seq, uint16_t* v_seq, uint32_t n_layers, uint32_t capacity,
                         uint32_t kv_dim, uint32_t seq_pos, uint32_t keep_recent) {
    moe::ModelHyperparams hp;
    hp.n_layers = n_layers;
    hp.kv_dim = kv_dim;
    hp.kv_cache_capacity = capacity;
    moe::KVCacheSlot slot;
    slot.init(0, hp);
    const size_t per_layer = static_cast<size_t>(capacity) * kv_dim;
    for (uint32_t l = 0; l < n_layers; ++l) {
        std::memcpy(slot.k_cache[l].data(), k_seq + l * per_layer, per_layer * 2);
        std::memcpy(slot.v_cache[l].data(), v_seq + l * per_layer, per_layer * 2);
    }
    slot.seq_pos = seq_pos;
    slot.token_history.assign(seq_pos, 0u);
    slot.compact(hp, keep_recent);
    for (uint32_t l = 0; l < n_layers; ++l) {
        std::memcpy(k_seq + l * per_layer, slot.k_cache[l].data(), per_layer * 2);
        std::memcpy(v_seq + l * per_layer, slot.v_cache[l].data(), per_layer * 2);
    }
    return slot.seq_pos;
}

// KVCacheSlot::rollback (src/transformer.cpp:32-39): returns the new seq_pos.
uint32_t jxr_rollback(uint32_t seq_pos, uint32_t new_seq_pos) {
    moe::KVCacheSlot slot;
    slot.seq_pos = seq_pos;
    slot.rollback(new_seq_pos);
    return slot.seq_pos;
}

int jxr_max_threads(void) {
#if defined(_OPENMP)
    return omp_get_max_threads();
#else
    return 1;
#endif
}

}  // extern "C"
