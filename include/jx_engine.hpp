// jx_engine.hpp -- C++ drop-in for jxai's KVCacheSlot and the attention block
// of MoETransformerEngine::forward_token, over the C ABI of jx_attn.h.
//
// The reference keeps each slot's cache in host vectors (include/transformer.h:
// 115-131) and runs RoPE, the KV append and grouped-query attention inline per
// layer (src/transformer.cpp:2497-2567) on host q/k/v vectors.  Here the cache
// lives in HBM (one jx_kv handle for all slots) and the block is one library
// call per layer; the engine's surrounding code keeps its host vectors:
//
//   jx::DeviceKVCache cache(hp, max_slots);            // KVCacheSlot::init for all slots
//   jx::KVCacheSlot& slot = ...; slot.init(id, cache);
//   jx::AttentionBlock attn(cache);                     // pinned staging buffers
//   // per layer, in place of transformer.cpp:2497-2567:
//   attn.forward(slot, layer_desc, q.data(), k.data(), v.data(), attn_out.data(), pos);
//   // after the last layer, as transformer.cpp:2792:
//   slot.seq_pos++;
//
// Two wider forms of the same block: forward_batch runs one layer for several
// slots at once (one token each, at each slot's seq_pos), and forward_prompt
// runs one layer for n consecutive prompt tokens of one slot (the prompt loop
// of transformer.cpp:3092-3095 done layer by layer instead of token by token).
//
// Header-only; link with libjxattn.so and the CUDA runtime.  Every call
// returns a jx status (0 = JX_OK); jx_last_error_string() has the message.
#ifndef JX_ENGINE_HPP
#define JX_ENGINE_HPP

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "jx_attn.h"

namespace jx {

// The attention-related fields of jxai's ModelHyperparams.
struct Hyper {
    uint32_t n_layers = 0;
    uint32_t n_heads = 0;
    uint32_t n_kv_heads = 0;
    uint32_t q_dim = 0;              // max over layers (row stride of q / attn_out)
    uint32_t kv_dim = 0;             // max over layers (row stride of the cache and k / v)
    uint32_t kv_cache_capacity = 0;
    uint32_t sliding_window = 0;
    float yarn_scale = 1.0f;
    float attn_logit_softcapping = 0.0f;
    bool rope_neox = true;
    bool unit_scale = false;         // gemma4: scale 1 instead of 1/sqrt(head_dim)
};

// The cache of every slot: KVCacheSlot::init's allocation for max_slots slots.
class DeviceKVCache {
  public:
    DeviceKVCache(const Hyper& hp, uint32_t max_slots, jx_dtype dtype = JX_F16_TRUNC,
                  int device = 0)
        : hp_(hp), max_slots_(max_slots) {
        jx_kv_desc d{};
        d.n_seqs = max_slots;
        d.n_layers = hp.n_layers;
        d.capacity = hp.kv_cache_capacity > 0 ? hp.kv_cache_capacity : 1;
        d.row_stride = hp.kv_dim;
        d.dtype = dtype;
        d.device = device;
        d.pos_base = 0;
        status_ = jx_kv_create(&d, &kv_);
    }
    ~DeviceKVCache() { jx_kv_destroy(kv_); }
    DeviceKVCache(const DeviceKVCache&) = delete;
    DeviceKVCache& operator=(const DeviceKVCache&) = delete;

    int status() const { return status_; }  // JX_OK when the allocation succeeded
    jx_kv* handle() const { return kv_; }
    const Hyper& hyper() const { return hp_; }
    uint32_t max_slots() const { return max_slots_; }

  private:
    Hyper hp_;
    uint32_t max_slots_ = 0;
    jx_kv* kv_ = nullptr;
    int status_ = JX_ERR_INVALID;
};

// moe::KVCacheSlot with its cache on the device: the same members and methods
// (transformer.cpp:13-66).  seq_pos is the engine's to advance, as in the
// reference; the device copy of it is synchronised by every call below.
struct KVCacheSlot {
    uint32_t slot_id = 0;
    uint32_t seq_pos = 0;
    uint32_t compactions = 0;
    std::vector<uint32_t> token_history;
    DeviceKVCache* cache = nullptr;

    int init(uint32_t id, DeviceKVCache& c) {
        cache = &c;
        slot_id = id;
        compactions = 0;
        token_history.clear();
        return clear();
    }
    // zero rows, seq_pos 0 (transformer.cpp:25-30)
    int clear(cudaStream_t stream = nullptr) {
        seq_pos = 0;
        token_history.clear();
        return jx_kv_clear(cache->handle(), slot_id, stream);
    }
    // never moves forward (transformer.cpp:32-39)
    int rollback(uint32_t new_seq_pos) {
        if (new_seq_pos < seq_pos) seq_pos = new_seq_pos;
        if (token_history.size() > new_seq_pos) token_history.resize(new_seq_pos);
        return jx_kv_set_seq_pos(cache->handle(), slot_id, seq_pos);
    }
    // 4 sink rows + the last keep_recent rows (transformer.cpp:41-66)
    int compact(uint32_t keep_recent = 128, cudaStream_t stream = nullptr) {
        int rc = jx_kv_set_seq_pos(cache->handle(), slot_id, seq_pos);
        if (rc) return rc;
        const uint32_t before = seq_pos;
        rc = jx_kv_compact(cache->handle(), slot_id, keep_recent, stream);
        if (rc) return rc;
        uint32_t after = before;
        rc = jx_kv_get_seq_pos(cache->handle(), slot_id, &after);
        if (rc) return rc;
        if (after != before) {
            seq_pos = after;
            if (token_history.size() > after) token_history.resize(after);
            compactions++;
        }
        return JX_OK;
    }
};

// The per-layer attention fields of jxai's LayerDenseWeights.
struct LayerAttn {
    uint32_t head_dim = 0;
    uint32_t rope_dim = 0;
    float rope_freq_base = 10000.0f;
    uint32_t kv_source_layer = 0;
    bool is_swa = false;
    bool shares_kv = false;
    const float* rope_freqs = nullptr;  // host, rope_dim/2 factors (Neox, global layers)
};

// How the block's host rows cross PCIe.
enum class Staging {
    // The CPU copies q/k/v into pinned host buffers the library reads directly
    // (one staging kernel brings them into device memory, chained to the
    // decode launch) and the decode kernel writes attn_out into a pinned
    // buffer, which the CPU copies out after the stream synchronises: no
    // copy-engine transfers on the per-layer critical path.
    PinnedHost,
    // cudaMemcpyAsync of q, k and v from the engine's (pageable) vectors into
    // device buffers, and of attn_out back.
    DeviceCopies,
};

// transformer.cpp:2497-2567 for one layer of one slot, host vectors in and
// out: q (n_heads*head_dim) and k, v (n_kv_heads*head_dim) go up, attn_out
// (n_heads*head_dim) comes down.  As in the reference, q and k are the
// un-rotated projections and the call rotates them; unlike the reference the
// host q and k are left unrotated (nothing reads them afterwards).
class AttentionBlock {
  public:
    explicit AttentionBlock(DeviceKVCache& c, cudaStream_t stream = nullptr,
                            Staging staging = Staging::PinnedHost)
        : cache_(c), stream_(stream), staging_(staging) {
        status_ = reserve(1);
    }
    ~AttentionBlock() { release(); }
    AttentionBlock(const AttentionBlock&) = delete;
    AttentionBlock& operator=(const AttentionBlock&) = delete;

    int status() const { return status_; }

    int forward(KVCacheSlot& slot, const LayerAttn& lw, const float* q, const float* k,
                const float* v, float* attn_out, uint32_t pos) {
        if (status_) return status_;
        const Hyper& hp = cache_.hyper();
        const size_t q_dim = static_cast<size_t>(hp.n_heads) * lw.head_dim;
        const size_t kv_dim = static_cast<size_t>(hp.n_kv_heads) * lw.head_dim;
        int rc = put_rows(q, q_dim, k, v, kv_dim);
        if (rc) return rc;
        int32_t seq = static_cast<int32_t>(slot.slot_id), p = static_cast<int32_t>(pos);
        jx_layer_desc L = desc(lw);
        jx_step_args a = args(lw, 1, &seq, &p);
        rc = jx_attn_step(cache_.handle(), &L, 1, &a, stream_);
        if (rc) return rc;
        return fetch(attn_out, q_dim * 4);
    }

    // One layer for n slots at once, one token each at slots[i]->seq_pos (a
    // serving loop's batched decode in place of one forward_token per request
    // under engine_mtx_, transformer.cpp:2361).  Host rows: q and attn_out
    // [n][hp.q_dim], k and v [n][hp.kv_dim]; row i belongs to slots[i].  A slot
    // appears at most once per call.
    int forward_batch(KVCacheSlot* const* slots, uint32_t n, const LayerAttn& lw,
                      const float* q, const float* k, const float* v, float* attn_out) {
        if (status_) return status_;
        if (n == 0) return JX_OK;
        if (!slots) return JX_ERR_INVALID;
        int rc = reserve(n);
        if (rc) return rc;
        seq_.resize(n);
        pos_.resize(n);
        for (uint32_t i = 0; i < n; ++i) {
            if (!slots[i]) return JX_ERR_INVALID;
            seq_[i] = static_cast<int32_t>(slots[i]->slot_id);
            pos_[i] = static_cast<int32_t>(slots[i]->seq_pos);
        }
        if ((rc = upload(q, k, v, n))) return rc;
        jx_layer_desc L = desc(lw);
        jx_step_args a = args(lw, n, seq_.data(), pos_.data());
        if ((rc = jx_attn_step(cache_.handle(), &L, 1, &a, stream_))) return rc;
        return fetch(attn_out, static_cast<size_t>(n) * cache_.hyper().q_dim * 4);
    }

    // One layer for n_tokens consecutive prompt tokens of one slot, at
    // positions pos0, pos0+1, ...: each token's k and v are appended and each
    // token attends causally over the rows up to its own position, the same
    // result as feeding the tokens one at a time (transformer.cpp:3092-3095).
    // Host rows as in forward_batch, one per token.  The caller advances
    // slot.seq_pos by n_tokens after the last layer.
    int forward_prompt(KVCacheSlot& slot, const LayerAttn& lw, const float* q, const float* k,
                       const float* v, float* attn_out, uint32_t n_tokens, uint32_t pos0) {
        if (status_) return status_;
        if (n_tokens == 0) return JX_OK;
        int rc = reserve(n_tokens);
        if (rc) return rc;
        seq_.assign(n_tokens, static_cast<int32_t>(slot.slot_id));
        pos_.resize(n_tokens);
        for (uint32_t t = 0; t < n_tokens; ++t) pos_[t] = static_cast<int32_t>(pos0 + t);
        if ((rc = upload(q, k, v, n_tokens))) return rc;
        jx_layer_desc L = desc(lw);
        jx_step_args a = args(lw, n_tokens, seq_.data(), pos_.data());
        if ((rc = jx_attn_prefill(cache_.handle(), &L, 1, &a, stream_))) return rc;
        return fetch(attn_out, static_cast<size_t>(n_tokens) * cache_.hyper().q_dim * 4);
    }

  private:
    // staging for `rows` rows of q/k/v/out (grown, never shrunk): pinned host
    // buffers or device buffers, by the staging mode
    int reserve(uint32_t rows) {
        if (rows <= rows_) return JX_OK;
        release();
        const Hyper& hp = cache_.hyper();
        const size_t qb = sizeof(float) * hp.q_dim * rows, kb = sizeof(float) * hp.kv_dim * rows;
        void* p[4] = {nullptr, nullptr, nullptr, nullptr};
        const size_t sz[4] = {qb, kb, kb, qb};
        for (int i = 0; i < 4; ++i) {
            const cudaError_t e = staging_ == Staging::PinnedHost
                                      ? cudaHostAlloc(&p[i], sz[i], cudaHostAllocDefault)
                                      : cudaMalloc(&p[i], sz[i]);
            if (e != cudaSuccess) {
                for (int j = 0; j < i; ++j) free_buf(p[j]);
                return JX_ERR_NOMEM;
            }
        }
        q_ = static_cast<float*>(p[0]);
        k_ = static_cast<float*>(p[1]);
        v_ = static_cast<float*>(p[2]);
        out_ = static_cast<float*>(p[3]);
        rows_ = rows;
        return JX_OK;
    }
    void free_buf(void* p) {
        if (staging_ == Staging::PinnedHost) cudaFreeHost(p);
        else cudaFree(p);
    }
    void release() {
        free_buf(q_);
        free_buf(k_);
        free_buf(v_);
        free_buf(out_);
        q_ = k_ = v_ = out_ = nullptr;
        rows_ = 0;
    }
    // one row of q (q_n floats) and of k, v (kv_n floats)
    int put_rows(const float* q, size_t q_n, const float* k, const float* v, size_t kv_n) {
        if (staging_ == Staging::PinnedHost) {
            std::memcpy(q_, q, q_n * 4);
            std::memcpy(k_, k, kv_n * 4);
            std::memcpy(v_, v, kv_n * 4);
            return JX_OK;
        }
        if (cudaMemcpyAsync(q_, q, q_n * 4, cudaMemcpyHostToDevice, stream_) != cudaSuccess ||
            cudaMemcpyAsync(k_, k, kv_n * 4, cudaMemcpyHostToDevice, stream_) != cudaSuccess ||
            cudaMemcpyAsync(v_, v, kv_n * 4, cudaMemcpyHostToDevice, stream_) != cudaSuccess)
            return JX_ERR_CUDA;
        return JX_OK;
    }
    int upload(const float* q, const float* k, const float* v, uint32_t rows) {
        const Hyper& hp = cache_.hyper();
        return put_rows(q, static_cast<size_t>(hp.q_dim) * rows, k, v,
                        static_cast<size_t>(hp.kv_dim) * rows);
    }
    int fetch(float* attn_out, size_t bytes) {
        if (staging_ == Staging::PinnedHost) {
            if (cudaStreamSynchronize(stream_) != cudaSuccess) return JX_ERR_CUDA;
            std::memcpy(attn_out, out_, bytes);
            return JX_OK;
        }
        if (cudaMemcpyAsync(attn_out, out_, bytes, cudaMemcpyDeviceToHost, stream_) !=
                cudaSuccess ||
            cudaStreamSynchronize(stream_) != cudaSuccess)
            return JX_ERR_CUDA;
        return JX_OK;
    }
    static jx_layer_desc desc(const LayerAttn& lw) {
        jx_layer_desc L{};
        L.head_dim = lw.head_dim;
        L.rope_dim = lw.rope_dim;
        L.rope_freq_base = lw.rope_freq_base;
        L.kv_source_layer = lw.kv_source_layer;
        L.is_swa = lw.is_swa ? 1 : 0;
        L.shares_kv = lw.shares_kv ? 1 : 0;
        L.rope_freqs = lw.rope_freqs;
        return L;
    }
    jx_step_args args(const LayerAttn& lw, uint32_t n, const int32_t* seq,
                      const int32_t* pos) const {
        const Hyper& hp = cache_.hyper();
        jx_step_args a{};
        a.n_heads = hp.n_heads;
        a.n_kv_heads = hp.n_kv_heads;
        a.n_seqs = n;
        a.seq_ids = seq;
        a.pos = pos;
        a.q = q_;
        a.k = k_;
        a.v = v_;
        a.out = out_;
        a.q_stride = hp.q_dim;
        a.kv_stride = hp.kv_dim;
        a.scale = hp.unit_scale ? 1.0f : 1.0f / std::sqrt(static_cast<float>(lw.head_dim));
        a.softcap = hp.attn_logit_softcapping;
        a.sliding_window = hp.sliding_window;
        a.yarn_scale = hp.yarn_scale;
        a.rope_neox = hp.rope_neox ? 1 : 0;
        return a;
    }

    DeviceKVCache& cache_;
    cudaStream_t stream_;
    Staging staging_;
    // q/k/v/out rows: pinned host memory (PinnedHost) or device memory (DeviceCopies)
    float *q_ = nullptr, *k_ = nullptr, *v_ = nullptr, *out_ = nullptr;
    uint32_t rows_ = 0;
    std::vector<int32_t> seq_, pos_;
    int status_ = JX_ERR_INVALID;
};

}  // namespace jx

#endif  // JX_ENGINE_HPP
