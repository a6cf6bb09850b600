// Drives jx_engine.hpp the way MoETransformerEngine::forward_token drives its
// KVCacheSlot and attention block (src/transformer.cpp:2366-2375, 2497-2567,
// 2792), on host vectors read from a script file; writes every layer's
// attn_out.  tests/test_gpu_engine.py replays the script through the CPU
// oracle and compares.
//
// Script (little-endian): int32 n_layers, n_heads, n_kv_heads, head_dim,
// capacity, neox, dtype, n_ops; float32 rope_base; then n_ops ops:
//   int32 1, then per layer q[n_heads*head_dim], k[n_kv*head_dim], v[n_kv*head_dim]
//            -- one token through all layers;
//   int32 2, int32 lcp -- prefix reuse: the slot rolls back to lcp
//            (transformer.cpp:3071-3089).
// Output: per token, per layer, attn_out[n_heads*head_dim] float32; then
// int32 seq_pos, compactions.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "jx_engine.hpp"

static bool rd(FILE* f, void* p, size_t n) { return fread(p, 1, n, f) == n; }

int main(int argc, char** argv) {
    if (argc != 3) {
        fprintf(stderr, "usage: %s script.bin out.bin\n", argv[0]);
        return 2;
    }
    FILE* in = fopen(argv[1], "rb");
    FILE* out = fopen(argv[2], "wb");
    if (!in || !out) return 2;
    int32_t h[8];
    float rope_base = 0.0f;
    if (!rd(in, h, sizeof h) || !rd(in, &rope_base, 4)) return 2;
    const int L = h[0], H = h[1], HK = h[2], HD = h[3], cap = h[4], neox = h[5], dtype = h[6];
    const int n_ops = h[7];

    jx::Hyper hp;
    hp.n_layers = L;
    hp.n_heads = H;
    hp.n_kv_heads = HK;
    hp.q_dim = H * HD;
    hp.kv_dim = HK * HD;
    hp.kv_cache_capacity = cap;
    hp.rope_neox = neox != 0;
    jx::DeviceKVCache cache(hp, 2, static_cast<jx_dtype>(dtype));
    if (cache.status()) {
        fprintf(stderr, "cache: %s\n", jx_last_error_string());
        return 1;
    }
    jx::KVCacheSlot slot;
    // slot 1 of 2, so the slot id reaches the library
    if (slot.init(1, cache)) return 1;
    jx::AttentionBlock attn(cache);
    if (attn.status()) return 1;
    std::vector<jx::LayerAttn> layers(L);
    for (int l = 0; l < L; ++l) {
        layers[l].head_dim = HD;
        layers[l].rope_dim = HD;
        layers[l].rope_freq_base = rope_base;
        layers[l].kv_source_layer = l;
    }
    std::vector<float> q(H * HD), k(HK * HD), v(HK * HD), o(H * HD);
    uint32_t token = 0;
    for (int op = 0; op < n_ops; ++op) {
        int32_t code = 0;
        if (!rd(in, &code, 4)) return 2;
        if (code == 2) {
            int32_t lcp = 0;
            if (!rd(in, &lcp, 4) || slot.rollback(static_cast<uint32_t>(lcp))) return 1;
            continue;
        }
        // forward_token: compact on overflow, position, history (:2373-2376)
        if (slot.seq_pos >= hp.kv_cache_capacity) {
            if (slot.compact(hp.kv_cache_capacity / 2)) {
                fprintf(stderr, "compact: %s\n", jx_last_error_string());
                return 1;
            }
        }
        const uint32_t pos = slot.seq_pos;
        slot.token_history.push_back(token++);
        for (int l = 0; l < L; ++l) {
            if (!rd(in, q.data(), q.size() * 4) || !rd(in, k.data(), k.size() * 4) ||
                !rd(in, v.data(), v.size() * 4))
                return 2;
            if (attn.forward(slot, layers[l], q.data(), k.data(), v.data(), o.data(), pos)) {
                fprintf(stderr, "forward: %s\n", jx_last_error_string());
                return 1;
            }
            fwrite(o.data(), 4, o.size(), out);
        }
        slot.seq_pos++;  // transformer.cpp:2792
    }
    const int32_t tail[2] = {static_cast<int32_t>(slot.seq_pos),
                             static_cast<int32_t>(slot.compactions)};
    fwrite(tail, 4, 2, out);
    fclose(out);
    fclose(in);
    return 0;
}
