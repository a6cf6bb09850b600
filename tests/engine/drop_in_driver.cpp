// Drives jx_engine.hpp the way MoETransformerEngine::forward_token drives its
// KVCacheSlot and attention block (src/transformer.cpp:2366-2375, 2497-2567,
// 2792), on host vectors read from a script file; writes every layer's
// attn_out.  The optional third argument picks the block's staging
// (jx::Staging::PinnedHost by default, "copies" for DeviceCopies).
// tests/test_gpu_engine.py replays the script through the CPU
// oracle and compares.
//
// Script (little-endian): int32 n_layers, n_heads, n_kv_heads, head_dim,
// capacity, neox, dtype, n_slots, n_ops; float32 rope_base; then n_ops ops:
//   int32 1, int32 slot, then per layer q[n_heads*head_dim],
//            k[n_kv*head_dim], v[n_kv*head_dim] -- one token of one slot
//            through all layers (AttentionBlock::forward);
//   int32 2, int32 slot, int32 lcp -- prefix reuse: the slot rolls back to
//            lcp (transformer.cpp:3071-3089);
//   int32 3, int32 m, int32 slot[m], then per layer q[m][..], k[m][..],
//            v[m][..] -- one token of each listed slot, one call per layer
//            (AttentionBlock::forward_batch);
//   int32 4, int32 slot, int32 n, then per layer q[n][..], k[n][..], v[n][..]
//            -- n prompt tokens of one slot, one call per layer
//            (AttentionBlock::forward_prompt).
// Rows are n_heads*head_dim (q) and n_kv*head_dim (k, v) floats, the engine's
// q_dim and kv_dim.  Output: the attn_out rows of every op in op, layer, row
// order, float32; then int32 seq_pos, compactions per slot.
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "jx_engine.hpp"

static bool rd(FILE* f, void* p, size_t n) { return fread(p, 1, n, f) == n; }

int main(int argc, char** argv) {
    if (argc != 3 && argc != 4) {
        fprintf(stderr, "usage: %s script.bin out.bin [pinned|copies]\n", argv[0]);
        return 2;
    }
    const jx::Staging staging = argc == 4 && std::string(argv[3]) == "copies"
                                    ? jx::Staging::DeviceCopies
                                    : jx::Staging::PinnedHost;
    FILE* in = fopen(argv[1], "rb");
    FILE* out = fopen(argv[2], "wb");
    if (!in || !out) return 2;
    int32_t h[9];
    float rope_base = 0.0f;
    if (!rd(in, h, sizeof h) || !rd(in, &rope_base, 4)) return 2;
    const int L = h[0], H = h[1], HK = h[2], HD = h[3], cap = h[4], neox = h[5], dtype = h[6];
    const int n_slots = h[7], n_ops = h[8];

    jx::Hyper hp;
    hp.n_layers = L;
    hp.n_heads = H;
    hp.n_kv_heads = HK;
    hp.q_dim = H * HD;
    hp.kv_dim = HK * HD;
    hp.kv_cache_capacity = cap;
    hp.rope_neox = neox != 0;
    jx::DeviceKVCache cache(hp, n_slots, static_cast<jx_dtype>(dtype));
    if (cache.status()) {
        fprintf(stderr, "cache: %s\n", jx_last_error_string());
        return 1;
    }
    std::vector<jx::KVCacheSlot> slots(n_slots);
    for (int s = 0; s < n_slots; ++s)
        if (slots[s].init(s, cache)) return 1;
    jx::AttentionBlock attn(cache, nullptr, staging);
    if (attn.status()) return 1;
    std::vector<jx::LayerAttn> layers(L);
    for (int l = 0; l < L; ++l) {
        layers[l].head_dim = HD;
        layers[l].rope_dim = HD;
        layers[l].rope_freq_base = rope_base;
        layers[l].kv_source_layer = l;
    }
    const size_t qd = hp.q_dim, kd = hp.kv_dim;
    std::vector<float> q, k, v, o;
    // reads one layer's n rows of q, k, v
    auto read_rows = [&](size_t n) {
        q.resize(n * qd);
        k.resize(n * kd);
        v.resize(n * kd);
        o.resize(n * qd);
        return rd(in, q.data(), q.size() * 4) && rd(in, k.data(), k.size() * 4) &&
               rd(in, v.data(), v.size() * 4);
    };
    // forward_token: compact on overflow before the token (:2373-2375)
    auto make_room = [&](jx::KVCacheSlot& s) {
        if (s.seq_pos >= hp.kv_cache_capacity && s.compact(hp.kv_cache_capacity / 2)) {
            fprintf(stderr, "compact: %s\n", jx_last_error_string());
            return false;
        }
        return true;
    };
    uint32_t token = 0;
    for (int op = 0; op < n_ops; ++op) {
        int32_t code = 0, sid = 0;
        if (!rd(in, &code, 4)) return 2;
        if (code == 1 || code == 2 || code == 4) {
            if (!rd(in, &sid, 4) || sid < 0 || sid >= n_slots) return 2;
        }
        if (code == 2) {
            int32_t lcp = 0;
            if (!rd(in, &lcp, 4) || slots[sid].rollback(static_cast<uint32_t>(lcp))) return 1;
        } else if (code == 1) {
            jx::KVCacheSlot& s = slots[sid];
            if (!make_room(s)) return 1;
            const uint32_t pos = s.seq_pos;
            s.token_history.push_back(token++);
            for (int l = 0; l < L; ++l) {
                if (!read_rows(1)) return 2;
                if (attn.forward(s, layers[l], q.data(), k.data(), v.data(), o.data(), pos)) {
                    fprintf(stderr, "forward: %s\n", jx_last_error_string());
                    return 1;
                }
                fwrite(o.data(), 4, o.size(), out);
            }
            s.seq_pos++;  // transformer.cpp:2792
        } else if (code == 3) {
            int32_t m = 0;
            if (!rd(in, &m, 4) || m <= 0 || m > n_slots) return 2;
            std::vector<int32_t> ids(m);
            if (!rd(in, ids.data(), 4 * m)) return 2;
            std::vector<jx::KVCacheSlot*> batch(m);
            for (int i = 0; i < m; ++i) {
                if (ids[i] < 0 || ids[i] >= n_slots) return 2;
                batch[i] = &slots[ids[i]];
                if (!make_room(*batch[i])) return 1;
                batch[i]->token_history.push_back(token++);
            }
            for (int l = 0; l < L; ++l) {
                if (!read_rows(m)) return 2;
                if (attn.forward_batch(batch.data(), m, layers[l], q.data(), k.data(), v.data(),
                                       o.data())) {
                    fprintf(stderr, "forward_batch: %s\n", jx_last_error_string());
                    return 1;
                }
                fwrite(o.data(), 4, o.size(), out);
            }
            for (jx::KVCacheSlot* s : batch) s->seq_pos++;
        } else if (code == 4) {
            int32_t n = 0;
            if (!rd(in, &n, 4) || n <= 0) return 2;
            jx::KVCacheSlot& s = slots[sid];
            const uint32_t pos0 = s.seq_pos;
            for (int t = 0; t < n; ++t) s.token_history.push_back(token++);
            for (int l = 0; l < L; ++l) {
                if (!read_rows(n)) return 2;
                if (attn.forward_prompt(s, layers[l], q.data(), k.data(), v.data(), o.data(), n,
                                        pos0)) {
                    fprintf(stderr, "forward_prompt: %s\n", jx_last_error_string());
                    return 1;
                }
                fwrite(o.data(), 4, o.size(), out);
            }
            s.seq_pos += n;
        } else {
            return 2;
        }
    }
    for (const jx::KVCacheSlot& s : slots) {
        const int32_t tail[2] = {static_cast<int32_t>(s.seq_pos),
                                 static_cast<int32_t>(s.compactions)};
        fwrite(tail, 4, 2, out);
    }
    fclose(out);
    fclose(in);
    return 0;
}
