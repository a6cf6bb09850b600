// Per-token latency of the attention block through jx_engine.hpp, driven the
// way MoETransformerEngine::forward_token drives its inline block
// (src/transformer.cpp:2497-2567, 2792): for every layer the engine's host
// q/k/v vectors go in, the block runs, and attn_out comes back to the host
// before the next layer (the CPU's Wo matmul, :2572, needs it), so each layer
// is one synchronous round trip.  The wall time of one token over all layers
// is the counterpart of the reference's attention_ms (:2499, 2567).
//
// One slot whose cache holds T-1 rows (seeded N(0,1), generated on the
// device); every token appends at T-1 and attends over T rows, then the slot
// rolls back to T-1 so that every token does the same work.
//
// usage: engine_latency dtype(0 f32|1 bf16|2 f16) T n_layers n_heads n_kv_heads
//                       head_dim neox rope_base tokens warmup staging(pinned|copies)
// Prints one JSON object: tokens, ms_per_token (mean), p50/p90 of the tokens,
// us_per_layer.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "jx_engine.hpp"

int main(int argc, char** argv) {
    if (argc != 12) {
        fprintf(stderr,
                "usage: %s dtype T n_layers n_heads n_kv_heads head_dim neox rope_base tokens "
                "warmup pinned|copies\n",
                argv[0]);
        return 2;
    }
    const int dtype = std::atoi(argv[1]);
    const uint32_t T = static_cast<uint32_t>(std::atol(argv[2]));
    const int L = std::atoi(argv[3]), H = std::atoi(argv[4]), HK = std::atoi(argv[5]);
    const int HD = std::atoi(argv[6]), neox = std::atoi(argv[7]);
    const float rope_base = static_cast<float>(std::atof(argv[8]));
    const int tokens = std::atoi(argv[9]), warmup = std::atoi(argv[10]);
    const jx::Staging staging =
        std::string(argv[11]) == "copies" ? jx::Staging::DeviceCopies : jx::Staging::PinnedHost;
    if (T < 1 || L < 1 || H < 1 || HK < 1 || HD < 1 || tokens < 1 || warmup < 0) return 2;

    jx::Hyper hp;
    hp.n_layers = L;
    hp.n_heads = H;
    hp.n_kv_heads = HK;
    hp.q_dim = H * HD;
    hp.kv_dim = HK * HD;
    hp.kv_cache_capacity = T;
    hp.rope_neox = neox != 0;
    jx::DeviceKVCache cache(hp, 1, static_cast<jx_dtype>(dtype));
    if (cache.status()) {
        fprintf(stderr, "cache: %s\n", jx_last_error_string());
        return 1;
    }
    const uint32_t rows = T - 1;
    jx::KVCacheSlot slot;
    if (slot.init(0, cache)) return 1;  // KVCacheSlot::init: cleared rows, seq_pos 0
    if (jx_kv_fill_normal(cache.handle(), &rows, 0x6a78616900000001ull, nullptr) ||
        cudaDeviceSynchronize() != cudaSuccess) {
        fprintf(stderr, "fill: %s\n", jx_last_error_string());
        return 1;
    }
    slot.seq_pos = rows;
    jx::AttentionBlock attn(cache, nullptr, staging);
    if (attn.status()) {
        fprintf(stderr, "block: %s\n", jx_last_error_string());
        return 1;
    }
    std::vector<jx::LayerAttn> layers(L);
    for (int l = 0; l < L; ++l) {
        layers[l].head_dim = HD;
        layers[l].rope_dim = HD;
        layers[l].rope_freq_base = rope_base;
        layers[l].kv_source_layer = l;
    }
    // the engine's per-layer vectors (pageable host memory, as in forward_token)
    std::vector<float> q(static_cast<size_t>(H) * HD), k(static_cast<size_t>(HK) * HD),
        v(static_cast<size_t>(HK) * HD), o(static_cast<size_t>(H) * HD);
    uint64_t x = 12345;
    auto rnd = [&x]() {
        x = x * 6364136223846793005ull + 1442695040888963407ull;
        return static_cast<float>((x >> 40) & 0xFFFF) / 32768.0f - 1.0f;
    };
    for (float& f : q) f = rnd();
    for (float& f : k) f = rnd();
    for (float& f : v) f = rnd();

    std::vector<double> ms;
    ms.reserve(tokens);
    for (int t = 0; t < warmup + tokens; ++t) {
        const auto t0 = std::chrono::steady_clock::now();
        const uint32_t pos = slot.seq_pos;
        for (int l = 0; l < L; ++l) {
            if (attn.forward(slot, layers[l], q.data(), k.data(), v.data(), o.data(), pos)) {
                fprintf(stderr, "forward: %s\n", jx_last_error_string());
                return 1;
            }
        }
        slot.seq_pos++;  // transformer.cpp:2792
        const auto t1 = std::chrono::steady_clock::now();
        if (slot.rollback(rows)) return 1;  // same work for every token
        if (t >= warmup) ms.push_back(std::chrono::duration<double, std::milli>(t1 - t0).count());
    }
    int code = 0;
    if (jx_kv_check_device_error(cache.handle(), &code, nullptr) || code) {
        fprintf(stderr, "device error %d: %s\n", code, jx_last_error_string());
        return 1;
    }
    double sum = 0.0;
    for (double m : ms) sum += m;
    std::vector<double> sorted = ms;
    std::sort(sorted.begin(), sorted.end());
    const double mean = sum / ms.size();
    printf("{\"tokens\": %d, \"ms_per_token\": %.5f, \"p50_ms\": %.5f, \"p90_ms\": %.5f, "
           "\"us_per_layer\": %.3f, \"staging\": \"%s\"}\n",
           tokens, mean, sorted[sorted.size() / 2], sorted[(sorted.size() * 9) / 10],
           mean * 1e3 / L, staging == jx::Staging::PinnedHost ? "pinned" : "copies");
    return 0;
}
