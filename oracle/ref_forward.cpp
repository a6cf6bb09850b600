// ref_forward.cpp -- TEST INFRASTRUCTURE ONLY (a parity checker's fixture source).
//
// Runs the reference engine's own MoETransformerEngine::forward_token
// (src/transformer.cpp, built from the reference's sources by oracle/Makefile)
// on a GGUF model for a few tokens of slot 0, then writes what the engine left
// in that slot's KVCacheSlot (include/transformer.h:121-139): its seq_pos and
// the k_cache / v_cache rows of every layer.  tests/golden/gen_golden.py turns
// the output into a fixture; the CPU tests use it to check the cache layout
// this library mirrors (row `pos` at pos*kv_dim, kv head at kvh*head_dim,
// fp16-truncated values, untouched rows zero) and to compare the C
// restatement of the attention block with the reference's own build on the
// engine's real cache contents.  The product library never uses this file.
//
// usage: ref_forward model.gguf n_tokens out.bin
// out.bin (little-endian): int32 n_layers, n_heads, n_kv_heads, head_dim,
// kv_dim, rope_dim, rope_neox, seq_pos, rows_written, capacity; float32
// rope_freq_base; then per layer the first rows_written rows (seq_pos + 2, so
// that two never-written rows are included) of k_cache, then of v_cache, as
// uint16 [rows_written][kv_dim].
#include <cstdint>
#include <cstdio>
#include <algorithm>
#include <cstdlib>
#include <string>
#include <vector>

#include "transformer.h"

using moe::KVCacheSlot;
using moe::ModelHyperparams;
using moe::MoETransformerEngine;

int main(int argc, char** argv) {
    if (argc != 4) {
        std::fprintf(stderr, "usage: %s model.gguf n_tokens out.bin\n", argv[0]);
        return 2;
    }
    const int n_tokens = std::atoi(argv[2]);
    MoETransformerEngine eng;
    std::string err;
    if (!eng.load_model(argv[1], err)) {
        std::fprintf(stderr, "load_model: %s\n", err.c_str());
        return 1;
    }
    const ModelHyperparams& hp = eng.hparams();
    for (int t = 0; t < n_tokens; ++t) {
        const uint32_t token = static_cast<uint32_t>((7 * t + 3) % std::max<uint32_t>(hp.vocab_size, 1));
        eng.forward_token(token, 0, nullptr, /*compute_logits=*/false);
    }
    KVCacheSlot& slot = eng.get_or_create_slot(0);
    const uint32_t kv_dim = hp.kv_dim;
    const uint32_t capacity =
        slot.k_cache.empty() || kv_dim == 0 ? 0 : static_cast<uint32_t>(slot.k_cache[0].size() / kv_dim);
    const uint32_t rows = std::min<uint32_t>(slot.seq_pos + 2, capacity);
    FILE* f = std::fopen(argv[3], "wb");
    if (!f) return 1;
    const int32_t hdr[10] = {static_cast<int32_t>(hp.n_layers), static_cast<int32_t>(hp.n_heads),
                             static_cast<int32_t>(hp.n_kv_heads), static_cast<int32_t>(hp.head_dim),
                             static_cast<int32_t>(kv_dim), static_cast<int32_t>(hp.rope_dim),
                             hp.rope_neox ? 1 : 0, static_cast<int32_t>(slot.seq_pos),
                             static_cast<int32_t>(rows), static_cast<int32_t>(capacity)};
    std::fwrite(hdr, sizeof hdr, 1, f);
    const float base = hp.rope_freq_base;
    std::fwrite(&base, sizeof base, 1, f);
    for (uint32_t l = 0; l < hp.n_layers; ++l)
        std::fwrite(slot.k_cache[l].data(), sizeof(uint16_t), static_cast<size_t>(rows) * kv_dim, f);
    for (uint32_t l = 0; l < hp.n_layers; ++l)
        std::fwrite(slot.v_cache[l].data(), sizeof(uint16_t), static_cast<size_t>(rows) * kv_dim, f);
    std::fclose(f);
    return 0;
}
