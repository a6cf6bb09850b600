/*
 * Sanitizer run of the CPU oracle (oracle/jx_oracle.c, test infrastructure):
 * built together with it under AddressSanitizer and UndefinedBehaviorSanitizer
 * by tests/test_host_logic.py.  Every exported oracle function runs on small
 * cases whose buffers are allocated to their exact sizes, so any read or write
 * past a cache, q/k/v/out row or score buffer, and any undefined arithmetic,
 * stops the program.  Cases: all 65,536 half and bf16 bit patterns and float
 * edge values through the converters; decode steps over all three cache types,
 * both RoPE styles, head_dim 32/64/128/256, partial rotary dims, frequency
 * factors, soft-cap, sliding windows, shared-KV layers, first and last
 * positions; a position past the cache (refused); compaction.
 * Prints "ok <steps>" and exits 0.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

float jxo_fp16_to_fp32(uint16_t h);
uint16_t jxo_fp32_to_fp16(float f);
float jxo_bf16_to_fp32(uint16_t b);
uint16_t jxo_fp32_to_bf16(float f);
void jxo_rope_cos_sin(uint32_t head_dim, uint32_t rope_dim, uint32_t pos, float freq_base,
                      float yarn_scale, int is_neox, const float* rope_freqs, float* cs);
int jxo_step(void* k_cache, void* v_cache, int dtype, uint32_t capacity, uint32_t row_stride,
             uint32_t n_cache_layers, uint32_t n_seqs, const int32_t* pos,
             uint32_t n_layers, const uint32_t* rope_dim, const float* rope_base,
             const int32_t* is_swa, const int32_t* shares_kv, const uint32_t* kv_source_layer,
             const float* q, const float* k, const float* v, float* out,
             uint32_t q_stride, uint32_t kv_stride, uint32_t n_heads, uint32_t n_kv_heads,
             uint32_t head_dim, float scale, float softcap, uint32_t sliding_window,
             float yarn_scale, int is_neox, const float* rope_freqs);
uint32_t jxo_compact(void* k_seq, void* v_seq, int dtype, uint32_t n_layers, uint32_t capacity,
                     uint32_t row_stride, uint32_t seq_pos, uint32_t keep_recent);

static uint64_t rng_state = 0x6a78616900000001ull;
static uint64_t next(void) {
    rng_state = rng_state * 6364136223846793005ull + 1442695040888963407ull;
    return rng_state;
}
static float rnd(void) { return (float)((next() >> 40) & 0xFFFFFF) / 8388608.0f - 1.0f; }

static float* fbuf(size_t n) {
    float* p = (float*)malloc(n * sizeof(float));
    for (size_t i = 0; i < n; ++i) p[i] = rnd();
    return p;
}

static int failures = 0;
#define CHECK(cond, ...)                                  \
    do {                                                  \
        if (!(cond)) {                                    \
            fprintf(stderr, __VA_ARGS__);                 \
            fputc('\n', stderr);                          \
            ++failures;                                   \
        }                                                 \
    } while (0)

static void converters(void) {
    for (uint32_t b = 0; b < 65536; ++b) {
        volatile float h = jxo_fp16_to_fp32((uint16_t)b);
        volatile float g = jxo_bf16_to_fp32((uint16_t)b);
        (void)jxo_fp32_to_fp16(h);
        (void)jxo_fp32_to_bf16(g);
    }
    const float edge[] = {0.0f, -0.0f, 1.0f, -1.0f, 65504.0f, 65520.0f, 1e-8f, -1e-8f,
                          5.9604645e-8f, 6.1035156e-5f, 3.4028235e38f, -3.4028235e38f,
                          1.17549435e-38f, 1e-45f, INFINITY, -INFINITY, NAN};
    for (size_t i = 0; i < sizeof edge / sizeof edge[0]; ++i) {
        (void)jxo_fp32_to_fp16(edge[i]);
        (void)jxo_fp32_to_bf16(edge[i]);
    }
    float cs[2 * 128 + 2];
    const uint32_t pos[] = {0, 1, 4095, 131071, 4294967295u};
    for (size_t i = 0; i < sizeof pos / sizeof pos[0]; ++i) {
        jxo_rope_cos_sin(256, 256, pos[i], 1e6f, 1.0f, 1, NULL, cs);
        jxo_rope_cos_sin(64, 32, pos[i], 5e5f, 4.0f, 0, NULL, cs);
    }
}

/* One decode step of 2 sequences x 3 layers (layer 2 reads layer 1's cache,
 * layer 0 is sliding-window) with exactly sized buffers. */
static int one_case(int dtype, int neox, uint32_t hd, uint32_t rope_dim, uint32_t n_heads,
                    uint32_t n_kv, uint32_t cap, const int32_t* pos, float softcap,
                    uint32_t window, int with_factors) {
    const uint32_t n_seqs = 2, n_layers = 3, n_cache_layers = 2;
    const uint32_t row_stride = n_kv * hd;
    const size_t esz = dtype == 0 ? 4 : 2;
    const size_t cache_elems = (size_t)n_seqs * n_cache_layers * cap * row_stride;
    unsigned char* kc = (unsigned char*)malloc(cache_elems * esz);
    unsigned char* vc = (unsigned char*)malloc(cache_elems * esz);
    for (size_t i = 0; i < cache_elems * esz; ++i) {
        kc[i] = (unsigned char)(next() >> 56);
        vc[i] = (unsigned char)(next() >> 56);
    }
    if (dtype != 0) { /* keep 16-bit values finite: clear the exponent's top bit */
        for (size_t i = 1; i < cache_elems * esz; i += 2) {
            kc[i] &= 0x3F;
            vc[i] &= 0x3F;
        }
    } else {
        float* kf = (float*)kc;
        float* vf = (float*)vc;
        for (size_t i = 0; i < cache_elems; ++i) {
            kf[i] = rnd();
            vf[i] = rnd();
        }
    }
    const uint32_t q_stride = n_heads * hd, kv_stride = n_kv * hd;
    const size_t rows = (size_t)n_seqs * n_layers;
    float* q = fbuf(rows * q_stride);
    float* k = fbuf(rows * kv_stride);
    float* v = fbuf(rows * kv_stride);
    float* out = fbuf(rows * q_stride);
    const uint32_t rdim = rope_dim;
    float* factors = NULL;
    if (with_factors) {
        factors = fbuf((hd < rdim ? hd : rdim) / 2);
        for (uint32_t i = 0; i < (hd < rdim ? hd : rdim) / 2; ++i) factors[i] = 1.0f + fabsf(factors[i]);
    }
    const uint32_t rope_dims[3] = {rdim, rdim, rdim};
    const float bases[3] = {1e4f, 1e6f, 5e5f};
    const int32_t is_swa[3] = {1, 0, 0};
    const int32_t shares[3] = {0, 0, 1};
    const uint32_t src[3] = {0, 1, 1};
    const int rc = jxo_step(kc, vc, dtype, cap, row_stride, n_cache_layers, n_seqs, pos, n_layers,
                            rope_dims, bases, is_swa, shares, src, q, k, v, out, q_stride,
                            kv_stride, n_heads, n_kv, hd, 1.0f / sqrtf((float)hd), softcap, window,
                            1.0f, neox, factors);
    int finite = 1;
    if (rc == 0)
        for (size_t i = 0; i < rows * q_stride; ++i) finite &= isfinite(out[i]) ? 1 : 0;
    if (rc == 0) {
        const uint32_t keep = cap / 4;
        const uint32_t n = jxo_compact(kc, vc, dtype, n_cache_layers, cap, row_stride,
                                       (uint32_t)pos[0] + 1, keep);
        CHECK(n <= (uint32_t)pos[0] + 1, "compact grew the sequence");
    }
    free(kc);
    free(vc);
    free(q);
    free(k);
    free(v);
    free(out);
    free(factors);
    CHECK(rc != 0 || finite, "non-finite output (dtype %d hd %u)", dtype, hd);
    return rc;
}

int main(void) {
    converters();
    int steps = 0;
    const uint32_t hds[] = {32, 64, 128, 256};
    for (int dtype = 0; dtype < 3; ++dtype)
        for (int neox = 0; neox < 2; ++neox)
            for (size_t h = 0; h < 4; ++h) {
                const uint32_t hd = hds[h];
                const uint32_t cap = 40;
                const int32_t pos_a[2] = {0, 39};   /* first and last row */
                const int32_t pos_b[2] = {17, 33};
                CHECK(one_case(dtype, neox, hd, hd, 8, 2, cap, pos_a, 0.0f, 0, 0) == 0,
                      "step failed (a)");
                CHECK(one_case(dtype, neox, hd, hd / 2, 7, 1, cap, pos_b, 30.0f, 8, neox) == 0,
                      "step failed (b)");
                CHECK(one_case(dtype, neox, hd, hd + 32, 4, 4, cap, pos_b, 0.0f, 64, 0) == 0,
                      "step failed (c)");
                steps += 3;
            }
    /* a position past the cache is refused without touching memory */
    const int32_t bad[2] = {3, 40};
    CHECK(one_case(0, 1, 64, 64, 8, 2, 40, bad, 0.0f, 0, 0) != 0, "position past the cache accepted");
    if (failures) return 1;
    printf("ok %d\n", steps);
    return 0;
}
