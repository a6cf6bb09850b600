// jx_internal.h -- types shared by the host library and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace jx {

// One (step sequence, call layer) pair of a decode step.  Pairs are stored in
// step order (sequence-major); `off` is the prefix sum of n_kv*len over the
// pairs before it, i.e. the pair's first index in the flattened
// (pair, kv head, attended row) space the persistent CTAs split evenly.
struct PairRow {
    long long off;
    int seq;          // cache sequence
    int io;           // row of q/k/v/out: step_seq * n_call_layers + call_layer
    int cache_layer;  // kv_source_layer: cache layer read (and appended)
    int row0;         // first attended local cache row
    int len;          // attended local rows (0 only in partial mode)
    int append_row;   // local row receiving this step's k/v, or -1
    int rope_row;     // row of the cos/sin table for (rope config, pos)
    int rope_half;    // rotated pairs per head = min(head_dim, rope_dim) / 2
    // A prefill block: nq > 1 consecutive tokens of one sequence share the
    // pair (their rows stream once for all of them).  Token j has q/out row
    // io + j*io_step, position row tok_row0 + j, cos/sin row rope_row + j, and
    // attends local rows [max(row0, tok_row0 + j - window + 1), tok_row0 + j]
    // (window 0: from row0).  nq <= 1: an ordinary pair.
    int nq;
    int io_step;
    int tok_row0;
    int window;
    int pad[2];
};
static_assert(sizeof(PairRow) == 64, "PairRow layout");

struct DecodeArgs {
    const PairRow* pairs;
    const int* cta_pair;  // per CTA: the pair holding its first row (or null: binary search)
    const long long* cta_begin;  // [P+1] slice boundaries, or null: CTA c takes [cN/P, (c+1)N/P)
    const int* seg_owner;        // with cta_begin: [segments][2] first and last CTA of a segment
    int n_pairs;
    int n_kv;       // kv heads
    int G;          // query heads per kv head
    int n_heads;
    long long total;  // flattened rows
    const float* q;
    const float* k_in;
    const float* v_in;
    float* out;
    long long q_stride;   // floats between (seq, layer) rows of q/out
    long long kv_stride;  // floats between (seq, layer) rows of k/v
    void* k_cache;
    void* v_cache;
    long long seq_stride;    // cache elements between sequences
    long long layer_stride;  // cache elements between layers
    long long row_stride;    // cache elements between rows
    const float2* rope;      // rows of head_dim/2 (cos, sin) pairs
    float scale;
    float softcap;
    float inv_softcap;
    int neox;
    float* scratch;  // split partials, (P + n_segments) slots
    int* counters;   // per segment arrival counters (self-resetting)
    float* part_out; // partial mode output, or null
    int* err;        // device error word
    int n_stages;
    int n_consumers; // consumer warps that take tiles (1..4), a multiple of the warps per
                     // tile (kv heads per tile row); n_stages % (warps / per tile) == 0
    // extents, used by the optional device-side checks (JX_DEVICE_CHECKS builds)
    long long n_io;          // rows of q/k/v/out
    long long cache_elems;   // elements of K (and of V)
    long long scratch_floats;
    long long n_segments;
    int n_rope_rows;
    int capacity;
    int n_cache_layers;
    int n_cache_seqs;
    int smem_bytes;          // dynamic shared memory of the launch
    int* dbg;                // [8]: first failed check (code, block, values)
    int q_bulk;              // 1: q rows and the rope table allow 16-byte bulk copies
                             // (the producer prefetches each piece's q into shared memory)
    int skip_append;         // 1: rows were appended by an earlier launch (prefill)
    int test_wait_cta;       // > 0: CTA test_wait_cta-1 makes one bounded wait on a barrier
                             // nothing arrives at (exercises the wait-timeout error path)
    long long wait_limit;    // SM cycles after which a pipeline wait gives up
};

// Host-side launch request for one fused decode launch.
struct DecodeLaunch {
    DecodeArgs args;
    const CUtensorMap* tmK;
    const CUtensorMap* tmV;
    int head_dim;
    int gp;      // padded group size (1, 2, 4, 8)
    int kp;      // kv heads per tile row (kv_pack)
    int dtype;   // 0 f32, 1 bf16, 2 f16 trunc
    int grid;
    int stages;
    int pdl;     // launch with programmatic stream serialisation
    cudaStream_t stream;
};

// One work item of the tensor-core prefill kernel: `ntok` consecutive prompt
// tokens of one sequence (local cache rows tok_row0 ..), one layer, one kv
// head.  Token j has q/out row io0 + j*io_step and cos/sin row rope_row0 + j,
// and attends local rows [max(row0, tok_row0 + j - window + 1), tok_row0 + j]
// (window 0: from row0).  The kernel streams cache rows [kv_lo, kv_lo +
// n_tiles*BN) of the item.
struct PrefillTile {
    int seq, cache_layer, kvh, io0;
    int io_step, tok_row0, ntok, row0;
    int window, rope_row0, rope_half, kv_lo;
    int n_tiles;
    int pad[3];
};
static_assert(sizeof(PrefillTile) == 64, "PrefillTile layout");

struct PrefillArgs {
    const PrefillTile* tiles;
    const int* cta_first;  // CTA b runs tiles [cta_first[b], cta_first[b + 1])
    int n_items;
    int neox;
    int q_vec;  // 1: q rows start 16-byte aligned (16-byte loads)
    const float* q;
    float* out;
    long long q_stride;
    const float2* rope;  // rows of head_dim/2 (cos, sin) pairs
    float scale;
    float softcap;
    float inv_softcap;
    int* err;
    int* dbg;
    long long wait_limit;
};

// Tensor-core prefill for (head_dim, cache dtype, query group) -- 16-bit
// caches, head_dim 64/128, groups 1/2/4/8; cache rows per K/V tile of the
// kernel for a head_dim (the TMA box height); launch of one grid.
bool prefill_tc_supported(int head_dim, int dtype, int G);
int prefill_tc_rows(int head_dim);
cudaError_t prefill_tc_launch(const PrefillArgs& a, const CUtensorMap* tmK, const CUtensorMap* tmV,
                              int head_dim, int dtype, int G, int grid, cudaStream_t stream);

// kv heads that share one tile row: 2 for 16-bit caches whose kv-head rows
// are under 256 bytes (head_dim 32, 64) when the heads pair up evenly and the
// query group needs no padding, 1 otherwise.  With 2, each tile row the TMA
// fetches is one contiguous run over two kv heads (256 bytes at head_dim 64);
// separate 128-byte runs at a 1 KB row stride cost ~1.5x their bytes in DRAM
// traffic on B200.  A segment then covers kp kv heads and kp*G query heads,
// and each tile goes to kp consumer warps, one per kv head.
inline int kv_pack(int head_dim, int esz, unsigned n_kv, unsigned G, int gp) {
    return (esz == 2 && head_dim * esz < 256 && n_kv % 2 == 0 && static_cast<int>(G) == gp) ? 2 : 1;
}
// Dynamic shared memory bytes of the kernel for (head_dim, gp, kp, dtype,
// stages), or -1 when that combination is not compiled.
int decode_smem_bytes(int head_dim, int gp, int kp, int dtype, int stages);
// Resident CTAs per SM for that configuration (occupancy calculator).
int decode_ctas_per_sm(int head_dim, int gp, int kp, int dtype, int stages);
// Launches; returns a cudaError_t.
cudaError_t decode_launch(const DecodeLaunch& L);
// Consumer warps for a ring of `stages` with `split` warps per tile.
int consumers_for(int stages, int split);
// Default ring depth and CTAs per SM for one kernel configuration.
void default_shape(int hd, int gp, int kp, int dtype, int* stages, int* cps);
// SM cycles of a bounded pipeline wait for a limit in milliseconds (0: default).
long long wait_limit_cycles(int ms);
// Sets the calling thread's jx_last_error_string() message.
void set_last_error(const char* msg);
// (cos, sin) of every rotated pair at `pos`, as apply_rope computes them;
// writes `width` entries (zeros past the rotated pairs).
void rope_row(uint32_t head_dim, uint32_t rope_dim, uint32_t pos, float base, float yarn_scale,
              bool neox, const float* rope_freqs, float2* out, int width);

}  // namespace jx
