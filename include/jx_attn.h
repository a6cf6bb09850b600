/*
 * jx_attn.h -- C ABI of the B200 decode-attention library (libjxattn.so).
 *
 * Replaces jxai's per-token attention step: the RoPE rotation, the KV-cache
 * append and the grouped-query decode attention that
 * MoETransformerEngine::forward_token runs inline for every layer
 * (src/transformer.cpp:2497-2567), and the KVCacheSlot cache that step reads
 * and writes (include/transformer.h:115-131, src/transformer.cpp:13-66).
 *
 * Conventions
 *   - Every entry point returns 0 (JX_OK) or a negative JX_ERR_* status; no
 *     exception, abort or device trap crosses this boundary.  The message of
 *     the last failure on the calling thread is jx_last_error_string().
 *   - All argument checks happen on the host before anything is launched.
 *   - Device work is asynchronous on the caller's CUDA stream (`stream` is a
 *     cudaStream_t; NULL is the legacy default stream).  Calls on one jx_kv
 *     must be ordered on one stream, as forward_token is serialised by
 *     engine_mtx_ (src/transformer.cpp:2361).  Distinct handles are independent.
 *   - q/k/v/out and partial buffers are caller-owned pointers to the cache's
 *     device memory or to pinned (page-locked) host memory -- the kernel then
 *     reads the inputs and writes the output over PCIe itself, with no copy
 *     of its own; pageable host memory is refused (JX_ERR_INVALID).  Position
 *     and descriptor arrays are HOST pointers.
 *   - There is no CPU implementation behind this header: without a B200 the
 *     library reports JX_ERR_CUDA.
 */
#ifndef JX_ATTN_H
#define JX_ATTN_H

#include <stdint.h>

#if defined(__GNUC__)
#define JX_API __attribute__((visibility("default")))
#else
#define JX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
    JX_OK = 0,
    JX_ERR_INVALID = -1,     /* bad argument (null pointer, shape mismatch, ...) */
    JX_ERR_CUDA = -2,        /* a CUDA runtime/driver call failed */
    JX_ERR_NOMEM = -3,       /* device or pinned-host allocation failed */
    JX_ERR_UNSUPPORTED = -4, /* shape outside the compiled kernel set */
    JX_ERR_RANGE = -5,       /* position outside the cache (caller must compact first) */
    JX_ERR_DEVICE = -6,      /* a kernel reported a device-side error (bounded wait ran out) */
    JX_ERR_TIMEOUT = -7,     /* a sharded step did not complete in time (or a peer rank was
                                not alive); its work stays queued and the communicator is
                                untouched: whether to call ncclCommAbort is the caller's choice */
    JX_ERR_COMM = -8         /* an NCCL call failed or NCCL is not available */
};

/* KV element type.  JX_F16_TRUNC is jxai's native cache: fp16 written with the
 * truncating fp32_to_fp16 of src/quant.cpp:906-925 (not round-to-nearest).
 * JX_BF16 rounds with fp32_to_bf16 (src/quant.cpp:934-939).  JX_F32 stores the
 * rotated values unchanged. */
typedef enum { JX_F32 = 0, JX_BF16 = 1, JX_F16_TRUNC = 2 } jx_dtype;

typedef struct jx_kv jx_kv;

/* Replaces KVCacheSlot::init (src/transformer.cpp:13-23) for n_seqs slots.
 * Device layout: K and V each [n_seqs][n_layers][capacity][row_stride], the
 * row layout of KVCacheSlot::k_cache[layer] (row t at t*row_stride, kv head
 * kvh at kvh*head_dim; transformer.cpp:2514-2515, 2540). */
typedef struct {
    uint32_t n_seqs;     /* independent sequences (slots) held by this handle */
    uint32_t n_layers;   /* cache layers = hp.n_layers */
    uint32_t capacity;   /* rows per (sequence, layer) = hp.kv_cache_capacity */
    uint32_t row_stride; /* elements per row = hp.kv_dim, the max kv_dim over layers */
    int32_t dtype;       /* jx_dtype */
    int32_t device;      /* CUDA device ordinal */
    uint32_t pos_base;   /* global position of local row 0: a shard of one long
                            sequence holds positions [pos_base, pos_base+capacity);
                            0 for an ordinary cache */
} jx_kv_desc;

/* Per-layer attention fields of LayerDenseWeights (include/transformer.h:50-58). */
typedef struct {
    uint32_t head_dim;        /* lw.head_dim */
    uint32_t rope_dim;        /* lw.rope_dim */
    float rope_freq_base;     /* lw.rope_freq_base (the _swa base on SWA layers) */
    uint32_t kv_source_layer; /* lw.kv_source_layer: cache layer read (and written) */
    int32_t is_swa;           /* lw.is_swa: attend the last sliding_window rows only */
    int32_t shares_kv;        /* lw.shares_kv: do not append, read kv_source_layer */
    const float* rope_freqs;  /* HOST; Neox frequency factors (rope_freqs.weight) with
                                 >= rope_dim/2 entries, or NULL; ignored on SWA
                                 layers and in interleaved mode (transformer.cpp:2501-2503, 89) */
} jx_layer_desc;

/* One decode step: for each listed sequence s and each call layer l, rotate
 * q[s][l] and k[s][l] at position pos[s], append k/v at that position of cache
 * layer layers[l].kv_source_layer, and write attention over the attended rows
 * to out[s][l].  Same math as transformer.cpp:2497-2566. */
typedef struct {
    uint32_t n_heads;         /* hp.n_heads */
    uint32_t n_kv_heads;      /* hp.n_kv_heads */
    uint32_t n_seqs;          /* sequences in this step */
    const int32_t* seq_ids;   /* HOST [n_seqs] cache sequence of each step row, or NULL
                                 for sequences 0..n_seqs-1 */
    const int32_t* pos;       /* HOST [n_seqs] position written this step (slot.seq_pos) */
    const float* q;           /* DEVICE or pinned HOST [n_seqs][n_layers][q_stride] fp32
                                 (not modified) */
    const float* k;           /* DEVICE or pinned HOST [n_seqs][n_layers][kv_stride] fp32 */
    const float* v;           /* DEVICE or pinned HOST [n_seqs][n_layers][kv_stride] fp32 */
    float* out;               /* DEVICE or pinned HOST [n_seqs][n_layers][q_stride] fp32
                                 (attn_out) */
    uint32_t q_stride;        /* >= n_heads*head_dim (hp.q_dim for the engine's q vector) */
    uint32_t kv_stride;       /* >= n_kv_heads*head_dim */
    float scale;              /* 1/sqrt(head_dim), or 1.0 for gemma4 (transformer.cpp:2525) */
    float softcap;            /* hp.attn_logit_softcapping; 0 = off */
    uint32_t sliding_window;  /* hp.sliding_window (used on is_swa layers) */
    float yarn_scale;         /* hp.yarn_scale */
    int32_t rope_neox;        /* hp.rope_neox: 1 rotate-half, 0 interleaved pairs */
} jx_step_args;

/* ---- cache lifetime: KVCacheSlot (include/transformer.h:115-131) ---------- */

/* KVCacheSlot::init (transformer.cpp:13-23): allocates and zero-fills. */
JX_API int jx_kv_create(const jx_kv_desc* desc, jx_kv** out);
JX_API int jx_kv_destroy(jx_kv* kv);
/* KVCacheSlot::clear (transformer.cpp:25-30): zero the rows, seq_pos = 0. */
JX_API int jx_kv_clear(jx_kv* kv, uint32_t seq, void* stream);
/* KVCacheSlot::rollback (transformer.cpp:32-39): seq_pos = min(seq_pos, new_seq_pos). */
JX_API int jx_kv_rollback(jx_kv* kv, uint32_t seq, uint32_t new_seq_pos);
/* KVCacheSlot::compact (transformer.cpp:41-66): keep rows [0,4) and the last
 * keep_recent rows of every layer; seq_pos becomes 4+keep_recent.  No-op when
 * seq_pos <= 4+keep_recent. */
JX_API int jx_kv_compact(jx_kv* kv, uint32_t seq, uint32_t keep_recent, void* stream);
/* KVCacheSlot::seq_pos accessors (the engine reads it as `pos`, transformer.cpp:2376,
 * and increments it after the layers, :2792). */
JX_API int jx_kv_get_seq_pos(const jx_kv* kv, uint32_t seq, uint32_t* seq_pos);
JX_API int jx_kv_set_seq_pos(jx_kv* kv, uint32_t seq, uint32_t seq_pos);
JX_API int jx_kv_get_desc(const jx_kv* kv, jx_kv_desc* desc);

/* Direct row access (integration and test plumbing; replaces indexing
 * slot.k_cache[layer] / slot.v_cache[layer]).  which: 0 = K, 1 = V.
 * buf may be host or device memory; to_cache = 1 copies buf -> cache. */
JX_API int jx_kv_copy_rows(jx_kv* kv, uint32_t seq, uint32_t layer, int which, uint32_t row0,
                    uint32_t n_rows, void* buf, int to_cache, void* stream);
/* Device address of row 0 of (seq, layer) for K (which=0) or V (which=1). */
JX_API int jx_kv_layer_ptr(jx_kv* kv, uint32_t seq, uint32_t layer, int which, void** ptr);

/* ---- the hot path: transformer.cpp:2497-2567 ------------------------------ */

/* One fused launch per step (two when a shares_kv layer reads a cache layer
 * that another layer of the same call appends to): RoPE + append + split-KV
 * decode attention + log-sum-exp merge, all layers and sequences together.
 * Requires every attended position to be local (pos_base <= window start and
 * pos < pos_base + capacity); otherwise JX_ERR_RANGE. */
JX_API int jx_attn_step(jx_kv* kv, const jx_layer_desc* layers, uint32_t n_layers,
                 const jx_step_args* args, void* stream);

/* Multi-token prefill: many tokens per call (the reference feeds a prompt
 * token by token through forward_token, transformer.cpp:3092-3095).  Rows of
 * `args` are tokens: args->seq_ids[i] (may repeat; NULL = all sequence 0) and
 * args->pos[i], each (sequence, position) once; q/k/v/out are
 * [n_rows][n_layers][stride] as in a step.  Every row's k and v are rotated
 * and appended first (one launch), then every row attends over its
 * sequence's rows up to its own position (window rules as in a step) --
 * causal attention, the result of running the rows through jx_attn_step one
 * position at a time.  Each row reads its own attended rows (no reuse of a
 * K/V tile across query rows). */
JX_API int jx_attn_prefill(jx_kv* kv, const jx_layer_desc* layers, uint32_t n_layers,
                           const jx_step_args* args, void* stream);

/* Sequence-sharded variant for one long context split across GPUs: the same
 * step over this shard's rows only, writing per (sequence, layer, head) the
 * unnormalised partial [o[0..head_dim), m, l] (head_dim+2 floats, row-major
 * [n_seqs][n_layers][n_heads]) to `partials` (DEVICE) instead of args->out.
 * A shard holding no attended row writes o = 0, m = -inf, l = 0.  The shard
 * that holds pos appends.  args->out is ignored. */
JX_API int jx_attn_step_partial(jx_kv* kv, const jx_layer_desc* layers, uint32_t n_layers,
                         const jx_step_args* args, float* partials, void* stream);

/* Log-sum-exp merge of n_shards partial buffers laid out back to back
 * (shard r at gathered + r*shard_stride floats, each as written by
 * jx_attn_step_partial): out[g*out_stride + h*head_dim + d] for n_groups
 * groups (= n_seqs*n_layers) of n_heads heads. */
JX_API int jx_lse_merge(const float* gathered, uint32_t n_shards, uint64_t shard_stride,
                 uint32_t n_groups, uint32_t n_heads, uint32_t head_dim, float* out,
                 uint32_t out_stride, void* stream);

/* The whole sequence-sharded step over NCCL: jx_attn_step_partial on this
 * rank's shard (the positions [desc.pos_base, desc.pos_base + capacity) of the
 * handle), one ncclAllGather of every rank's partials over `nccl_comm` (an
 * ncclComm_t of all ranks, rank order = shard order), and the log-sum-exp
 * merge into args->out (row stride args->q_stride) -- every rank receives the
 * full output.  All layers of the call share head_dim.  Partial and gather
 * buffers belong to the handle.  NCCL is the process's libnccl.so.2, found at
 * run time (JX_ERR_COMM when absent).
 * timeout_ms = 0: asynchronous on `stream`, like jx_attn_step.  timeout_ms > 0:
 * the call also waits for the step to complete, polling NCCL's asynchronous
 * error; if it has not completed within timeout_ms (a rank that never joins)
 * it returns JX_ERR_TIMEOUT, on an NCCL error JX_ERR_COMM.  The work stays
 * queued and the communicator untouched: aborting it is the caller's
 * decision (ncclCommAbort).  (Callers with their own
 * collectives can still compose jx_attn_step_partial, an all-gather and
 * jx_lse_merge.)  The reference has no multi-GPU path: this extends
 * transformer.cpp:2497-2567 to one context sharded by position. */
JX_API int jx_attn_step_sharded(jx_kv* kv, const jx_layer_desc* layers, uint32_t n_layers,
                                const jx_step_args* args, void* nccl_comm, uint32_t timeout_ms,
                                void* stream);

/* The same step as jx_attn_step for callers that cannot allocate GPU memory.
 * No counterpart in the reference (its cache lives in host vectors).  For an
 * engine that gives all of HBM to its own arena or pool, or a serving loop
 * that must not run into cudaMalloc/cudaFree (and their implicit device
 * synchronisation) mid-token: the caller passes the K and V caches as its own
 * device buffers laid out as jx_kv_create lays them out ([n_seqs][n_layers]
 * [capacity][row_stride] of desc->dtype; desc->device must be current), and
 * the call allocates nothing -- its scratch (split partials, arrival
 * counters, work plan) is one fixed 8 MiB array per GPU, reserved while the
 * library is loaded.  Steps needing more scratch are rejected with
 * JX_ERR_RANGE.  All calls share that array: calls that overlap on the GPU
 * race.  The call cannot be captured into a CUDA graph (it returns
 * JX_ERR_UNSUPPORTED while its stream is capturing: its plan is copied from
 * a host slot that later calls reuse).  All layers of one call share head_dim, and no
 * shares_kv layer may read a cache layer appended in the same call. */
JX_API int jx_attn_step_noalloc(const jx_kv_desc* desc, void* k_cache, void* v_cache,
                                const jx_layer_desc* layers, uint32_t n_layers,
                                const jx_step_args* args, void* stream);

/* Reads and clears the device error word of the no-allocation path on
 * `device` (it synchronises `stream`).  No counterpart in the reference.  The
 * word is shared by every jx_attn_step_noalloc call on that device and keeps
 * the first error since it was last read: *code = 0 when no kernel reported
 * one; otherwise *code is the kernel's error (1: a bounded wait ran out) and
 * the call returns JX_ERR_DEVICE with the site in jx_last_error_string().
 * Call it after the steps it covers have been queued, before relying on
 * their outputs.  Allocates nothing. */
JX_API int jx_noalloc_check_device_error(int device, int* code, void* stream);

/* Options of the no-allocation path (it has no handle; they apply to every
 * later jx_attn_step_noalloc call in the process): "wait_limit_ms" and
 * "test_wait_cta" as in jx_kv_set_option.  No counterpart in the reference. */
JX_API int jx_noalloc_set_option(const char* key, int value);

/* ---- diagnostics, tuning, harness helpers --------------------------------- */

/* Reads and clears the handle's device error word (synchronises the stream).
 * *code = 0 when no kernel reported an error. */
JX_API int jx_kv_check_device_error(jx_kv* kv, int* code, void* stream);

/* Launch options: "ctas_per_sm", "stages" and "grid" override the launch shape
 * (tuning sweeps; 0 restores the default); "pdl" 1 (default) / 0 turns
 * programmatic dependent launch of the decode kernel on / off (with it, a
 * step's launch and set-up overlap the previous kernel's tail; its data
 * accesses still wait for that kernel to complete); "timing" 1 records events around every
 * jx_attn_step / jx_attn_step_partial (not while a stream is being captured);
 * "split_penalty_us" (-1 = default: 5 for fp32 caches, 8 for 16-bit; 0 =
 * uniform slices) is the time an extra piece costs a CTA, used to size the
 * CTAs' slices; "wait_limit_ms" (0 = default, ~4 s) bounds every pipeline
 * wait inside the kernel, after which the CTA gives up, sets the device error
 * word and finishes (the step's output is then invalid);
 * "test_wait_cta" N > 0 makes CTA N-1 of every launch wait once on a barrier
 * nothing arrives at -- a test of that error path (use with a short
 * "wait_limit_ms"; 0 = off); "prefill_tc" 1 (default) / 0 runs prompts on
 * 16-bit caches on the tensor-core kernel / the decode kernel's token blocks;
 * "prefill_l2_mb" (default 32) is the L2 budget for the K/V rows the
 * tensor-core prefill's CTAs read at one time: when a call's K/V rows exceed
 * L2, its work items go in batches of as many (sequence, layer, kv head)
 * streams as fit it (0, or rows that fit L2: all items largest first,
 * strided over the CTAs). */
JX_API int jx_kv_set_option(jx_kv* kv, const char* key, int value);

/* Device time of the last step recorded with option "timing" (waits for it):
 * the counterpart of forward_token's attention_ms (transformer.cpp:2499, 2567),
 * the wall time of RoPE + append + attention. */
JX_API int jx_kv_last_step_ms(jx_kv* kv, float* ms);

/* Number of kernels the last jx_attn_step / jx_attn_step_partial launched. */
JX_API int jx_kv_last_launch_count(const jx_kv* kv, int* count);

/* Seeded N(0,1) fill of rows [0, rows_per_seq[s]) of every layer of every
 * sequence, K and V, converted to the cache dtype (benchmark inputs).
 * rows_per_seq is a HOST array of n_seqs entries. */
JX_API int jx_kv_fill_normal(jx_kv* kv, const uint32_t* rows_per_seq, uint64_t seed, void* stream);
/* Seeded N(0,1) fill of n floats at dst (DEVICE); `stream_id` separates streams
 * of values drawn from one seed. */
JX_API int jx_fill_normal_f32(float* dst, uint64_t n, uint64_t seed, uint32_t stream_id, void* stream);

JX_API const char* jx_last_error_string(void);
/* Library version string. */
JX_API const char* jx_version(void);

#ifdef __cplusplus
}
#endif

#endif /* JX_ATTN_H */
