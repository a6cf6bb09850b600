// jx_lib.cu -- host side of libjxattn.so: the C ABI declared in
// include/jx_attn.h.  Owns the device KV cache (the B200 counterpart of
// KVCacheSlot, include/transformer.h:115-131), turns each decode step (or
// prefill) into a flattened work plan with balanced CTA slices, and launches
// the fused kernel (jx_decode.cuh); plus the log-sum-exp merge of sequence
// shards, the NCCL-sharded step, the prefill append pass and the seeded fill
// used by benches.
#include <cudaTypedefs.h>
#include <dlfcn.h>
#include <nccl.h>  // types and enum values only: the functions are resolved at run time

#include <chrono>
#include <thread>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <type_traits>
#include <vector>

#include "jx_attn.h"
#include "jx_device.cuh"
#include "jx_internal.h"
#include "jx_plan.h"

namespace jx {
bool decode_dispatch_dt0(int, int, int, int, int, const DecodeLaunch*, int*, cudaError_t*);
bool decode_dispatch_dt1(int, int, int, int, int, const DecodeLaunch*, int*, cudaError_t*);
bool decode_dispatch_dt2(int, int, int, int, int, const DecodeLaunch*, int*, cudaError_t*);

static bool dispatch(int dtype, int hd, int gp, int kp, int op, int stages, const DecodeLaunch* L,
                     int* oi, cudaError_t* oe) {
    switch (dtype) {
        case 0: return decode_dispatch_dt0(hd, gp, kp, op, stages, L, oi, oe);
        case 1: return decode_dispatch_dt1(hd, gp, kp, op, stages, L, oi, oe);
        case 2: return decode_dispatch_dt2(hd, gp, kp, op, stages, L, oi, oe);
        default: return false;
    }
}

int decode_smem_bytes(int hd, int gp, int kp, int dtype, int stages) {
    int v = -1;
    cudaError_t e = cudaSuccess;
    if (!dispatch(dtype, hd, gp, kp, 0, stages, nullptr, &v, &e)) return -1;
    return v;
}

int decode_ctas_per_sm(int hd, int gp, int kp, int dtype, int stages) {
    int v = 0;
    cudaError_t e = cudaSuccess;
    if (!dispatch(dtype, hd, gp, kp, 1, stages, nullptr, &v, &e)) return 0;
    return v;
}

cudaError_t decode_launch(const DecodeLaunch& L) {
    int v = 0;
    cudaError_t e = cudaErrorInvalidValue;
    if (!dispatch(L.dtype, L.head_dim, L.gp, L.kp, 2, L.stages, &L, &v, &e))
        return cudaErrorInvalidValue;
    return e;
}

// ------------------------------------------------------------------ kernels

__global__ void lse_merge_kernel(const float* __restrict__ gathered, int n_shards,
                                 long long shard_stride, int n_rows, int n_heads, int hd,
                                 float* __restrict__ out, long long out_stride) {
    const int row = blockIdx.x;  // (group, head)
    if (row >= n_rows) return;
    const int grp = row / n_heads, h = row % n_heads;
    const long long base = static_cast<long long>(row) * (hd + 2);
    float M = -INFINITY;
    for (int r = 0; r < n_shards; ++r) M = fmaxf(M, gathered[r * shard_stride + base + hd]);
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float Ls = 0.0f, O = 0.0f;
        for (int r = 0; r < n_shards; ++r) {
            const float* src = gathered + r * shard_stride + base;
            const float m = src[hd];
            const float f = m == -INFINITY ? 0.0f : ex2_approx((m - M) * 1.4426950408889634f);
            Ls += src[hd + 1] * f;
            O += src[d] * f;
        }
        out[static_cast<long long>(grp) * out_stride + static_cast<long long>(h) * hd + d] =
            O * (1.0f / Ls);
    }
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// Counter-based N(0,1): splitmix64 of (seed, stream, index) -> Box-Muller.
__device__ __forceinline__ float normal_at(uint64_t seed, uint32_t stream_id, uint64_t idx) {
    const uint64_t h = splitmix64(seed ^ splitmix64((static_cast<uint64_t>(stream_id) << 56) ^ idx));
    const float u1 = (static_cast<float>(h >> 40) + 1.0f) * (1.0f / 16777216.0f);
    const float u2 = static_cast<float>(h & 0xFFFFFFull) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

template <int DT>
__global__ void fill_cache_kernel(void* k, void* v, const uint32_t* __restrict__ rows,
                                  uint32_t n_seqs, uint32_t n_layers, uint32_t cap, uint32_t rs,
                                  uint64_t seed) {
    const long long per_seq = static_cast<long long>(n_layers) * cap * rs;
    const long long total = per_seq * n_seqs;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const uint32_t s = static_cast<uint32_t>(i / per_seq);
        const uint32_t row = static_cast<uint32_t>((i / rs) % cap);
        if (row >= rows[s]) continue;
        store_kv<DT>(k, i, normal_at(seed, 1, static_cast<uint64_t>(i)));
        store_kv<DT>(v, i, normal_at(seed, 2, static_cast<uint64_t>(i)));
    }
}

__global__ void fill_f32_kernel(float* dst, uint64_t n, uint64_t seed, uint32_t stream_id) {
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        dst[i] = normal_at(seed, stream_id, i);
}

// Multi-token prefill, first pass: every pair's k row rotated and k, v stored
// at its position (the append of transformer.cpp:2506-2520 for all tokens of
// the call) before any of them attends.  One block per pair.
template <int DT>
__global__ void append_rows_kernel(const PairRow* __restrict__ pairs, int n_pairs,
                                   const float2* __restrict__ rope, int rope_width,
                                   const float* __restrict__ k_in, const float* __restrict__ v_in,
                                   long long kv_stride, int n_kv, int hd, int neox, void* kc,
                                   void* vc, long long seq_stride, long long layer_stride,
                                   long long row_stride) {
    const int i = blockIdx.x;
    if (i >= n_pairs) return;
    const PairRow pr = pairs[i];
    if (pr.append_row < 0) return;
    const int nq = pr.nq > 1 ? pr.nq : 1;  // tokens of a prefill block
    for (int j = 0; j < nq; ++j) {
        const float2* cs = rope + static_cast<long long>(pr.rope_row + j) * rope_width;
        const long long io = pr.io + static_cast<long long>(j) * pr.io_step;
        const long long dst0 = static_cast<long long>(pr.seq) * seq_stride +
                               static_cast<long long>(pr.cache_layer) * layer_stride +
                               static_cast<long long>(pr.append_row + j) * row_stride;
        for (int idx = threadIdx.x; idx < n_kv * hd; idx += blockDim.x) {
            const int kvh = idx / hd, d = idx % hd;
            const float* kin = k_in + io * kv_stride + kvh * hd;
            const float kr = rope_elem(kin, d, pr.rope_half, cs, neox != 0);
            store_kv<DT>(kc, dst0 + idx, kr);
            store_kv<DT>(vc, dst0 + idx, v_in[io * kv_stride + idx]);
        }
    }
}

// Copies up to three host-resident (pinned) input buffers into device memory
// at the start of a step: many threads in flight, each input byte crossing
// PCIe once.  It lets the step's decode launch be scheduled at once
// (programmatic dependent launch); that launch waits for this grid before it
// reads the copies.
__global__ void stage_inputs_kernel(const float* s0, float* d0, long long n0, const float* s1,
                                    float* d1, long long n1, const float* s2, float* d2,
                                    long long n2) {
    pdl_launch_dependents();
    const long long tid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long nthr = static_cast<long long>(gridDim.x) * blockDim.x;
    const float* src[3] = {s0, s1, s2};
    float* dst[3] = {d0, d1, d2};
    const long long n[3] = {n0, n1, n2};
    for (int b = 0; b < 3; ++b) {
        if (!src[b] || n[b] <= 0) continue;
        const bool vec = (reinterpret_cast<uintptr_t>(src[b]) | reinterpret_cast<uintptr_t>(dst[b])) %
                             16 == 0;
        const long long n4 = vec ? n[b] / 4 : 0;
        const float4* s4 = reinterpret_cast<const float4*>(src[b]);
        float4* d4 = reinterpret_cast<float4*>(dst[b]);
        for (long long i = tid; i < n4; i += nthr) d4[i] = s4[i];
        for (long long i = 4 * n4 + tid; i < n[b]; i += nthr) dst[b][i] = src[b][i];
    }
}

// Consumer warps for a ring of `stages` when `split` warps share each tile:
// every stage must be consumed by one group of warps only, so the number of
// tile streams (warps / split) divides the ring size.
int consumers_for(int stages, int split) {
    for (int c = 4; c >= split; --c)
        if (c % split == 0 && stages % (c / split) == 0) return c;
    return split;
}

// Default pipeline depth / residency for one kernel configuration: a ring of
// 8 or 4 stages (all four consumer warps busy) with two CTAs per SM if shared
// memory and registers allow it, else with one CTA per SM, else the deepest
// ring that fits one CTA.
void default_shape(int hd, int gp, int kp, int dtype, int* stages, int* cps) {
    const int per_sm = 227 * 1024;
    for (int c = 2; c >= 1; --c)
        for (int ns : {8, 4}) {
            const int bytes = decode_smem_bytes(hd, gp, kp, dtype, ns);
            if (bytes < 0 || bytes + 1024 * (c - 1) > per_sm / c) continue;
            if (decode_ctas_per_sm(hd, gp, kp, dtype, ns) < c) continue;
            *stages = ns;
            *cps = c;
            return;
        }
    int best = 2;
    for (int ns = 7; ns >= 2; --ns)
        if (decode_smem_bytes(hd, gp, kp, dtype, ns) <= per_sm) { best = ns; break; }
    *stages = best;
    *cps = 1;
}

// Inverse frequency of every rotated pair (half = min(head_dim, rope_dim) / 2
// entries), computed with the same float expressions as apply_rope
// (src/transformer.cpp:82-92, 112-116).  It does not depend on the position,
// so a step computes it once per RoPE configuration.
void rope_inv_freqs(uint32_t head_dim, uint32_t rope_dim, float base, bool neox,
                    const float* rope_freqs, float* freq) {
    const uint32_t rdim = std::min(head_dim, rope_dim);
    const uint32_t half = rdim / 2;
    for (uint32_t j = 0; j < half; ++j) {
        float f;
        if (neox) {
            f = 1.0f / std::pow(base, (2.0f * static_cast<float>(j)) / static_cast<float>(rdim));
            if (rope_freqs) f /= rope_freqs[j];
        } else {
            const uint32_t d = 2 * j;
            f = 1.0f / std::pow(base, static_cast<float>(d) / static_cast<float>(rdim));
        }
        freq[j] = f;
    }
}

// (cos, sin) of the `half` rotated pairs at `pos` from their inverse
// frequencies; writes `width` entries (zeros past the rotated pairs).
void rope_row_freqs(const float* freq, uint32_t half, uint32_t pos, float yarn_scale, float2* out,
                    int width) {
    const float pos_scaled = static_cast<float>(pos) / std::max(1e-4f, yarn_scale);
    for (int j = 0; j < width; ++j) out[j] = make_float2(0.0f, 0.0f);
    for (uint32_t j = 0; j < half; ++j) {
        const float angle = pos_scaled * freq[j];
        out[j] = make_float2(std::cos(angle), std::sin(angle));
    }
}

// (cos, sin) of every rotated pair at `pos`, as apply_rope computes them.
void rope_row(uint32_t head_dim, uint32_t rope_dim, uint32_t pos, float base, float yarn_scale,
              bool neox, const float* rope_freqs, float2* out, int width) {
    float freq[128];  // head_dim <= 256
    const uint32_t half = std::min(std::min(head_dim, rope_dim) / 2, 128u);
    rope_inv_freqs(std::min(head_dim, 256u), rope_dim, base, neox, rope_freqs, freq);
    rope_row_freqs(freq, half, pos, yarn_scale, out, width);
}

}  // namespace jx

using namespace jx;

// ------------------------------------------------------------------ errors

static thread_local std::string g_err;

static int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
static int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

void jx::set_last_error(const char* msg) { g_err = msg; }

#define JX_CUDA(call)                                                                    \
    do {                                                                                 \
        cudaError_t e_ = (call);                                                         \
        if (e_ != cudaSuccess)                                                           \
            return fail(JX_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_));    \
    } while (0)

namespace {

// Sets the handle's device for the duration of a call and restores the
// caller's current device afterwards.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) return;
        ok = prev == dev || cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (ok && prev >= 0) cudaSetDevice(prev);
    }
};

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// A work plan in device memory.  A decode loop whose positions change every
// step uploads a new plan per call: plans go to a ring of kStaging device
// buffers, each filled from its own pinned host buffer by a copy on a side
// stream, and the step's stream waits only for that copy's event.  The
// step's stream thus runs staging kernel -> decode kernel with no copy-engine
// operation between them (which cost ~25 us of GPU time per step), and the
// host runs up to kStaging calls ahead.  A ring buffer is refilled only after
// the launches that last read it (ev_used) and the copy that last read its
// host buffer (ev_copy) are done.  While a stream is being captured into a
// graph, the copy stays on that stream (a captured stream cannot wait for an
// uncaptured one).
constexpr int kStaging = 4;
struct PlanSlot {
    std::vector<unsigned char> cached;  // bytes last uploaded
    void* d_buf = nullptr;              // the buffer holding `cached`
    int cur = -1;                       // its ring index
    void* d_ring[kStaging] = {};
    size_t d_cap[kStaging] = {};
    void* h_buf[kStaging] = {};  // pinned staging
    size_t h_cap[kStaging] = {};
    cudaEvent_t ev_copy[kStaging] = {};
    bool copy_pending[kStaging] = {};
    cudaEvent_t ev_used[kStaging] = {};
    bool used_pending[kStaging] = {};
    int next = 0;
};

}  // namespace

struct jx_kv {
    jx_kv_desc d{};
    size_t esz = 4;
    void* k = nullptr;
    void* v = nullptr;
    long long seq_stride = 0, layer_stride = 0;  // elements
    // tensor maps by TMA box inner extent: [0] = 128-byte boxes, [1] = 64-byte boxes
    CUtensorMap tmK[2], tmV[2];
    bool tm_ok[2] = {false, false};
    // tensor maps of the tensor-core prefill (128-byte boxes, 128-byte swizzle) by box
    // height: [0] = 128 rows (head_dim 64), [1] = 64 rows (head_dim 128)
    CUtensorMap tmKp[2], tmVp[2];
    bool tmp_ok[2] = {false, false};
    int opt_prefill_tc = 1;  // 16-bit caches: prefill attention on the tensor cores (tcgen05)
    int opt_prefill_l2_mb = 32;  // L2 budget of the K/V streams prefill CTAs share at one time
    std::vector<uint32_t> seq_pos;
    int num_sms = 0;
    int* d_err = nullptr;
    int* d_dbg = nullptr;        // [8] first failed device check (checked builds)
    uint32_t* d_rows = nullptr;  // fill helper
    float* d_scratch = nullptr;
    size_t scratch_floats = 0;
    int* d_counters = nullptr;
    size_t counters_n = 0;
    std::vector<PlanSlot> slots;
    int opt_ctas_per_sm = 0, opt_stages = 0, opt_grid = 0;
    int opt_pdl = -1;  // programmatic dependent launch: -1 auto, 0 off, 1 on
    int opt_timing = 0;  // 1: events around every step (jx_kv_last_step_ms)
    float opt_split_penalty_us = -1.0f;  // cost of an extra piece in a CTA's slice; -1: auto
    int opt_wait_limit_ms = 0;   // bound of the kernel's pipeline waits; 0: the default (~4 s)
    int opt_test_wait_cta = 0;   // test hook: CTA + 1 that waits on a barrier nothing arrives at
    cudaEvent_t ev_t0 = nullptr, ev_t1 = nullptr;
    bool timed = false;  // a timed step was recorded
    int last_launches = 0;
    // launch shape per (head_dim, group, stages override): {stages, ctas per SM}
    std::map<std::tuple<int, int, int, int>, std::pair<int, int>> shapes;
    // per (segments + 1, CTAs): the slice budget of the last plan (warm start)
    std::map<std::pair<long long, long long>, long long> split_hints;
    // Replay of the last step: a call identical to the previous one (same
    // arguments, positions, layers, buffers, stream, options) relaunches the
    // launches built for it, as long as no plan buffer or scratch changed since.
    uint64_t generation = 0;  // bumped whenever a plan buffer or the scratch changes
    uint64_t replay_generation = ~0ull;
    std::vector<unsigned char> replay_key;
    std::vector<DecodeLaunch> replay;
    // sequence-sharded step: this rank's partials and the gathered partials
    float* d_part = nullptr;
    float* d_gather = nullptr;
    size_t part_floats = 0, gather_floats = 0;
    // device copies of a step's host-resident q/k/v (stage_host_inputs)
    float* d_stage = nullptr;
    size_t stage_floats = 0;
    cudaStream_t up_stream = nullptr;  // plan copies (upload_plan)
    // copies of host-resident q/k/v decided by stage_host_inputs, launched by
    // the step right before its first kernel (after its plan uploads)
    struct PendingStage {
        bool active = false;
        const float* src[3] = {};
        float* dst[3] = {};
        long long n[3] = {};
        int grid = 0;
    } pend;
    std::vector<int> used_slots;       // plan slots the current call's launches read
    std::vector<int> replay_slots;     // plan slots the recorded launches read
};

namespace {

int encode_maps(jx_kv* kv, int box_kind) {
    if (kv->tm_ok[box_kind]) return JX_OK;
    auto enc = tensor_map_encoder();
    if (!enc) return fail(JX_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[4] = {kv->d.row_stride, kv->d.capacity, kv->d.n_layers, kv->d.n_seqs};
    const cuuint64_t strides[3] = {
        static_cast<cuuint64_t>(kv->d.row_stride) * kv->esz,
        static_cast<cuuint64_t>(kv->d.row_stride) * kv->esz * kv->d.capacity,
        static_cast<cuuint64_t>(kv->d.row_stride) * kv->esz * kv->d.capacity * kv->d.n_layers};
    const uint32_t box_bytes = box_kind == 0 ? 128 : 64;
    const cuuint32_t box[4] = {static_cast<cuuint32_t>(box_bytes / kv->esz), 32, 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUtensorMapDataType dt =
        kv->esz == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
    const CUtensorMapSwizzle sw =
        box_kind == 0 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    for (int which = 0; which < 2; ++which) {
        CUresult r = enc(which == 0 ? &kv->tmK[box_kind] : &kv->tmV[box_kind], dt, 4,
                         which == 0 ? kv->k : kv->v, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(JX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    }
    kv->tm_ok[box_kind] = true;
    return JX_OK;
}

// Tensor maps of the tensor-core prefill: boxes of 64 16-bit elements (128
// bytes, one head-row slab) x `rows` cache rows, 128-byte swizzle -- the
// K-major / MN-major operand layout the kernel's MMAs read.
int encode_prefill_maps(jx_kv* kv, int kind, int rows) {
    if (kv->tmp_ok[kind]) return JX_OK;
    auto enc = tensor_map_encoder();
    if (!enc) return fail(JX_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    if (kv->esz != 2) return fail(JX_ERR_UNSUPPORTED, "tensor-core prefill needs a 16-bit cache");
    const cuuint64_t dims[4] = {kv->d.row_stride, kv->d.capacity, kv->d.n_layers, kv->d.n_seqs};
    const cuuint64_t strides[3] = {
        static_cast<cuuint64_t>(kv->d.row_stride) * 2,
        static_cast<cuuint64_t>(kv->d.row_stride) * 2 * kv->d.capacity,
        static_cast<cuuint64_t>(kv->d.row_stride) * 2 * kv->d.capacity * kv->d.n_layers};
    const cuuint32_t box[4] = {64, static_cast<cuuint32_t>(rows), 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    for (int which = 0; which < 2; ++which) {
        CUresult r = enc(which == 0 ? &kv->tmKp[kind] : &kv->tmVp[kind],
                         CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, which == 0 ? kv->k : kv->v, dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(JX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    }
    kv->tmp_ok[kind] = true;
    return JX_OK;
}

int upload_plan(jx_kv* kv, size_t slot_i, const std::vector<unsigned char>& bytes,
                cudaStream_t stream) {
    if (kv->slots.size() <= slot_i) kv->slots.resize(slot_i + 1);
    PlanSlot& s = kv->slots[slot_i];
    kv->used_slots.push_back(static_cast<int>(slot_i));
    if (s.cached == bytes && s.d_buf) return JX_OK;
    const int b = s.next;
    s.next = (b + 1) % kStaging;
    if (s.d_cap[b] < bytes.size()) {
        if (s.d_ring[b]) JX_CUDA(cudaFree(s.d_ring[b]));  // (synchronises the device)
        s.d_ring[b] = nullptr;
        s.d_cap[b] = 0;
        s.used_pending[b] = false;
        const size_t cap = std::max<size_t>(bytes.size() * 2, 4096);
        if (cudaMalloc(&s.d_ring[b], cap) != cudaSuccess)
            return fail(JX_ERR_NOMEM, "plan buffer allocation of %zu bytes failed", cap);
        s.d_cap[b] = cap;
    }
    if (!s.ev_copy[b]) JX_CUDA(cudaEventCreateWithFlags(&s.ev_copy[b], cudaEventDisableTiming));
    if (!s.ev_used[b]) JX_CUDA(cudaEventCreateWithFlags(&s.ev_used[b], cudaEventDisableTiming));
    if (s.copy_pending[b]) {
        JX_CUDA(cudaEventSynchronize(s.ev_copy[b]));  // the host buffer's previous copy ran
        s.copy_pending[b] = false;
    }
    if (s.h_cap[b] < bytes.size()) {
        if (s.h_buf[b]) JX_CUDA(cudaFreeHost(s.h_buf[b]));
        s.h_buf[b] = nullptr;
        s.h_cap[b] = 0;
        const size_t cap = std::max<size_t>(bytes.size() * 2, 4096);
        if (cudaHostAlloc(&s.h_buf[b], cap, cudaHostAllocDefault) != cudaSuccess)
            return fail(JX_ERR_NOMEM, "pinned staging allocation of %zu bytes failed", cap);
        s.h_cap[b] = cap;
    }
    std::memcpy(s.h_buf[b], bytes.data(), bytes.size());
    ++kv->generation;
    cudaStreamCaptureStatus cap_st = cudaStreamCaptureStatusNone;
    JX_CUDA(cudaStreamIsCapturing(stream, &cap_st));
    if (cap_st != cudaStreamCaptureStatusNone) {
        // captured: the copy is a node of the stream's graph
        JX_CUDA(cudaMemcpyAsync(s.d_ring[b], s.h_buf[b], bytes.size(), cudaMemcpyHostToDevice,
                                stream));
    } else {
        const cudaError_t busy = cudaStreamQuery(stream);
        if (busy == cudaErrorNotReady && cudaPeekAtLastError() == cudaErrorNotReady)
            cudaGetLastError();  // a status, not an error of the caller's
        if (busy == cudaSuccess) {
            // nothing queued on the stream (a caller that synchronises every
            // call): copy in it, with no cross-stream wait before the launch
            JX_CUDA(cudaMemcpyAsync(s.d_ring[b], s.h_buf[b], bytes.size(), cudaMemcpyHostToDevice,
                                    stream));
            JX_CUDA(cudaEventRecord(s.ev_copy[b], stream));
        } else {
            // work in flight: copy on the side stream once the launches that
            // last read this buffer have run, so the copy overlaps that work
            if (!kv->up_stream)
                JX_CUDA(cudaStreamCreateWithFlags(&kv->up_stream, cudaStreamNonBlocking));
            if (s.used_pending[b]) JX_CUDA(cudaStreamWaitEvent(kv->up_stream, s.ev_used[b], 0));
            JX_CUDA(cudaMemcpyAsync(s.d_ring[b], s.h_buf[b], bytes.size(), cudaMemcpyHostToDevice,
                                    kv->up_stream));
            JX_CUDA(cudaEventRecord(s.ev_copy[b], kv->up_stream));
            JX_CUDA(cudaStreamWaitEvent(stream, s.ev_copy[b], 0));
        }
        s.copy_pending[b] = true;
    }
    s.d_buf = s.d_ring[b];
    s.cur = b;
    s.cached = bytes;
    return JX_OK;
}

// Launches the copies of host-resident step inputs that stage_host_inputs
// decided on, once per call, before the call's first kernel: after the plan
// uploads, so that no stream wait separates the staging kernel from the
// launch it feeds.
int flush_staging(jx_kv* kv, cudaStream_t stream) {
    if (!kv->pend.active) return JX_OK;
    auto& p = kv->pend;
    p.active = false;
    stage_inputs_kernel<<<p.grid, 256, 0, stream>>>(p.src[0], p.dst[0], p.n[0], p.src[1], p.dst[1],
                                                    p.n[1], p.src[2], p.dst[2], p.n[2]);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(JX_ERR_CUDA, "input staging launch: %s", cudaGetErrorString(e));
    return JX_OK;
}

// After a call's launches: each plan buffer they read is marked as read up
// to this point of `stream` (upload_plan refills it only after that).
int mark_plans_used(jx_kv* kv, const std::vector<int>& slots, cudaStream_t stream) {
    for (int si : slots) {
        PlanSlot& s = kv->slots[static_cast<size_t>(si)];
        if (s.cur < 0) continue;
        JX_CUDA(cudaEventRecord(s.ev_used[s.cur], stream));
        s.used_pending[s.cur] = true;
    }
    return JX_OK;
}

int ensure_scratch(jx_kv* kv, size_t floats, size_t counters) {
    if (kv->scratch_floats < floats || kv->counters_n < counters) ++kv->generation;
    if (kv->scratch_floats < floats) {
        if (kv->d_scratch) JX_CUDA(cudaFree(kv->d_scratch));
        kv->d_scratch = nullptr;
        kv->scratch_floats = 0;
        if (cudaMalloc(&kv->d_scratch, floats * sizeof(float)) != cudaSuccess)
            return fail(JX_ERR_NOMEM, "scratch allocation of %zu floats failed", floats);
        kv->scratch_floats = floats;
    }
    if (kv->counters_n < counters) {
        if (kv->d_counters) JX_CUDA(cudaFree(kv->d_counters));
        kv->d_counters = nullptr;
        kv->counters_n = 0;
        if (cudaMalloc(&kv->d_counters, counters * sizeof(int)) != cudaSuccess)
            return fail(JX_ERR_NOMEM, "counter allocation failed");
        JX_CUDA(cudaMemset(kv->d_counters, 0, counters * sizeof(int)));
        kv->counters_n = counters;
    }
    return JX_OK;
}

uint64_t hash_floats(const float* p, size_t n) {
    uint64_t h = 1469598103934665603ull;
    const unsigned char* b = reinterpret_cast<const unsigned char*>(p);
    for (size_t i = 0; i < n * 4; ++i) h = (h ^ b[i]) * 1099511628211ull;
    return h;
}

int gp_of(uint32_t g) {
    if (g <= 1) return 1;
    if (g <= 2) return 2;
    if (g <= 4) return 4;
    if (g <= 8) return 8;
    return 0;
}

template <typename T>
void put(std::vector<unsigned char>& k, const T& v) {
    const unsigned char* p = reinterpret_cast<const unsigned char*>(&v);
    k.insert(k.end(), p, p + sizeof(T));
}

// Everything a step's launches depend on, field by field (no padding bytes).
std::vector<unsigned char> call_key(const jx_kv* kv, const jx_layer_desc* layers,
                                    uint32_t n_layers, const jx_step_args* a,
                                    const float* partials, cudaStream_t stream) {
    std::vector<unsigned char> k;
    k.reserve(128 + 8 * a->n_seqs + 40 * n_layers);
    put(k, a->n_heads); put(k, a->n_kv_heads); put(k, a->n_seqs);
    put(k, a->q); put(k, a->k); put(k, a->v); put(k, a->out);
    put(k, a->q_stride); put(k, a->kv_stride); put(k, a->scale); put(k, a->softcap);
    put(k, a->sliding_window); put(k, a->yarn_scale); put(k, a->rope_neox);
    put(k, partials); put(k, stream);
    put(k, kv->opt_stages); put(k, kv->opt_ctas_per_sm); put(k, kv->opt_grid); put(k, kv->opt_pdl);
    put(k, kv->opt_split_penalty_us); put(k, kv->opt_wait_limit_ms); put(k, kv->opt_test_wait_cta);
    for (uint32_t s = 0; s < a->n_seqs; ++s) {
        put(k, a->pos[s]);
        put(k, a->seq_ids ? a->seq_ids[s] : -1);
    }
    for (uint32_t l = 0; l < n_layers; ++l) {
        const jx_layer_desc& L = layers[l];
        put(k, L.head_dim); put(k, L.rope_dim); put(k, L.rope_freq_base);
        put(k, L.kv_source_layer); put(k, L.is_swa); put(k, L.shares_kv);
        put(k, L.rope_freqs ? hash_floats(L.rope_freqs, std::min(L.head_dim, L.rope_dim) / 2)
                            : uint64_t(0));
    }
    return k;
}

}  // namespace

// SM cycles of a bounded pipeline wait for a limit in milliseconds (counted at
// 2 GHz, about B200's top SM clock, so a wait lasts at least that long); 0
// selects the kernel's default of ~4 s.
long long jx::wait_limit_cycles(int ms) {
    return ms > 0 ? static_cast<long long>(ms) * 2000000ll : kWaitLimitCycles;
}

namespace {

// Rows one CTA streams per microsecond when all P CTAs share HBM evenly
// (~6.5 TB/s on B200): converts a per-piece time cost into rows.
double split_rows_per_us(const jx_kv* kv, size_t bytes_per_row, long long P) {
    (void)kv;
    if (bytes_per_row == 0 || P <= 0) return 0.0;
    return 6.5e6 / static_cast<double>(P) / static_cast<double>(bytes_per_row);
}

// q/k/v/out (and partials) may live in this device's memory or in pinned
// (page-locked) host memory, which the kernel reads and writes over PCIe;
// pageable host memory or another device's memory is refused, since a
// kernel touching it would fault.  *host tells which.
int check_step_ptr(const void* p, const char* name, int device, bool* host) {
    cudaPointerAttributes at{};
    const cudaError_t e = cudaPointerGetAttributes(&at, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(JX_ERR_INVALID, "%s: not a CUDA-visible pointer (%s)", name, cudaGetErrorString(e));
    }
    if (at.type == cudaMemoryTypeHost) {
        *host = true;
        return JX_OK;
    }
    *host = false;
    if ((at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) && at.device == device)
        return JX_OK;
    return fail(JX_ERR_INVALID,
                "%s must be memory of device %d or pinned host memory (pageable host memory "
                "or another device's memory would fault the kernel)", name, device);
}

// Plan and launch of the tensor-core prefill for one launch group (layers of
// one head_dim; their rows were appended already).  Rows of the call that
// belong to one sequence at consecutive positions (in call order) form runs;
// each run is cut into tiles of 128/G tokens, and a work item is (tile, layer,
// kv head).  Items go largest first (streamed K/V tiles) so the persistent
// CTAs, which take items c, c + P, ..., finish close together.  Each tile has
// its own run of (cos, sin) rows, computed with apply_rope's expressions.
int prefill_tc(jx_kv* kv, const jx_layer_desc* layers, uint32_t n_layers,
               const std::vector<uint32_t>& grp_layers, const jx_step_args* a,
               const std::vector<int>& seqs, int hd, uint32_t G, bool neox, float inv_cap,
               size_t gi, cudaStream_t stream) {
    const jx_kv_desc& D = kv->d;
    const int TQ = 128 / static_cast<int>(G);
    const int BN = prefill_tc_rows(hd);
    const int kind = hd == 64 ? 0 : 1;
    int rc = encode_prefill_maps(kv, kind, BN);
    if (rc) return rc;
    std::vector<std::pair<uint32_t, uint32_t>> chunks;  // (first row, tokens)
    for (uint32_t r = 0; r < a->n_seqs;) {
        uint32_t nb = 1;
        while (nb < static_cast<uint32_t>(TQ) && r + nb < a->n_seqs && seqs[r + nb] == seqs[r] &&
               a->pos[r + nb] == a->pos[r] + static_cast<int32_t>(nb))
            ++nb;
        chunks.emplace_back(r, nb);
        r += nb;
    }
    const int width = hd / 2;
    std::vector<PrefillTile> items;
    items.reserve(chunks.size() * grp_layers.size() * a->n_kv_heads);
    std::vector<PairRow> appends;  // append pass: one row per (chunk, layer)
    appends.reserve(chunks.size() * grp_layers.size());
    std::vector<float2> rope;
    std::map<std::tuple<uint32_t, uint32_t, uint32_t, uint64_t, uint32_t, uint32_t>, int> rope_ids;
    std::map<std::tuple<uint32_t, uint32_t, uint64_t>, std::vector<float>> inv_freqs;
    int n_rope = 0;
    const uint32_t W = a->sliding_window;
    for (const auto& ch : chunks) {
        const uint32_t r0 = ch.first, nt = ch.second;
        const uint32_t pos0 = static_cast<uint32_t>(a->pos[r0]);
        for (uint32_t l : grp_layers) {
            const jx_layer_desc& L = layers[l];
            // every row the chunk attends must be in this cache (as for a step)
            const uint64_t t0 = (L.is_swa && W > 0 && pos0 >= W) ? pos0 - W + 1 : 0;
            const uint64_t last = static_cast<uint64_t>(pos0) + nt - 1;
            if (t0 < D.pos_base || last >= static_cast<uint64_t>(D.pos_base) + D.capacity)
                return fail(JX_ERR_RANGE,
                            "position %llu (window start %llu) is outside the cache rows "
                            "[%u, %llu); compact or roll back first",
                            static_cast<unsigned long long>(last),
                            static_cast<unsigned long long>(t0), D.pos_base,
                            static_cast<unsigned long long>(D.pos_base) + D.capacity);
            const uint32_t rdim = std::min(L.head_dim, L.rope_dim);
            const float* rf = (neox && !L.is_swa && L.rope_freqs) ? L.rope_freqs : nullptr;
            uint32_t base_bits, yarn_bits;
            std::memcpy(&base_bits, &L.rope_freq_base, 4);
            std::memcpy(&yarn_bits, &a->yarn_scale, 4);
            const uint64_t fh = rf ? hash_floats(rf, rdim / 2) : 0;
            const auto key = std::make_tuple(rdim, base_bits, yarn_bits, fh, pos0, nt);
            auto itk = rope_ids.find(key);
            int rid;
            if (itk == rope_ids.end()) {
                rid = n_rope;
                rope_ids.emplace(key, rid);
                n_rope += static_cast<int>(nt);
                rope.resize(static_cast<size_t>(n_rope) * width);
                const auto fkey = std::make_tuple(rdim, base_bits, fh);
                auto itf = inv_freqs.find(fkey);
                if (itf == inv_freqs.end()) {
                    std::vector<float> f(rdim / 2);
                    rope_inv_freqs(L.head_dim, L.rope_dim, L.rope_freq_base, neox, rf, f.data());
                    itf = inv_freqs.emplace(fkey, std::move(f)).first;
                }
                for (uint32_t j = 0; j < nt; ++j)
                    rope_row_freqs(itf->second.data(), rdim / 2, pos0 + j, a->yarn_scale,
                                   rope.data() + static_cast<size_t>(rid + j) * width, width);
            } else {
                rid = itk->second;
            }
            PrefillTile t{};
            t.seq = seqs[r0];
            t.cache_layer = static_cast<int>(L.kv_source_layer);
            t.io0 = static_cast<int>(r0 * n_layers + l);
            t.io_step = static_cast<int>(n_layers);
            t.tok_row0 = static_cast<int>(pos0) - static_cast<int>(D.pos_base);
            t.ntok = static_cast<int>(nt);
            t.row0 = 0;  // local row 0: non-window layers need pos_base == 0 (checked above)
            t.window = (L.is_swa && W > 0) ? static_cast<int>(W) : 0;
            t.rope_row0 = rid;
            t.rope_half = static_cast<int>(rdim / 2);
            t.kv_lo = t.window > 0 ? std::max(0, t.tok_row0 - t.window + 1) : 0;
            t.n_tiles = (t.tok_row0 + t.ntok - t.kv_lo + BN - 1) / BN;
            for (uint32_t h = 0; h < a->n_kv_heads; ++h) {
                t.kvh = static_cast<int>(h);
                items.push_back(t);
            }
            // the chunk's rows of this layer, appended before any is attended
            // (one block per chunk and layer; shares-KV layers append nothing)
            PairRow ap{};
            ap.seq = t.seq;
            ap.io = t.io0;
            ap.io_step = t.io_step;
            ap.nq = t.ntok;
            ap.cache_layer = t.cache_layer;
            ap.append_row = L.shares_kv ? -1 : t.tok_row0;
            ap.rope_row = rid;
            ap.rope_half = t.rope_half;
            appends.push_back(ap);
        }
    }
    // The kernel trusts the plan: validate every item here.
    for (const PrefillTile& t : items) {
        const bool ok =
            t.seq >= 0 && t.seq < static_cast<int>(D.n_seqs) && t.cache_layer >= 0 &&
            t.cache_layer < static_cast<int>(D.n_layers) && t.kvh >= 0 &&
            static_cast<uint64_t>(t.kvh + 1) * hd <= D.row_stride && t.ntok >= 1 && t.ntok <= TQ &&
            t.tok_row0 >= 0 && static_cast<uint64_t>(t.tok_row0) + t.ntok <= D.capacity &&
            t.kv_lo >= 0 && t.kv_lo <= t.tok_row0 && t.n_tiles >= 1 && t.io0 >= 0 &&
            static_cast<long long>(t.io0) + static_cast<long long>(t.ntok - 1) * t.io_step <
                static_cast<long long>(a->n_seqs) * n_layers &&
            t.rope_row0 >= 0 && t.rope_row0 + t.ntok <= n_rope && t.rope_half >= 0 &&
            t.rope_half <= hd / 2;
        if (!ok) return fail(JX_ERR_INVALID, "internal: inconsistent prefill work item");
    }
    const int grid = static_cast<int>(std::min<size_t>(std::max(kv->num_sms, 1), items.size()));
    std::vector<int> cta_first;
    {
        std::vector<long long> stream(items.size());
        std::vector<int> tiles(items.size());
        for (size_t i = 0; i < items.size(); ++i) {
            const PrefillTile& t = items[i];
            stream[i] = (static_cast<long long>(t.seq) * D.n_layers + t.cache_layer) *
                            static_cast<long long>(a->n_kv_heads) + t.kvh;
            tiles[i] = t.n_tiles;
        }
        // Streams per batch: as many as fit the L2 budget (option
        // prefill_l2_mb), once all streams' rows together exceed L2 (126 MB);
        // below that they stay in L2 whatever the order, and striding the
        // items largest first balances the CTAs best.  Measured (bf16, one
        // prompt): 2048-token Llama-3.2-1B (67 MB of K/V) strided 1.46 ms,
        // batched 2.0-2.2; 8192-token Llama-3.2-1B (268 MB) 16.8 / 15.9 ms;
        // 8192-token Mistral-7B (1.07 GB) 60.4 / 54.3 ms.
        int window = 0;
        if (kv->opt_prefill_l2_mb > 0) {
            std::map<long long, int> stream_tiles;
            for (size_t i = 0; i < tiles.size(); ++i)
                stream_tiles[stream[i]] = std::max(stream_tiles[stream[i]], tiles[i]);
            double all_bytes = 0, max_bytes = 1;
            for (const auto& st : stream_tiles) {
                const double b = 2.0 * st.second * BN * hd * 2;  // K and V rows, 16-bit
                all_bytes += b;
                max_bytes = std::max(max_bytes, b);
            }
            if (all_bytes > 126.0 * 1048576.0)
                window = static_cast<int>(std::max(
                    1.0, std::floor(kv->opt_prefill_l2_mb * 1048576.0 / max_bytes)));
        }
        const std::vector<size_t> order = schedule_items(stream, tiles, grid, 2, window, cta_first);
        std::vector<PrefillTile> sorted(items.size());
        for (size_t i = 0; i < order.size(); ++i) sorted[i] = items[order[i]];
        items.swap(sorted);
    }
    for (const PairRow& ap : appends) {
        const bool ok = ap.append_row < 0 ||
                        (ap.append_row >= 0 &&
                         static_cast<uint64_t>(ap.append_row) + ap.nq <= D.capacity &&
                         ap.rope_row + ap.nq <= n_rope &&
                         static_cast<uint64_t>(a->n_kv_heads) * hd <= D.row_stride &&
                         static_cast<uint64_t>(a->n_kv_heads) * hd <= a->kv_stride);
        if (!ok) return fail(JX_ERR_INVALID, "internal: inconsistent prefill append row");
    }
    const size_t item_bytes = items.size() * sizeof(PrefillTile);
    const size_t first_off = (item_bytes + 255) & ~static_cast<size_t>(255);
    const size_t first_bytes = cta_first.size() * sizeof(int);
    const size_t app_off = (first_off + first_bytes + 255) & ~static_cast<size_t>(255);
    const size_t app_bytes = appends.size() * sizeof(PairRow);
    const size_t rope_off = (app_off + app_bytes + 255) & ~static_cast<size_t>(255);
    std::vector<unsigned char> bytes(rope_off + rope.size() * sizeof(float2), 0);
    std::memcpy(bytes.data(), items.data(), item_bytes);
    std::memcpy(bytes.data() + first_off, cta_first.data(), first_bytes);
    std::memcpy(bytes.data() + app_off, appends.data(), app_bytes);
    if (!rope.empty()) std::memcpy(bytes.data() + rope_off, rope.data(), rope.size() * sizeof(float2));
    const size_t slot = gi;
    rc = upload_plan(kv, slot, bytes, stream);
    if (rc) return rc;
    rc = flush_staging(kv, stream);
    if (rc) return rc;
    {
        unsigned char* dplan = static_cast<unsigned char*>(kv->slots[slot].d_buf);
        const PairRow* dp = reinterpret_cast<const PairRow*>(dplan + app_off);
        const float2* dr = reinterpret_cast<const float2*>(dplan + rope_off);
        const int np = static_cast<int>(appends.size());
        const int nkv = static_cast<int>(a->n_kv_heads);
        if (D.dtype == JX_BF16)
            append_rows_kernel<DT_BF16><<<np, 256, 0, stream>>>(
                dp, np, dr, width, a->k, a->v, a->kv_stride, nkv, hd, neox ? 1 : 0, kv->k, kv->v,
                kv->seq_stride, kv->layer_stride, D.row_stride);
        else
            append_rows_kernel<DT_F16T><<<np, 256, 0, stream>>>(
                dp, np, dr, width, a->k, a->v, a->kv_stride, nkv, hd, neox ? 1 : 0, kv->k, kv->v,
                kv->seq_stride, kv->layer_stride, D.row_stride);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess)
            return fail(JX_ERR_CUDA, "append launch failed: %s", cudaGetErrorString(e));
    }
    PrefillArgs pa{};
    pa.tiles = static_cast<const PrefillTile*>(kv->slots[slot].d_buf);
    pa.cta_first = reinterpret_cast<const int*>(static_cast<unsigned char*>(kv->slots[slot].d_buf) +
                                                first_off);
    pa.n_items = static_cast<int>(items.size());
    pa.neox = neox ? 1 : 0;
    pa.q_vec = (reinterpret_cast<uintptr_t>(a->q) % 16 == 0 && a->q_stride % 4 == 0) ? 1 : 0;
    pa.q = a->q;
    pa.out = a->out;
    pa.q_stride = a->q_stride;
    pa.rope = reinterpret_cast<const float2*>(static_cast<unsigned char*>(kv->slots[slot].d_buf) +
                                              rope_off);
    pa.scale = a->scale;
    pa.softcap = a->softcap;
    pa.inv_softcap = inv_cap;
    pa.err = kv->d_err;
    pa.dbg = kv->d_dbg;
    pa.wait_limit = wait_limit_cycles(kv->opt_wait_limit_ms);
    const cudaError_t e = prefill_tc_launch(pa, &kv->tmKp[kind], &kv->tmVp[kind], hd, D.dtype,
                                            static_cast<int>(G), grid, stream);
    if (e != cudaSuccess)
        return fail(JX_ERR_CUDA, "tensor-core prefill launch failed: %s", cudaGetErrorString(e));
    return JX_OK;
}

int step_impl(jx_kv* kv, const jx_layer_desc* layers, uint32_t n_layers, const jx_step_args* a,
              float* partials, cudaStream_t stream, bool prefill = false) {
    if (!kv || !layers || !a) return fail(JX_ERR_INVALID, "null handle, layers or args");
    if (n_layers == 0 || a->n_seqs == 0) return fail(JX_ERR_INVALID, "empty step");
    if (!a->pos || !a->q || !a->k || !a->v) return fail(JX_ERR_INVALID, "null pos/q/k/v");
    if (prefill && partials) return fail(JX_ERR_INVALID, "prefill writes outputs, not partials");
    std::vector<unsigned char> key = call_key(kv, layers, n_layers, a, partials, stream);
    if (!prefill && kv->replay_generation == kv->generation && key == kv->replay_key) {
        DeviceGuard guard(kv->d.device);
        if (!guard.ok) return fail(JX_ERR_CUDA, "cannot select device %d", kv->d.device);
        {
            const int rc = flush_staging(kv, stream);
            if (rc) return rc;
        }
        for (const DecodeLaunch& Lc : kv->replay) {
            const cudaError_t e = decode_launch(Lc);
            if (e != cudaSuccess)
                return fail(JX_ERR_CUDA, "decode launch failed: %s", cudaGetErrorString(e));
        }
        kv->last_launches = static_cast<int>(kv->replay.size());
        cudaStreamCaptureStatus cap_st = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(stream, &cap_st) == cudaSuccess && cap_st == cudaStreamCaptureStatusNone)
            return mark_plans_used(kv, kv->replay_slots, stream);
        return JX_OK;
    }
    kv->used_slots.clear();
    kv->replay_generation = ~0ull;
    kv->replay.clear();
    std::vector<DecodeLaunch> launched;
    const bool partial = partials != nullptr;
    if (!partial && !a->out) return fail(JX_ERR_INVALID, "null out");
    bool q_host = false, k_host = false, v_host = false;
    {
        bool h = false;
        int rc0 = check_step_ptr(a->q, "q", kv->d.device, &q_host);
        if (!rc0) rc0 = check_step_ptr(a->k, "k", kv->d.device, &k_host);
        if (!rc0) rc0 = check_step_ptr(a->v, "v", kv->d.device, &v_host);
        if (!rc0 && a->out) rc0 = check_step_ptr(a->out, "out", kv->d.device, &h);
        if (!rc0 && partial) rc0 = check_step_ptr(partials, "partials", kv->d.device, &h);
        if (rc0) return rc0;
    }
    if (a->n_kv_heads == 0 || a->n_heads == 0 || a->n_heads % a->n_kv_heads != 0)
        return fail(JX_ERR_UNSUPPORTED, "n_heads (%u) must be a multiple of n_kv_heads (%u)",
                    a->n_heads, a->n_kv_heads);
    const uint32_t G = a->n_heads / a->n_kv_heads;
    const int gp = gp_of(G);
    if (!gp) return fail(JX_ERR_UNSUPPORTED, "query group of %u heads exceeds 8", G);
    if (!(a->yarn_scale > 0.0f) && a->yarn_scale != 0.0f)
        return fail(JX_ERR_INVALID, "yarn_scale must not be negative or NaN");
    const jx_kv_desc& D = kv->d;
    std::vector<int> seqs(a->n_seqs);
    {
        // a step lists each sequence once; a prefill lists a sequence once per
        // token, each (sequence, position) once
        std::vector<char> seen(prefill ? 0 : D.n_seqs, 0);
        std::vector<std::pair<int, int>> rows;
        for (uint32_t s = 0; s < a->n_seqs; ++s) {
            const int sid = a->seq_ids ? a->seq_ids[s] : (prefill ? 0 : static_cast<int>(s));
            if (sid < 0 || static_cast<uint32_t>(sid) >= D.n_seqs)
                return fail(JX_ERR_INVALID, "sequence id %d outside [0, %u)", sid, D.n_seqs);
            if (a->pos[s] < 0) return fail(JX_ERR_INVALID, "negative position");
            if (prefill) {
                rows.emplace_back(sid, a->pos[s]);
            } else {
                if (seen[sid]) return fail(JX_ERR_INVALID, "sequence id %d listed twice", sid);
                seen[sid] = 1;
            }
            seqs[s] = sid;
        }
        if (prefill) {
            std::sort(rows.begin(), rows.end());
            if (std::adjacent_find(rows.begin(), rows.end()) != rows.end())
                return fail(JX_ERR_INVALID, "a (sequence, position) is listed twice");
        }
    }
    std::vector<char> appended(D.n_layers, 0);
    for (uint32_t l = 0; l < n_layers; ++l) {
        const jx_layer_desc& L = layers[l];
        const uint32_t hd = L.head_dim;
        if (hd != 32 && hd != 64 && hd != 128 && hd != 256)
            return fail(JX_ERR_UNSUPPORTED, "head_dim %u (compiled: 32, 64, 128, 256)", hd);
        if (hd * kv->esz < 64)
            return fail(JX_ERR_UNSUPPORTED, "head rows below 64 bytes are not supported");
        if (static_cast<uint64_t>(a->n_kv_heads) * hd > D.row_stride)
            return fail(JX_ERR_INVALID, "layer %u: kv_dim %u exceeds row_stride %u", l,
                        a->n_kv_heads * hd, D.row_stride);
        if (L.kv_source_layer >= D.n_layers)
            return fail(JX_ERR_INVALID, "layer %u: kv_source_layer %u >= %u", l, L.kv_source_layer,
                        D.n_layers);
        if (a->q_stride < a->n_heads * hd || a->kv_stride < a->n_kv_heads * hd)
            return fail(JX_ERR_INVALID, "q_stride/kv_stride smaller than the layer's rows");
        if (!L.shares_kv) appended[L.kv_source_layer] = 1;
    }
    const bool neox = a->rope_neox != 0;
    const float inv_cap = a->softcap > 0.0f ? 1.0f / a->softcap : 0.0f;

    // Launch groups: wave 0 = layers that do not read a cache layer appended
    // in this call by another layer; wave 1 = the rest.  Within a wave, one
    // launch per head_dim.
    struct Group {
        int hd;
        std::vector<uint32_t> layers;
    };
    std::vector<Group> groups;
    for (int wave = 0; wave < 2; ++wave) {
        const size_t first = groups.size();
        for (uint32_t l = 0; l < n_layers; ++l) {
            const jx_layer_desc& L = layers[l];
            const int w = (L.shares_kv && appended[L.kv_source_layer]) ? 1 : 0;
            if (w != wave) continue;
            Group* g = nullptr;
            for (size_t i = first; i < groups.size(); ++i)
                if (groups[i].hd == static_cast<int>(L.head_dim)) g = &groups[i];
            if (!g) {
                groups.push_back(Group{static_cast<int>(L.head_dim), {}});
                g = &groups.back();
            }
            g->layers.push_back(l);
        }
    }

    DeviceGuard guard(D.device);
    if (!guard.ok) return fail(JX_ERR_CUDA, "cannot select device %d", D.device);
    int launches = 0;
    for (size_t gi = 0; gi < groups.size(); ++gi) {
        const Group& grp = groups[gi];
        const int hd = grp.hd;
        if (prefill && kv->opt_prefill_tc && gp == static_cast<int>(G) &&
            prefill_tc_supported(hd, D.dtype, static_cast<int>(G))) {
            // 16-bit cache: append pass, then the prompt's attention on the
            // tensor cores, every K/V tile shared by 128/G tokens x G heads
            const int rc = prefill_tc(kv, layers, n_layers, grp.layers, a, seqs, hd, G, neox,
                                      inv_cap, gi, stream);
            if (rc) return rc;
            ++launches;
            continue;
        }
        // Prefill blocks: up to 8/G consecutive tokens of a sequence share one
        // pair (8 query columns: token x head), so their rows stream once.
        const int nq_max =
            (prefill && gp == static_cast<int>(G) && G <= 4) ? 8 / static_cast<int>(G) : 1;
        const bool blocks = nq_max > 1;
        const int gp_l = blocks ? 8 : gp;  // kernel query columns per segment
        const int kp = blocks ? 1 : kv_pack(hd, kv->esz, a->n_kv_heads, G, gp);
        const uint32_t n_kv = a->n_kv_heads / kp;  // segments per (sequence, layer) pair
        const int box_kind = kp * hd * kv->esz >= 128 ? 0 : 1;
        int rc = encode_maps(kv, box_kind);
        if (rc) return rc;
        // ---- pairs and rope rows
        std::vector<PairRow> pairs;
        pairs.reserve(static_cast<size_t>(a->n_seqs) * grp.layers.size());
        std::map<std::tuple<uint32_t, uint32_t, uint32_t, uint32_t, uint64_t, uint32_t>, int>
            rope_ids;
        std::vector<float2> rope;
        // inverse frequencies per RoPE configuration (rotated dims, base, factors)
        std::map<std::tuple<uint32_t, uint32_t, uint64_t>, std::vector<float>> inv_freqs;
        const int width = hd / 2;
        int n_rope_rows = 0;
        // step rows grouped into blocks (first row, tokens): single rows, or
        // in prefill runs of rows of one sequence at consecutive positions
        std::vector<std::pair<uint32_t, uint32_t>> blk;
        for (uint32_t r = 0; r < a->n_seqs;) {
            uint32_t nb = 1;
            if (blocks)
                while (nb < static_cast<uint32_t>(nq_max) && r + nb < a->n_seqs &&
                       seqs[r + nb] == seqs[r] &&
                       a->pos[r + nb] == a->pos[r] + static_cast<int32_t>(nb))
                    ++nb;
            blk.emplace_back(r, nb);
            r += nb;
        }
        long long off = 0;
        for (const auto& bk : blk) {
            const uint32_t s = bk.first, nb = bk.second;
            const uint32_t pos = static_cast<uint32_t>(a->pos[s]);  // first token
            const uint32_t pos_last = pos + nb - 1;
            for (uint32_t l : grp.layers) {
                const jx_layer_desc& L = layers[l];
                const uint32_t W = a->sliding_window;
                const uint64_t t0 = (L.is_swa && W > 0 && pos >= W) ? pos - W + 1 : 0;
                const uint64_t lo = std::max<uint64_t>(t0, D.pos_base);
                const uint64_t hi = std::min<uint64_t>(
                    pos_last, static_cast<uint64_t>(D.pos_base) + D.capacity - 1);
                const long long len = hi >= lo ? static_cast<long long>(hi - lo + 1) : 0;
                if (!partial && (lo != t0 || hi != pos_last))
                    return fail(JX_ERR_RANGE,
                                "position %u (window start %llu) is outside the cache rows "
                                "[%u, %llu); compact or roll back first",
                                pos_last, static_cast<unsigned long long>(t0), D.pos_base,
                                static_cast<unsigned long long>(D.pos_base) + D.capacity);
                PairRow pr{};
                pr.off = off;
                pr.seq = seqs[s];
                pr.io = static_cast<int>(s * n_layers + l);
                pr.cache_layer = static_cast<int>(L.kv_source_layer);
                pr.row0 = len > 0 ? static_cast<int>(lo - D.pos_base) : 0;
                pr.len = static_cast<int>(len);
                pr.append_row = (!L.shares_kv && pos >= D.pos_base &&
                                 static_cast<uint64_t>(pos_last) <
                                     static_cast<uint64_t>(D.pos_base) + D.capacity)
                                    ? static_cast<int>(pos - D.pos_base)
                                    : -1;
                pr.nq = static_cast<int>(nb);
                pr.io_step = static_cast<int>(n_layers);
                pr.tok_row0 = static_cast<int>(pos) - static_cast<int>(D.pos_base);
                pr.window = (L.is_swa && W > 0) ? static_cast<int>(W) : 0;
                const uint32_t rdim = std::min(L.head_dim, L.rope_dim);
                pr.rope_half = static_cast<int>(rdim / 2);
                const float* rf = (neox && !L.is_swa && L.rope_freqs) ? L.rope_freqs : nullptr;
                uint32_t base_bits, yarn_bits;
                std::memcpy(&base_bits, &L.rope_freq_base, 4);
                std::memcpy(&yarn_bits, &a->yarn_scale, 4);
                const uint64_t fh = rf ? hash_floats(rf, rdim / 2) : 0;
                // nb consecutive rows of the table: positions pos .. pos_last
                const auto key = std::make_tuple(rdim, base_bits, yarn_bits, pos, fh,
                                                 static_cast<uint32_t>(L.head_dim) * 16 + nb);
                auto itk = rope_ids.find(key);
                int rid;
                if (itk == rope_ids.end()) {
                    rid = n_rope_rows;
                    rope_ids.emplace(key, rid);
                    n_rope_rows += static_cast<int>(nb);
                    rope.resize(static_cast<size_t>(n_rope_rows) * width);
                    // the configuration's inverse frequencies, once per call
                    const auto fkey = std::make_tuple(rdim, base_bits, fh);
                    auto itf = inv_freqs.find(fkey);
                    if (itf == inv_freqs.end()) {
                        std::vector<float> f(rdim / 2);
                        rope_inv_freqs(L.head_dim, L.rope_dim, L.rope_freq_base, neox, rf,
                                       f.data());
                        itf = inv_freqs.emplace(fkey, std::move(f)).first;
                    }
                    for (uint32_t j = 0; j < nb; ++j)
                        rope_row_freqs(itf->second.data(), rdim / 2, pos + j, a->yarn_scale,
                                       rope.data() + static_cast<size_t>(rid + j) * width, width);
                } else {
                    rid = itk->second;
                }
                pr.rope_row = rid;
                pairs.push_back(pr);
                off += len * n_kv;
            }
        }
        const long long total = off;
        // The kernel trusts the plan: validate every row of it here.
        {
            long long o = 0;
            for (const PairRow& pr : pairs) {
                const bool ok = pr.off == o && pr.len >= 0 && pr.row0 >= 0 &&
                                static_cast<long long>(pr.row0) + pr.len <= D.capacity &&
                                pr.nq >= 1 && pr.nq <= nq_max &&
                                (pr.append_row < 0 ||
                                 (pr.append_row >= pr.row0 &&
                                  pr.append_row + pr.nq - 1 < pr.row0 + pr.len)) &&
                                pr.rope_row >= 0 && pr.rope_row + pr.nq - 1 < n_rope_rows &&
                                pr.io >= 0 &&
                                pr.io + (pr.nq - 1) * pr.io_step <
                                    static_cast<int>(a->n_seqs * n_layers) &&
                                pr.cache_layer >= 0 && pr.cache_layer < static_cast<int>(D.n_layers) &&
                                pr.seq >= 0 && pr.seq < static_cast<int>(D.n_seqs) &&
                                pr.rope_half >= 0 && pr.rope_half <= hd / 2;
                if (!ok) return fail(JX_ERR_INVALID, "internal: inconsistent work plan row");
                o += static_cast<long long>(pr.len) * n_kv;
            }
        }
        // ---- launch shape (cached per configuration)
        int stages = 0, cps = 0;
        const auto skey = std::make_tuple(hd, gp_l * 16 + kp, kv->opt_stages, kv->opt_ctas_per_sm);
        auto sit = kv->shapes.find(skey);
        if (sit != kv->shapes.end()) {
            stages = sit->second.first;
            cps = sit->second.second;
        } else {
            default_shape(hd, gp_l, kp, D.dtype, &stages, &cps);
            if (kv->opt_stages) stages = kv->opt_stages;
            if (decode_smem_bytes(hd, gp_l, kp, D.dtype, stages) < 0)
                return fail(JX_ERR_UNSUPPORTED, "no kernel for head_dim %d group %d dtype %d", hd,
                            gp, D.dtype);
            const int occ = decode_ctas_per_sm(hd, gp_l, kp, D.dtype, stages);
            if (occ <= 0)
                return fail(JX_ERR_UNSUPPORTED, "kernel does not fit with %d stages", stages);
            if (kv->opt_ctas_per_sm) cps = kv->opt_ctas_per_sm;
            cps = std::max(1, std::min(cps, occ));
            kv->shapes.emplace(skey, std::make_pair(stages, cps));
        }
        long long P = static_cast<long long>(kv->num_sms) * cps;
        P = std::min<long long>(P, std::max<long long>(1, (total + 63) / 64));
        if (kv->opt_grid) P = kv->opt_grid;
        if (total == 0) P = 1;
        // Slice boundaries: equal rows plus a cost per piece (merge, next q) --
        // a CTA whose slice crosses segment boundaries gets fewer rows.  With
        // the penalty at 0, uniform (CTA c takes rows [c*N/P, (c+1)*N/P)).
        const long long n_kv_segs = static_cast<long long>(pairs.size()) * n_kv;
        std::vector<long long> cta_begin;
        std::vector<int> seg_owner;  // [n_segs][2]: first and last CTA of each segment
        // measured best on B200 (c1/c2 sweeps): ~5 us per extra piece with the
        // CUDA-core consumer, ~8 us with the tensor-core one
        const double penalty_us = kv->opt_split_penalty_us >= 0.0f ? kv->opt_split_penalty_us
                                                                    : (kv->esz == 2 ? 8.0 : 5.0);
        const double penalty_rows =
            penalty_us * split_rows_per_us(kv, static_cast<size_t>(kp) * hd * kv->esz * 2, P);
        if (penalty_rows > 0.0 && total > 0) {
            std::vector<long long> seg_off;  // flattened start of each non-empty segment
            seg_off.reserve(static_cast<size_t>(n_kv_segs) + 1);
            for (const PairRow& pr : pairs)
                for (uint32_t h = 0; h < n_kv; ++h)
                    if (pr.len > 0) seg_off.push_back(pr.off + static_cast<long long>(h) * pr.len);
            seg_off.push_back(total);
            // the previous call's budget for this layout size as a warm start
            if (kv->split_hints.size() > 64) kv->split_hints.clear();
            long long& hint = kv->split_hints[std::make_pair(static_cast<long long>(seg_off.size()), P)];
            cta_begin = balanced_split(seg_off, total, P, penalty_rows, -1, &hint);
            seg_owner.assign(static_cast<size_t>(n_kv_segs) * 2, 0);
            size_t c = 0;
            long long si = 0;
            for (const PairRow& pr : pairs)
                for (uint32_t h = 0; h < n_kv; ++h, ++si) {
                    if (pr.len <= 0) continue;
                    const long long first = pr.off + static_cast<long long>(h) * pr.len;
                    const long long last = first + pr.len - 1;
                    while (c + 1 < static_cast<size_t>(P) && cta_begin[c + 1] <= first) ++c;
                    size_t d = c;
                    while (d + 1 < static_cast<size_t>(P) && cta_begin[d + 1] <= last) ++d;
                    seg_owner[2 * si] = static_cast<int>(c);
                    seg_owner[2 * si + 1] = static_cast<int>(d);
                }
        }
        // each CTA's first pair (the kernel then needs no search to find its slice)
        std::vector<int> cta_pair(static_cast<size_t>(P), 0);
        for (long long c = 0; c < P; ++c) {
            const long long x = cta_begin.empty() ? total * c / P : cta_begin[c];
            int lo = 0, hi = static_cast<int>(pairs.size()) - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (pairs[mid].off <= x) lo = mid; else hi = mid - 1;
            }
            cta_pair[c] = lo;
        }
        const size_t pair_bytes = pairs.size() * sizeof(PairRow);
        const size_t rope_off = (pair_bytes + 255) & ~static_cast<size_t>(255);
        const size_t rope_bytes = rope.size() * sizeof(float2);
        const size_t cta_off = (rope_off + rope_bytes + 255) & ~static_cast<size_t>(255);
        const size_t begin_off =
            (cta_off + cta_pair.size() * sizeof(int) + 255) & ~static_cast<size_t>(255);
        const size_t owner_off =
            (begin_off + cta_begin.size() * sizeof(long long) + 255) & ~static_cast<size_t>(255);
        std::vector<unsigned char> bytes(owner_off + seg_owner.size() * sizeof(int), 0);
        std::memcpy(bytes.data(), pairs.data(), pair_bytes);
        if (!rope.empty()) std::memcpy(bytes.data() + rope_off, rope.data(), rope_bytes);
        std::memcpy(bytes.data() + cta_off, cta_pair.data(), cta_pair.size() * sizeof(int));
        if (!cta_begin.empty()) {
            std::memcpy(bytes.data() + begin_off, cta_begin.data(),
                        cta_begin.size() * sizeof(long long));
            std::memcpy(bytes.data() + owner_off, seg_owner.data(), seg_owner.size() * sizeof(int));
        }
        rc = upload_plan(kv, gi, bytes, stream);
        if (rc) return rc;
        rc = flush_staging(kv, stream);
        if (rc) return rc;
        if (prefill && !pairs.empty()) {
            // all of this group's rows are stored before any of them is attended
            const PairRow* dp = static_cast<const PairRow*>(kv->slots[gi].d_buf);
            const float2* dr = reinterpret_cast<const float2*>(
                static_cast<unsigned char*>(kv->slots[gi].d_buf) + rope_off);
            const int np = static_cast<int>(pairs.size());
            const int nkv = static_cast<int>(a->n_kv_heads);
#define JX_APPEND(DTV)                                                                      \
    append_rows_kernel<DTV><<<np, 128, 0, stream>>>(dp, np, dr, width, a->k, a->v,          \
                                                    a->kv_stride, nkv, hd, neox ? 1 : 0,     \
                                                    kv->k, kv->v, kv->seq_stride,            \
                                                    kv->layer_stride, D.row_stride)
            if (D.dtype == JX_F32) JX_APPEND(DT_F32);
            else if (D.dtype == JX_BF16) JX_APPEND(DT_BF16);
            else JX_APPEND(DT_F16T);
#undef JX_APPEND
            const cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess)
                return fail(JX_ERR_CUDA, "append launch failed: %s", cudaGetErrorString(e));
        }
        const long long n_segs = static_cast<long long>(pairs.size()) * n_kv;
        rc = ensure_scratch(kv, static_cast<size_t>(P + n_segs) * gp_l * kp * (hd + 2),
                            static_cast<size_t>(std::max<long long>(n_segs, 1)));
        if (rc) return rc;

        DecodeLaunch Lc{};
        DecodeArgs& A = Lc.args;
        A.pairs = static_cast<const PairRow*>(kv->slots[gi].d_buf);
        A.cta_pair = reinterpret_cast<const int*>(static_cast<unsigned char*>(kv->slots[gi].d_buf) +
                                                  cta_off);
        A.cta_begin = cta_begin.empty() ? nullptr
                                        : reinterpret_cast<const long long*>(
                                              static_cast<unsigned char*>(kv->slots[gi].d_buf) +
                                              begin_off);
        A.seg_owner = seg_owner.empty() ? nullptr
                                        : reinterpret_cast<const int*>(
                                              static_cast<unsigned char*>(kv->slots[gi].d_buf) +
                                              owner_off);
        A.n_pairs = static_cast<int>(pairs.size());
        A.n_kv = static_cast<int>(n_kv);
        A.G = static_cast<int>(G) * kp;
        A.n_heads = static_cast<int>(a->n_heads);
        A.total = total;
        A.q = a->q;
        A.k_in = a->k;
        A.v_in = a->v;
        A.out = a->out;
        A.q_stride = a->q_stride;
        A.kv_stride = a->kv_stride;
        A.k_cache = kv->k;
        A.v_cache = kv->v;
        A.seq_stride = kv->seq_stride;
        A.layer_stride = kv->layer_stride;
        A.row_stride = D.row_stride;
        A.rope = reinterpret_cast<const float2*>(static_cast<unsigned char*>(kv->slots[gi].d_buf) +
                                                 rope_off);
        A.scale = a->scale;
        A.softcap = a->softcap;
        A.inv_softcap = inv_cap;
        A.neox = neox ? 1 : 0;
        A.scratch = kv->d_scratch;
        A.counters = kv->d_counters;
        A.part_out = partial ? partials : nullptr;
        A.err = kv->d_err;
        A.n_stages = stages;
        A.n_consumers = consumers_for(stages, kp);
        // bulk prefetch of q (and of the k/v rows the step appends): device
        // memory, 16-byte rows (prefill blocks and host-resident inputs are
        // read with ordinary loads)
        A.q_bulk = (!blocks && !q_host && !k_host && !v_host &&
                    reinterpret_cast<uintptr_t>(a->q) % 16 == 0 && a->q_stride % 4 == 0 &&
                    reinterpret_cast<uintptr_t>(a->k) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(a->v) % 16 == 0 && a->kv_stride % 4 == 0)
                       ? 1 : 0;
        A.skip_append = prefill ? 1 : 0;
        A.test_wait_cta = kv->opt_test_wait_cta;
        A.wait_limit = wait_limit_cycles(kv->opt_wait_limit_ms);
        A.n_io = static_cast<long long>(a->n_seqs) * n_layers;
        A.cache_elems = kv->seq_stride * D.n_seqs;
        A.scratch_floats = static_cast<long long>(kv->scratch_floats);
        A.n_segments = n_segs;
        A.n_rope_rows = n_rope_rows;
        A.capacity = static_cast<int>(D.capacity);
        A.n_cache_layers = static_cast<int>(D.n_layers);
        A.n_cache_seqs = static_cast<int>(D.n_seqs);
        A.smem_bytes = decode_smem_bytes(hd, gp_l, kp, D.dtype, stages);
        A.dbg = kv->d_dbg;
        Lc.tmK = &kv->tmK[box_kind];
        Lc.tmV = &kv->tmV[box_kind];
        Lc.head_dim = hd;
        Lc.gp = gp_l;
        Lc.kp = kp;
        Lc.dtype = D.dtype;
        Lc.grid = static_cast<int>(P);
        Lc.stages = stages;
        // Default on: measured -3 % (c2), -5 % (c2 bf16), -7 % (c1) per step.
        Lc.pdl = kv->opt_pdl >= 0 ? kv->opt_pdl : 1;
        Lc.stream = stream;
        if (total == 0 && !partial) continue;
        const cudaError_t e = decode_launch(Lc);
        if (e != cudaSuccess)
            return fail(JX_ERR_CUDA, "decode launch failed: %s", cudaGetErrorString(e));
        ++launches;
        launched.push_back(Lc);
    }
    kv->last_launches = launches;
    {
        const int rc = flush_staging(kv, stream);
        if (rc) return rc;
    }
    {
        cudaStreamCaptureStatus cap_st = cudaStreamCaptureStatusNone;
        JX_CUDA(cudaStreamIsCapturing(stream, &cap_st));
        if (cap_st == cudaStreamCaptureStatusNone) {
            const int rc = mark_plans_used(kv, kv->used_slots, stream);
            if (rc) return rc;
        }
    }
    if (prefill) return JX_OK;  // not replayed: its append launches are not recorded
    kv->replay_key = std::move(key);
    kv->replay = std::move(launched);
    kv->replay_slots = kv->used_slots;
    kv->replay_generation = kv->generation;
    return JX_OK;
}

// NCCL entry points used by the sharded step, taken from the process's
// libnccl.so.2 (the copy a framework already loaded, else the system one), so
// the library has no link-time NCCL dependency.
struct NcclApi {
    bool ok = false;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*comm_user_rank)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    const char* (*get_error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl_api() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.comm_count = reinterpret_cast<decltype(api.comm_count)>(dlsym(h, "ncclCommCount"));
        api.comm_user_rank =
            reinterpret_cast<decltype(api.comm_user_rank)>(dlsym(h, "ncclCommUserRank"));
        api.comm_get_async_error = reinterpret_cast<decltype(api.comm_get_async_error)>(
            dlsym(h, "ncclCommGetAsyncError"));
        api.get_error_string =
            reinterpret_cast<decltype(api.get_error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.all_gather && api.comm_count && api.comm_user_rank &&
                 api.comm_get_async_error && api.get_error_string;
    });
    return api;
}

int grow(float** p, size_t* have, size_t need) {
    if (*have >= need) return JX_OK;
    if (*p) JX_CUDA(cudaFree(*p));
    *p = nullptr;
    *have = 0;
    if (cudaMalloc(p, need * sizeof(float)) != cudaSuccess)
        return fail(JX_ERR_NOMEM, "allocation of %zu floats failed", need);
    *have = need;
    return JX_OK;
}

// Waits for `stream` to reach the point of the call, polling NCCL's
// asynchronous error.  It never aborts the communicator itself: whether to
// abort (and how the process recovers) stays with the caller.
int wait_sharded(const NcclApi& nc, ncclComm_t comm, cudaStream_t stream, uint32_t timeout_ms) {
    cudaEvent_t ev = nullptr;
    JX_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    cudaError_t e = cudaEventRecord(ev, stream);
    if (e != cudaSuccess) {
        cudaEventDestroy(ev);
        return fail(JX_ERR_CUDA, "cudaEventRecord: %s", cudaGetErrorString(e));
    }
    const auto t0 = std::chrono::steady_clock::now();
    int rc = JX_OK;
    for (;;) {
        e = cudaEventQuery(ev);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) {
            rc = fail(JX_ERR_CUDA, "sharded step: %s", cudaGetErrorString(e));
            break;
        }
        ncclResult_t ae = ncclSuccess;
        if (nc.comm_get_async_error(comm, &ae) == ncclSuccess && ae != ncclSuccess &&
            ae != ncclInProgress) {
            rc = fail(JX_ERR_COMM, "NCCL asynchronous error: %s", nc.get_error_string(ae));
            break;
        }
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0)
                            .count();
        if (ms > static_cast<long long>(timeout_ms)) {
            rc = fail(JX_ERR_TIMEOUT,
                      "sharded step did not complete within %u ms (a rank did not join?)",
                      timeout_ms);
            break;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    cudaEventDestroy(ev);
    return rc;
}

}  // namespace

namespace {

// step_impl between two events when the handle's "timing" option is on: the
// device time of everything the step queued (plan upload when it changed,
// launches) -- the counterpart of forward_token's attention_ms
// (transformer.cpp:2499, 2567).
// Host-resident (pinned) q, k and v are copied into device memory by one
// small kernel at the start of the step, and the step then reads the copies:
// read in place over PCIe, every CTA that shares a segment fetched the same
// q rows, and each piece's q (and the new row's k, v) stalled its consumers
// for a PCIe round trip.  *staged receives the arguments to use (unchanged
// when nothing is host-resident).  The copies cover exactly the rows the
// step reads: [rows - 1] strides plus the last row.
int stage_host_inputs(jx_kv* kv, const jx_layer_desc* layers, uint32_t n_layers,
                      const jx_step_args* a, cudaStream_t stream, jx_step_args* staged) {
    *staged = *a;
    if (!a->q || !a->k || !a->v || n_layers == 0 || a->n_seqs == 0) return JX_OK;
    // arguments step_impl would refuse are left to it: nothing is read here
    if (a->n_kv_heads == 0 || a->n_heads == 0 || a->n_heads % a->n_kv_heads != 0) return JX_OK;
    for (uint32_t l = 0; l < n_layers; ++l) {
        const uint32_t hd = layers[l].head_dim;
        if ((hd != 32 && hd != 64 && hd != 128 && hd != 256) ||
            a->q_stride < static_cast<uint64_t>(a->n_heads) * hd ||
            a->kv_stride < static_cast<uint64_t>(a->n_kv_heads) * hd)
            return JX_OK;
    }
    bool host[3] = {false, false, false};
    const void* ptr[3] = {a->q, a->k, a->v};
    for (int b = 0; b < 3; ++b) {
        // queried on every call: a buffer freed and replaced at the same
        // address may no longer be pinned
        cudaPointerAttributes at{};
        if (cudaPointerGetAttributes(&at, ptr[b]) != cudaSuccess) {
            cudaGetLastError();
            return JX_OK;  // step_impl reports the bad pointer
        }
        host[b] = at.type == cudaMemoryTypeHost;
    }
    if (!host[0] && !host[1] && !host[2]) return JX_OK;
    const long long rows = static_cast<long long>(a->n_seqs) * n_layers;
    const long long hd_last = layers[n_layers - 1].head_dim;
    const long long n_q = (rows - 1) * a->q_stride + static_cast<long long>(a->n_heads) * hd_last;
    const long long n_kv = (rows - 1) * a->kv_stride + static_cast<long long>(a->n_kv_heads) * hd_last;
    if (n_q <= 0 || n_kv <= 0) return JX_OK;  // step_impl reports the bad shape
    const long long off_k = (n_q + 3) & ~3ll, off_v = off_k + ((n_kv + 3) & ~3ll);
    float* before = kv->d_stage;
    int rc = grow(&kv->d_stage, &kv->stage_floats, static_cast<size_t>(off_v + n_kv));
    if (rc) return rc;
    if (kv->d_stage != before) ++kv->generation;  // recorded launches name the old copy
    const float* src[3] = {host[0] ? a->q : nullptr, host[1] ? a->k : nullptr,
                           host[2] ? a->v : nullptr};
    float* dst[3] = {kv->d_stage, kv->d_stage + off_k, kv->d_stage + off_v};
    const long long work = (host[0] ? n_q : 0) + (host[1] ? 2 * n_kv : 0);
    const int grid = static_cast<int>(std::min<long long>(
        std::max<long long>((work / 4 + 255) / 256, 1), 4ll * std::max(kv->num_sms, 1)));
    // launched by the step (flush_staging) right before its first kernel
    auto& p = kv->pend;
    p.active = true;
    p.grid = grid;
    const long long nn[3] = {n_q, n_kv, n_kv};
    for (int b = 0; b < 3; ++b) {
        p.src[b] = src[b];
        p.dst[b] = dst[b];
        p.n[b] = nn[b];
    }
    if (host[0]) staged->q = dst[0];
    if (host[1]) staged->k = dst[1];
    if (host[2]) staged->v = dst[2];
    return JX_OK;
}

int timed_step(jx_kv* kv, const jx_layer_desc* layers, uint32_t n_layers, const jx_step_args* a,
               float* partials, cudaStream_t stream, bool prefill = false) {
    if (!kv || !layers || !a) return step_impl(kv, layers, n_layers, a, partials, stream, prefill);
    DeviceGuard guard(kv->d.device);
    if (!guard.ok) return fail(JX_ERR_CUDA, "cannot select device %d", kv->d.device);
    if (kv->opt_timing) {
        if (!kv->ev_t0) JX_CUDA(cudaEventCreate(&kv->ev_t0));
        if (!kv->ev_t1) JX_CUDA(cudaEventCreate(&kv->ev_t1));
        JX_CUDA(cudaEventRecord(kv->ev_t0, stream));
    }
    jx_step_args staged{};
    int rc = stage_host_inputs(kv, layers, n_layers, a, stream, &staged);
    if (!rc) rc = step_impl(kv, layers, n_layers, &staged, partials, stream, prefill);
    kv->pend.active = false;  // a call that failed before its first launch copies nothing
    if (kv->opt_timing) {
        JX_CUDA(cudaEventRecord(kv->ev_t1, stream));
        kv->timed = rc == JX_OK;
    }
    return rc;
}

}  // namespace

// ================================================================== C ABI

extern "C" {

const char* jx_last_error_string(void) { return g_err.c_str(); }

const char* jx_version(void) { return "jxai_b200 decode-attention 0.1 (sm_100a)"; }

int jx_kv_create(const jx_kv_desc* desc, jx_kv** out) {
    if (!desc || !out) return fail(JX_ERR_INVALID, "null desc/out");
    *out = nullptr;
    const jx_kv_desc& d = *desc;
    if (d.n_seqs == 0 || d.n_layers == 0 || d.capacity == 0 || d.row_stride == 0)
        return fail(JX_ERR_INVALID, "n_seqs, n_layers, capacity and row_stride must be positive");
    if (d.dtype < 0 || d.dtype > 2) return fail(JX_ERR_INVALID, "unknown dtype %d", d.dtype);
    const size_t esz = d.dtype == JX_F32 ? 4 : 2;
    if ((d.row_stride * esz) % 16 != 0)
        return fail(JX_ERR_UNSUPPORTED, "row_stride*element size must be a multiple of 16 bytes");
    if (static_cast<uint64_t>(d.pos_base) + d.capacity > (1ull << 31))
        return fail(JX_ERR_INVALID, "positions must stay below 2^31");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return fail(JX_ERR_CUDA, "no CUDA device (this library has no CPU path)");
    if (d.device < 0 || d.device >= ndev) return fail(JX_ERR_INVALID, "device %d absent", d.device);
    DeviceGuard guard(d.device);
    if (!guard.ok) return fail(JX_ERR_CUDA, "cannot select device %d", d.device);
    cudaDeviceProp prop;
    JX_CUDA(cudaGetDeviceProperties(&prop, d.device));
    if (prop.major < 10)
        return fail(JX_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", d.device,
                    prop.major, prop.minor);
    jx_kv* kv = new jx_kv();
    kv->d = d;
    kv->esz = esz;
    kv->num_sms = prop.multiProcessorCount;
    kv->layer_stride = static_cast<long long>(d.capacity) * d.row_stride;
    kv->seq_stride = kv->layer_stride * d.n_layers;
    kv->seq_pos.assign(d.n_seqs, 0);
    const size_t bytes = static_cast<size_t>(kv->seq_stride) * d.n_seqs * esz;
    auto cleanup = [&](int code) {
        jx_kv_destroy(kv);
        return code;
    };
    if (cudaMalloc(&kv->k, bytes) != cudaSuccess || cudaMalloc(&kv->v, bytes) != cudaSuccess) {
        cudaGetLastError();
        return cleanup(fail(JX_ERR_NOMEM, "KV cache allocation of 2 x %zu bytes failed", bytes));
    }
    if (cudaMemset(kv->k, 0, bytes) != cudaSuccess || cudaMemset(kv->v, 0, bytes) != cudaSuccess ||
        cudaMalloc(&kv->d_err, sizeof(int)) != cudaSuccess ||
        cudaMemset(kv->d_err, 0, sizeof(int)) != cudaSuccess ||
        cudaMalloc(&kv->d_dbg, 8 * sizeof(int)) != cudaSuccess ||
        cudaMemset(kv->d_dbg, 0, 8 * sizeof(int)) != cudaSuccess ||
        cudaMalloc(&kv->d_rows, sizeof(uint32_t) * d.n_seqs) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess)
        return cleanup(fail(JX_ERR_CUDA, "cache initialisation failed"));
    *out = kv;
    return JX_OK;
}

int jx_kv_destroy(jx_kv* kv) {
    if (!kv) return JX_OK;
    DeviceGuard guard(kv->d.device);
    cudaDeviceSynchronize();
    cudaFree(kv->k);
    cudaFree(kv->v);
    cudaFree(kv->d_err);
    cudaFree(kv->d_dbg);
    cudaFree(kv->d_rows);
    cudaFree(kv->d_scratch);
    cudaFree(kv->d_counters);
    cudaFree(kv->d_part);
    cudaFree(kv->d_gather);
    cudaFree(kv->d_stage);
    if (kv->ev_t0) cudaEventDestroy(kv->ev_t0);
    if (kv->ev_t1) cudaEventDestroy(kv->ev_t1);
    for (PlanSlot& s : kv->slots) {
        for (int b = 0; b < kStaging; ++b) {
            if (s.ev_copy[b]) cudaEventDestroy(s.ev_copy[b]);
            if (s.ev_used[b]) cudaEventDestroy(s.ev_used[b]);
            if (s.h_buf[b]) cudaFreeHost(s.h_buf[b]);
            cudaFree(s.d_ring[b]);
        }
    }
    if (kv->up_stream) cudaStreamDestroy(kv->up_stream);
    delete kv;
    return JX_OK;
}

int jx_kv_get_desc(const jx_kv* kv, jx_kv_desc* desc) {
    if (!kv || !desc) return fail(JX_ERR_INVALID, "null argument");
    *desc = kv->d;
    return JX_OK;
}

int jx_kv_get_seq_pos(const jx_kv* kv, uint32_t seq, uint32_t* seq_pos) {
    if (!kv || !seq_pos || seq >= kv->d.n_seqs) return fail(JX_ERR_INVALID, "bad handle/sequence");
    *seq_pos = kv->seq_pos[seq];
    return JX_OK;
}

int jx_kv_set_seq_pos(jx_kv* kv, uint32_t seq, uint32_t seq_pos) {
    if (!kv || seq >= kv->d.n_seqs) return fail(JX_ERR_INVALID, "bad handle/sequence");
    if (seq_pos > kv->d.capacity) return fail(JX_ERR_RANGE, "seq_pos beyond capacity");
    kv->seq_pos[seq] = seq_pos;
    return JX_OK;
}

int jx_kv_clear(jx_kv* kv, uint32_t seq, void* stream) {
    if (!kv || seq >= kv->d.n_seqs) return fail(JX_ERR_INVALID, "bad handle/sequence");
    DeviceGuard guard(kv->d.device);
    const size_t bytes = static_cast<size_t>(kv->seq_stride) * kv->esz;
    const size_t off = static_cast<size_t>(seq) * bytes;
    JX_CUDA(cudaMemsetAsync(static_cast<char*>(kv->k) + off, 0, bytes, (cudaStream_t)stream));
    JX_CUDA(cudaMemsetAsync(static_cast<char*>(kv->v) + off, 0, bytes, (cudaStream_t)stream));
    kv->seq_pos[seq] = 0;
    return JX_OK;
}

int jx_kv_rollback(jx_kv* kv, uint32_t seq, uint32_t new_seq_pos) {
    if (!kv || seq >= kv->d.n_seqs) return fail(JX_ERR_INVALID, "bad handle/sequence");
    if (new_seq_pos < kv->seq_pos[seq]) kv->seq_pos[seq] = new_seq_pos;
    return JX_OK;
}

int jx_kv_compact(jx_kv* kv, uint32_t seq, uint32_t keep_recent, void* stream) {
    if (!kv || seq >= kv->d.n_seqs) return fail(JX_ERR_INVALID, "bad handle/sequence");
    const uint32_t sink = 4;
    const uint32_t sp = kv->seq_pos[seq];
    if (sp <= sink + keep_recent) return JX_OK;
    DeviceGuard guard(kv->d.device);
    const uint32_t src_start = sp - keep_recent;
    const size_t row_b = static_cast<size_t>(kv->d.row_stride) * kv->esz;
    const size_t layer_b = static_cast<size_t>(kv->layer_stride) * kv->esz;
    const size_t seq_off = static_cast<size_t>(seq) * kv->seq_stride * kv->esz;
    cudaStream_t st = (cudaStream_t)stream;
    // memmove of rows [src_start, src_start + keep) down to row `sink` in
    // every layer (transformer.cpp:48-60).  Source and destination overlap when
    // keep > src_start - sink, so the rows go in chunks of d = src_start - sink
    // rows, front to back: chunk i reads rows that no earlier chunk writes and
    // writes only rows chunk i-1 already read, and copies on one stream run in
    // order -- memmove's result with no temporary buffer, no allocation and no
    // host wait.  The reference's own trigger (keep = capacity/2 at seq_pos =
    // capacity, :2373) takes two chunks per tensor.
    const uint32_t d = src_start - sink;
    for (uint32_t r = 0; r < keep_recent; r += d) {
        const uint32_t n = std::min(d, keep_recent - r);
        for (int which = 0; which < 2; ++which) {
            char* basep = static_cast<char*>(which == 0 ? kv->k : kv->v) + seq_off;
            JX_CUDA(cudaMemcpy2DAsync(basep + (sink + r) * row_b, layer_b,
                                      basep + (src_start + r) * row_b, layer_b,
                                      static_cast<size_t>(n) * row_b, kv->d.n_layers,
                                      cudaMemcpyDeviceToDevice, st));
        }
    }
    kv->seq_pos[seq] = sink + keep_recent;
    return JX_OK;
}

int jx_kv_copy_rows(jx_kv* kv, uint32_t seq, uint32_t layer, int which, uint32_t row0,
                    uint32_t n_rows, void* buf, int to_cache, void* stream) {
    if (!kv || !buf || seq >= kv->d.n_seqs || layer >= kv->d.n_layers || (which != 0 && which != 1))
        return fail(JX_ERR_INVALID, "bad copy_rows arguments");
    if (static_cast<uint64_t>(row0) + n_rows > kv->d.capacity)
        return fail(JX_ERR_RANGE, "rows [%u, %u) beyond capacity %u", row0, row0 + n_rows,
                    kv->d.capacity);
    DeviceGuard guard(kv->d.device);
    const size_t row_b = static_cast<size_t>(kv->d.row_stride) * kv->esz;
    char* p = static_cast<char*>(which == 0 ? kv->k : kv->v) +
              (static_cast<size_t>(seq) * kv->seq_stride +
               static_cast<size_t>(layer) * kv->layer_stride) * kv->esz +
              static_cast<size_t>(row0) * row_b;
    const size_t n = static_cast<size_t>(n_rows) * row_b;
    if (to_cache)
        JX_CUDA(cudaMemcpyAsync(p, buf, n, cudaMemcpyDefault, (cudaStream_t)stream));
    else
        JX_CUDA(cudaMemcpyAsync(buf, p, n, cudaMemcpyDefault, (cudaStream_t)stream));
    return JX_OK;
}

int jx_kv_layer_ptr(jx_kv* kv, uint32_t seq, uint32_t layer, int which, void** ptr) {
    if (!kv || !ptr || seq >= kv->d.n_seqs || layer >= kv->d.n_layers || (which != 0 && which != 1))
        return fail(JX_ERR_INVALID, "bad layer_ptr arguments");
    *ptr = static_cast<char*>(which == 0 ? kv->k : kv->v) +
           (static_cast<size_t>(seq) * kv->seq_stride + static_cast<size_t>(layer) * kv->layer_stride) *
               kv->esz;
    return JX_OK;
}

int jx_attn_step(jx_kv* kv, const jx_layer_desc* layers, uint32_t n_layers,
                 const jx_step_args* args, void* stream) {
    return timed_step(kv, layers, n_layers, args, nullptr, (cudaStream_t)stream);
}

int jx_attn_step_partial(jx_kv* kv, const jx_layer_desc* layers, uint32_t n_layers,
                         const jx_step_args* args, float* partials, void* stream) {
    if (!partials) return fail(JX_ERR_INVALID, "null partials");
    return timed_step(kv, layers, n_layers, args, partials, (cudaStream_t)stream);
}

int jx_attn_prefill(jx_kv* kv, const jx_layer_desc* layers, uint32_t n_layers,
                    const jx_step_args* args, void* stream) {
    return timed_step(kv, layers, n_layers, args, nullptr, (cudaStream_t)stream, true);
}

int jx_kv_last_step_ms(jx_kv* kv, float* ms) {
    if (!kv || !ms) return fail(JX_ERR_INVALID, "null argument");
    if (!kv->timed) return fail(JX_ERR_INVALID, "no timed step (set option \"timing\" to 1)");
    DeviceGuard guard(kv->d.device);
    JX_CUDA(cudaEventSynchronize(kv->ev_t1));
    JX_CUDA(cudaEventElapsedTime(ms, kv->ev_t0, kv->ev_t1));
    return JX_OK;
}

int jx_attn_step_sharded(jx_kv* kv, const jx_layer_desc* layers, uint32_t n_layers,
                         const jx_step_args* args, void* nccl_comm, uint32_t timeout_ms,
                         void* stream) {
    if (!kv || !layers || !args || !nccl_comm || !args->out || n_layers == 0)
        return fail(JX_ERR_INVALID, "null handle, layers, args, communicator or output");
    const uint32_t hd = layers[0].head_dim;
    for (uint32_t l = 1; l < n_layers; ++l)
        if (layers[l].head_dim != hd)
            return fail(JX_ERR_UNSUPPORTED, "all layers of a sharded step must share head_dim");
    if (args->n_seqs == 0 || args->n_heads == 0 || hd == 0)
        return fail(JX_ERR_INVALID, "empty step");
    if (args->q_stride < static_cast<uint64_t>(args->n_heads) * hd)
        return fail(JX_ERR_INVALID, "q_stride smaller than n_heads*head_dim");
    const NcclApi& nc = nccl_api();
    if (!nc.ok) return fail(JX_ERR_COMM, "NCCL (libnccl.so.2) is not available in this process");
    ncclComm_t comm = static_cast<ncclComm_t>(nccl_comm);
    int world = 0, rank = -1;
    if (nc.comm_count(comm, &world) != ncclSuccess || nc.comm_user_rank(comm, &rank) != ncclSuccess ||
        world <= 0 || rank < 0 || rank >= world)
        return fail(JX_ERR_COMM, "cannot query the communicator's size and rank");
    const uint64_t groups = static_cast<uint64_t>(args->n_seqs) * n_layers;
    const size_t per = static_cast<size_t>(groups * args->n_heads * (hd + 2));
    DeviceGuard guard(kv->d.device);
    if (!guard.ok) return fail(JX_ERR_CUDA, "cannot select device %d", kv->d.device);
    int rc = grow(&kv->d_part, &kv->part_floats, per);
    if (!rc) rc = grow(&kv->d_gather, &kv->gather_floats, per * static_cast<size_t>(world));
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    rc = jx_attn_step_partial(kv, layers, n_layers, args, kv->d_part, stream);
    if (rc) return rc;
    const ncclResult_t r = nc.all_gather(kv->d_part, kv->d_gather, per, ncclFloat32, comm, st);
    if (r == ncclInProgress) {
        // A non-blocking communicator (blocking = 0) may still be connecting:
        // the all-gather is accepted and goes on in the background; no other
        // NCCL call may be made on it until its state leaves ncclInProgress.
        const uint32_t limit_ms = timeout_ms > 0 ? timeout_ms : 120000;
        const auto t0 = std::chrono::steady_clock::now();
        for (;;) {
            ncclResult_t ae = ncclInProgress;
            if (nc.comm_get_async_error(comm, &ae) != ncclSuccess)
                return fail(JX_ERR_COMM, "ncclCommGetAsyncError failed");
            if (ae == ncclSuccess) break;
            if (ae != ncclInProgress)
                return fail(JX_ERR_COMM, "ncclAllGather: %s", nc.get_error_string(ae));
            const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                                std::chrono::steady_clock::now() - t0).count();
            if (ms > static_cast<long long>(limit_ms))
                return fail(JX_ERR_TIMEOUT,
                            "ncclAllGather still in progress after %u ms (a rank that never "
                            "joined?)", limit_ms);
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
    } else if (r != ncclSuccess) {
        return fail(JX_ERR_COMM, "ncclAllGather: %s", nc.get_error_string(r));
    }
    rc = jx_lse_merge(kv->d_gather, static_cast<uint32_t>(world), per, static_cast<uint32_t>(groups),
                      args->n_heads, hd, args->out, static_cast<uint32_t>(args->q_stride), stream);
    if (rc) return rc;
    if (timeout_ms > 0) return wait_sharded(nc, comm, st, timeout_ms);
    return JX_OK;
}

int jx_lse_merge(const float* gathered, uint32_t n_shards, uint64_t shard_stride,
                 uint32_t n_groups, uint32_t n_heads, uint32_t head_dim, float* out,
                 uint32_t out_stride, void* stream) {
    if (!gathered || !out || n_shards == 0 || n_groups == 0 || n_heads == 0 || head_dim == 0)
        return fail(JX_ERR_INVALID, "bad lse_merge arguments");
    if (shard_stride < static_cast<uint64_t>(n_groups) * n_heads * (head_dim + 2))
        return fail(JX_ERR_INVALID, "shard_stride smaller than one shard's partials");
    if (out_stride < n_heads * head_dim) return fail(JX_ERR_INVALID, "out_stride too small");
    const int rows = static_cast<int>(n_groups * n_heads);
    lse_merge_kernel<<<rows, 128, 0, (cudaStream_t)stream>>>(
        gathered, static_cast<int>(n_shards), static_cast<long long>(shard_stride), rows,
        static_cast<int>(n_heads), static_cast<int>(head_dim), out, out_stride);
    JX_CUDA(cudaGetLastError());
    return JX_OK;
}

int jx_kv_check_device_error(jx_kv* kv, int* code, void* stream) {
    if (!kv || !code) return fail(JX_ERR_INVALID, "null argument");
    DeviceGuard guard(kv->d.device);
    int h = 0, dbg[8] = {0};
    cudaStream_t st = (cudaStream_t)stream;
    JX_CUDA(cudaMemcpyAsync(&h, kv->d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
    JX_CUDA(cudaMemcpyAsync(dbg, kv->d_dbg, sizeof dbg, cudaMemcpyDeviceToHost, st));
    JX_CUDA(cudaStreamSynchronize(st));
    JX_CUDA(cudaMemsetAsync(kv->d_err, 0, sizeof(int), st));
    JX_CUDA(cudaMemsetAsync(kv->d_dbg, 0, sizeof dbg, st));
    JX_CUDA(cudaStreamSynchronize(st));
    *code = h;
    if (h == kDevErrWaitTimeout)
        return fail(JX_ERR_DEVICE,
                    "a decode kernel's bounded wait ran out: site %d block %d thread %d tile %d "
                    "after %lld cycles (%d ms of global timer)",
                    dbg[0] - 100, dbg[1], dbg[2], dbg[5],
                    static_cast<long long>((static_cast<uint64_t>(static_cast<uint32_t>(dbg[4])) << 32) |
                                           static_cast<uint32_t>(dbg[3])),
                    dbg[6]);
    if (h)
        return fail(JX_ERR_DEVICE,
                    "device check %d failed in block %d thread %d: values %lld %d %d (error %d)",
                    dbg[0], dbg[1], dbg[2],
                    static_cast<long long>((static_cast<uint64_t>(static_cast<uint32_t>(dbg[4])) << 32) |
                                           static_cast<uint32_t>(dbg[3])),
                    dbg[5], dbg[6], h);
    return JX_OK;
}

int jx_kv_set_option(jx_kv* kv, const char* key, int value) {
    if (!kv || !key) return fail(JX_ERR_INVALID, "bad option");
    if (value < 0 && std::strcmp(key, "pdl") != 0 && std::strcmp(key, "split_penalty_us") != 0)
        return fail(JX_ERR_INVALID, "option '%s' takes a non-negative value", key);
    if (!std::strcmp(key, "ctas_per_sm")) kv->opt_ctas_per_sm = value;
    else if (!std::strcmp(key, "stages")) {
        if (value == 1 || value > 16) return fail(JX_ERR_INVALID, "stages must be 2..16");
        kv->opt_stages = value;
    } else if (!std::strcmp(key, "grid")) kv->opt_grid = value;
    else if (!std::strcmp(key, "pdl")) kv->opt_pdl = value < 0 ? -1 : (value ? 1 : 0);
    else if (!std::strcmp(key, "timing")) kv->opt_timing = value ? 1 : 0;
    else if (!std::strcmp(key, "split_penalty_us"))
        kv->opt_split_penalty_us = value < 0 ? -1.0f : static_cast<float>(value);
    else if (!std::strcmp(key, "wait_limit_ms")) kv->opt_wait_limit_ms = value;
    else if (!std::strcmp(key, "prefill_tc")) kv->opt_prefill_tc = value ? 1 : 0;
    else if (!std::strcmp(key, "prefill_l2_mb")) {
        if (value < 0) return fail(JX_ERR_INVALID, "prefill_l2_mb must be >= 0");
        kv->opt_prefill_l2_mb = value;
    }
    else if (!std::strcmp(key, "test_wait_cta")) kv->opt_test_wait_cta = value;
    else return fail(JX_ERR_INVALID, "unknown option '%s'", key);
    return JX_OK;
}

int jx_kv_last_launch_count(const jx_kv* kv, int* count) {
    if (!kv || !count) return fail(JX_ERR_INVALID, "null argument");
    *count = kv->last_launches;
    return JX_OK;
}

int jx_kv_fill_normal(jx_kv* kv, const uint32_t* rows_per_seq, uint64_t seed, void* stream) {
    if (!kv || !rows_per_seq) return fail(JX_ERR_INVALID, "null argument");
    for (uint32_t s = 0; s < kv->d.n_seqs; ++s)
        if (rows_per_seq[s] > kv->d.capacity) return fail(JX_ERR_RANGE, "rows beyond capacity");
    DeviceGuard guard(kv->d.device);
    cudaStream_t st = (cudaStream_t)stream;
    JX_CUDA(cudaMemcpyAsync(kv->d_rows, rows_per_seq, sizeof(uint32_t) * kv->d.n_seqs,
                            cudaMemcpyHostToDevice, st));
    const int grid = kv->num_sms * 8;
    const auto& d = kv->d;
    if (d.dtype == JX_F32)
        fill_cache_kernel<DT_F32><<<grid, 256, 0, st>>>(kv->k, kv->v, kv->d_rows, d.n_seqs, d.n_layers,
                                                        d.capacity, d.row_stride, seed);
    else if (d.dtype == JX_BF16)
        fill_cache_kernel<DT_BF16><<<grid, 256, 0, st>>>(kv->k, kv->v, kv->d_rows, d.n_seqs,
                                                         d.n_layers, d.capacity, d.row_stride, seed);
    else
        fill_cache_kernel<DT_F16T><<<grid, 256, 0, st>>>(kv->k, kv->v, kv->d_rows, d.n_seqs,
                                                         d.n_layers, d.capacity, d.row_stride, seed);
    JX_CUDA(cudaGetLastError());
    // the host rows array may be released once this returns
    JX_CUDA(cudaStreamSynchronize(st));
    return JX_OK;
}

int jx_fill_normal_f32(float* dst, uint64_t n, uint64_t seed, uint32_t stream_id, void* stream) {
    if (!dst) return fail(JX_ERR_INVALID, "null dst");
    if (n == 0) return JX_OK;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    fill_f32_kernel<<<sms * 8, 256, 0, (cudaStream_t)stream>>>(dst, n, seed, stream_id);
    JX_CUDA(cudaGetLastError());
    return JX_OK;
}

}  // extern "C"
