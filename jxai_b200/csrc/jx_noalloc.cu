// jx_noalloc.cu -- jx_attn_step_noalloc: the decode step for callers that must
// not allocate GPU memory.
//
// jx_attn_step keeps its scratch (split partials, per-segment arrival
// counters, the per-step work plan) in buffers the library allocates and grows
// on demand.  Some callers cannot let a library call cudaMalloc: an engine
// that hands every byte of HBM to its own arena or pool allocator, a serving
// loop that must never hit cudaMalloc/cudaFree's implicit device
// synchronisation in the middle of a token, or code running where a new
// allocation is simply not allowed.  This entry point takes the KV cache as
// caller-owned device buffers and keeps all of its scratch in one fixed array
// below, reserved once per GPU when the library's device code is loaded.
//
// Limits and rules:
//   * The scratch array holds kNoAllocScratchBytes (8 MiB) per GPU and stays
//     reserved on every GPU that loads this library until the process exits.
//     A step whose partials, counters and plan need more is rejected with
//     JX_ERR_RANGE and a message giving both sizes (a few thousand
//     (sequence, layer, kv head) segments fit; the 256-sequence ragged batch
//     of the benchmark does not).
//   * All calls share that one array and it keeps the last call's contents.
//     Each call clears the part that must start at zero (the per-segment
//     arrival counters) on its own stream before its launch.  Calls that
//     overlap on the GPU -- on different streams, or from different threads
//     without ordering -- race on the array and give wrong results.
//   * A kernel that reports an error (a bounded wait that ran out) sets the
//     device error word at the start of the array; it stays set until
//     jx_noalloc_check_device_error reads and clears it, so one check after a
//     run of steps reports the first error among them.
//   * The first call on each device does its set-up: it looks up the array's
//     device address (cudaGetSymbolAddress) with that device current and
//     creates that device's plan-copy events; the first call in the process
//     also page-locks the fixed host buffer the plan is built in
//     (cudaHostRegister of the library's own static buffer -- no memory is
//     allocated).  The call refuses stream capture (JX_ERR_UNSUPPORTED): a
//     captured plan copy would replay from a slot later calls overwrite.
//   * Nothing here calls cudaMalloc, cudaFree, cudaMallocAsync, cudaHostAlloc
//     or any other allocating routine: the work plan is built in one of four
//     slots of the fixed host buffer (not on the heap) and copied into the
//     array with cudaMemcpyAsync; a slot is reused only after the copy that
//     last read it has run (its event), so the host runs up to four steps
//     ahead of the GPU without waiting.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>

#include "jx_attn.h"
#include "jx_device.cuh"
#include "jx_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // per GPU
constexpr size_t kHeaderBytes = 256;                       // err word + dbg[8]
constexpr int kPlanSlots = 4;                              // host plan buffers in flight
constexpr size_t kPlanSlotBytes = size_t(1) << 20;         // one step's plan
constexpr size_t kMaxPairs = kPlanSlotBytes / sizeof(jx::PairRow);
constexpr int kMaxDevices = 64;

// The scratch itself.  In host code `g_noalloc_scratch` is only a stand-in
// symbol, never a usable address: its device address comes from
// cudaGetSymbolAddress (per device) and is what the kernel receives.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Host side of the plan: kPlanSlots slots, page-locked once per process.
alignas(4096) unsigned char g_plan_host[kPlanSlots * kPlanSlotBytes];
struct RopeKey { uint32_t rdim, base, pos; const float* rf; };
RopeKey g_rope_keys[kMaxPairs];        // plan building only (host)
std::mutex g_mu;                       // one plan build / upload at a time
bool g_plan_pinned = false;            // cudaHostRegister of g_plan_host succeeded
bool g_pin_tried = false;
int g_next_slot = 0;
int g_slot_dev[kPlanSlots] = {-1, -1, -1, -1};  // device of each slot's last copy
struct DeviceState {
    unsigned char* scratch = nullptr;  // device address of g_noalloc_scratch
    cudaEvent_t ev[kPlanSlots] = {};   // recorded after each slot's plan copy
};
DeviceState g_dev[kMaxDevices];
std::atomic<int> g_opt_wait_limit_ms{0};
std::atomic<int> g_opt_test_wait_cta{0};

// Reports a failure through jx_last_error_string() (the calling thread's message).
int nfail(int code, const char* fmt, ...) {
    char msg[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, sizeof msg, fmt, ap);
    va_end(ap);
    jx::set_last_error(msg);
    return code;
}

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// Pointer check as jx_attn_step makes it: device memory of `dev` or (where
// allowed) pinned host memory; pageable host memory or another device's
// memory would fault the kernel.  An error this query raises is cleared only
// when the caller had none pending, so a caller's unread error survives.
int check_ptr(const void* p, const char* name, int dev, bool host_ok, bool* host) {
    const cudaError_t pending = cudaPeekAtLastError();
    cudaPointerAttributes at{};
    const cudaError_t e = cudaPointerGetAttributes(&at, p);
    if (e != cudaSuccess) {
        if (pending == cudaSuccess) cudaGetLastError();
        return nfail(JX_ERR_INVALID, "%s: not a CUDA-visible pointer (%s)", name,
                     cudaGetErrorString(e));
    }
    if (at.type == cudaMemoryTypeHost && host_ok) {
        *host = true;
        return JX_OK;
    }
    *host = false;
    if ((at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) && at.device == dev)
        return JX_OK;
    return nfail(JX_ERR_INVALID, "%s must be memory of device %d%s", name, dev,
                 host_ok ? " or pinned host memory" : "");
}

// Once per device (with it current): the scratch array's device address and
// the plan-copy events; once per process: page-lock the host plan buffer.
// Called with g_mu held.
int setup_device(int dev) {
    if (!g_pin_tried) {
        g_pin_tried = true;
        const cudaError_t pending = cudaPeekAtLastError();
        g_plan_pinned = cudaHostRegister(g_plan_host, sizeof g_plan_host,
                                         cudaHostRegisterPortable) == cudaSuccess;
        // without it the copies still work, from pageable memory
        if (!g_plan_pinned && pending == cudaSuccess) cudaGetLastError();
    }
    DeviceState& st = g_dev[dev];
    if (st.scratch) return JX_OK;
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
        return nfail(JX_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
    for (int i = 0; i < kPlanSlots; ++i)
        if (!st.ev[i] && cudaEventCreateWithFlags(&st.ev[i], cudaEventDisableTiming) != cudaSuccess)
            return nfail(JX_ERR_CUDA, "event creation failed");
    st.scratch = static_cast<unsigned char*>(p);
    return JX_OK;
}

int current_device(int want) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices || dev != want)
        return -1;
    return dev;
}

}  // namespace

using namespace jx;

extern "C" JX_API int jx_attn_step_noalloc(const jx_kv_desc* desc, void* k_cache, void* v_cache,
                                           const jx_layer_desc* layers, uint32_t n_layers,
                                           const jx_step_args* a, void* stream_ptr) {
    if (!desc || !k_cache || !v_cache || !layers || !a || n_layers == 0 || a->n_seqs == 0)
        return nfail(JX_ERR_INVALID, "null argument or empty step");
    if (!a->pos || !a->q || !a->k || !a->v || !a->out)
        return nfail(JX_ERR_INVALID, "null pos/q/k/v/out");
    const jx_kv_desc& D = *desc;
    if (D.dtype < 0 || D.dtype > 2 || D.n_seqs == 0 || D.n_layers == 0 || D.capacity == 0 ||
        D.row_stride == 0)
        return nfail(JX_ERR_INVALID, "bad cache descriptor");
    const size_t esz = D.dtype == JX_F32 ? 4 : 2;
    if ((D.row_stride * esz) % 16 != 0 || (reinterpret_cast<uintptr_t>(k_cache) % 16) != 0 ||
        (reinterpret_cast<uintptr_t>(v_cache) % 16) != 0)
        return nfail(JX_ERR_UNSUPPORTED, "cache rows and base addresses must be 16-byte aligned");
    if (a->n_kv_heads == 0 || a->n_heads % a->n_kv_heads != 0)
        return nfail(JX_ERR_UNSUPPORTED, "n_heads must be a multiple of n_kv_heads");
    const uint32_t G = a->n_heads / a->n_kv_heads;
    const int gp = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : G <= 8 ? 8 : 0;
    if (!gp) return nfail(JX_ERR_UNSUPPORTED, "query group above 8 heads");
    const uint32_t hd = layers[0].head_dim;
    if (hd != 32 && hd != 64 && hd != 128 && hd != 256)
        return nfail(JX_ERR_UNSUPPORTED, "head_dim %u (compiled: 32, 64, 128, 256)", hd);
    if (hd * esz < 64) return nfail(JX_ERR_UNSUPPORTED, "head rows below 64 bytes");
    const int kp = kv_pack(static_cast<int>(hd), static_cast<int>(esz), a->n_kv_heads, G, gp);
    const uint32_t n_kv = a->n_kv_heads / kp;  // segments per (sequence, layer) pair
    if (static_cast<uint64_t>(a->n_kv_heads) * hd > D.row_stride ||
        a->q_stride < a->n_heads * hd || a->kv_stride < a->n_kv_heads * hd)
        return nfail(JX_ERR_INVALID, "strides smaller than the layer's rows");
    for (uint32_t l = 0; l < n_layers; ++l) {
        if (layers[l].head_dim != hd)
            return nfail(JX_ERR_UNSUPPORTED, "all layers of one call must share head_dim");
        if (layers[l].kv_source_layer >= D.n_layers)
            return nfail(JX_ERR_INVALID, "kv_source_layer out of range");
    }
    // one launch only: a shares-KV layer must not read a cache layer appended in this call
    for (uint32_t l = 0; l < n_layers; ++l) {
        if (!layers[l].shares_kv) continue;
        for (uint32_t m = 0; m < n_layers; ++m)
            if (!layers[m].shares_kv && layers[m].kv_source_layer == layers[l].kv_source_layer)
                return nfail(JX_ERR_UNSUPPORTED,
                             "a shares-KV layer reads a cache layer appended in the same call; "
                             "split the call");
    }
    const size_t n_pairs = static_cast<size_t>(a->n_seqs) * n_layers;
    if (n_pairs > kMaxPairs)
        return nfail(JX_ERR_RANGE, "step of %zu (sequence, layer) pairs exceeds the %zu the "
                                   "no-allocation path plans", n_pairs, kMaxPairs);
    const int dev = current_device(D.device);
    if (dev < 0)
        return nfail(JX_ERR_INVALID, "make the cache's device (%d) current before the call",
                     D.device);
    // the same pointer rules as jx_attn_step: inputs and output in this device's
    // memory or pinned host memory, the caches in this device's memory
    bool q_host = false, k_host = false, v_host = false, o_host = false, c_host = false;
    int rc = check_ptr(a->q, "q", dev, true, &q_host);
    if (!rc) rc = check_ptr(a->k, "k", dev, true, &k_host);
    if (!rc) rc = check_ptr(a->v, "v", dev, true, &v_host);
    if (!rc) rc = check_ptr(a->out, "out", dev, true, &o_host);
    if (!rc) rc = check_ptr(k_cache, "k_cache", dev, false, &c_host);
    if (!rc) rc = check_ptr(v_cache, "v_cache", dev, false, &c_host);
    if (rc) return rc;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    // a captured plan copy would replay from a host slot that later calls
    // overwrite, so the path refuses capture instead of recording it
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    const cudaError_t ce = cudaStreamIsCapturing(stream, &cap);
    if (ce != cudaSuccess)
        return nfail(JX_ERR_CUDA, "cudaStreamIsCapturing failed: %s", cudaGetErrorString(ce));
    if (cap != cudaStreamCaptureStatusNone)
        return nfail(JX_ERR_UNSUPPORTED,
                     "jx_attn_step_noalloc cannot be captured into a CUDA graph (its work plan "
                     "is copied from a host slot that later calls reuse)");

    std::lock_guard<std::mutex> lk(g_mu);
    rc = setup_device(dev);
    if (rc) return rc;
    unsigned char* scratch = g_dev[dev].scratch;

    // ---- work plan, built in the next host slot: pairs, then rope rows.  The
    // slot is reused only once the copy that last read it has run.
    const int slot = g_next_slot;
    if (g_slot_dev[slot] >= 0) {
        const cudaError_t e = cudaEventSynchronize(g_dev[g_slot_dev[slot]].ev[slot]);
        if (e != cudaSuccess)
            return nfail(JX_ERR_CUDA, "plan slot wait failed: %s", cudaGetErrorString(e));
        g_slot_dev[slot] = -1;
    }
    unsigned char* plan_host = g_plan_host + static_cast<size_t>(slot) * kPlanSlotBytes;
    const size_t pair_bytes = n_pairs * sizeof(PairRow);
    const size_t rope_off = round_up(pair_bytes, 256);
    const int width = static_cast<int>(hd / 2);
    const size_t row_bytes = static_cast<size_t>(width) * sizeof(float2);
    if (rope_off + n_pairs * row_bytes > kPlanSlotBytes)
        return nfail(JX_ERR_RANGE, "step of %zu (sequence, layer) pairs exceeds the %zu-byte plan "
                                   "slot of the no-allocation path", n_pairs, kPlanSlotBytes);
    PairRow* pairs = reinterpret_cast<PairRow*>(plan_host);
    float2* rope = reinterpret_cast<float2*>(plan_host + rope_off);
    RopeKey* keys = g_rope_keys;
    int n_rope = 0;
    long long off = 0;
    const bool neox = a->rope_neox != 0;
    for (uint32_t s = 0; s < a->n_seqs; ++s) {
        const int sid = a->seq_ids ? a->seq_ids[s] : static_cast<int>(s);
        if (sid < 0 || static_cast<uint32_t>(sid) >= D.n_seqs || a->pos[s] < 0)
            return nfail(JX_ERR_INVALID, "sequence id or position out of range");
        for (uint32_t t = 0; t < s; ++t)
            if ((a->seq_ids ? a->seq_ids[t] : static_cast<int>(t)) == sid)
                return nfail(JX_ERR_INVALID, "sequence id %d listed twice", sid);
        const uint32_t pos = static_cast<uint32_t>(a->pos[s]);
        for (uint32_t l = 0; l < n_layers; ++l) {
            const jx_layer_desc& L = layers[l];
            const uint32_t W = a->sliding_window;
            const uint64_t t0 = (L.is_swa && W > 0 && pos >= W) ? pos - W + 1 : 0;
            if (t0 < D.pos_base || static_cast<uint64_t>(pos) >= static_cast<uint64_t>(D.pos_base) + D.capacity)
                return nfail(JX_ERR_RANGE, "position %u outside the cache rows", pos);
            PairRow& pr = pairs[s * n_layers + l];
            std::memset(&pr, 0, sizeof pr);
            pr.off = off;
            pr.seq = sid;
            pr.io = static_cast<int>(s * n_layers + l);
            pr.cache_layer = static_cast<int>(L.kv_source_layer);
            pr.row0 = static_cast<int>(t0 - D.pos_base);
            pr.len = static_cast<int>(pos - t0 + 1);
            pr.append_row = L.shares_kv ? -1 : static_cast<int>(pos - D.pos_base);
            const uint32_t rdim = std::min(L.head_dim, L.rope_dim);
            pr.rope_half = static_cast<int>(rdim / 2);
            const float* rf = (neox && !L.is_swa && L.rope_freqs) ? L.rope_freqs : nullptr;
            uint32_t base_bits;
            std::memcpy(&base_bits, &L.rope_freq_base, 4);
            int rid = -1;
            for (int r = 0; r < n_rope; ++r)
                if (keys[r].rdim == rdim && keys[r].base == base_bits && keys[r].pos == pos &&
                    keys[r].rf == rf) {
                    rid = r;
                    break;
                }
            if (rid < 0) {
                rid = n_rope++;
                keys[rid] = RopeKey{rdim, base_bits, pos, rf};
                rope_row(L.head_dim, L.rope_dim, pos, L.rope_freq_base, a->yarn_scale, neox, rf,
                         rope + static_cast<size_t>(rid) * width, width);
            }
            pr.rope_row = rid;
            off += static_cast<long long>(pr.len) * n_kv;
        }
    }
    const long long total = off;
    const size_t plan_bytes = rope_off + static_cast<size_t>(n_rope) * row_bytes;

    // ---- launch shape and scratch layout
    int stages = 0, cps = 0;
    default_shape(static_cast<int>(hd), gp, kp, D.dtype, &stages, &cps);
    const int occ = decode_ctas_per_sm(static_cast<int>(hd), gp, kp, D.dtype, stages);
    if (occ <= 0) return nfail(JX_ERR_UNSUPPORTED, "kernel does not fit");
    cps = std::max(1, std::min(cps, occ));
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return nfail(JX_ERR_CUDA, "cannot query the SM count");
    long long P = std::min<long long>(static_cast<long long>(sms) * cps,
                                      std::max<long long>(1, (total + 63) / 64));
    const long long n_segs = static_cast<long long>(n_pairs) * n_kv;
    const size_t counters_off = kHeaderBytes;
    const size_t partials_off = round_up(counters_off + static_cast<size_t>(n_segs) * 4, 256);
    const size_t partial_floats = static_cast<size_t>(P + n_segs) * gp * kp * (hd + 2);
    const size_t plan_off = round_up(partials_off + partial_floats * 4, 256);
    const size_t need = plan_off + plan_bytes;
    if (need > kNoAllocScratchBytes)
        return nfail(JX_ERR_RANGE,
                     "step needs %zu bytes of scratch (%lld segments); the no-allocation "
                     "scratch holds %zu bytes -- use jx_attn_step",
                     need, n_segs, kNoAllocScratchBytes);

    // ---- tensor maps for the caller's cache (host-side encoding only)
    auto enc = encoder();
    if (!enc) return nfail(JX_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    CUtensorMap tmK, tmV;
    const uint32_t box_bytes = kp * hd * esz >= 128 ? 128 : 64;
    const cuuint64_t dims[4] = {D.row_stride, D.capacity, D.n_layers, D.n_seqs};
    const cuuint64_t strides[3] = {
        static_cast<cuuint64_t>(D.row_stride) * esz,
        static_cast<cuuint64_t>(D.row_stride) * esz * D.capacity,
        static_cast<cuuint64_t>(D.row_stride) * esz * D.capacity * D.n_layers};
    const cuuint32_t box[4] = {static_cast<cuuint32_t>(box_bytes / esz), 32, 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUtensorMapDataType dt =
        esz == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
    const CUtensorMapSwizzle sw =
        box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    for (int which = 0; which < 2; ++which) {
        const CUresult r = enc(which == 0 ? &tmK : &tmV, dt, 4, which == 0 ? k_cache : v_cache,
                               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return nfail(JX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    }

    // ---- clear the counters (the error word stays until it is read), upload
    // the plan from its slot, launch
    cudaError_t e = cudaMemsetAsync(scratch + counters_off, 0, partials_off - counters_off, stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(scratch + plan_off, plan_host, plan_bytes, cudaMemcpyHostToDevice,
                            stream);
    if (e == cudaSuccess) e = cudaEventRecord(g_dev[dev].ev[slot], stream);
    if (e != cudaSuccess) return nfail(JX_ERR_CUDA, "scratch set-up failed: %s", cudaGetErrorString(e));
    g_slot_dev[slot] = dev;
    g_next_slot = (slot + 1) % kPlanSlots;

    DecodeLaunch Lc{};
    DecodeArgs& A = Lc.args;
    A.pairs = reinterpret_cast<const PairRow*>(scratch + plan_off);
    A.n_pairs = static_cast<int>(n_pairs);
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
    A.k_cache = k_cache;
    A.v_cache = v_cache;
    A.layer_stride = static_cast<long long>(D.capacity) * D.row_stride;
    A.seq_stride = A.layer_stride * D.n_layers;
    A.row_stride = D.row_stride;
    A.rope = reinterpret_cast<const float2*>(scratch + plan_off + rope_off);
    A.scale = a->scale;
    A.softcap = a->softcap;
    A.inv_softcap = a->softcap > 0.0f ? 1.0f / a->softcap : 0.0f;
    A.neox = neox ? 1 : 0;
    A.scratch = reinterpret_cast<float*>(scratch + partials_off);
    A.counters = reinterpret_cast<int*>(scratch + counters_off);
    A.part_out = nullptr;
    A.err = reinterpret_cast<int*>(scratch);
    A.dbg = reinterpret_cast<int*>(scratch) + 8;
    A.n_stages = stages;
    A.n_consumers = consumers_for(stages, kp);
    // q and the appended k/v rows are bulk-prefetched from device memory with
    // 16-byte rows; host-resident (pinned) inputs are read with ordinary loads
    A.q_bulk = (!q_host && !k_host && !v_host && reinterpret_cast<uintptr_t>(a->q) % 16 == 0 &&
                a->q_stride % 4 == 0 && reinterpret_cast<uintptr_t>(a->k) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(a->v) % 16 == 0 && a->kv_stride % 4 == 0)
                   ? 1 : 0;
    A.test_wait_cta = g_opt_test_wait_cta.load();
    A.wait_limit = wait_limit_cycles(g_opt_wait_limit_ms.load());
    A.n_io = static_cast<long long>(n_pairs);
    A.cache_elems = A.seq_stride * D.n_seqs;
    A.scratch_floats = static_cast<long long>(partial_floats);
    A.n_segments = n_segs;
    A.n_rope_rows = n_rope;
    A.capacity = static_cast<int>(D.capacity);
    A.n_cache_layers = static_cast<int>(D.n_layers);
    A.n_cache_seqs = static_cast<int>(D.n_seqs);
    A.smem_bytes = decode_smem_bytes(static_cast<int>(hd), gp, kp, D.dtype, stages);
    Lc.tmK = &tmK;
    Lc.tmV = &tmV;
    Lc.head_dim = static_cast<int>(hd);
    Lc.gp = gp;
    Lc.kp = kp;
    Lc.dtype = D.dtype;
    Lc.grid = static_cast<int>(P);
    Lc.stages = stages;
    Lc.pdl = 1;  // as jx_attn_step's default
    Lc.stream = stream;
    e = decode_launch(Lc);
    if (e != cudaSuccess) return nfail(JX_ERR_CUDA, "decode launch failed: %s", cudaGetErrorString(e));
    return JX_OK;
}

// Reads and clears the error word and the record of where the first error
// happened (header of the scratch array), in stream order after the steps
// queued on `stream`.
extern "C" JX_API int jx_noalloc_check_device_error(int device, int* code, void* stream_ptr) {
    if (!code) return nfail(JX_ERR_INVALID, "null code");
    *code = 0;
    const int dev = current_device(device);
    if (dev < 0) return nfail(JX_ERR_INVALID, "make device %d current before the call", device);
    cudaStream_t st = static_cast<cudaStream_t>(stream_ptr);
    std::lock_guard<std::mutex> lk(g_mu);
    int rc = setup_device(dev);
    if (rc) return rc;
    unsigned char* scratch = g_dev[dev].scratch;
    int hdr[16] = {0};  // err word, padding, dbg[8] at int offset 8
    cudaError_t e = cudaMemcpyAsync(hdr, scratch, sizeof hdr, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess && hdr[0] != 0) {
        e = cudaMemsetAsync(scratch, 0, kHeaderBytes, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    }
    if (e != cudaSuccess) return nfail(JX_ERR_CUDA, "error word read failed: %s", cudaGetErrorString(e));
    *code = hdr[0];
    const int* dbg = hdr + 8;
    const long long v = static_cast<long long>(
        (static_cast<uint64_t>(static_cast<uint32_t>(dbg[4])) << 32) | static_cast<uint32_t>(dbg[3]));
    if (hdr[0] == kDevErrWaitTimeout)
        return nfail(JX_ERR_DEVICE,
                     "a no-allocation step's bounded wait ran out: site %d block %d thread %d "
                     "tile %d after %lld cycles",
                     dbg[0] - 100, dbg[1], dbg[2], dbg[5], v);
    if (hdr[0])
        return nfail(JX_ERR_DEVICE, "device check %d failed in block %d thread %d (error %d)",
                     dbg[0], dbg[1], dbg[2], hdr[0]);
    return JX_OK;
}

extern "C" JX_API int jx_noalloc_set_option(const char* key, int value) {
    if (!key) return nfail(JX_ERR_INVALID, "null option");
    if (value < 0) return nfail(JX_ERR_INVALID, "option '%s' takes a non-negative value", key);
    if (!std::strcmp(key, "wait_limit_ms")) g_opt_wait_limit_ms = value;
    else if (!std::strcmp(key, "test_wait_cta")) g_opt_test_wait_cta = value;
    else return nfail(JX_ERR_INVALID, "unknown option '%s'", key);
    return JX_OK;
}
