// jx_device.cuh -- device helpers shared by the decode-attention kernels:
// inline-PTX wrappers for mbarriers, TMA tile loads and proxy fences, bounded
// waits, and bit-exact copies of jxai's scalar KV conversions.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace jx {

// ---------------------------------------------------------------- addressing
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarriers
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes freshly initialised barriers visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// A wait that always ends.  Elapsed time is measured with the SM's own cycle
// counter (clock64, monotonic per SM) and checked only after a floor of polls,
// so a jump of the global nanosecond timer cannot end a wait early.  After
// `limit` cycles the wait raises the CTA's abort flag and the device error
// word, records where it gave up in dbg[0..7], and returns false.  Once the
// CTA has aborted, later waits that honour the flag return false at once (the
// caller carries on through its barriers so no warp waits on another).
constexpr long long kWaitLimitCycles = 8000000000ll;   // ~4 s at 1.965 GHz
constexpr long long kDrainLimitCycles = 30000000000ll; // ~15 s: copies in flight at exit
constexpr int kDevErrWaitTimeout = 1;
constexpr int kPollFloor = 4096;

__device__ __noinline__ static void report_timeout(int* err, int* dbg, int site, int tile,
                                                   long long cycles, uint64_t g0) {
    const uint64_t g1 = global_timer_ns();
    if (atomicCAS(dbg, 0, 100 + site) == 0) {
        dbg[1] = static_cast<int>(blockIdx.x);
        dbg[2] = static_cast<int>(threadIdx.x);
        dbg[3] = static_cast<int>(cycles);
        dbg[4] = static_cast<int>(cycles >> 32);
        dbg[5] = tile;
        dbg[6] = static_cast<int>((static_cast<long long>(g1 - g0)) / 1000000);  // ms
        __threadfence();
    }
    atomicExch(err, kDevErrWaitTimeout);
}

__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  volatile int* abort_flag, int* err, int* dbg,
                                                  int site, int tile, bool honour_abort = true,
                                                  long long limit = kWaitLimitCycles) {
    if (mbar_try_wait(bar, parity)) return true;
    if (honour_abort && *abort_flag) return false;
    const long long c0 = clock64();
    const uint64_t g0 = global_timer_ns();
    int polls = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (honour_abort && *abort_flag) return false;
        if (++polls < kPollFloor) continue;
        polls = 0;
        const long long dc = clock64() - c0;
        if (dc > limit) {
            *abort_flag = 1;
            report_timeout(err, dbg, site, tile, dc, g0);
            return false;
        }
    }
    return true;
}

// ---------------------------------------------------------------- optional device checks
// Built with -DJX_DEVICE_CHECKS=1, every global/shared index and TMA coordinate
// the decode kernel uses is validated first; a failed check records the first
// violation in dbg[0..7] (code, block, three values), raises the device error
// word, and the access is skipped -- nothing traps.
#ifndef JX_DEVICE_CHECKS
#define JX_DEVICE_CHECKS 0
#endif
constexpr int kDevErrCheck = 2;

static __device__ __noinline__ void report_check(int* err, int* dbg, int code, long long v0, long long v1,
                                          long long v2) {
    if (atomicCAS(dbg, 0, code) == 0) {
        dbg[1] = static_cast<int>(blockIdx.x);
        dbg[2] = static_cast<int>(threadIdx.x);
        dbg[3] = static_cast<int>(v0);
        dbg[4] = static_cast<int>(v0 >> 32);
        dbg[5] = static_cast<int>(v1);
        dbg[6] = static_cast<int>(v2);
        __threadfence();
    }
    atomicExch(err, kDevErrCheck);
}

// `ok` evaluates to the condition; on failure the violation is reported.
#define JX_CHECKED(args, cond, code, v0, v1, v2)                                  \
    ((!JX_DEVICE_CHECKS) || (cond) ||                                             \
     (::jx::report_check((args).err, (args).dbg, (code), (long long)(v0),         \
                         (long long)(v1), (long long)(v2)),                       \
      false))

// ---------------------------------------------------------------- TMA
// Tiled 4-D load global -> this CTA's shared memory, completion counted on an
// mbarrier.  No multicast: every CTA fetches its own tiles.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

// Untiled bulk copy global -> this CTA's shared memory (no multicast),
// completion counted on an mbarrier.  Both addresses 16-byte aligned, `bytes`
// a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(dst),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (TMA) writes of the same bytes.
__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Atomic add with acquire-release semantics at GPU scope.  Issued by one
// thread after a CTA barrier, it publishes every write the CTA made before the
// barrier and observes every write published by earlier arrivals.
__device__ __forceinline__ int atomic_add_acq_rel_gpu(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Atomic add with release semantics at GPU scope: publishes the writes the
// CTA made before a preceding barrier without waiting for other CTAs' writes.
__device__ __forceinline__ int atomic_add_release_gpu(int* p, int v) {
    int old;
    asm volatile("atom.release.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Acquire-release fence at GPU scope (after reading a counter that earlier
// writers released, before reading their data).
__device__ __forceinline__ void fence_acq_rel_gpu() {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

// Programmatic dependent launch.  launch_dependents lets the next kernel of
// the stream (launched with programmatic stream serialisation) be scheduled
// onto SMs this grid frees; wait blocks until every prerequisite grid has
// completed and its memory is visible -- nothing a previous kernel may have
// written is read or written before it.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Named barrier over `count` threads (count a multiple of 32).
__device__ __forceinline__ void named_bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---------------------------------------------------------------- math
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------- KV element conversions
// Bit-for-bit copies of jxai's scalar conversions (src/quant.cpp:876-939).
enum { DT_F32 = 0, DT_BF16 = 1, DT_F16T = 2 };

// fp32_to_bf16 (quant.cpp:934-939): round to nearest even, no NaN special case.
__device__ __forceinline__ uint16_t f32_to_bf16_ref(float f) {
    const uint32_t u = __float_as_uint(f);
    return static_cast<uint16_t>((u + (((u >> 16) & 1u) + 0x7FFFu)) >> 16);
}

// fp32_to_fp16 (quant.cpp:906-925): truncates the mantissa; exponent overflow,
// Inf and NaN become +-Inf; values below the smallest subnormal become +-0.
__device__ __forceinline__ uint16_t f32_to_f16_trunc_ref(float f) {
    const uint32_t u = __float_as_uint(f);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const int ex = static_cast<int>((u >> 23) & 0xFFu) - 127 + 15;
    uint32_t mant = u & 0x007FFFFFu;
    if (ex <= 0) {
        if (ex < -10) return static_cast<uint16_t>(sign);
        mant |= 0x00800000u;
        return static_cast<uint16_t>(sign | (mant >> (14 - ex)));
    }
    if (ex >= 31) return static_cast<uint16_t>(sign | 0x7C00u);
    return static_cast<uint16_t>(sign | (static_cast<uint32_t>(ex) << 10) | (mant >> 13));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

// Exact IEEE half -> float (fp16_to_fp32, quant.cpp:876-904).
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

template <int DT>
__device__ __forceinline__ void store_kv(void* base, long long i, float x) {
    if constexpr (DT == DT_F32) {
        static_cast<float*>(base)[i] = x;
    } else if constexpr (DT == DT_BF16) {
        static_cast<uint16_t*>(base)[i] = f32_to_bf16_ref(x);
    } else {
        static_cast<uint16_t*>(base)[i] = f32_to_f16_trunc_ref(x);
    }
}

// Unpacks one 16-byte chunk of stored elements into floats.
template <int DT>
__device__ __forceinline__ void unpack16(const uint4& r, float* out) {
    if constexpr (DT == DT_F32) {
        out[0] = __uint_as_float(r.x);
        out[1] = __uint_as_float(r.y);
        out[2] = __uint_as_float(r.z);
        out[3] = __uint_as_float(r.w);
    } else {
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (DT == DT_BF16) {
                out[2 * i] = __uint_as_float(w[i] << 16);
                out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
            } else {
                out[2 * i] = f16_bits_to_f32(w[i] & 0xFFFFu);
                out[2 * i + 1] = f16_bits_to_f32(w[i] >> 16);
            }
        }
    }
}

// ---------------------------------------------------------------- warp MMA (16-bit caches)
// m16n8k16 with fp32 accumulation; A row-major, B column-major.  Lane L holds
// A rows L/4 and L/4+8, B column L/4 and C rows L/4, L/4+8 (columns 2(L%4), +1).
template <int DT>
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    if constexpr (DT == DT_BF16) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
            "{%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
            "{%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}

// Four 8x8 16-bit matrices from shared memory; lane L supplies the address of
// row L%8 of matrix L/8.  `trans` delivers each matrix transposed.
template <bool trans>
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    if constexpr (trans)
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                     : "r"(addr));
    else
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                     : "r"(addr));
}

// Transposes an 8x8 16-bit matrix held one row pair per lane (lane L: row
// L/4, columns 2(L%4), 2(L%4)+1) into the same layout.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

// Two floats as a 16-bit pair (x in the low half) rounded to nearest, plus the
// pair of what the rounding left over: x = hi + lo to ~2^-16 relative.
template <int DT>
__device__ __forceinline__ void split_pair(float x, float y, uint32_t& hi, uint32_t& lo) {
    if constexpr (DT == DT_BF16) {
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(y), "f"(x));
        const float xh = __uint_as_float(hi << 16), yh = __uint_as_float(hi & 0xFFFF0000u);
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(y - yh), "f"(x - xh));
    } else {
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(y), "f"(x));
        const float xh = f16_bits_to_f32(hi & 0xFFFFu), yh = f16_bits_to_f32(hi >> 16);
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(y - yh), "f"(x - xh));
    }
}

// d0 += a0 * b0 and d1 += a1 * b1 as one fp32x2 fused multiply-add (each
// half rounded once, as __fmaf_rn): half the FMA instructions of two scalar
// ones for the CUDA-core dot products.
__device__ __forceinline__ void fma_x2(float& d0, float& d1, float a0, float a1, float b0,
                                       float b1) {
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rd, {%0, %1};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rd;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "+f"(d0), "+f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// max(a, b, c) in one instruction (a NaN operand is ignored, as by fmaxf).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// (d0, d1) += (a0, a1) and (d0, d1) = (a0 - b0, a1 - b1): one packed fp32
// instruction each, every lane rounded to nearest like a scalar add / sub.
__device__ __forceinline__ void add_x2(float& d0, float& d1, float a0, float a1) {
    asm("{\n\t.reg .b64 ra, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rd, {%0, %1};\n\t"
        "add.rn.f32x2 rd, rd, ra;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "+f"(d0), "+f"(d1)
        : "f"(a0), "f"(a1));
}

__device__ __forceinline__ void sub_x2(float& d0, float& d1, float a0, float a1, float b0,
                                       float b1) {
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "sub.rn.f32x2 rd, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// ---------------------------------------------------------------- RoPE
// One element of a rotated head, rounded as jxai's build rounds apply_rope
// (src/transformer.cpp:76-138, gcc -O3 -mfma):
//   Neox pair (j, j+half):   x[j] = fma(a, c, -(b*s)),  x[j+half] = fma(a, s, b*c)
//   interleaved (2j, 2j+1):  x[2j] = a*c - b*s,        x[2j+1]   = a*s + b*c
// Dimensions at or beyond 2*half are returned unchanged.  cs[j] = (cos, sin).
__device__ __forceinline__ float rope_elem(const float* x, int d, int half, const float2* cs,
                                           bool neox) {
    if (d >= 2 * half) return x[d];
    if (neox) {
        const int j = d < half ? d : d - half;
        const float2 t = cs[j];
        const float a = x[j], b = x[j + half];
        return d < half ? __fmaf_rn(a, t.x, -__fmul_rn(b, t.y))
                        : __fmaf_rn(a, t.y, __fmul_rn(b, t.x));
    }
    const int j = d >> 1;
    const float2 t = cs[j];
    const float a = x[2 * j], b = x[2 * j + 1];
    return (d & 1) == 0 ? __fsub_rn(__fmul_rn(a, t.x), __fmul_rn(b, t.y))
                        : __fadd_rn(__fmul_rn(a, t.y), __fmul_rn(b, t.x));
}

}  // namespace jx
