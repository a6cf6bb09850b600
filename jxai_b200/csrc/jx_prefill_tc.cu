// jx_prefill_tc.cu -- causal prompt attention on the 5th-generation tensor
// cores (tcgen05, TMEM accumulators) for 16-bit KV caches.
//
// jxai feeds a prompt token by token through forward_token
// (src/transformer.cpp:3092-3095): token j appends its row and attends over
// every earlier row of its sequence (sliding-window layers: the last W rows,
// :2524-2527), with the block of :2530-2566.  jx_attn_prefill appends every
// row first (append_rows_kernel); this kernel then computes all tokens'
// attention at once, sharing every K/V tile across a tile of query rows:
//
//  * Work item = (run of consecutive prompt tokens of one sequence, layer,
//    kv head): TQ = 128/G tokens x the G query heads of that kv head are the
//    M = 128 rows of the MMAs (row r = token r/G, head r%G).
//  * Warp 0 streams K and V tiles of 128 cache rows into a ring (4 stages at
//    head_dim 64, 2 at head_dim 128) with TMA (128-byte swizzle, no
//    multicast).  Warp 1 owns the tensor memory (512 columns) and issues the
//    MMAs from one thread: S = Q.K^T into one of two TMEM buffers (Q read
//    from TMEM), then O += P.V into the item's TMEM accumulator.  Warps 2-9
//    (two per TMEM lane quarter, each with half of a row's columns; one
//    thread per query row = TMEM lane) rotate and stage Q into TMEM, read S
//    with tcgen05.ld, apply the scale, soft-cap and each row's causal /
//    window limits, run the online softmax (row maxima exchanged between the
//    two halves; the running maximum moves lazily, O rescaled in TMEM when
//    it does), stage P, and write each item's O / l.
//  * Precision.  q and p are fp32; each is split into two 16-bit parts
//    (hi = rn(x), lo = rn(x - hi)) and both parts are multiplied into the same
//    fp32 accumulator, while cache values are exact in the operand type -- the
//    fp32-level result the 1e-4 bar needs (a numpy model of this arithmetic
//    stays within 1.3e-6 of float64 attention; one 16-bit part is 2-7e-4).
//    fp16 q rows are scaled by a power of two into [2^14, 2^15) first and the
//    scale is taken off S exactly.
//  * Unattended V rows past the prompt's last row in the last tile are
//    cleared in shared memory before P.V (0 * Inf would otherwise leak).
//  * Every mbarrier wait is bounded; a wait that runs out raises the CTA's
//    abort flag and the device error word, and every role finishes its
//    control flow, waits for its copies / MMAs in flight and frees TMEM.
#include "jx_device.cuh"
#include "jx_internal.h"

namespace jx {
namespace {

constexpr float kLog2eP = 1.4426950408889634f;
constexpr int kSoftmaxWarps = 8;                       // warps 2-9
// + TMA warp, MMA warp.  Ten warps put three on two of the SM's four
// sub-partitions (16K registers each): at most 170 registers per thread.
constexpr int kPfThreads = 32 * (2 + kSoftmaxWarps);

// Loads 32 consecutive 32-bit TMEM columns of this thread's lane and waits
// for them (one asm statement: the registers are valid when it ends).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// Loads 64 consecutive 32-bit TMEM columns of this thread's lane and waits
// for them (one asm statement: the registers are valid when it ends).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr)
        : "memory");
}

// Stores 32 consecutive 32-bit TMEM columns of this thread's lane and waits
// until the stores are done (before a thread synchronisation hands the
// columns to the tensor cores).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n\t"
        "tcgen05.wait::st.sync.aligned;"
        :
        : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// As tmem_st32, 16 columns.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n\t"
        "tcgen05.wait::st.sync.aligned;"
        :
        : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
// Orders tcgen05 operations before / after a thread synchronisation (an
// mbarrier arrive / wait or a CTA barrier).
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// The mbarrier completes once every tcgen05 operation this thread issued
// before has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T, one CTA, 16-bit operands, fp32 accumulator.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u),
        "r"(0u), "r"(0u)
        : "memory");
}

// D[tmem] (+)= A[tmem] . B[smem]^T: A read from tensor memory (lane = row,
// each 32-bit column two consecutive 16-bit elements, the even one in the
// low half), one CTA, fp32 accumulator.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u),
        "r"(0u), "r"(0u)
        : "memory");
}

// Shared-memory matrix descriptor of a 128-byte-swizzled operand tile (the
// layout TMA's SWIZZLE_128B writes: 128-byte rows, 16-byte chunk c of row r at
// chunk c ^ (r % 8), tile base 1024-byte aligned).  lbo / sbo in bytes:
// K-major operands: lbo unused (16), sbo = 1024 (8 rows of 128 bytes);
// MN-major operands: lbo = distance between 64-element column blocks, sbo =
// 1024 (8 K-rows).  Bits 46-47 = 1 (tcgen05 descriptor), 61-63 = 2 (128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) |
           (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16 with fp32 accumulation: A and B both
// bf16 (DT_BF16) or both fp16, A K-major, B K-major or MN-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int dt, int M, int N, bool b_mn) {
    return (1u << 4) | ((dt == DT_BF16 ? 1u : 0u) << 7) | ((dt == DT_BF16 ? 1u : 0u) << 10) |
           ((b_mn ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ float f4_at(const float4& v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

template <int HD>
struct PfCfg {
    static constexpr int BN = 128;                  // cache rows per K/V tile
    // K/V ring stages: 32 KB (head_dim 64) or 64 KB (128) each
    static constexpr int NS = HD == 64 ? 4 : 2;
    // Q buffers in TMEM: two (the next item's Q staged while the current
    // item's S MMAs still read theirs) where the columns allow
    static constexpr int QBUF = HD == 64 ? 2 : 1;
    static constexpr int NSLAB = HD / 64;           // 128-byte slabs of a head row
    static constexpr int KSLAB = BN * 128;          // one slab of a K or V tile
    static constexpr int TILE_B = KSLAB * NSLAB;    // K (or V) tile
    static constexpr int STAGE_B = 2 * TILE_B;
    static constexpr int PSLAB = 128 * 128;
    static constexpr int PNSLAB = BN / 64;
    static constexpr int PPART = PSLAB * PNSLAB;    // one 16-bit part of P
    static constexpr int OFF_P = NS * STAGE_B;
    static constexpr int OFF_BAR = OFF_P + 2 * PPART;
    // barriers: kv_full[NS], kv_empty[NS], q_full[2], q_empty[2], s_full[2],
    // s_empty[2], p_full, p_empty, o_full (each P.V done), o_empty (an item's
    // O read), done
    static constexpr int B_KVF = 0, B_KVE = NS, B_QF = 2 * NS, B_QE = B_QF + 2, B_SF = B_QE + 2,
                         B_SE = B_SF + 2, B_PF = B_SE + 2, B_PE = B_PF + 1, B_OF = B_PE + 1,
                         B_OE = B_OF + 1, B_DONE = B_OE + 1, NBARS = B_DONE + 1;
    static constexpr int OFF_MISC = OFF_BAR + NBARS * 8;  // TMEM base, abort flag
    static constexpr int OFF_XCH = OFF_MISC + 32;         // [2][2][128] floats: row exchanges
    static constexpr int SMEM = OFF_XCH + 2 * 2 * 128 * 4 + 1024;  // + alignment slack
    static constexpr int TMEM_COLS = 512;
    static constexpr int COL_S = 0;        // S buffers: columns [0, 2 BN)
    static constexpr int COL_O = 2 * BN;   // the item's O accumulator: [2 BN, 2 BN + HD)
    // Q of QBUF items: buffer b at [COL_Q + b HD, +HD), its hi part in the
    // first HD/2 columns
    static constexpr int COL_Q = 2 * BN + HD;
    static_assert(COL_Q + QBUF * HD <= TMEM_COLS, "TMEM budget");
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

template <int HD, int DT, int G>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      const PrefillArgs a) {
    using C = PfCfg<HD>;
    constexpr int BN = C::BN;
    static_assert(128 % G == 0 && G <= 8, "query group");
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;  // 128-byte-swizzled tiles: 1024-byte aligned
    unsigned char* base = smem_raw + (sbase - raw);
    const uint32_t bars = sbase + C::OFF_BAR;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + C::OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(base + C::OFF_MISC + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long wlim = a.wait_limit > 0 ? a.wait_limit : kWaitLimitCycles;
    // this CTA's items: a contiguous run of the plan (the host's schedule)
    const int it_begin = a.cta_first[blockIdx.x], it_end = a.cta_first[blockIdx.x + 1];
#define BAR(i) (bars + 8u * static_cast<uint32_t>(i))
#define WAIT(i, par, site, idx) \
    mbar_wait_bounded(BAR(i), (par), abort_flag, a.err, a.dbg, (site), (idx), true, wlim)

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::NS; ++s) {
            mbar_init(BAR(C::B_KVF + s), 1);
            mbar_init(BAR(C::B_KVE + s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(BAR(C::B_QF + b), kSoftmaxWarps);
            mbar_init(BAR(C::B_QE + b), 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(BAR(C::B_SF + s), 1);
            mbar_init(BAR(C::B_SE + s), kSoftmaxWarps);
        }
        mbar_init(BAR(C::B_OF), 1);
        mbar_init(BAR(C::B_OE), kSoftmaxWarps);
        mbar_init(BAR(C::B_PF), kSoftmaxWarps);
        mbar_init(BAR(C::B_PE), 1);
        mbar_init(BAR(C::B_DONE), 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tensormap(&tmK);
            prefetch_tensormap(&tmV);
        }
        int g = 0, n_issued = 0;
        for (int it = it_begin; it < it_end; ++it) {
            const PrefillTile tl = a.tiles[it];
            if (it + 1 < it_end) {
                // the next item's 128 q rows and their (cos, sin) rows into L2
                // (this warp is idle most of the time): its Q staging then
                // reads L2, not DRAM
                const PrefillTile nx = a.tiles[it + 1];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int r = lane * 4 + k, jj = r / G, hh = r % G;
                    if (jj < nx.ntok) {
                        const char* qrow = reinterpret_cast<const char*>(
                            a.q + (static_cast<long long>(nx.io0) + static_cast<long long>(jj) * nx.io_step) *
                                      a.q_stride +
                            static_cast<long long>(nx.kvh * G + hh) * HD);
                        const char* crow = reinterpret_cast<const char*>(
                            a.rope + static_cast<long long>(nx.rope_row0 + jj) * (HD / 2));
#pragma unroll
                        for (int b = 0; b < HD * 4; b += 128) {
                            asm volatile("prefetch.global.L2 [%0];" ::"l"(qrow + b));
                            asm volatile("prefetch.global.L2 [%0];" ::"l"(crow + b));
                        }
                    }
                }
            }
            for (int t = 0; t < tl.n_tiles; ++t, ++g) {
                const int st = g % C::NS;
                if (g >= C::NS) WAIT(C::B_KVE + st, ((g / C::NS) & 1) ^ 1u, 21, g);
                const bool issue = __shfl_sync(0xffffffffu, *abort_flag == 0 ? 1 : 0, 0) != 0;
                if (!issue) continue;
                n_issued = g + 1;
                if (lane == 0) {
                    const uint32_t fb = BAR(C::B_KVF + st);
                    mbar_arrive_expect_tx(fb, C::STAGE_B);
                    const uint32_t dk = sbase + st * C::STAGE_B, dv = dk + C::TILE_B;
                    const int row = tl.kv_lo + t * BN;
#pragma unroll
                    for (int b = 0; b < C::NSLAB; ++b) {
                        const int x = tl.kvh * HD + b * 64;
                        tma_load_4d(dk + b * C::KSLAB, &tmK, fb, x, row, tl.cache_layer, tl.seq);
                        tma_load_4d(dv + b * C::KSLAB, &tmV, fb, x, row, tl.cache_layer, tl.seq);
                    }
                }
                __syncwarp();
            }
        }
        // every issued tile lands before the CTA exits
        for (int k = n_issued > C::NS ? n_issued - C::NS : 0; k < n_issued; ++k)
            mbar_wait_bounded(BAR(C::B_KVF + k % C::NS), (k / C::NS) & 1, abort_flag, a.err, a.dbg,
                              23, k, false, kDrainLimitCycles);
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        constexpr uint32_t ID_S = idesc_f16(DT, 128, BN, false);
        constexpr uint32_t ID_PV = idesc_f16(DT, 128, HD, true);
        int g = 0, itc = 0;
        for (int it = it_begin; it < it_end; ++it, ++itc) {
            const PrefillTile tl = a.tiles[it];
            const int n = tl.n_tiles;
            const int qb = itc % C::QBUF;
            WAIT(C::B_QF + qb, (itc / C::QBUF) & 1, 24, itc);  // Q of this item staged
            tc_fence_after();
            const uint32_t qa = tmem + C::COL_Q + qb * HD;
            // S = Q_hi.K^T + Q_lo.K^T for global tile gg
            auto issue_s = [&](int gg) {
                const int st = gg % C::NS;
                WAIT(C::B_KVF + st, (gg / C::NS) & 1, 25, gg);
                const int sb = gg & 1;
                if (gg >= 2) WAIT(C::B_SE + sb, ((gg >> 1) - 1) & 1, 26, gg);
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t d = tmem + C::COL_S + sb * BN;
                    const uint32_t kb = sbase + st * C::STAGE_B;
#pragma unroll
                    for (int part = 0; part < 2; ++part)
#pragma unroll
                        for (int ks = 0; ks < HD / 16; ++ks) {
                            const uint64_t bd =
                                sw128_desc(kb + (ks / 4) * C::KSLAB + (ks % 4) * 32, 16, 1024);
                            tc_mma_ts(d, qa + part * (HD / 2) + ks * 8, bd, ID_S,
                                      (part | ks) != 0 ? 1u : 0u);
                        }
                    tc_commit(BAR(C::B_SF + sb));
                }
                __syncwarp();
            };
            if (n > 0) issue_s(g);
            for (int t = 0; t < n; ++t, ++g) {
                if (t + 1 < n) issue_s(g + 1);
                WAIT(C::B_PF, g & 1, 27, g);  // P(g) staged
                // the item's first P.V overwrites O: the previous item's O read
                if (t == 0 && itc > 0) WAIT(C::B_OE, (itc - 1) & 1, 28, itc);
                tc_fence_after();
                const int st = g % C::NS;
                const uint32_t vb = sbase + st * C::STAGE_B + C::TILE_B;
                if (t == n - 1) {
                    // rows past the prompt's last row: V := 0 (p is 0 there)
                    const int z0 = tl.tok_row0 + tl.ntok - (tl.kv_lo + t * BN);
                    if (z0 < BN) {
                        unsigned char* vt = base + st * C::STAGE_B + C::TILE_B;
                        for (int b = 0; b < C::NSLAB; ++b)
                            for (int idx = lane; idx < (BN - z0) * 8; idx += 32)
                                *reinterpret_cast<uint4*>(vt + b * C::KSLAB + (z0 + idx / 8) * 128 +
                                                          (idx % 8) * 16) = make_uint4(0u, 0u, 0u, 0u);
                        fence_proxy_async_shared();
                    }
                    __syncwarp();
                }
                if (lane == 0) {
                    // O += P.V, in TMEM across the item's tiles
                    const uint32_t d = tmem + C::COL_O;
#pragma unroll
                    for (int part = 0; part < 2; ++part)
#pragma unroll
                        for (int kb = 0; kb < BN / 16; ++kb) {
                            const uint64_t ad = sw128_desc(sbase + C::OFF_P + part * C::PPART +
                                                               (kb / 4) * C::PSLAB + (kb % 4) * 32,
                                                           16, 1024);
                            const uint64_t bd = sw128_desc(vb + kb * 16 * 128, C::KSLAB, 1024);
                            tc_mma(d, ad, bd, ID_PV, (t | part | kb) != 0 ? 1u : 0u);
                        }
                    tc_commit(BAR(C::B_OF));
                    tc_commit(BAR(C::B_PE));
                    tc_commit(BAR(C::B_KVE + st));
                }
                __syncwarp();
            }
            if (lane == 0) tc_commit(BAR(C::B_QE + qb));  // this item's Q is no longer read
            __syncwarp();
        }
        // every MMA this thread issued completes before TMEM is freed
        if (lane == 0) tc_commit(BAR(C::B_DONE));
        __syncwarp();
        mbar_wait_bounded(BAR(C::B_DONE), 0u, abort_flag, a.err, a.dbg, 29, 0, false,
                          kDrainLimitCycles);
    } else {
        // ------------------------------------------------------------ softmax warps
        // Warps 2-9: warp w takes TMEM lane quarter w % 4 (its 32 query rows)
        // and half hf of the columns -- S columns [hf*BN/2, +BN/2), O / head
        // dims [hf*HD/2, +HD/2).  The two warps of a quarter exchange row
        // maxima (and at an item's end row sums) through shared memory under a
        // 64-thread named barrier; exchange buffers alternate, so one barrier
        // per exchange keeps a write from overtaking the partner's read.
        constexpr int SW = BN / 2, HW = HD / 2;
        const int q4 = warp & 3;
        const int hf = (warp - 2) >> 2;
        const int r = q4 * 32 + lane;      // query row of the tile = TMEM lane
        const int j = r / G, h = r % G;    // token of the tile, head within the kv group
        const uint32_t lane_addr = static_cast<uint32_t>(q4 * 32) << 16;
        float* xch = reinterpret_cast<float*>(base + C::OFF_XCH);  // [2 buffers][2 halves][128]
        int xu = 0;
        auto exchange = [&](float mine) {  // the partner warp's value for this row
            float* buf = xch + (xu & 1) * 256;
            ++xu;
            buf[hf * 128 + r] = mine;
            named_bar_sync(1 + q4, 64);
            return buf[(hf ^ 1) * 128 + r];
        };
        // Rotates this warp's half of item tl's query rows, splits them into
        // hi / lo 16-bit parts and stores them to TMEM Q buffer qi % QBUF (the MMA
        // warp's A operand); returns the power of two S is to be scaled back by.
        auto stage_q = [&](const PrefillTile& tl, int qi) -> float {
            const int qb = qi % C::QBUF;
            const bool live = j < tl.ntok;
            const long long io = static_cast<long long>(tl.io0) + static_cast<long long>(j) * tl.io_step;
            if (qi >= C::QBUF) WAIT(C::B_QE + qb, ((qi / C::QBUF) - 1) & 1, 30, qi);
            float unscale = 1.0f;
            {
                // rotation of this warp's half of the row (dims [hf*HW, +HW)),
                // 16 dims at a time: each batch's operands are loaded together
                // (independent loads in flight), then rotated with the rounding
                // forms of rope_elem -- Neox pairs (j, j + HD/2), which for full
                // rotary put half 0 at j = d and half 1 at j = d - HD/2;
                // interleaved pairs (2j, 2j + 1) within the half
                const float* qin = a.q + io * a.q_stride + static_cast<long long>(tl.kvh * G + h) * HD;
                const float2* cs = a.rope + static_cast<long long>(tl.rope_row0 + j) * (HD / 2);
                float qr[HW];
                float mx = 0.0f;
                if (!live) {
#pragma unroll
                    for (int dd = 0; dd < HW; ++dd) qr[dd] = 0.0f;
                } else if (tl.rope_half == HD / 2 && a.q_vec) {
                    // 16-byte loads: every lane reads its own row, so each
                    // warp-wide load touches 32 lines -- a quarter as many
                    // requests as 4-byte loads
                    const float4* q4 = reinterpret_cast<const float4*>(qin);
                    const float4* c4 = reinterpret_cast<const float4*>(cs);  // 2 (cos, sin) pairs each
                    if (a.neox) {
#pragma unroll
                        for (int b0 = 0; b0 < HW; b0 += 16) {
                            float4 xa[4], xb[4], cc[8];
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                xa[i] = __ldg(q4 + b0 / 4 + i);
                                xb[i] = __ldg(q4 + (HD / 2 + b0) / 4 + i);
                            }
#pragma unroll
                            for (int i = 0; i < 8; ++i) cc[i] = __ldg(c4 + b0 / 2 + i);
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const float va = f4_at(xa[i / 4], i % 4), vb = f4_at(xb[i / 4], i % 4);
                                const float cx = (i & 1) ? cc[i / 2].z : cc[i / 2].x;
                                const float sy = (i & 1) ? cc[i / 2].w : cc[i / 2].y;
                                qr[b0 + i] = hf == 0 ? __fmaf_rn(va, cx, -__fmul_rn(vb, sy))
                                                     : __fmaf_rn(va, sy, __fmul_rn(vb, cx));
                            }
                        }
                    } else {
#pragma unroll
                        for (int b0 = 0; b0 < HW; b0 += 16) {
                            const int d0 = hf * HW + b0;
                            float4 x4[4], cc[4];
#pragma unroll
                            for (int i = 0; i < 4; ++i) x4[i] = __ldg(q4 + d0 / 4 + i);
#pragma unroll
                            for (int i = 0; i < 4; ++i) cc[i] = __ldg(c4 + d0 / 4 + i);
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const float aa = f4_at(x4[i / 4], i % 4 & ~1);
                                const float bb = f4_at(x4[i / 4], (i % 4) | 1);
                                // pair i/2 -> (cos, sin) entry i/2: float4 i/4, half (i/2) & 1
                                const float cx = ((i / 2) & 1) ? cc[i / 4].z : cc[i / 4].x;
                                const float sy = ((i / 2) & 1) ? cc[i / 4].w : cc[i / 4].y;
                                qr[b0 + i] = (i & 1) == 0 ? __fsub_rn(__fmul_rn(aa, cx), __fmul_rn(bb, sy))
                                                          : __fadd_rn(__fmul_rn(aa, sy), __fmul_rn(bb, cx));
                            }
                        }
                    }
                } else if (tl.rope_half == HD / 2 && a.neox) {
#pragma unroll
                    for (int b0 = 0; b0 < HW; b0 += 16) {
                        float xa[16], xb[16];
                        float2 c[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            xa[i] = __ldg(qin + b0 + i);
                            xb[i] = __ldg(qin + HD / 2 + b0 + i);
                            c[i] = __ldg(cs + b0 + i);
                        }
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            qr[b0 + i] = hf == 0 ? __fmaf_rn(xa[i], c[i].x, -__fmul_rn(xb[i], c[i].y))
                                                 : __fmaf_rn(xa[i], c[i].y, __fmul_rn(xb[i], c[i].x));
                    }
                } else if (tl.rope_half == HD / 2) {
#pragma unroll
                    for (int b0 = 0; b0 < HW; b0 += 16) {
                        const int d0 = hf * HW + b0;
                        float x[16];
                        float2 c[8];
#pragma unroll
                        for (int i = 0; i < 16; ++i) x[i] = __ldg(qin + d0 + i);
#pragma unroll
                        for (int i = 0; i < 8; ++i) c[i] = __ldg(cs + d0 / 2 + i);
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const float aa = x[i & ~1], bb = x[i | 1];
                            const float2 t = c[i >> 1];
                            qr[b0 + i] = (i & 1) == 0 ? __fsub_rn(__fmul_rn(aa, t.x), __fmul_rn(bb, t.y))
                                                      : __fadd_rn(__fmul_rn(aa, t.y), __fmul_rn(bb, t.x));
                        }
                    }
                } else {
                    // partial rotary
#pragma unroll
                    for (int dd = 0; dd < HW; ++dd)
                        qr[dd] = rope_elem(qin, hf * HW + dd, tl.rope_half, cs, a.neox != 0);
                }
#pragma unroll
                for (int dd = 0; dd < HW; ++dd) mx = fmaxf(mx, fabsf(qr[dd]));
                float up = 1.0f;
                if constexpr (DT == DT_F16T) {
                    mx = fmaxf(mx, exchange(mx));  // the whole row's largest |q|
                    const int e = static_cast<int>((__float_as_uint(mx) >> 23) & 0xFFu) - 127;
                    const int sh = min(60, max(-60, 14 - e));
                    up = __uint_as_float(static_cast<uint32_t>(127 + sh) << 23);
                    unscale = __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);
                }
                // this half's dims [hf*HW, +HW) are columns [hf*HW/2, +HW/2) of
                // each part (two elements per column, the even one low)
                uint32_t hw[HW / 2], lw[HW / 2];
#pragma unroll
                for (int i = 0; i < HW / 2; ++i)
                    split_pair<DT>(qr[2 * i] * up, qr[2 * i + 1] * up, hw[i], lw[i]);
                __syncwarp();  // converged for the .sync.aligned stores
                const uint32_t qc = tmem + lane_addr + C::COL_Q + qb * HD + hf * (HW / 2);
                if constexpr (HW / 2 == 16) {
                    tmem_st16(qc, hw);
                    tmem_st16(qc + HD / 2, lw);
                } else {
                    tmem_st32(qc, hw);
                    tmem_st32(qc + HD / 2, lw);
                }
            }
            tc_fence_before();  // TMEM stores done (wait::st) -> the MMA warp
            __syncwarp();
            if (lane == 0) mbar_arrive(BAR(C::B_QF + qb));
            return unscale;
        };
        int g = 0, itc = 0;
        float unscale = it_begin < it_end ? stage_q(a.tiles[it_begin], 0) : 1.0f;
        for (int it = it_begin; it < it_end; ++it, ++itc) {
            const PrefillTile tl = a.tiles[it];
            const bool live = j < tl.ntok;
            const int hi_r = live ? tl.tok_row0 + j : -1;
            const int lo_r = live ? (tl.window > 0 ? max(tl.row0, hi_r - tl.window + 1) : tl.row0) : 0;
            const long long io = static_cast<long long>(tl.io0) + static_cast<long long>(j) * tl.io_step;

            // Running maximum m (the reference p = exp(s - m) is taken against)
            // and this half's sum l.  O accumulates in TMEM across the item's
            // tiles; m moves only when a tile's maximum exceeds it by more
            // than kLazy (p then stays below e^kLazy = 256, exact in the
            // fp32 sums), and O and l are rescaled then -- rarely after the
            // first tiles, so the softmax does not wait for each tile's P.V.
            constexpr float kLazy = 5.545177444479562f;  // 8 ln 2
            float m = -INFINITY, l = 0.0f;
            const int n = tl.n_tiles;
            // unscale is a power of two: (S * unscale) * scale rounds once, as
            // the reference's dot * scale does
            const float sc_mul = a.scale * unscale;
            const bool capped = a.softcap > 0.0f;
            // columns every live row of the item attends: [lo_all, hi_all]
            const int hi_all = tl.tok_row0;  // the first token's row
            const int lo_all = tl.window > 0
                                   ? max(tl.row0, tl.tok_row0 + tl.ntok - 1 - tl.window + 1)
                                   : tl.row0;
            for (int t = 0; t < n; ++t, ++g) {
                const int sb = g & 1;
                WAIT(C::B_SF + sb, (g >> 1) & 1, 32, g);
                __syncwarp();  // converged for the .sync.aligned load
                tc_fence_after();
                uint32_t sr[SW];
                if constexpr (SW == 64) tmem_ld64(tmem + lane_addr + C::COL_S + sb * BN + hf * SW, sr);
                else tmem_ld32(tmem + lane_addr + C::COL_S + sb * BN + hf * SW, sr);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(BAR(C::B_SE + sb));
                // scores of this row's columns: scale, soft-cap, and -- on tiles
                // that cross a row's causal or window limit -- each row's [lo, hi]
                const int c0 = tl.kv_lo + t * BN + hf * SW;
                const int tile0 = tl.kv_lo + t * BN;
                const bool masked = tile0 + BN - 1 > hi_all || tile0 < lo_all;
                float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                // plain tiles keep S unscaled: the scale goes into the
                // exponent's fused multiply-add below, and the row maximum is
                // scaled once (x -> x * sc_mul is monotone, sc_mul > 0)
                const bool raw = !capped && !masked;
                if (raw) {
#pragma unroll
                    for (int c = 0; c < SW; c += 2)
                        mx4[(c >> 1) & 3] = fmax3(mx4[(c >> 1) & 3], __uint_as_float(sr[c]),
                                                  __uint_as_float(sr[c + 1]));
#pragma unroll
                    for (int i = 0; i < 4; ++i) mx4[i] = __fmul_rn(mx4[i], sc_mul);
                } else {
#pragma unroll
                    for (int c = 0; c < SW; ++c) {
                        float v = __fmul_rn(__uint_as_float(sr[c]), sc_mul);
                        if (capped) v = __fmul_rn(a.softcap, tanhf(__fmul_rn(v, a.inv_softcap)));
                        const int col = c0 + c;
                        if (masked) v = (col >= lo_r && col <= hi_r) ? v : -INFINITY;
                        sr[c] = __float_as_uint(v);
                        mx4[c & 3] = fmaxf(mx4[c & 3], v);
                    }
                }
                float mt = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
                mt = fmaxf(mt, exchange(mt));  // the row's maximum over both halves
                // both warps of a row see the same mt and m, so they move m together
                const bool move = mt > m + kLazy || (m == -INFINITY && mt > -INFINITY);
                if (__any_sync(0xffffffffu, move)) {
                    const float alpha = (!move || m == -INFINITY) ? (move ? 0.0f : 1.0f)
                                                                    : ex2_approx((m - mt) * kLog2eP);
                    if (move) {
                        l *= alpha;
                        m = mt;
                    }
                    // O holds P.V of tiles [0, t): rescale this half of it once the
                    // last of those has landed.  A row whose m was -inf has O = 0
                    // (all its p were 0) and alpha = 0.
                    if (t > 0) {
                        WAIT(C::B_OF, (g - 1) & 1, 31, g);
                        __syncwarp();
                        tc_fence_after();
#pragma unroll
                        for (int c = 0; c < HW; c += 32) {
                            uint32_t t32[32];
                            tmem_ld32(tmem + lane_addr + C::COL_O + hf * HW + c, t32);
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                t32[i] = __float_as_uint(__uint_as_float(t32[i]) * alpha);
                            tmem_st32(tmem + lane_addr + C::COL_O + hf * HW + c, t32);
                        }
                    }
                }
                // p = exp(s - m) and its hi / lo 16-bit parts, in registers before
                // waiting for the P buffer (this overlaps the previous P.V).
                // ex2(-inf) is +0, so masked columns need no test once m is
                // finite (a row with no attended column yet uses 0).
                const float mref = m == -INFINITY ? 0.0f : m;
                // exponent x = s * a_mul - mref * log2(e), two columns per
                // fp32x2 FMA (s unscaled on plain tiles: a_mul = scale * log2(e))
                const float a_mul = raw ? sc_mul * kLog2eP : kLog2eP;
                const float b_add = -mref * kLog2eP;
                uint32_t hw[SW / 2], lw[SW / 2];
                // row-sum partials: two pairs, two columns per packed add
                float ls4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int c = 0; c < SW; c += 2) {
                    float x0 = b_add, x1 = b_add;
                    fma_x2(x0, x1, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]), a_mul, a_mul);
                    const float p0 = ex2_approx(x0);
                    const float p1 = ex2_approx(x1);
                    add_x2(ls4[((c >> 1) & 1) * 2], ls4[((c >> 1) & 1) * 2 + 1], p0, p1);
                    if constexpr (DT == DT_BF16) {
                        // hi: p truncated to bf16 (exact bit mask); lo = p - hi
                        // (exact), rounded to the nearest bf16 by adding half
                        // an ulp to its bits (ties away from zero: the same
                        // half-ulp bound as ties to even) -- integer work that
                        // leaves the special-function pipe to ex2
                        const uint32_t b0 = __float_as_uint(p0) & 0xFFFF0000u;
                        const uint32_t b1 = __float_as_uint(p1) & 0xFFFF0000u;
                        hw[c / 2] = __byte_perm(b0, b1, 0x7632);
                        float d0, d1;
                        sub_x2(d0, d1, p0, p1, __uint_as_float(b0), __uint_as_float(b1));
                        const uint32_t r0 = __float_as_uint(d0) + 0x8000u;
                        const uint32_t r1 = __float_as_uint(d1) + 0x8000u;
                        lw[c / 2] = __byte_perm(r0, r1, 0x7632);
                    } else {
                        split_pair<DT>(p0, p1, hw[c / 2], lw[c / 2]);
                    }
                }
                l += (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);  // this half's columns
                if (g >= 1) WAIT(C::B_PE, (g - 1) & 1, 33, g);  // P.V of the previous tile read P
#pragma unroll
                for (int cc = 0; cc < SW / 8; ++cc) {
                    const int c8 = hf * (SW / 8) + cc;
                    const int off =
                        C::OFF_P + (c8 / 8) * C::PSLAB + r * 128 + (((c8 % 8) ^ (r & 7)) * 16);
                    *reinterpret_cast<uint4*>(base + off) =
                        make_uint4(hw[4 * cc], hw[4 * cc + 1], hw[4 * cc + 2], hw[4 * cc + 3]);
                    *reinterpret_cast<uint4*>(base + off + C::PPART) =
                        make_uint4(lw[4 * cc], lw[4 * cc + 1], lw[4 * cc + 2], lw[4 * cc + 3]);
                }
                fence_proxy_async_shared();
                tc_fence_before();  // the O rescale's TMEM stores, before P.V reads O
                __syncwarp();
                if (lane == 0) mbar_arrive(BAR(C::B_PF));
            }
            // the next item's Q, while this item's last P.V runs (the MMA warp
            // can start the next item's S as soon as it is staged)
            const float unscale_next = it + 1 < it_end ? stage_q(a.tiles[it + 1], itc + 1) : 1.0f;
            // ---- this half of the output row: O / (l of both halves), once the
            // item's last P.V has landed
            const float lt = l + exchange(l);
            if (n > 0) {
                WAIT(C::B_OF, (g - 1) & 1, 34, g);
                __syncwarp();
                tc_fence_after();
                float* dst = a.out + io * a.q_stride + static_cast<long long>(tl.kvh * G + h) * HD +
                             hf * HW;
                const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
#pragma unroll
                for (int c = 0; c < HW; c += 32) {
                    uint32_t t32[32];
                    tmem_ld32(tmem + lane_addr + C::COL_O + hf * HW + c, t32);
                    if (live && lt > 0.0f) {
#pragma unroll
                        for (int d = 0; d < 32; d += 4)
                            *reinterpret_cast<float4*>(dst + c + d) = make_float4(
                                __uint_as_float(t32[d]) * inv, __uint_as_float(t32[d + 1]) * inv,
                                __uint_as_float(t32[d + 2]) * inv, __uint_as_float(t32[d + 3]) * inv);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(BAR(C::B_OE));  // O may be overwritten
            unscale = unscale_next;
        }
    }
#undef WAIT
#undef BAR
    // every role is done with TMEM: tcgen05.ld completed (wait::ld), MMAs
    // observed through the done barrier
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

template <int HD, int DT, int G>
cudaError_t launch_one(const PrefillArgs& a, const CUtensorMap* tk, const CUtensorMap* tv, int grid,
                       cudaStream_t st) {
    constexpr int smem = PfCfg<HD>::SMEM;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel<HD, DT, G>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    prefill_tc_kernel<HD, DT, G><<<grid, kPfThreads, smem, st>>>(*tk, *tv, a);
    return cudaGetLastError();
}

template <int HD, int DT>
cudaError_t launch_g(const PrefillArgs& a, const CUtensorMap* tk, const CUtensorMap* tv, int G,
                     int grid, cudaStream_t st) {
    switch (G) {
        case 1: return launch_one<HD, DT, 1>(a, tk, tv, grid, st);
        case 2: return launch_one<HD, DT, 2>(a, tk, tv, grid, st);
        case 4: return launch_one<HD, DT, 4>(a, tk, tv, grid, st);
        case 8: return launch_one<HD, DT, 8>(a, tk, tv, grid, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

bool prefill_tc_supported(int head_dim, int dtype, int G) {
    return (head_dim == 64 || head_dim == 128) && (dtype == DT_BF16 || dtype == DT_F16T) &&
           (G == 1 || G == 2 || G == 4 || G == 8);
}

int prefill_tc_rows(int head_dim) { return head_dim == 64 ? PfCfg<64>::BN : PfCfg<128>::BN; }

cudaError_t prefill_tc_launch(const PrefillArgs& a, const CUtensorMap* tmK, const CUtensorMap* tmV,
                              int head_dim, int dtype, int G, int grid, cudaStream_t stream) {
    if (!prefill_tc_supported(head_dim, dtype, G)) return cudaErrorInvalidValue;
    if (head_dim == 64)
        return dtype == DT_BF16 ? launch_g<64, DT_BF16>(a, tmK, tmV, G, grid, stream)
                                : launch_g<64, DT_F16T>(a, tmK, tmV, G, grid, stream);
    return dtype == DT_BF16 ? launch_g<128, DT_BF16>(a, tmK, tmV, G, grid, stream)
                            : launch_g<128, DT_F16T>(a, tmK, tmV, G, grid, stream);
}

}  // namespace jx
