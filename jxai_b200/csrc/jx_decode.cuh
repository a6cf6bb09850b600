// jx_decode.cuh -- the fused decode-attention kernel for sm_100a.
//
// One launch performs, for every (sequence, layer) pair of a step, the work
// jxai's forward_token does inline per layer (src/transformer.cpp:2497-2566):
// RoPE on q and k, the append of k and v at `pos`, and grouped-query attention
// over every attended cache row.  Design:
//
//  * Work space.  Rows are flattened over (pair, segment, row), a segment being
//    one kv head of a pair (two for 16-bit caches with short head rows); each
//    of the P persistent CTAs takes a contiguous slice of that space -- equal
//    in rows, or (with few segments per CTA) sized on the host so that rows
//    plus a cost per extra piece come out equal -- so bytes are balanced
//    across SMs however ragged the sequences are.  A slice cuts segments into
//    pieces.
//  * Pipeline.  Warp 4 is the producer: it streams 32-row K and V tiles of the
//    current piece into a ring of shared-memory stages with 4-D TMA tile loads
//    (128-byte swizzle, no multicast), completion tracked by mbarriers, and
//    bulk-copies each piece's q and RoPE row (and the raw k/v rows the piece
//    appends) into one of two q slots.
//    Warps 0-3 are consumers; tile k goes to stream k % S (S = consumer warps /
//    warps per tile) with the ring size a multiple of S, so every use of a
//    given stage is consumed by the same warps, in order.  (A stage whose
//    successive uses went to different warps could be waited on two phases
//    ahead, which mbarrier parity cannot tell apart.)  The kernel lets the next
//    kernel of the stream launch early (programmatic dependent launch) and
//    waits for the previous one before touching data.
//  * fp32 caches: math on CUDA cores (~1 flop per KV byte at group 4, well
//    under the FMA rate at HBM speed).  QK: lane = cache row, dot product over
//    head_dim in ascending order with fused multiply-adds (the reference's
//    `dot += q[d]*k[d]` order), q of the whole query group broadcast from
//    shared memory.  Online softmax per tile with warp-shuffle max; PV: lane =
//    head dimensions, p broadcast from shared memory.
//  * bf16 / fp16 caches: twice the flops per byte plus a conversion per
//    element made the CUDA-core form FMA-issue-bound (~60% of HBM), so QK and
//    PV run on the tensor cores (MmaWarp: warp-level m16n8k16, q and p split
//    into two 16-bit parts for fp32-level accuracy).  Two kv heads share a
//    tile row where head rows are under 256 bytes (kv_pack), each handled by
//    its own consumer warp.
//  * Merge.  At the end of a piece the four warps' (m, l, o) are merged through
//    shared memory.  A piece that is a whole segment writes the normalised
//    output directly; otherwise it writes a partial to scratch and counts
//    itself in on the segment's counter (no waiting); the CTA that counts in
//    last merges all partials by log-sum-exp after its own last piece and
//    resets the counter.
//  * Append.  The consumer warp whose tile holds a segment's newest row
//    rotates k, converts both rows to the cache type, and stores them to the
//    cache (for later steps) and into the landed tile (for this one); the raw
//    rows come with the piece's q in the prefetch.  The tile's load does not
//    wait for the global store, so no generic->async proxy fence on global
//    memory holds the ring back.
//
// Template parameters: HD = head_dim, GP = query heads per kv head rounded up
// to 1/2/4/8, DT = cache element type (DT_F32 / DT_BF16 / DT_F16T), KP = kv
// heads per tile row (1, or 2 for 16-bit caches with short head rows).
#pragma once

#include "jx_device.cuh"
#include "jx_internal.h"

namespace jx {

constexpr int kConsumerWarps = 4;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kTileRows = 32;
constexpr float kLog2e = 1.4426950408889634f;

template <int HD, int DT>
struct Geo {
    static constexpr int ESZ = DT == DT_F32 ? 4 : 2;
    static constexpr int ROWB = HD * ESZ;                // bytes of one kv-head row
    static constexpr int BOX = ROWB < 128 ? ROWB : 128;  // TMA box inner extent (bytes)
    static constexpr int NB = ROWB / BOX;                // boxes per row
    static constexpr int BOXE = BOX / ESZ;               // box inner extent (elements)
    static constexpr int TILEB = kTileRows * ROWB;       // one K (or V) tile
    static constexpr int SWZ = BOX / 16 - 1;             // swizzle row mask
    static constexpr int EPC = 16 / ESZ;                 // elements per 16-byte chunk
    static constexpr int CHUNKS = ROWB / 16;             // chunks per row
    static constexpr int CPB = BOX / 16;                 // chunks per box row
    static constexpr int DPL = HD / 32;                  // head dims per lane in PV
    static constexpr int LANEB = DPL * ESZ;              // bytes per lane per V row
    static_assert(ROWB % 64 == 0, "row bytes must be a multiple of 64");
};

// Shared-memory carve-up, identical on host and device.  KP kv heads share a
// tile row (16-bit caches), so a segment has GP*KP query heads.
template <int HD, int GP, int DT, int KP = 1>
struct SmemLayout {
    using G = Geo<HD * KP, DT>;
    static constexpr int GS = GP * KP;
    static constexpr int q_bytes = GS * HD * 4;       // rotated q of the current piece
    static constexpr int qraw_bytes = 2 * GS * HD * 4;  // raw q of two pieces (bulk copies)
    static constexpr int rope_bytes = 2 * HD * 4;       // (cos, sin) rows of two pieces
    static constexpr int p_bytes = DT == DT_F32 ? kConsumerWarps * kTileRows * GS * 4 : 0;
    static constexpr int o_bytes = kConsumerWarps * GS * HD * 4;
    static constexpr int ml_bytes = kConsumerWarps * GS * 2 * 4;
    static constexpr int lohi_bytes = 2 * GS * 4;       // per-column row limits (prefill blocks)
    static constexpr int misc_bytes = 16 + 2 * 48 + 48;  // flags, two split records, new-row record
    static constexpr int n_extra_bars = 5;  // q full[2], q empty[2], test (never arrived at)
    static __host__ __device__ constexpr int stages_bytes(int ns) { return ns * 2 * G::TILEB; }
    static __host__ __device__ constexpr int bars_offset(int ns) {
        return stages_bytes(ns) + q_bytes + qraw_bytes + rope_bytes + p_bytes + o_bytes +
               ml_bytes + lohi_bytes + misc_bytes;
    }
    static __host__ __device__ constexpr int bars_end(int ns) {
        return bars_offset(ns) + (ns * 2 + n_extra_bars) * 8;
    }
    // Optional, after the barriers: the raw k and v rows of the two prefetched
    // pieces (the new row's inputs), when they fit the 227 KB a CTA may have.
    static constexpr int kvraw_bytes = 2 * 2 * KP * HD * 4;
    static constexpr int kMaxBytes = 227 * 1024;
    static __host__ __device__ constexpr int kvraw_offset(int ns) { return (bars_end(ns) + 15) & ~15; }
    static __host__ __device__ constexpr bool kv_prefetch(int ns) {
        return kvraw_offset(ns) + kvraw_bytes + 1024 <= kMaxBytes;
    }
    static __host__ __device__ constexpr int total(int ns) {
        return (kv_prefetch(ns) ? kvraw_offset(ns) + kvraw_bytes : bars_end(ns)) +
               1024;  // + alignment slack
    }
};

// Byte offset inside a TMA-written tile (rows of BOX bytes per box, boxes of
// 32 rows placed one after another) with the hardware swizzle applied.
template <int HD, int DT>
__device__ __forceinline__ uint32_t tile_off(int row, int byte_in_row) {
    using G = Geo<HD, DT>;
    const int b = byte_in_row / G::BOX;
    const uint32_t off =
        static_cast<uint32_t>(b * kTileRows * G::BOX + row * G::BOX + (byte_in_row % G::BOX));
    return off ^ (((off >> 7) & G::SWZ) << 4);
}

// Walks one CTA's slice [b0, b1) of the flattened row space piece by piece.
struct PieceIter {
    const PairRow* pairs;
    int n_pairs, n_kv;
    long long x, b1;
    int i;
    // current piece
    PairRow pr;
    int pi, kvh, r, n;
    long long seg_start;

    __device__ void init(const PairRow* p, int np, int nkv, long long b0_, long long b1_,
                         const int* start_hint) {
        pairs = p;
        n_pairs = np;
        n_kv = nkv;
        x = b0_;
        b1 = b1_;
        if (start_hint) {  // precomputed by the host for this CTA
            i = start_hint[blockIdx.x];
            return;
        }
        // largest i with pairs[i].off <= x (zero-length pairs share the next offset)
        int lo = 0, hi = np - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (pairs[mid].off <= x) lo = mid; else hi = mid - 1;
        }
        i = lo;
    }

    int bad = 0;  // set when the plan is inconsistent (checked builds report it)

    __device__ bool next() {
        if (x >= b1) return false;
        if (JX_DEVICE_CHECKS && (i < 0 || i >= n_pairs)) {
            bad = 1;
            return false;
        }
        pr = pairs[i];
        if (JX_DEVICE_CHECKS && (pr.len <= 0 || x < pr.off || x >= pr.off + (long long)n_kv * pr.len)) {
            bad = 2;
            return false;
        }
        pi = i;
        const long long rel = x - pr.off;
        kvh = static_cast<int>(rel / pr.len);
        r = static_cast<int>(rel - static_cast<long long>(kvh) * pr.len);
        seg_start = pr.off + static_cast<long long>(kvh) * pr.len;
        const long long seg_end = seg_start + pr.len;
        const long long pend = seg_end < b1 ? seg_end : b1;
        n = static_cast<int>(pend - x);
        x = pend;
        if (x == seg_end && kvh == n_kv - 1) {
            ++i;
            while (i < n_pairs && pairs[i].len == 0) ++i;
        }
        return true;
    }
};

// CTA that owns flattened row x when `total` rows are split over P CTAs with
// CTA c taking [floor(c*total/P), floor((c+1)*total/P)).
__device__ __forceinline__ long long owner_cta(long long x, long long total, long long P) {
    return ((x + 1) * P - 1) / total;
}

// The step's new row (transformer.cpp:2506-2520) for one kv head: k rotated
// at the row's position, both converted to the cache type, written to the
// cache in HBM for later steps and into the landed tile's row `rr` in shared
// memory for this one.  One warp.  The tile was fetched by TMA without waiting
// for the global store (a generic-proxy global write would need a proxy fence
// that drains the CTA's loads in flight); the shared-memory copy is the one
// this step reads, and the fence before the stage is released orders these
// generic writes before the stage's next TMA write.
struct PatchRec {
    long long dst;     // cache element of the row's first kv head
    const float* kin;  // raw k of that head (shared memory or global)
    const float* vin;  // raw v of that head
    const float2* cs;  // (cos, sin) row
    int rr;            // row within its tile
    int rope_half;
    int pad[2];
};
static_assert(sizeof(PatchRec) == 48, "PatchRec layout");

template <int HD, int RW, int DT>
__device__ __forceinline__ void patch_new_row(const DecodeArgs& a, const PatchRec& pp, int h_local,
                                              unsigned char* Kt, unsigned char* Vt, int lane) {
    constexpr int ESZ = DT == DT_F32 ? 4 : 2;
    const long long dst = pp.dst + static_cast<long long>(h_local) * HD;
    const float* kin = pp.kin + h_local * HD;
    const float* vin = pp.vin + h_local * HD;
    const int rr = pp.rr;
    if (JX_CHECKED(a, dst >= 0 && dst + HD <= a.cache_elems && rr >= 0 && rr < kTileRows, 11, dst,
                   rr, h_local)) {
#pragma unroll 2
        for (int d = lane; d < HD; d += 32) {
            const float kr = rope_elem(kin, d, pp.rope_half, pp.cs, a.neox != 0);
            const float vr = vin[d];
            store_kv<DT>(a.k_cache, dst + d, kr);
            store_kv<DT>(a.v_cache, dst + d, vr);
            const uint32_t off = tile_off<RW, DT>(rr, (h_local * HD + d) * ESZ);
            if constexpr (DT == DT_F32) {
                *reinterpret_cast<float*>(Kt + off) = kr;
                *reinterpret_cast<float*>(Vt + off) = vr;
            } else if constexpr (DT == DT_BF16) {
                *reinterpret_cast<uint16_t*>(Kt + off) = f32_to_bf16_ref(kr);
                *reinterpret_cast<uint16_t*>(Vt + off) = f32_to_bf16_ref(vr);
            } else {
                *reinterpret_cast<uint16_t*>(Kt + off) = f32_to_f16_trunc_ref(kr);
                *reinterpret_cast<uint16_t*>(Vt + off) = f32_to_f16_trunc_ref(vr);
            }
        }
    }
    fence_proxy_async_shared();  // before the stage's next TMA write
    __syncwarp();
}

// Writes one merged (g, d) element of a finished segment: normalised output,
// or the partial (o, m, l) in partial mode.
template <int HD>
__device__ __forceinline__ void emit_final(const DecodeArgs& a, int io, int h, int d, float M,
                                           float L, float O) {
    if (!JX_CHECKED(a, io >= 0 && io < a.n_io && h < a.n_heads && d < HD, 20, io, h, d)) return;
    if (a.part_out) {
        const long long base = (static_cast<long long>(io) * a.n_heads + h) * (HD + 2);
        a.part_out[base + d] = O;
        if (d == 0) {
            a.part_out[base + HD] = M;
            a.part_out[base + HD + 1] = L;
        }
    } else {
        a.out[static_cast<long long>(io) * a.q_stride + h * HD + d] = O * (1.0f / L);
    }
}

// A piece that is not a whole segment.  Its partial (o, m, l) goes to scratch
// slot (cta + seg) when the piece ends and the CTA counts it in on the
// segment's counter -- at once (release only, nobody waits) when more pieces
// follow in the CTA, else after the CTA's last piece.  The CTA that counts in
// last merges the segment after its last piece.
struct SplitRec {
    long long seg;        // segment index: pair * n_kv + kv head (of the segment)
    long long seg_start;  // flattened index of the segment's first row
    int len;              // segment rows
    int io;               // q/out row of the pair
    int kvh;              // kv head (of the segment) within the pair
    int early;            // 1: counted in when the piece ended (more pieces followed)
    int nq;               // tokens of a prefill block (1 otherwise)
    int io_step;          // io distance between the block's tokens
    int c_first, c_last;  // first and last CTA of the segment
};
static_assert(sizeof(SplitRec) == 48, "SplitRec layout");

// Last-arriver merge of segment `r`: the partials of CTAs c_first..c_last are
// combined by log-sum-exp and the output written.  Each consumer thread owns
// E (head, dim) elements and issues the loads of QC pieces for all of them
// before using any (one round trip per QC pieces); no barriers.  Inlined: a
// call would give the kernel a stack frame, which measurably slows launches.
template <int HD, int GS>
__device__ __forceinline__ void merge_split(const DecodeArgs& a, const SplitRec& r, long long c_first,
                                         long long c_last, int ctid) {
    constexpr int E = (GS * HD + kConsumerThreads - 1) / kConsumerThreads;
    constexpr int QC = (24 / E) < 1 ? 1 : ((24 / E) > 8 ? 8 : (24 / E));
    const int np = static_cast<int>(c_last - c_first + 1);
    const int Gn = a.G;
    const int ncol = Gn * (r.nq > 1 ? r.nq : 1);  // (token, head) columns
    const long long step = static_cast<long long>(GS) * (HD + 2);
    const float* base_p = a.scratch + (c_first + r.seg) * step;
    float M[E], Ls[E], O[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        M[e] = -INFINITY;
        Ls[e] = 0.0f;
        O[e] = 0.0f;
    }
    for (int q0 = 0; q0 < np; q0 += QC) {
        float mv[E][QC], lv[E][QC], ov[E][QC];
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const int idx = ctid + e * kConsumerThreads;
            const int g = idx / HD, d = idx % HD;
            const float* src = base_p + static_cast<long long>(g) * (HD + 2);
#pragma unroll
            for (int qq = 0; qq < QC; ++qq) {
                const bool ok = idx < ncol * HD && q0 + qq < np;
                const float* pq = src + (q0 + qq) * step;
                mv[e][qq] = ok ? __ldcg(pq + HD) : -INFINITY;
                lv[e][qq] = ok ? __ldcg(pq + HD + 1) : 0.0f;
                ov[e][qq] = ok ? __ldcg(pq + d) : 0.0f;
            }
        }
#pragma unroll
        for (int e = 0; e < E; ++e) {
            float Mn = M[e];
#pragma unroll
            for (int qq = 0; qq < QC; ++qq) Mn = fmaxf(Mn, mv[e][qq]);
            if (Mn == -INFINITY) continue;
            const float f0 = M[e] == -INFINITY ? 0.0f : ex2_approx((M[e] - Mn) * kLog2e);
            Ls[e] *= f0;
            O[e] *= f0;
#pragma unroll
            for (int qq = 0; qq < QC; ++qq) {
                const float f = mv[e][qq] == -INFINITY ? 0.0f : ex2_approx((mv[e][qq] - Mn) * kLog2e);
                Ls[e] += lv[e][qq] * f;
                O[e] += ov[e][qq] * f;
            }
            M[e] = Mn;
        }
    }
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int idx = ctid + e * kConsumerThreads;
        if (idx < ncol * HD) {
            const int g = idx / HD, d = idx % HD;
            const int j = g / Gn, h = g - j * Gn;
            emit_final<HD>(a, r.io + j * r.io_step, r.kvh * Gn + h, d, M[e], Ls[e], O[e]);
        }
    }
}

// ---------------------------------------------------------------- 16-bit caches: warp MMA
// One consumer warp's attention state for bf16 / fp16 caches, on the tensor
// cores (mma.sync m16n8k16, fp32 accumulation).  Per 32-row tile:
//   S^T[row][col] = K[row][:] . Qc[col][:]     rows as M (two blocks of 16)
//   O^T[d][col]  += V^T[d][row] . Pc[row][col]  head dims as M (HD/16 blocks)
// The 8 columns of an n8 block are (part, head) pairs, col = part*GP + head:
// q and p are fp32, so each is split into two 16-bit parts, hi = rn(x) and
// lo = rn(x - hi), and the parts' columns are summed back in fp32.  Cache
// values are exact in the MMA's operand type, so the products carry q and p
// to ~2^-17 relative (bf16) or ~2^-22 (fp16), inside the fp32-path tolerance.
// fp16 q is first scaled by a power of two so the group's largest |q| sits in
// [2^14, 2^15) (no overflow, no lost low bits); the scale is undone on S
// exactly.  Lane L holds, after the column sums, S and O for the rows / dims
// of its C fragment and heads (2(L%4) + j) % GP, j = 0, 1 ("slots").
template <int HD, int GP, int DT, int KP>
struct MmaWarp {
    static constexpr int RW = HD * KP;            // tile row: KP kv heads side by side
    using G = Geo<RW, DT>;
    static constexpr int NBC = (2 * GP + 7) / 8;  // n8 blocks of (part, head) columns
    static constexpr int KS = HD / 16;            // k16 steps of QK = m16 blocks of PV
    static_assert(DT != DT_F32, "fp32 caches use the CUDA-core consumer");
    static_assert(HD % 16 == 0, "head_dim must be a multiple of 16");

    int kp;                   // the kv head of the tile row this warp attends with
    uint32_t qf[KS][NBC][2];  // Q^T B fragments
    float o[KS][NBC][4];      // O^T accumulators
    float m[2], l[2];         // running max / lane-partial sum per slot
    float s_unscale;          // 2^-shift of the fp16 q scaling (1 for bf16)
    bool blocked;             // prefill block: per-slot attended rows [row_lo, row_hi]
    int row_lo[2], row_hi[2];

    // Sum of a value over the columns that hold the same head (see above).
    __device__ __forceinline__ static float col_sum(const float (&x)[NBC][4], int r) {
        float v = x[0][r];
        if constexpr (NBC == 2) v += x[1][r];
        if constexpr (GP == 1) v += x[0][r ^ 1];
        if constexpr (GP <= 2) v += __shfl_xor_sync(0xffffffffu, v, 1);
        if constexpr (GP <= 4) v += __shfl_xor_sync(0xffffffffu, v, 2);
        return v;
    }

    // This lane's 16-bit pair for column block nb from the hi / lo pairs.
    __device__ __forceinline__ static uint32_t pick(uint32_t hi, uint32_t lo, int nb, int t) {
        if constexpr (GP == 8) return nb == 0 ? hi : lo;
        else if constexpr (GP == 4) return t < 2 ? hi : lo;
        else if constexpr (GP == 2) return t == 0 ? hi : (t == 1 ? lo : 0u);
        else return t == 0 ? ((hi & 0xFFFFu) | (lo << 16)) : 0u;  // cols 0, 1 = hi, lo
    }

    // q_s: rotated q of the segment's KP*GP heads, [head][HD]; this warp takes
    // kv head `kp_` of the tile row and its GP query heads.
    __device__ __forceinline__ void begin_piece(const float* q_s, int lane, int kp_,
                                                const int* lohi) {
        kp = kp_;
        const int g = lane >> 2, t = lane & 3;
        blocked = lohi != nullptr;
        if (blocked) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int hs = kp * GP + (2 * t + j) % GP;
                row_lo[j] = lohi[hs];
                row_hi[j] = lohi[KP * GP + hs];
            }
        }
        float x[KS][NBC][4];
        float mx = 0.0f;
#pragma unroll
        for (int nb = 0; nb < NBC; ++nb) {
            const int col = nb * 8 + g;
            const int part = col / GP, h = col % GP;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const float* src = q_s + (kp * GP + h) * HD + ks * 16 + 2 * t;
                const bool use = part < 2;
                x[ks][nb][0] = use ? src[0] : 0.0f;
                x[ks][nb][1] = use ? src[1] : 0.0f;
                x[ks][nb][2] = use ? src[8] : 0.0f;
                x[ks][nb][3] = use ? src[9] : 0.0f;
#pragma unroll
                for (int e = 0; e < 4; ++e) mx = fmaxf(mx, fabsf(x[ks][nb][e]));
            }
        }
        float up = 1.0f;
        s_unscale = 1.0f;
        if constexpr (DT == DT_F16T) {
            const float gm = warp_max(mx);
            const int e = static_cast<int>((__float_as_uint(gm) >> 23) & 0xFFu) - 127;
            const int sh = min(60, max(-60, 14 - e));
            up = __uint_as_float(static_cast<uint32_t>(127 + sh) << 23);
            s_unscale = __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);
        }
#pragma unroll
        for (int nb = 0; nb < NBC; ++nb) {
            const int part = (nb * 8 + g) / GP;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                uint32_t h01, l01, h23, l23;
                split_pair<DT>(x[ks][nb][0] * up, x[ks][nb][1] * up, h01, l01);
                split_pair<DT>(x[ks][nb][2] * up, x[ks][nb][3] * up, h23, l23);
                qf[ks][nb][0] = part == 0 ? h01 : (part == 1 ? l01 : 0u);
                qf[ks][nb][1] = part == 0 ? h23 : (part == 1 ? l23 : 0u);
            }
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            m[j] = -INFINITY;
            l[j] = 0.0f;
        }
#pragma unroll
        for (int mh = 0; mh < KS; ++mh)
#pragma unroll
            for (int nb = 0; nb < NBC; ++nb)
#pragma unroll
                for (int r = 0; r < 4; ++r) o[mh][nb][r] = 0.0f;
    }

    // One tile of kTileRows rows; rows [nvalid, kTileRows) are not attended.
    __device__ __forceinline__ void tile(uint32_t Kt, unsigned char* Vt_ptr, uint32_t Vt,
                                         int nvalid, int row_first, int lane, float scale,
                                         float softcap, float inv_cap) {
        const int g = lane >> 2, t = lane & 3;
        const int i8 = lane >> 3, r8 = lane & 7;
        const int cb = kp * HD * 2;  // this kv head's first byte in a tile row
        if (nvalid < kTileRows) {
            // p is 0 there, but 0 * (Inf or NaN) is not: clear this kv head's
            // unattended V rows
            constexpr int CH = HD * 2 / 16;
            for (int idx = lane; idx < (kTileRows - nvalid) * CH; idx += 32) {
                const int row = nvalid + idx / CH;
                *reinterpret_cast<uint4*>(Vt_ptr + tile_off<RW, DT>(row, cb + (idx % CH) * 16)) =
                    make_uint4(0u, 0u, 0u, 0u);
            }
            fence_proxy_async_shared();  // before the stage's next TMA write
            __syncwarp();
        }
        // ---- S^T = K Qc^T
        float acc[2][NBC][4];
#pragma unroll
        for (int mb = 0; mb < 2; ++mb)
#pragma unroll
            for (int nb = 0; nb < NBC; ++nb)
#pragma unroll
                for (int r = 0; r < 4; ++r) acc[mb][nb][r] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
            for (int mb = 0; mb < 2; ++mb) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4<false>(Kt + tile_off<RW, DT>(mb * 16 + (i8 & 1) * 8 + r8,
                                                     cb + ks * 32 + (i8 >> 1) * 16),
                               a0, a1, a2, a3);
#pragma unroll
                for (int nb = 0; nb < NBC; ++nb)
                    mma_16816<DT>(acc[mb][nb], a0, a1, a2, a3, qf[ks][nb][0], qf[ks][nb][1]);
            }
        }
        // ---- scores, online softmax (rows mb*16 + (r>>1)*8 + g, slot r&1)
        float s[2][4];
#pragma unroll
        for (int mb = 0; mb < 2; ++mb)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                float sc = __fmul_rn(col_sum(acc[mb], r) * s_unscale, scale);
                if (softcap > 0.0f) sc = __fmul_rn(softcap, tanhf(__fmul_rn(sc, inv_cap)));
                const int rt = mb * 16 + (r >> 1) * 8 + g;  // row within the tile
                bool keep = rt < nvalid;
                if (blocked)
                    keep = keep && row_first + rt >= row_lo[r & 1] && row_first + rt <= row_hi[r & 1];
                s[mb][r] = keep ? sc : -INFINITY;
            }
        float alpha[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            float mt = fmaxf(fmaxf(s[0][j], s[0][j + 2]), fmaxf(s[1][j], s[1][j + 2]));
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
            const float mn = fmaxf(m[j], mt);
            alpha[j] = m[j] == -INFINITY ? 0.0f : ex2_approx((m[j] - mn) * kLog2e);
            m[j] = mn;
        }
        float p[2][4];
        float ls[2] = {0.0f, 0.0f};
#pragma unroll
        for (int mb = 0; mb < 2; ++mb)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                p[mb][r] = s[mb][r] == -INFINITY ? 0.0f : ex2_approx((s[mb][r] - m[r & 1]) * kLog2e);
                ls[r & 1] += p[mb][r];
            }
#pragma unroll
        for (int j = 0; j < 2; ++j) l[j] = l[j] * alpha[j] + ls[j];
#pragma unroll
        for (int mh = 0; mh < KS; ++mh)
#pragma unroll
            for (int nb = 0; nb < NBC; ++nb)
#pragma unroll
                for (int r = 0; r < 4; ++r) o[mh][nb][r] *= alpha[r & 1];
        // ---- P as B fragments: C layout of (rows, columns) -> transposed
        uint32_t bp[2][NBC][2];
#pragma unroll
        for (int mb = 0; mb < 2; ++mb)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                uint32_t hi, lo;
                split_pair<DT>(p[mb][2 * hf], p[mb][2 * hf + 1], hi, lo);
#pragma unroll
                for (int nb = 0; nb < NBC; ++nb) bp[mb][nb][hf] = movmatrix_trans(pick(hi, lo, nb, t));
            }
        // ---- O^T += V^T Pc
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
            if (kb == 1 && nvalid <= 16) break;
#pragma unroll
            for (int mh = 0; mh < KS; ++mh) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4<true>(Vt + tile_off<RW, DT>(kb * 16 + (i8 >> 1) * 8 + r8,
                                                    cb + mh * 32 + (i8 & 1) * 16),
                              a0, a1, a2, a3);
#pragma unroll
                for (int nb = 0; nb < NBC; ++nb)
                    mma_16816<DT>(o[mh][nb], a0, a1, a2, a3, bp[kb][nb][0], bp[kb][nb][1]);
            }
        }
    }

    // Writes this warp's (m, l) and unnormalised o per head into the merge
    // staging area ([warp][KP*GP heads]), in the layout of the CUDA-core
    // consumer; the heads of the row's other kv heads get the empty state.
    __device__ __forceinline__ void finish(float* o_s, float* ml_s, int warp, int lane) {
        constexpr int GS = KP * GP;
        const int g = lane >> 2, t = lane & 3;
        float lt[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            float v = l[j];
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            lt[j] = v;
        }
        // lanes holding a head's first copy write it
        const bool w0 = GP == 8 || (GP == 4 && t < 2) || (GP <= 2 && t == 0);
        const bool w1 = w0 && GP != 1;
#pragma unroll
        for (int mh = 0; mh < KS; ++mh)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float v = col_sum(o[mh], r);
                const int j = r & 1;
                if (j == 0 ? w0 : w1) {
                    const int h = kp * GP + (2 * t + j) % GP;
                    o_s[(warp * GS + h) * HD + mh * 16 + (r >> 1) * 8 + g] = v;
                }
            }
        if (g == 0) {
#pragma unroll
            for (int j = 0; j < 2; ++j)
                if (j == 0 ? w0 : w1) {
                    const int h = kp * GP + (2 * t + j) % GP;
                    ml_s[(warp * GS + h) * 2] = m[j];
                    ml_s[(warp * GS + h) * 2 + 1] = lt[j];
                }
        }
        if constexpr (KP > 1) {
            for (int idx = lane; idx < GS * HD; idx += 32) {
                const int h = idx / HD;
                if (h / GP == kp) continue;
                o_s[(warp * GS + h) * HD + idx % HD] = 0.0f;
                if (idx % HD == 0) {
                    ml_s[(warp * GS + h) * 2] = -INFINITY;
                    ml_s[(warp * GS + h) * 2 + 1] = 0.0f;
                }
            }
        }
    }
};

// Register cap per configuration.  A 5-warp CTA pair puts three warps on
// some SM sub-partition (16K registers each), so two CTAs per SM need at most
// 170 registers per thread; configurations whose shared memory allows two
// CTAs are held to 168, the others may use all 255.  (The tensor-core
// consumer at head_dim 128 and group 8 would spill under the cap: it runs one
// CTA per SM with a deeper ring instead.)
template <int HD, int GP, int DT, int KP>
struct RegCap {
    static constexpr bool two_ctas =
        SmemLayout<HD, GP, DT, KP>::total(4) + 1024 <= (227 * 1024) / 2 &&
        !(DT != DT_F32 && HD >= 128 && GP * KP >= 8);
    static constexpr int value = two_ctas ? 168 : 255;
};

template <int HD, int GP, int DT, int KP>
__global__ void __launch_bounds__(kThreads) __maxnreg__((RegCap<HD, GP, DT, KP>::value))
    decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const DecodeArgs a) {
    constexpr int RW = HD * KP;  // tile row width (elements): KP kv heads side by side
    constexpr int GS = GP * KP;  // padded query heads of a segment
    static_assert(KP == 1 || DT != DT_F32, "kv-head packing is for 16-bit caches");
    constexpr bool kMma = DT != DT_F32;  // 16-bit caches: tensor-core consumer
    constexpr int kSplit = KP;           // consumer warps per tile
    using G = Geo<RW, DT>;
    using L = SmemLayout<HD, GP, DT, KP>;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
    unsigned char* base = smem_raw + (base_u32 - raw_u32);
    const int NS = a.n_stages;
    float* q_s = reinterpret_cast<float*>(base + L::stages_bytes(NS));
    float* qraw_s = q_s + L::q_bytes / 4;                                  // [2][GS*HD]
    float2* rope_s = reinterpret_cast<float2*>(qraw_s + L::qraw_bytes / 4);  // [2][HD/2]
    float* p_s = reinterpret_cast<float*>(rope_s) + L::rope_bytes / 4;
    // raw k and v rows of the new row, [2 q slots][k, v][KP*HD], when they fit
    const bool kv_pre = L::kv_prefetch(NS);
    float* kvraw_s = reinterpret_cast<float*>(base + L::kvraw_offset(NS));
    float* o_s = p_s + L::p_bytes / 4;
    float* ml_s = o_s + L::o_bytes / 4;
    int* lohi_s = reinterpret_cast<int*>(ml_s + L::ml_bytes / 4);  // [GS] lo, [GS] hi
    int* misc = lohi_s + 2 * GS;  // [1] abort, [2..3] last flags
    SplitRec* recs = reinterpret_cast<SplitRec*>(misc + 4);     // [2]
    PatchRec* patch = reinterpret_cast<PatchRec*>(recs + 2);    // the piece's new row
    // full[s] at bars+8s, empty[s] at bars+8(NS+s), q full[2], q empty[2] after them
    const uint32_t bars = base_u32 + L::bars_offset(NS);
    const uint32_t qfull = bars + 8 * (2 * NS);
    const uint32_t qempty = qfull + 16;
    const uint32_t test_bar = qempty + 16;  // nothing ever arrives here
    volatile int* abort_flag = misc + 1;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // bound of every pipeline wait (0 in the arguments: the default)
    const long long wlim = a.wait_limit > 0 ? a.wait_limit : kWaitLimitCycles;
    // The next step may be scheduled onto SMs as this grid frees them; it
    // waits (pdl_wait) for this grid's completion before touching any data.
    pdl_launch_dependents();
    if (!JX_CHECKED(a, static_cast<int>(base_u32 - raw_u32) +
                               (kv_pre ? L::kvraw_offset(NS) + L::kvraw_bytes : L::bars_end(NS)) <=
                               a.smem_bytes &&
                           a.n_consumers >= kSplit && a.n_consumers <= kConsumerWarps &&
                           a.n_consumers % kSplit == 0 && NS % (a.n_consumers / kSplit) == 0,
                    1, a.smem_bytes, NS, a.n_consumers))
        return;  // every thread takes this branch together

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(bars + 8 * s, 1);
            mbar_init(bars + 8 * (NS + s), kSplit);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(qfull + 8 * s, 1);
            mbar_init(qempty + 8 * s, 1);
        }
        mbar_init(test_bar, 1);
        misc[0] = 0;
        misc[1] = 0;
        fence_barrier_init();
    }
    __syncthreads();

    const long long P = gridDim.x;
    const long long c = blockIdx.x;
    const long long b0 = a.cta_begin ? a.cta_begin[c] : a.total * c / P;
    const long long b1 = a.cta_begin ? a.cta_begin[c + 1] : a.total * (c + 1) / P;

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            prefetch_tensormap(&tmK);
            prefetch_tensormap(&tmV);
        }
        PieceIter it;
        it.init(a.pairs, a.n_pairs, a.n_kv, b0, b1, a.cta_pair);
        int tile = 0;
        int stage = 0;         // tile % NS
        uint32_t phase = 0;    // (tile / NS) & 1
        int n_issued = 0;  // tiles [0, n_issued) had their loads issued
        int piece = 0;
        while (it.next()) {
            // the work plan was read above; everything below may touch data an
            // earlier kernel of the stream wrote (q/k/v inputs, cache rows)
            if (piece == 0) pdl_wait();
            const PairRow& pr = it.pr;
            const int ntiles = (it.n + kTileRows - 1) / kTileRows;
            if (!JX_CHECKED(a, it.kvh >= 0 && it.kvh < a.n_kv && pr.cache_layer >= 0 &&
                                   pr.cache_layer < a.n_cache_layers && pr.seq >= 0 &&
                                   pr.seq < a.n_cache_seqs && pr.row0 >= 0 &&
                                   pr.row0 + pr.len <= a.capacity,
                            30, it.kvh, pr.cache_layer, pr.row0 + pr.len))
                break;
            // The segment's newest row, when this piece holds it: its consumer
            // warp writes it (cache and landed tile) from the raw k/v rows.
            bool has_app = false;
            if (kv_pre && pr.append_row >= 0 && !a.skip_append) {
                const int al = pr.append_row - pr.row0;
                has_app = al >= it.r && al < it.r + it.n;
            }
            // this piece's raw q (the segment's query heads), (cos, sin) row and,
            // with the new row, raw k and v -> q slot piece % 2, ahead of the
            // consumers that use them
            if (a.q_bulk) {
                const int qs = piece & 1;
                if (piece >= 2)
                    mbar_wait_bounded(qempty + 8 * qs, ((piece >> 1) & 1) ^ 1u, abort_flag, a.err,
                                      a.dbg, 4, piece, true, wlim);
                if (lane == 0 && *abort_flag == 0 &&
                    JX_CHECKED(a, pr.io >= 0 && pr.io < a.n_io && pr.rope_row >= 0 &&
                                      pr.rope_row < a.n_rope_rows &&
                                      (it.kvh + 1) * a.G <= a.n_heads &&
                                      (it.kvh + 1) * KP * HD <= a.kv_stride,
                               32, pr.io, pr.rope_row, it.kvh)) {
                    const uint32_t qb = static_cast<uint32_t>(a.G) * HD * 4;
                    constexpr uint32_t kvb = KP * HD * 4;
                    mbar_arrive_expect_tx(qfull + 8 * qs, qb + HD * 4 + (has_app ? 2 * kvb : 0));
                    if (has_app) {
                        const long long kv_off = static_cast<long long>(pr.io) * a.kv_stride +
                                                 static_cast<long long>(it.kvh) * KP * HD;
                        bulk_load(smem_u32(kvraw_s + qs * 2 * KP * HD), a.k_in + kv_off, kvb,
                                  qfull + 8 * qs);
                        bulk_load(smem_u32(kvraw_s + qs * 2 * KP * HD + KP * HD), a.v_in + kv_off,
                                  kvb, qfull + 8 * qs);
                    }
                    bulk_load(smem_u32(qraw_s + qs * GS * HD),
                              a.q + static_cast<long long>(pr.io) * a.q_stride +
                                  static_cast<long long>(it.kvh) * a.G * HD,
                              qb, qfull + 8 * qs);
                    bulk_load(smem_u32(rope_s + qs * (HD / 2)),
                              a.rope + static_cast<long long>(pr.rope_row) * (HD / 2), HD * 4,
                              qfull + 8 * qs);
                } else if (lane == 0) {
                    mbar_arrive(qfull + 8 * qs);  // complete the phase without data
                }
                __syncwarp();
            }
            ++piece;
            for (int t = 0; t < ntiles; ++t, ++tile) {
                const int cur_stage = stage;
                const uint32_t cur_phase = phase;
                if (++stage == NS) {
                    stage = 0;
                    phase ^= 1u;
                }
                // wait until the previous use of this stage (tile - NS) has been released
                if (tile >= NS)
                    mbar_wait_bounded(bars + 8 * (NS + cur_stage), cur_phase ^ 1u, abort_flag,
                                      a.err, a.dbg, 1, tile, true, wlim);
                const bool issue = __shfl_sync(0xffffffffu, *abort_flag == 0 ? 1 : 0, 0) != 0;
                if (!issue) continue;
                n_issued = tile + 1;
                const int stage_ = cur_stage;
                if (lane == 0) {
                    const uint32_t fb = bars + 8 * stage_;
                    const uint32_t dk = base_u32 + stage_ * 2 * G::TILEB;
                    const uint32_t dv = dk + G::TILEB;
                    const int row = pr.row0 + it.r + t * kTileRows;
                    if (JX_CHECKED(a, stage_ >= 0 && stage_ < NS && row >= 0 && row < a.capacity &&
                                          (it.kvh + 1) * RW <= a.row_stride,
                                   31, row, stage_, it.kvh)) {
                        mbar_arrive_expect_tx(fb, 2 * G::TILEB);
#pragma unroll
                        for (int b = 0; b < G::NB; ++b) {
                            const int c0 = it.kvh * RW + b * G::BOXE;
                            tma_load_4d(dk + b * kTileRows * G::BOX, &tmK, fb, c0, row,
                                        pr.cache_layer, pr.seq);
                            tma_load_4d(dv + b * kTileRows * G::BOX, &tmV, fb, c0, row,
                                        pr.cache_layer, pr.seq);
                        }
                    } else {
                        mbar_arrive(fb);  // complete the phase without data
                    }
                }
                __syncwarp();
            }
        }
        (void)JX_CHECKED(a, it.bad == 0, 40 + it.bad, it.x, it.i, b1);
        // Drain: every issued tile load must land before the CTA exits.
        const int first = n_issued > NS ? n_issued - NS : 0;
        for (int k = first; k < n_issued; ++k)
            mbar_wait_bounded(bars + 8 * (k % NS), (k / NS) & 1, abort_flag, a.err, a.dbg, 3, k,
                              false, kDrainLimitCycles);
        if (a.q_bulk)
            for (int k = piece > 2 ? piece - 2 : 0; k < piece; ++k)
                mbar_wait_bounded(qfull + 8 * (k & 1), (k >> 1) & 1, abort_flag, a.err, a.dbg, 6,
                                  k, false, kDrainLimitCycles);
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int ctid = threadIdx.x;
    pdl_wait();  // outputs, partials and counters were last written by an earlier step
    if (a.test_wait_cta > 0 && blockIdx.x == a.test_wait_cta - 1 && warp == 0) {
        // Test hook for the error path: one bounded wait on a barrier nothing
        // arrives at.  It runs out after wlim cycles, raises the CTA's
        // abort flag and the device error word; every later wait of the CTA
        // then returns at once and the CTA finishes its control flow.
        mbar_wait_bounded(test_bar, 0u, abort_flag, a.err, a.dbg, 7, 0, true, wlim);
    }

    // Partial mode: pairs with no local rows still owe an (o=0, m=-inf, l=0) partial.
    if (a.part_out) {
        for (int i = blockIdx.x; i < a.n_pairs; i += gridDim.x) {
            const PairRow pr = a.pairs[i];
            if (pr.len != 0) continue;
            for (int idx = ctid; idx < a.n_heads * (HD + 2); idx += kConsumerThreads) {
                const int d = idx % (HD + 2);
                a.part_out[static_cast<long long>(pr.io) * a.n_heads * (HD + 2) + idx] =
                    d == HD ? -INFINITY : 0.0f;
            }
        }
    }

    PieceIter it;
    it.init(a.pairs, a.n_pairs, a.n_kv, b0, b1, a.cta_pair);
    const int C = a.n_consumers;
    const bool active = warp < C;
    // 16-bit caches with two kv heads per tile row: each tile goes to a pair of
    // warps, one per kv head (SPLIT arrivals release a stage)
    const int streams = C / kSplit;  // tile streams; stream i takes tiles i, i + streams, ...
    const int stream_id = warp / kSplit;
    int tile_base = 0;          // global index of the current piece's first tile
    int my_k = stream_id;       // this warp's next tile (global index)
    int my_stage = stream_id;   // my_k % NS
    uint32_t my_phase = 0;      // (my_k / NS) & 1
    const float scale = a.scale;
    const float softcap = a.softcap;
    const float inv_cap = a.inv_softcap;
    using MW = MmaWarp<HD, GP, (kMma ? DT : DT_BF16), KP>;
    MW mw;
    int cpiece = 0;       // pieces started
    int n_split = 0;      // pieces recorded in recs[]
    int early_prev = -1;  // thread 0: counter value before an early count-in
    long long pending_seg = -1;  // segment of an early count-in not issued yet
    while (it.next()) {
        const PairRow& pr = it.pr;
        const int kvh = it.kvh;
        const bool blocked = pr.nq > 1;  // a prefill block of several tokens
        // A piece that is not a whole segment is counted in after it ends,
        // against the first and last CTA of its segment: read them now, so
        // that the load is not on the count-in's path.
        int2 owner = make_int2(0, 0);
        if (ctid == 0 && !(it.r == 0 && it.n == pr.len)) {
            const long long sg = static_cast<long long>(it.pi) * a.n_kv + kvh;
            if (!a.seg_owner) {
                owner.x = static_cast<int>(owner_cta(it.seg_start, a.total, P));
                owner.y = static_cast<int>(owner_cta(it.seg_start + pr.len - 1, a.total, P));
            } else if (sg >= 0 && sg < a.n_segments) {
                owner = __ldg(reinterpret_cast<const int2*>(a.seg_owner) + sg);
            }
        }

        // The segment's newest row, when this piece holds it (index within the
        // piece): the consumer warp(s) of its tile write it (patch_new_row), and
        // the piece's q slot, which holds its raw k and v, is released after the
        // piece's tiles rather than after the q rotation.
        int app_row = -1;
        if (pr.append_row >= 0 && !a.skip_append) {
            const int al = pr.append_row - pr.row0;
            if (al >= it.r && al < it.r + it.n) app_row = al - it.r;
        }
        const int qs_piece = cpiece & 1;
        const bool slot_kv = a.q_bulk && kv_pre && app_row >= 0;  // inputs in the q slot
        if (app_row >= 0 && ctid == 0) {
            // read by the tile's warp(s) after the barrier below; the previous
            // piece's readers passed the barrier that ended its tiles
            PatchRec& pp = *patch;
            pp.dst = static_cast<long long>(pr.seq) * a.seq_stride +
                     static_cast<long long>(pr.cache_layer) * a.layer_stride +
                     static_cast<long long>(pr.append_row) * a.row_stride +
                     static_cast<long long>(kvh) * KP * HD;
            if (slot_kv) {
                pp.kin = kvraw_s + qs_piece * 2 * KP * HD;
                pp.vin = pp.kin + KP * HD;
                pp.cs = rope_s + qs_piece * (HD / 2);
            } else {
                const long long off = static_cast<long long>(pr.io) * a.kv_stride +
                                      static_cast<long long>(kvh) * KP * HD;
                pp.kin = a.k_in + off;
                pp.vin = a.v_in + off;
                pp.cs = a.rope + static_cast<long long>(pr.rope_row) * (HD / 2);
            }
            pp.rr = app_row & (kTileRows - 1);
            pp.rope_half = pr.rope_half;
        }

        // q rotation for this segment's query group -> q_s (padded heads = 0).
        // Every reader of q_s for the previous piece passed the barrier that
        // ended that piece's tiles.
        if (a.q_bulk) {
            const int qs = qs_piece;
            mbar_wait_bounded(qfull + 8 * qs, (cpiece >> 1) & 1, abort_flag, a.err, a.dbg, 5,
                              cpiece, true, wlim);
            const float* qr = qraw_s + qs * GS * HD;
            const float2* cs = rope_s + qs * (HD / 2);
            for (int idx = ctid; idx < GS * HD; idx += kConsumerThreads) {
                const int g = idx / HD, d = idx % HD;
                q_s[idx] = g < a.G ? rope_elem(qr + g * HD, d, pr.rope_half, cs, a.neox != 0) : 0.0f;
            }
            named_bar_sync(1, kConsumerThreads);
            if (ctid == 0 && !slot_kv) mbar_arrive(qempty + 8 * qs);
        } else {
        // q straight from global memory; a prefill block's column g is head
        // g % G of token g / G (its own q row and cos/sin row)
        named_bar_sync(1, kConsumerThreads);
        const int nq = pr.nq > 1 ? pr.nq : 1;
        if (JX_CHECKED(a, pr.io >= 0 && pr.io + (nq - 1) * pr.io_step < a.n_io &&
                              pr.rope_row >= 0 && pr.rope_row + nq - 1 < a.n_rope_rows &&
                              (kvh + 1) * a.G <= a.n_heads,
                       50, pr.io, pr.rope_row, kvh)) {
            for (int idx = ctid; idx < GS * HD; idx += kConsumerThreads) {
                const int g = idx / HD, d = idx % HD;
                const int j = g / a.G, h = g - j * a.G;
                float val = 0.0f;
                if (j < nq) {
                    const float* qin = a.q +
                                       static_cast<long long>(pr.io + j * pr.io_step) * a.q_stride +
                                       (static_cast<long long>(kvh) * a.G + h) * HD;
                    const float2* cs =
                        a.rope + static_cast<long long>(pr.rope_row + j) * (HD / 2);
                    val = rope_elem(qin, d, pr.rope_half, cs, a.neox != 0);
                }
                q_s[idx] = val;
            }
            if (nq > 1) {
                // per-column attended rows: token j sees [lo, tok_row0 + j]
                for (int g = ctid; g < GS; g += kConsumerThreads) {
                    const int j = g / a.G;
                    int lo = 1, hi = 0;  // padded column: nothing
                    if (j < nq) {
                        hi = pr.tok_row0 + j;
                        lo = pr.window > 0 ? max(pr.row0, hi - pr.window + 1) : pr.row0;
                    }
                    lohi_s[g] = lo;
                    lohi_s[GS + g] = hi;
                }
            }
        }
        named_bar_sync(1, kConsumerThreads);
        }
        ++cpiece;
        if (pending_seg >= 0) {
            // Every consumer thread's partial stores of the previous piece precede
            // the barrier just passed, so this release publishes them; only
            // warp 0 waits for it.
            if (ctid == 0 && JX_CHECKED(a, pending_seg < a.n_segments, 63, pending_seg, 0, 0))
                early_prev = atomic_add_release_gpu(a.counters + pending_seg, 1);
            pending_seg = -1;
        }

        float m[GS], l[GS], o[GS][G::DPL];
        if constexpr (kMma) {
            mw.begin_piece(q_s, lane, warp % kSplit, blocked ? lohi_s : nullptr);
        } else {
#pragma unroll
            for (int g = 0; g < GS; ++g) {
                m[g] = -INFINITY;
                l[g] = 0.0f;
#pragma unroll
                for (int k = 0; k < G::DPL; ++k) o[g][k] = 0.0f;
            }
        }

        const int ntiles = (it.n + kTileRows - 1) / kTileRows;
        const int tile_end = tile_base + ntiles;
        // this warp's tiles of the piece: my_k, my_k + C, ... (stage and phase tracked
        // incrementally; the ring size is a multiple of C)
        while (active && my_k < tile_end) {
            const int t = my_k - tile_base;
            mbar_wait_bounded(bars + 8 * my_stage, my_phase, abort_flag, a.err, a.dbg, 2, my_k,
                              true, wlim);
            const int nvalid = min(kTileRows, it.n - t * kTileRows);
            unsigned char* Kt = base + my_stage * 2 * G::TILEB;
            unsigned char* Vt = Kt + G::TILEB;
            if (app_row >= 0 && t == (app_row >> 5))  // the new row of this warp's kv head
                patch_new_row<HD, RW, DT>(a, *patch, kSplit > 1 ? warp % kSplit : 0, Kt, Vt, lane);
            if constexpr (kMma) {
                const uint32_t ku = base_u32 + my_stage * 2 * G::TILEB;
                mw.tile(ku, base + my_stage * 2 * G::TILEB + G::TILEB, ku + G::TILEB, nvalid,
                        pr.row0 + it.r + t * kTileRows, lane, scale, softcap, inv_cap);
            } else {

            // ---- scores: lane = row
            float s[GS];
            if (lane < nvalid) {
                // even and odd dims summed apart, two per fp32x2 FMA, then added
                float acc[GS], acc1[GS];
#pragma unroll
                for (int g = 0; g < GS; ++g) acc[g] = acc1[g] = 0.0f;
#pragma unroll 4
                for (int j = 0; j < G::CHUNKS; ++j) {
                    const uint4 raw = *reinterpret_cast<const uint4*>(
                        Kt + tile_off<RW, DT>(lane, j * 16));
                    float kv[G::EPC];
                    unpack16<DT>(raw, kv);
#pragma unroll
                    for (int e4 = 0; e4 < G::EPC; e4 += 4) {
#pragma unroll
                        for (int g = 0; g < GS; ++g) {
                            const float4 qv =
                                *reinterpret_cast<const float4*>(q_s + g * HD + j * G::EPC + e4);
                            fma_x2(acc[g], acc1[g], qv.x, qv.y, kv[e4 + 0], kv[e4 + 1]);
                            fma_x2(acc[g], acc1[g], qv.z, qv.w, kv[e4 + 2], kv[e4 + 3]);
                        }
                    }
                }
#pragma unroll
                for (int g = 0; g < GS; ++g) acc[g] = __fadd_rn(acc[g], acc1[g]);
#pragma unroll
                for (int g = 0; g < GS; ++g) {
                    float sc = __fmul_rn(acc[g], scale);
                    if (softcap > 0.0f) sc = __fmul_rn(softcap, tanhf(__fmul_rn(sc, inv_cap)));
                    s[g] = sc;
                }
                if (blocked) {  // prefill block: each token's causal / window limits
                    const int rowl = pr.row0 + it.r + t * kTileRows + lane;
#pragma unroll
                    for (int g = 0; g < GS; ++g)
                        if (rowl < lohi_s[g] || rowl > lohi_s[GS + g]) s[g] = -INFINITY;
                }
            } else {
#pragma unroll
                for (int g = 0; g < GS; ++g) s[g] = -INFINITY;
            }

            // ---- online softmax over this tile
            float pv[GS];
#pragma unroll
            for (int g = 0; g < GS; ++g) {
                const float mt = warp_max(s[g]);
                const float mn = fmaxf(m[g], mt);
                const float alpha = m[g] == -INFINITY ? 0.0f : ex2_approx((m[g] - mn) * kLog2e);
                const float p =
                    (lane < nvalid && s[g] != -INFINITY) ? ex2_approx((s[g] - mn) * kLog2e) : 0.0f;
                l[g] = l[g] * alpha + p;
#pragma unroll
                for (int k = 0; k < G::DPL; ++k) o[g][k] *= alpha;
                m[g] = mn;
                pv[g] = p;
            }
            float* pw = p_s + warp * kTileRows * GS;
            if constexpr (GS % 4 == 0) {
#pragma unroll
                for (int g4 = 0; g4 < GS; g4 += 4)
                    *reinterpret_cast<float4*>(pw + lane * GS + g4) =
                        make_float4(pv[g4], pv[g4 + 1], pv[g4 + 2], pv[g4 + 3]);
            } else {
#pragma unroll
                for (int g = 0; g < GS; ++g) pw[lane * GS + g] = pv[g];
            }
            __syncwarp();

            // ---- PV: lane = head dims [lane*DPL, lane*DPL + DPL)
            auto pv_row = [&](const int rr) {
                float pr_[GS];
                if constexpr (GS % 4 == 0) {
#pragma unroll
                    for (int g4 = 0; g4 < GS; g4 += 4) {
                        const float4 t4 = *reinterpret_cast<const float4*>(pw + rr * GS + g4);
                        pr_[g4] = t4.x;
                        pr_[g4 + 1] = t4.y;
                        pr_[g4 + 2] = t4.z;
                        pr_[g4 + 3] = t4.w;
                    }
                } else {
#pragma unroll
                    for (int g = 0; g < GS; ++g) pr_[g] = pw[rr * GS + g];
                }
                float vv[G::DPL];
                if constexpr (G::LANEB >= 16) {
#pragma unroll
                    for (int q16 = 0; q16 < G::LANEB / 16; ++q16) {
                        const uint4 raw = *reinterpret_cast<const uint4*>(
                            Vt + tile_off<RW, DT>(rr, lane * G::LANEB + q16 * 16));
                        unpack16<DT>(raw, vv + q16 * G::EPC);
                    }
                } else if constexpr (G::LANEB == 8) {
                    const uint2 raw =
                        *reinterpret_cast<const uint2*>(Vt + tile_off<RW, DT>(rr, lane * 8));
                    if constexpr (DT == DT_F32) {
                        vv[0] = __uint_as_float(raw.x);
                        vv[1] = __uint_as_float(raw.y);
                    } else {
                        const uint4 r4 = make_uint4(raw.x, raw.y, 0u, 0u);
                        float tmp[8];
                        unpack16<DT>(r4, tmp);
#pragma unroll
                        for (int k = 0; k < G::DPL; ++k) vv[k] = tmp[k];
                    }
                } else if constexpr (G::LANEB == 4) {
                    const uint32_t raw =
                        *reinterpret_cast<const uint32_t*>(Vt + tile_off<RW, DT>(rr, lane * 4));
                    if constexpr (DT == DT_F32) {
                        vv[0] = __uint_as_float(raw);
                    } else if constexpr (DT == DT_BF16) {
                        vv[0] = __uint_as_float(raw << 16);
                        vv[1] = __uint_as_float(raw & 0xFFFF0000u);
                    } else {
                        vv[0] = f16_bits_to_f32(raw & 0xFFFFu);
                        vv[1] = f16_bits_to_f32(raw >> 16);
                    }
                } else {  // 2 bytes: one 16-bit element
                    const uint32_t raw =
                        *reinterpret_cast<const uint16_t*>(Vt + tile_off<RW, DT>(rr, lane * 2));
                    vv[0] = DT == DT_BF16 ? bf16_bits_to_f32(raw) : f16_bits_to_f32(raw);
                }
#pragma unroll
                for (int g = 0; g < GS; ++g) {
                    if constexpr (G::DPL % 2 == 0) {
#pragma unroll
                        for (int k = 0; k < G::DPL; k += 2)
                            fma_x2(o[g][k], o[g][k + 1], pr_[g], pr_[g], vv[k], vv[k + 1]);
                    } else {
#pragma unroll
                        for (int k = 0; k < G::DPL; ++k) o[g][k] = __fmaf_rn(pr_[g], vv[k], o[g][k]);
                    }
                }
            
            };
            if (nvalid == kTileRows) {
#pragma unroll
                for (int rr = 0; rr < kTileRows; ++rr) pv_row(rr);
            } else {
#pragma unroll 2
                for (int rr = 0; rr < nvalid; ++rr) pv_row(rr);
            }
            }  // CUDA-core tile
            __syncwarp();
            if (lane == 0) mbar_arrive(bars + 8 * (NS + my_stage));
            my_k += streams;
            my_stage += streams;
            if (my_stage >= NS) {
                my_stage -= NS;
                my_phase ^= 1u;
            }
        }
        tile_base = tile_end;

        // ---- merge the four warps' states for this piece
        if constexpr (kMma) {
            mw.finish(o_s, ml_s, warp, lane);
        } else {
#pragma unroll
            for (int g = 0; g < GS; ++g) l[g] = warp_sum(l[g]);
            if (lane == 0) {
#pragma unroll
                for (int g = 0; g < GS; ++g) {
                    ml_s[(warp * GS + g) * 2] = m[g];
                    ml_s[(warp * GS + g) * 2 + 1] = l[g];
                }
            }
#pragma unroll
            for (int g = 0; g < GS; ++g)
#pragma unroll
                for (int k = 0; k < G::DPL; ++k)
                    o_s[(warp * GS + g) * HD + lane * G::DPL + k] = o[g][k];
        }
        named_bar_sync(1, kConsumerThreads);
        // every use of the piece's raw k and v precedes the barrier just passed
        if (slot_kv && ctid == 0) mbar_arrive(qempty + 8 * qs_piece);

        const bool whole = it.r == 0 && it.n == pr.len;
        const long long seg = static_cast<long long>(it.pi) * a.n_kv + kvh;
        const long long slot = c + seg;
        const int ncol = a.G * (blocked ? pr.nq : 1);  // (token, head) columns
        for (int idx = ctid; idx < ncol * HD; idx += kConsumerThreads) {
            const int g = idx / HD, d = idx % HD;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, ml_s[(w * GS + g) * 2]);
            float Lsum = 0.0f, O = 0.0f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
                const float mw = ml_s[(w * GS + g) * 2];
                const float f = mw == -INFINITY ? 0.0f : ex2_approx((mw - M) * kLog2e);
                Lsum += ml_s[(w * GS + g) * 2 + 1] * f;
                O += o_s[(w * GS + g) * HD + d] * f;
            }
            if (whole) {
                const int j = g / a.G, h = g - j * a.G;
                emit_final<HD>(a, pr.io + j * pr.io_step, kvh * a.G + h, d, M, Lsum, O);
            } else if (JX_CHECKED(a, (slot + 1) * GS * (HD + 2) <= a.scratch_floats, 60, slot, seg, 0)) {
                float* dst = a.scratch + (slot * GS + g) * (HD + 2);
                dst[d] = O;
                if (d == 0) {
                    dst[HD] = M;
                    dst[HD + 1] = Lsum;
                }
            }
        }
        if (!whole) {
            // counted in after the CTA's last piece (at most the first and the
            // last piece of a slice are not whole segments)
            if (n_split < 2) {
                const bool early = it.x < b1;  // more pieces follow in this CTA
                if (ctid == 0) {
                    SplitRec& r = recs[n_split];
                    r.seg = seg;
                    r.seg_start = it.seg_start;
                    r.len = pr.len;
                    r.io = pr.io;
                    r.kvh = kvh;
                    r.early = early ? 1 : 0;
                    r.nq = blocked ? pr.nq : 1;
                    r.io_step = pr.io_step;
                    r.c_first = owner.x;
                    r.c_last = owner.y;
                }
                if (early) pending_seg = seg;  // counted in after the next piece's first barrier
                ++n_split;
            } else {
                (void)JX_CHECKED(a, false, 62, n_split, seg, 0);
            }
        }
    }
    if (n_split > 0) {
        // Release: every writer of a partial reaches the barrier, then one
        // thread counts the CTA's last piece in with an acquire-release atomic
        // (the pattern of a grid-wide barrier); an early count-in that turned
        // out last gets an acquire fence.  The last CTA of a segment merges it.
        named_bar_sync(1, kConsumerThreads);
        if (ctid == 0) {
            bool fence = false;
            for (int k = 0; k < n_split; ++k) {
                const SplitRec& r = recs[k];
                const long long c_first = r.c_first, c_last = r.c_last;
                int last = 0;
                if (JX_CHECKED(a, r.seg >= 0 && r.seg < a.n_segments &&
                                      c_last + r.seg < P + a.n_segments && c_first >= 0 &&
                                      (c_last + r.seg + 1) * GS * (HD + 2) <= a.scratch_floats,
                               61, r.seg, c_first, c_last)) {
                    const int prev =
                        r.early ? early_prev : atomic_add_acq_rel_gpu(a.counters + r.seg, 1);
                    last = prev == static_cast<int>(c_last - c_first) ? 1 : 0;
                    if (last) {
                        a.counters[r.seg] = 0;  // every piece arrived: ready for the next step
                        fence = fence || r.early;
                    }
                }
                misc[2 + k] = last;
            }
            if (fence) fence_acq_rel_gpu();
        }
        named_bar_sync(1, kConsumerThreads);
        for (int k = 0; k < n_split; ++k) {
            if (!misc[2 + k]) continue;  // the same for every consumer thread
            const SplitRec r = recs[k];
            merge_split<HD, GS>(a, r, r.c_first, r.c_last, ctid);
        }
    }
    (void)JX_CHECKED(a, it.bad == 0, 45 + it.bad, it.x, it.i, b1);
}

}  // namespace jx
