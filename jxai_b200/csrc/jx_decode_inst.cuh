// jx_decode_inst.cuh -- instantiates the decode kernel for one cache element
// type (JX_INST_DT) over head_dim {32, 64, 128, 256} x group {1, 2, 4, 8}
// (plus, for 16-bit caches, head_dim {32, 64} with two kv heads per tile row)
// and provides that type's dispatcher.  Included once by each jx_decode_<dt>.cu so
// the three element types compile in parallel.
#include "jx_decode.cuh"

#ifndef JX_INST_DT
#error "define JX_INST_DT before including"
#endif

namespace jx {

namespace {

template <int HD, int GP, int KP>
struct Entry {
    static constexpr int DT = JX_INST_DT;
    static int smem(int stages) { return SmemLayout<HD, GP, DT, KP>::total(stages); }
    // Kernel attributes: the dynamic shared memory it asks for, and the largest
    // shared-memory carveout so that two CTAs of ~80-110 KB fit on one SM
    // (the default carveout choice can leave room for only one).
    static cudaError_t set_attributes(int bytes) {
        cudaError_t e = cudaFuncSetAttribute(decode_kernel<HD, GP, DT, KP>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e != cudaSuccess) return e;
        return cudaFuncSetAttribute(decode_kernel<HD, GP, DT, KP>,
                                    cudaFuncAttributePreferredSharedMemoryCarveout,
                                    cudaSharedmemCarveoutMaxShared);
    }
    static int occupancy(int stages) {
        const int bytes = smem(stages);
        if (set_attributes(bytes) != cudaSuccess) return 0;
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_kernel<HD, GP, DT, KP>, kThreads,
                                                          bytes) != cudaSuccess)
            return 0;
        return n;
    }
    static cudaError_t launch(const DecodeLaunch& L) {
        const int bytes = smem(L.stages);
        // the attribute is per device and per kernel: set it once per (device, size)
        static int set_bytes[64] = {0};
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= 64 || set_bytes[dev] < bytes) {
            e = set_attributes(bytes);
            if (e != cudaSuccess) return e;
            if (dev >= 0 && dev < 64) set_bytes[dev] = bytes;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(L.grid));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = static_cast<size_t>(bytes);
        cfg.stream = L.stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = L.pdl ? 1 : 0;
        return cudaLaunchKernelEx(&cfg, decode_kernel<HD, GP, DT, KP>, *L.tmK, *L.tmV, L.args);
    }
};

template <int HD, int KP>
bool pick_gp(int gp, int op, int stages, const DecodeLaunch* L, int* out_i, cudaError_t* out_e) {
    auto run = [&](auto entry) {
        using E = decltype(entry);
        if (op == 0) *out_i = E::smem(stages);
        else if (op == 1) *out_i = E::occupancy(stages);
        else *out_e = E::launch(*L);
    };
    switch (gp) {
        case 1: run(Entry<HD, 1, KP>{}); return true;
        case 2: run(Entry<HD, 2, KP>{}); return true;
        case 4: run(Entry<HD, 4, KP>{}); return true;
        case 8: run(Entry<HD, 8, KP>{}); return true;
        default: return false;
    }
}

bool dispatch(int head_dim, int gp, int kp, int op, int stages, const DecodeLaunch* L,
              int* out_i, cudaError_t* out_e) {
    if (kp == 2) {
        if constexpr (JX_INST_DT == DT_F32) {
            return false;
        } else {
            switch (head_dim) {
                case 32: return pick_gp<32, 2>(gp, op, stages, L, out_i, out_e);
                case 64: return pick_gp<64, 2>(gp, op, stages, L, out_i, out_e);
                default: return false;
            }
        }
    }
    if (kp != 1) return false;
    switch (head_dim) {
        case 32: return pick_gp<32, 1>(gp, op, stages, L, out_i, out_e);
        case 64: return pick_gp<64, 1>(gp, op, stages, L, out_i, out_e);
        case 128: return pick_gp<128, 1>(gp, op, stages, L, out_i, out_e);
        case 256: return pick_gp<256, 1>(gp, op, stages, L, out_i, out_e);
        default: return false;
    }
}

}  // namespace

#define JX_CAT2(a, b) a##b
#define JX_CAT(a, b) JX_CAT2(a, b)

bool JX_CAT(decode_dispatch_dt, JX_INST_DT)(int head_dim, int gp, int kp, int op, int stages,
                                           const DecodeLaunch* L, int* out_i, cudaError_t* out_e) {
    return dispatch(head_dim, gp, kp, op, stages, L, out_i, out_e);
}

}  // namespace jx
