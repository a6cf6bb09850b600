// Decode-kernel instantiations for one cache element type (see jx_decode_inst.cuh).
#define JX_INST_DT 0
#include "jx_decode_inst.cuh"
