"""jxai_b200 -- B200-native (sm_100a) replacement for jxai's per-token attention step.

The path: RoPE on q/k, append of k/v into the per-layer KV cache, and
grouped-query decode attention over every cached position
(jacxishipping/jxai src/transformer.cpp:2497-2567), run as one fused CUDA
launch per step from libjxattn.so (C ABI: include/jx_attn.h).
"""
from ._lib import (JX_BF16, JX_F16_TRUNC, JX_F32, JxError, EXPORTS, load as load_library,
                   lib_path)
from .attention import (KVCache, KVCacheSlot, Layer, StepPlan, attn_prefill, attn_step,
                        attn_step_partial, attn_step_sharded, fill_normal, lse_merge)

__all__ = [
    "JX_F32", "JX_BF16", "JX_F16_TRUNC", "JxError", "EXPORTS", "load_library", "lib_path",
    "KVCache", "KVCacheSlot", "Layer", "StepPlan", "attn_step", "attn_step_partial", "lse_merge",
    "attn_step_sharded", "attn_prefill", "fill_normal",
]
