"""Shared test helpers: seeded host inputs and the oracle side of a step."""
from __future__ import annotations

import numpy as np

from oracle.oracle import BF16, F16T, F32, Oracle


def random_cache(rng, shape, dtype):
    """Seeded cache contents: float32, or uint16 bit patterns of valid bf16/fp16 values."""
    x = rng.standard_normal(shape).astype(np.float32)
    if dtype == F32:
        return x
    if dtype == BF16:
        return (x.view(np.uint32) >> 16).astype(np.uint16)
    return x.astype(np.float16).view(np.uint16)


def np_dtype(dtype):
    return np.float32 if dtype == F32 else np.uint16


def layer_dicts(layers):
    return [dict(rope_dim=L.rope_dim, rope_base=L.rope_base, is_swa=int(L.is_swa),
                 shares_kv=int(L.shares_kv), kv_source_layer=L.kv_source_layer) for L in layers]


def oracle_step(kc, vc, dtype, pos, layers, q, k, v, n_heads, n_kv, head_dim, scale, softcap=0.0,
                window=0, yarn=1.0, neox=True, rope_freqs=None, kind="port"):
    """Runs the CPU oracle in place on host caches; returns out."""
    return Oracle(kind).step(kc, vc, dtype, pos, layer_dicts(layers), q, k, v, n_heads, n_kv,
                             head_dim, scale, softcap, window, yarn, neox, rope_freqs)
