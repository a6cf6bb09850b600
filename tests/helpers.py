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


_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(x):
    x = x + np.uint64(0x9E3779B97F4A7C15)
    x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return x ^ (x >> np.uint64(31))


def normal_at(seed: int, stream_id: int, idx) -> np.ndarray:
    """Host restatement of the library's seeded fill (jx_lib.cu normal_at):
    splitmix64 of (seed, stream, index), then Box-Muller.  The device uses
    logf / cospif in float32, this float64 numpy, so values agree to a few
    float32 ulps -- enough to rebuild the unrounded values behind a bf16 cache
    for the 2e-2 bar, not for bit-level checks."""
    with np.errstate(over="ignore"):
        idx = np.asarray(idx, dtype=np.uint64)
        inner = _splitmix64((np.uint64(stream_id) << np.uint64(56)) ^ idx)
        h = _splitmix64(np.uint64(seed) ^ inner)
    u1 = ((h >> np.uint64(40)).astype(np.float64) + 1.0) / 16777216.0
    u2 = (h & np.uint64(0xFFFFFF)).astype(np.float64) / 16777216.0
    return (np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)).astype(np.float32)
