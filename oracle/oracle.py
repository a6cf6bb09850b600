"""TEST INFRASTRUCTURE ONLY: ctypes front end to the CPU parity checkers.

Two shared objects sit behind this module:

* ``oracle/libjxoracle.so`` -- the plain-C restatement of jxai's attention step
  (``oracle/jx_oracle.c``), always buildable with gcc;
* ``oracle/_ref/libjxref.so`` -- the reference's own sources compiled in place
  with the reference's flags plus ``oracle/ref_block.cpp``; present only where
  the reference tree was available when ``make -C oracle`` ran.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm import this module.  The product library (``jxai_b200``) never
does; it has no CPU path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "libjxoracle.so")
REF_SO = os.path.join(HERE, "_ref", "libjxref.so")

F32, BF16, F16T = 0, 1, 2
_NP_DTYPE = {F32: np.float32, BF16: np.uint16, F16T: np.uint16}

_lock = threading.Lock()
_libs: dict[str, C.CDLL] = {}


def build(ref: str | None = None) -> None:
    """Run oracle/Makefile (restatement always; reference build when REF exists)."""
    cmd = ["make", "-s", "-C", HERE]
    if ref:
        cmd.append(f"REF={ref}")
    subprocess.run(cmd, check=True)


def _fp(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


def _declare(lib: C.CDLL, prefix: str) -> None:
    u16, u32, i32, f32, vp, i64 = C.c_uint16, C.c_uint32, C.c_int32, C.c_float, C.c_void_p, C.c_int64
    getattr(lib, prefix + "fp16_to_fp32").restype = f32
    getattr(lib, prefix + "fp16_to_fp32").argtypes = [u16]
    getattr(lib, prefix + "fp32_to_fp16").restype = u16
    getattr(lib, prefix + "fp32_to_fp16").argtypes = [f32]
    getattr(lib, prefix + "bf16_to_fp32").restype = f32
    getattr(lib, prefix + "bf16_to_fp32").argtypes = [u16]
    getattr(lib, prefix + "fp32_to_bf16").restype = u16
    getattr(lib, prefix + "fp32_to_bf16").argtypes = [f32]
    fn = getattr(lib, prefix + "apply_rope")
    fn.restype = None
    fn.argtypes = [vp, vp, u32, u32, u32, u32, u32, f32, f32, C.c_int, vp]
    fn = getattr(lib, prefix + "softmax")
    fn.restype = None
    fn.argtypes = [vp, i64]
    fn = getattr(lib, prefix + "append_attend")
    fn.restype = C.c_int
    fn.argtypes = [vp, vp, C.c_int, u32, vp, vp, vp, vp, u32, u32, u32, u32, u32, f32, f32,
                   C.c_int, vp, C.c_int, C.c_int, u32, f32, f32]
    fn = getattr(lib, prefix + "step")
    fn.restype = C.c_int
    fn.argtypes = [vp, vp, C.c_int, u32, u32, u32, u32, vp, u32, vp, vp, vp, vp, vp, vp, vp, vp,
                   vp, u32, u32, u32, u32, u32, f32, f32, u32, f32, C.c_int, vp]
    getattr(lib, prefix + "max_threads").restype = C.c_int


def _load(kind: str) -> C.CDLL:
    with _lock:
        if kind in _libs:
            return _libs[kind]
        path = PORT_SO if kind == "port" else REF_SO
        if kind == "port" and not os.path.exists(path):
            build()
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built (needs the reference tree)")
        lib = C.CDLL(path)
        prefix = "jxo_" if kind == "port" else "jxr_"
        _declare(lib, prefix)
        if kind == "port":
            lib.jxo_rope_cos_sin.restype = None
            lib.jxo_rope_cos_sin.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, C.c_float,
                                             C.c_float, C.c_int, C.c_void_p, C.c_void_p]
            lib.jxo_compact.restype = C.c_uint32
            lib.jxo_compact.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_uint32, C.c_uint32,
                                        C.c_uint32, C.c_uint32, C.c_uint32]
        else:
            lib.jxr_compact_u16.restype = C.c_uint32
            lib.jxr_compact_u16.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32,
                                            C.c_uint32, C.c_uint32, C.c_uint32]
            lib.jxr_rollback.restype = C.c_uint32
            lib.jxr_rollback.argtypes = [C.c_uint32, C.c_uint32]
        _libs[kind] = lib
        return lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


class Oracle:
    """One of the two CPU implementations behind a common numpy interface."""

    def __init__(self, kind: str = "port"):
        assert kind in ("port", "ref")
        self.kind = kind
        self.lib = _load(kind)
        self.p = "jxo_" if kind == "port" else "jxr_"

    def _f(self, name):
        return getattr(self.lib, self.p + name)

    # ---- scalar conversions (src/quant.cpp:876-939) ----
    def fp32_to_fp16(self, x: float) -> int:
        return int(self._f("fp32_to_fp16")(float(x)))

    def fp16_to_fp32(self, h: int) -> float:
        return float(self._f("fp16_to_fp32")(int(h)))

    def fp32_to_bf16(self, x: float) -> int:
        return int(self._f("fp32_to_bf16")(float(x)))

    def bf16_to_fp32(self, h: int) -> float:
        return float(self._f("bf16_to_fp32")(int(h)))

    def convert_array(self, x: np.ndarray, dtype: int) -> np.ndarray:
        """fp32 array -> stored representation (float32 or uint16 bit patterns)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if dtype == F32:
            return x.copy()
        f = self._f("fp32_to_bf16" if dtype == BF16 else "fp32_to_fp16")
        return np.array([f(float(v)) for v in x.ravel()], dtype=np.uint16).reshape(x.shape)

    def max_threads(self) -> int:
        return int(self._f("max_threads")())

    # ---- RoPE (src/transformer.cpp:76-138) ----
    def apply_rope(self, q, k, n_heads, n_kv_heads, head_dim, rope_dim, pos, base, yarn_scale=1.0,
                   neox=True, rope_freqs=None):
        q = np.ascontiguousarray(q, dtype=np.float32).copy()
        k = None if k is None else np.ascontiguousarray(k, dtype=np.float32).copy()
        rf = None if rope_freqs is None else np.ascontiguousarray(rope_freqs, dtype=np.float32)
        self._f("apply_rope")(_fp(q), _fp(k), n_heads, n_kv_heads, head_dim, rope_dim, pos, base,
                              yarn_scale, int(neox), _fp(rf))
        return q, k

    def softmax(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32).copy()
        self._f("softmax")(_fp(x), x.size)
        return x

    # ---- one decode step over [seq][layer] (transformer.cpp:2497-2566) ----
    def step(self, k_cache, v_cache, dtype, pos, layers, q, k, v, n_heads, n_kv_heads, head_dim,
             scale, softcap=0.0, sliding_window=0, yarn_scale=1.0, neox=True, rope_freqs=None):
        """Run the attention step in place on host caches.

        k_cache/v_cache: [n_seqs][n_cache_layers][capacity][row_stride] (float32 or uint16)
        q: [n_seqs][n_layers][q_stride] float32;  k, v: [n_seqs][n_layers][kv_stride]
        layers: list of dicts with rope_dim, rope_base, is_swa, shares_kv, kv_source_layer
        Returns out [n_seqs][n_layers][q_stride] float32.
        """
        assert k_cache.flags.c_contiguous and v_cache.flags.c_contiguous
        assert k_cache.dtype == _NP_DTYPE[dtype]
        n_seqs, n_cache_layers, capacity, row_stride = k_cache.shape
        n_layers = len(layers)
        q = np.ascontiguousarray(q, dtype=np.float32)
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        out = np.zeros_like(q)
        pos_a = np.ascontiguousarray(pos, dtype=np.int32)
        rd = np.array([L["rope_dim"] for L in layers], dtype=np.uint32)
        rb = np.array([L["rope_base"] for L in layers], dtype=np.float32)
        sw = np.array([int(L.get("is_swa", 0)) for L in layers], dtype=np.int32)
        sh = np.array([int(L.get("shares_kv", 0)) for L in layers], dtype=np.int32)
        src = np.array([L.get("kv_source_layer", i) for i, L in enumerate(layers)], dtype=np.uint32)
        rf = None if rope_freqs is None else np.ascontiguousarray(rope_freqs, dtype=np.float32)
        rc = self._f("step")(_fp(k_cache), _fp(v_cache), dtype, capacity, row_stride,
                             n_cache_layers, n_seqs, _fp(pos_a), n_layers, _fp(rd), _fp(rb),
                             _fp(sw), _fp(sh), _fp(src), _fp(q), _fp(k), _fp(v), _fp(out),
                             q.shape[-1], k.shape[-1], n_heads, n_kv_heads, head_dim, scale,
                             softcap, sliding_window, yarn_scale, int(neox), _fp(rf))
        if rc != 0:
            raise RuntimeError(f"oracle step failed: {rc}")
        return out

    # ---- KVCacheSlot::compact (transformer.cpp:41-66) on one sequence ----
    def compact(self, k_seq, v_seq, dtype, seq_pos, keep_recent):
        n_layers, capacity, row_stride = k_seq.shape
        if self.kind == "port":
            return int(self.lib.jxo_compact(_fp(k_seq), _fp(v_seq), dtype, n_layers, capacity,
                                            row_stride, seq_pos, keep_recent))
        assert k_seq.dtype == np.uint16, "the reference cache holds uint16 values"
        return int(self.lib.jxr_compact_u16(_fp(k_seq), _fp(v_seq), n_layers, capacity,
                                            row_stride, seq_pos, keep_recent))


def rope_cos_sin(head_dim, rope_dim, pos, base, yarn_scale=1.0, neox=True, rope_freqs=None):
    """(cos, sin) pairs as apply_rope computes them (port)."""
    lib = _load("port")
    rdim = min(head_dim, rope_dim)
    cs = np.zeros(rdim + 2, dtype=np.float32)
    rf = None if rope_freqs is None else np.ascontiguousarray(rope_freqs, dtype=np.float32)
    lib.jxo_rope_cos_sin(head_dim, rope_dim, pos, base, yarn_scale, int(neox), _fp(rf), _fp(cs))
    return cs[:rdim].reshape(-1, 2)
