"""ctypes binding of include/jx_attn.h (libjxattn.so).

The structures below mirror the header field for field.  Loading fails loudly
when the library is missing and cannot be built: there is no CPU path.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

from . import build as _build

JX_OK = 0
JX_ERR_INVALID = -1
JX_ERR_CUDA = -2
JX_ERR_NOMEM = -3
JX_ERR_UNSUPPORTED = -4
JX_ERR_RANGE = -5
JX_ERR_DEVICE = -6
JX_ERR_TIMEOUT = -7
JX_ERR_COMM = -8

JX_F32, JX_BF16, JX_F16_TRUNC = 0, 1, 2

# symbols include/jx_attn.h declares (checked by the tests)
EXPORTS = (
    "jx_kv_create", "jx_kv_destroy", "jx_kv_clear", "jx_kv_rollback", "jx_kv_compact",
    "jx_kv_get_seq_pos", "jx_kv_set_seq_pos", "jx_kv_get_desc", "jx_kv_copy_rows",
    "jx_kv_layer_ptr", "jx_attn_step", "jx_attn_step_partial", "jx_lse_merge",
    "jx_kv_check_device_error", "jx_kv_set_option", "jx_kv_last_launch_count",
    "jx_kv_fill_normal", "jx_fill_normal_f32", "jx_last_error_string", "jx_version",
    "jx_attn_step_noalloc", "jx_attn_step_sharded", "jx_kv_last_step_ms", "jx_attn_prefill",
    "jx_noalloc_check_device_error", "jx_noalloc_set_option",
)


class JxError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"jx error {code}: {msg}")
        self.code = code


class KvDesc(C.Structure):
    _fields_ = [("n_seqs", C.c_uint32), ("n_layers", C.c_uint32), ("capacity", C.c_uint32),
                ("row_stride", C.c_uint32), ("dtype", C.c_int32), ("device", C.c_int32),
                ("pos_base", C.c_uint32)]


class LayerDesc(C.Structure):
    _fields_ = [("head_dim", C.c_uint32), ("rope_dim", C.c_uint32),
                ("rope_freq_base", C.c_float), ("kv_source_layer", C.c_uint32),
                ("is_swa", C.c_int32), ("shares_kv", C.c_int32),
                ("rope_freqs", C.POINTER(C.c_float))]


class StepArgs(C.Structure):
    _fields_ = [("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32), ("n_seqs", C.c_uint32),
                ("seq_ids", C.POINTER(C.c_int32)), ("pos", C.POINTER(C.c_int32)),
                ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("out", C.c_void_p),
                ("q_stride", C.c_uint32), ("kv_stride", C.c_uint32), ("scale", C.c_float),
                ("softcap", C.c_float), ("sliding_window", C.c_uint32),
                ("yarn_scale", C.c_float), ("rope_neox", C.c_int32)]


_lock = threading.Lock()
_lib: C.CDLL | None = None


def _declare(lib: C.CDLL) -> None:
    vp, u32, u64, i32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int32
    sig = {
        "jx_kv_create": [C.POINTER(KvDesc), C.POINTER(vp)],
        "jx_kv_destroy": [vp],
        "jx_kv_clear": [vp, u32, vp],
        "jx_kv_rollback": [vp, u32, u32],
        "jx_kv_compact": [vp, u32, u32, vp],
        "jx_kv_get_seq_pos": [vp, u32, C.POINTER(u32)],
        "jx_kv_set_seq_pos": [vp, u32, u32],
        "jx_kv_get_desc": [vp, C.POINTER(KvDesc)],
        "jx_kv_copy_rows": [vp, u32, u32, C.c_int, u32, u32, vp, C.c_int, vp],
        "jx_kv_layer_ptr": [vp, u32, u32, C.c_int, C.POINTER(vp)],
        "jx_attn_step": [vp, C.POINTER(LayerDesc), u32, C.POINTER(StepArgs), vp],
        "jx_attn_step_partial": [vp, C.POINTER(LayerDesc), u32, C.POINTER(StepArgs), vp, vp],
        "jx_lse_merge": [vp, u32, u64, u32, u32, u32, vp, u32, vp],
        "jx_kv_check_device_error": [vp, C.POINTER(C.c_int), vp],
        "jx_kv_set_option": [vp, C.c_char_p, C.c_int],
        "jx_kv_last_launch_count": [vp, C.POINTER(C.c_int)],
        "jx_kv_fill_normal": [vp, C.POINTER(u32), u64, vp],
        "jx_fill_normal_f32": [vp, u64, u64, u32, vp],
        "jx_attn_step_noalloc": [C.POINTER(KvDesc), vp, vp, C.POINTER(LayerDesc), u32,
                                 C.POINTER(StepArgs), vp],
        "jx_attn_step_sharded": [vp, C.POINTER(LayerDesc), u32, C.POINTER(StepArgs), vp, u32, vp],
        "jx_kv_last_step_ms": [vp, C.POINTER(C.c_float)],
        "jx_attn_prefill": [vp, C.POINTER(LayerDesc), u32, C.POINTER(StepArgs), vp],
        "jx_noalloc_check_device_error": [C.c_int, C.POINTER(C.c_int), vp],
        "jx_noalloc_set_option": [C.c_char_p, C.c_int],
    }
    for name, args in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = C.c_int
    lib.jx_last_error_string.restype = C.c_char_p
    lib.jx_last_error_string.argtypes = []
    lib.jx_version.restype = C.c_char_p
    lib.jx_version.argtypes = []


def checked_build_requested() -> bool:
    """JXAI_B200_CHECKED=1 selects the diagnostic build with device-side index checks."""
    return os.environ.get("JXAI_B200_CHECKED", "0") not in ("", "0")


def lib_path() -> str:
    return _build.LIB_CHECKED if checked_build_requested() else _build.LIB


def load(build_if_missing: bool = True) -> C.CDLL:
    """The loaded libjxattn.so (built in-tree on first use if nvcc is present)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        checked = checked_build_requested()
        path = lib_path()
        if not os.path.exists(path) or not _build.up_to_date(checked):
            if not build_if_missing:
                raise FileNotFoundError(f"{path} is not built")
            _build.build(checked=checked)
        lib = C.CDLL(path)
        _declare(lib)
        _lib = lib
        return lib


def check(rc: int) -> None:
    if rc != JX_OK:
        msg = load().jx_last_error_string()
        raise JxError(rc, msg.decode() if msg else "")
