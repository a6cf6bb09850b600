"""Python host side of the B200 decode-attention path.

Mirrors the reference's interface for this path:

* ``KVCache`` owns the device cache of ``n_seqs`` slots (the storage of
  ``KVCacheSlot``, include/transformer.h:115-131);
* ``KVCacheSlot`` is a per-slot view with the reference's methods
  (``init/clear/rollback/compact``, ``seq_pos``, ``token_history``;
  src/transformer.cpp:13-66);
* ``attn_step`` is the per-token attention block of forward_token
  (src/transformer.cpp:2497-2567) for any number of slots and layers.

All compute goes through libjxattn.so (include/jx_attn.h); tensors are torch
CUDA tensors passed by address.  There is no CPU path: without the library or
a B200 every call raises ``JxError``.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from ._lib import (JX_BF16, JX_F16_TRUNC, JX_F32, JxError, KvDesc, LayerDesc, StepArgs, check,
                   load)

DTYPES = {"f32": JX_F32, "bf16": JX_BF16, "f16": JX_F16_TRUNC, "f16_trunc": JX_F16_TRUNC,
          JX_F32: JX_F32, JX_BF16: JX_BF16, JX_F16_TRUNC: JX_F16_TRUNC}
ELEM_SIZE = {JX_F32: 4, JX_BF16: 2, JX_F16_TRUNC: 2}


def _stream_ptr(stream) -> Optional[int]:
    if stream is not None:
        return int(getattr(stream, "cuda_stream", stream))
    try:
        import torch
        if torch.cuda.is_available():
            return int(torch.cuda.current_stream().cuda_stream)
    except ImportError:
        pass
    return None


def _dev_ptr(t, name: str, min_elems: int, host_ok: bool = False) -> int:
    """Address of a contiguous float32 tensor on the device -- or, where
    host_ok, in pinned host memory (the kernel then reads / writes it over
    PCIe, with no separate copy)."""
    import torch
    if not isinstance(t, torch.Tensor):
        raise JxError(-1, f"{name} must be a tensor")
    if not t.is_cuda and not (host_ok and t.device.type == "cpu" and t.is_pinned()):
        raise JxError(-1, f"{name} must be a CUDA tensor" + (" or pinned host tensor" if host_ok else ""))
    if t.dtype != torch.float32 or not t.is_contiguous():
        raise JxError(-1, f"{name} must be a contiguous float32 tensor")
    if t.numel() < min_elems:
        raise JxError(-1, f"{name} holds {t.numel()} floats, needs {min_elems}")
    return t.data_ptr()


@dataclass
class Layer:
    """Attention fields of one LayerDenseWeights (include/transformer.h:50-58)."""
    head_dim: int
    rope_dim: int
    rope_base: float
    kv_source_layer: int
    is_swa: bool = False
    shares_kv: bool = False
    rope_freqs: Optional[np.ndarray] = None


class KVCache:
    """Device KV cache: K and V each [n_seqs][n_layers][capacity][row_stride]."""

    def __init__(self, n_seqs: int, n_layers: int, capacity: int, row_stride: int,
                 dtype="f32", device: int = 0, pos_base: int = 0):
        self.lib = load()
        self.dtype = DTYPES[dtype]
        self.n_seqs, self.n_layers = n_seqs, n_layers
        self.capacity, self.row_stride = capacity, row_stride
        self.device, self.pos_base = device, pos_base
        d = KvDesc(n_seqs, n_layers, capacity, row_stride, self.dtype, device, pos_base)
        h = C.c_void_p()
        check(self.lib.jx_kv_create(C.byref(d), C.byref(h)))
        self.handle = h

    # lifetime ---------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.jx_kv_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def elem_size(self) -> int:
        return ELEM_SIZE[self.dtype]

    @property
    def nbytes(self) -> int:
        return 2 * self.n_seqs * self.n_layers * self.capacity * self.row_stride * self.elem_size

    # KVCacheSlot operations (src/transformer.cpp:25-66) --------------------
    def clear(self, seq: int, stream=None) -> None:
        check(self.lib.jx_kv_clear(self.handle, seq, _stream_ptr(stream)))

    def rollback(self, seq: int, new_seq_pos: int) -> None:
        check(self.lib.jx_kv_rollback(self.handle, seq, new_seq_pos))

    def compact(self, seq: int, keep_recent: int = 128, stream=None) -> None:
        check(self.lib.jx_kv_compact(self.handle, seq, keep_recent, _stream_ptr(stream)))

    def seq_pos(self, seq: int) -> int:
        v = C.c_uint32()
        check(self.lib.jx_kv_get_seq_pos(self.handle, seq, C.byref(v)))
        return v.value

    def set_seq_pos(self, seq: int, pos: int) -> None:
        check(self.lib.jx_kv_set_seq_pos(self.handle, seq, pos))

    # plumbing ------------------------------------------------------------------
    def _np_dtype(self):
        return np.float32 if self.dtype == JX_F32 else np.uint16

    def read_rows(self, seq: int, layer: int, which: int, row0: int, n_rows: int,
                  stream=None) -> np.ndarray:
        """Host copy of rows [row0, row0+n_rows) (float32, or uint16 bit patterns)."""
        out = np.empty((n_rows, self.row_stride), dtype=self._np_dtype())
        st = _stream_ptr(stream)
        check(self.lib.jx_kv_copy_rows(self.handle, seq, layer, which, row0, n_rows,
                                       out.ctypes.data_as(C.c_void_p), 0, st))
        self.synchronize(stream)
        return out

    def write_rows(self, seq: int, layer: int, which: int, row0: int, rows: np.ndarray,
                   stream=None) -> None:
        rows = np.ascontiguousarray(rows, dtype=self._np_dtype())
        assert rows.ndim == 2 and rows.shape[1] == self.row_stride
        st = _stream_ptr(stream)
        check(self.lib.jx_kv_copy_rows(self.handle, seq, layer, which, row0, rows.shape[0],
                                       rows.ctypes.data_as(C.c_void_p), 1, st))
        self.synchronize(stream)

    def layer_ptr(self, seq: int, layer: int, which: int) -> int:
        p = C.c_void_p()
        check(self.lib.jx_kv_layer_ptr(self.handle, seq, layer, which, C.byref(p)))
        return p.value

    def fill_normal(self, rows_per_seq: Sequence[int], seed: int, stream=None) -> None:
        arr = (C.c_uint32 * self.n_seqs)(*[int(r) for r in rows_per_seq])
        check(self.lib.jx_kv_fill_normal(self.handle, arr, C.c_uint64(seed), _stream_ptr(stream)))

    def set_option(self, key: str, value: int) -> None:
        check(self.lib.jx_kv_set_option(self.handle, key.encode(), value))

    def check_device_error(self, stream=None) -> int:
        code = C.c_int()
        rc = self.lib.jx_kv_check_device_error(self.handle, C.byref(code), _stream_ptr(stream))
        if rc not in (0, -6):
            check(rc)
        return code.value

    def last_launch_count(self) -> int:
        n = C.c_int()
        check(self.lib.jx_kv_last_launch_count(self.handle, C.byref(n)))
        return n.value

    def last_step_ms(self) -> float:
        """Device time of the last step (needs set_option("timing", 1)); the
        reference's attention_ms."""
        ms = C.c_float()
        check(self.lib.jx_kv_last_step_ms(self.handle, C.byref(ms)))
        return ms.value

    def synchronize(self, stream=None) -> None:
        try:
            import torch
            if stream is None:
                torch.cuda.current_stream(self.device).synchronize()
            else:
                stream.synchronize()
        except ImportError:
            pass


class KVCacheSlot:
    """One slot of a KVCache with KVCacheSlot's interface (transformer.h:115-131)."""

    def __init__(self, cache: KVCache, slot_id: int):
        self.cache = cache
        self.slot_id = slot_id
        self.token_history: list[int] = []
        self.compactions = 0

    @property
    def seq_pos(self) -> int:
        return self.cache.seq_pos(self.slot_id)

    @seq_pos.setter
    def seq_pos(self, v: int) -> None:
        self.cache.set_seq_pos(self.slot_id, v)

    def init(self, slot_id: int) -> None:  # transformer.cpp:13-23
        self.slot_id = slot_id
        self.compactions = 0
        self.token_history.clear()
        self.cache.clear(slot_id)

    def clear(self) -> None:  # transformer.cpp:25-30
        self.token_history.clear()
        self.cache.clear(self.slot_id)

    def rollback(self, new_seq_pos: int) -> None:  # transformer.cpp:32-39
        self.cache.rollback(self.slot_id, new_seq_pos)
        if len(self.token_history) > new_seq_pos:
            del self.token_history[new_seq_pos:]

    def compact(self, keep_recent: int = 128) -> None:  # transformer.cpp:41-66
        before = self.seq_pos
        self.cache.compact(self.slot_id, keep_recent)
        after = self.seq_pos
        if after != before:
            if len(self.token_history) > after:
                del self.token_history[after:]
            self.compactions += 1

    def pages_allocated(self, block_tokens: int = 16) -> int:  # transformer.h:127-129
        sp = self.seq_pos
        return 0 if sp == 0 else (sp + block_tokens - 1) // block_tokens


def _layer_array(layers: Sequence[Layer]):
    arr = (LayerDesc * len(layers))()
    keep = []
    for i, L in enumerate(layers):
        rf = None
        if L.rope_freqs is not None:
            a = np.ascontiguousarray(L.rope_freqs, dtype=np.float32)
            keep.append(a)
            rf = a.ctypes.data_as(C.POINTER(C.c_float))
        arr[i] = LayerDesc(L.head_dim, L.rope_dim, L.rope_base, L.kv_source_layer,
                           int(bool(L.is_swa)), int(bool(L.shares_kv)), rf)
    return arr, keep


def _step_args(cache, layers, q, k, v, out, pos, n_heads, n_kv_heads, scale, softcap,
               sliding_window, yarn_scale, neox, seq_ids, partial_floats):
    n = len(pos)
    hd = layers[0].head_dim
    q_stride = q.shape[-1]
    kv_stride = k.shape[-1]
    rows = n * len(layers)
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    pos_a = (C.c_int32 * n)(*[int(p) for p in pos])
    sid = None
    if seq_ids is not None:
        sid = (C.c_int32 * n)(*[int(s) for s in seq_ids])
    a = StepArgs()
    a.n_heads, a.n_kv_heads, a.n_seqs = n_heads, n_kv_heads, n
    a.seq_ids = C.cast(sid, C.POINTER(C.c_int32)) if sid is not None else None
    a.pos = C.cast(pos_a, C.POINTER(C.c_int32))
    a.q = _dev_ptr(q, "q", rows * q_stride, host_ok=True)
    a.k = _dev_ptr(k, "k", rows * kv_stride, host_ok=True)
    a.v = _dev_ptr(v, "v", rows * kv_stride, host_ok=True)
    a.out = _dev_ptr(out, "out", rows * q_stride, host_ok=True) if out is not None else None
    a.q_stride, a.kv_stride = q_stride, kv_stride
    a.scale, a.softcap = float(scale), float(softcap)
    a.sliding_window, a.yarn_scale, a.rope_neox = int(sliding_window), float(yarn_scale), int(neox)
    return a, (pos_a, sid)


def attn_step(cache: KVCache, layers: Sequence[Layer], q, k, v, out, pos: Sequence[int],
              n_heads: int, n_kv_heads: int, scale: Optional[float] = None, softcap: float = 0.0,
              sliding_window: int = 0, yarn_scale: float = 1.0, neox: bool = True,
              seq_ids: Optional[Sequence[int]] = None, stream=None) -> None:
    """RoPE + KV append + GQA decode attention for len(pos) slots x len(layers) layers.

    q/out: [n_seqs, n_layers, q_stride] float32 CUDA tensors;
    k/v: [n_seqs, n_layers, kv_stride].  Asynchronous on `stream`.
    """
    arr, keep = _layer_array(layers)
    a, keep2 = _step_args(cache, layers, q, k, v, out, pos, n_heads, n_kv_heads, scale, softcap,
                          sliding_window, yarn_scale, neox, seq_ids, 0)
    check(cache.lib.jx_attn_step(cache.handle, arr, len(layers), C.byref(a), _stream_ptr(stream)))


def attn_prefill(cache: KVCache, layers: Sequence[Layer], q, k, v, out, pos: Sequence[int],
                 n_heads: int, n_kv_heads: int, seq_ids: Optional[Sequence[int]] = None,
                 scale: Optional[float] = None, softcap: float = 0.0, sliding_window: int = 0,
                 yarn_scale: float = 1.0, neox: bool = True, stream=None) -> None:
    """Many tokens per call: row i is a token of sequence seq_ids[i] (default 0)
    at position pos[i]; all rows are appended, then each attends causally.
    q/out: [n_rows, n_layers, q_stride]; k/v: [n_rows, n_layers, kv_stride]."""
    if seq_ids is None:
        seq_ids = [0] * len(pos)
    arr, keep = _layer_array(layers)
    a, keep2 = _step_args(cache, layers, q, k, v, out, pos, n_heads, n_kv_heads, scale, softcap,
                          sliding_window, yarn_scale, neox, seq_ids, 0)
    check(cache.lib.jx_attn_prefill(cache.handle, arr, len(layers), C.byref(a),
                                    _stream_ptr(stream)))


def attn_step_partial(cache: KVCache, layers: Sequence[Layer], q, k, v, partials,
                      pos: Sequence[int], n_heads: int, n_kv_heads: int,
                      scale: Optional[float] = None, softcap: float = 0.0,
                      sliding_window: int = 0, yarn_scale: float = 1.0, neox: bool = True,
                      seq_ids: Optional[Sequence[int]] = None, stream=None) -> None:
    """Shard-local step writing (o, m, l) partials [n_seqs, n_layers, n_heads, head_dim+2]."""
    hd = layers[0].head_dim
    n = len(pos) * len(layers) * n_heads * (hd + 2)
    pp = _dev_ptr(partials, "partials", n)
    arr, keep = _layer_array(layers)
    a, keep2 = _step_args(cache, layers, q, k, v, None, pos, n_heads, n_kv_heads, scale, softcap,
                          sliding_window, yarn_scale, neox, seq_ids, n)
    check(cache.lib.jx_attn_step_partial(cache.handle, arr, len(layers), C.byref(a), pp,
                                         _stream_ptr(stream)))


def attn_step_sharded(cache: KVCache, layers: Sequence[Layer], q, k, v, out, pos: Sequence[int],
                      n_heads: int, n_kv_heads: int, comm, timeout_ms: int = 0,
                      scale: Optional[float] = None, softcap: float = 0.0,
                      sliding_window: int = 0, yarn_scale: float = 1.0, neox: bool = True,
                      seq_ids: Optional[Sequence[int]] = None, stream=None, heartbeat=None,
                      step: int = 0, liveness_timeout_s: float = 5.0) -> None:
    """One context sharded by position over the ranks of an NCCL communicator.

    This rank's cache holds positions [pos_base, pos_base + capacity); the call
    runs the shard's partial step, all-gathers every rank's (o, m, l) over
    `comm` (an ncclComm_t address, e.g. NcclComm.handle) and merges them into
    `out` on every rank.  timeout_ms > 0 also waits for completion and raises
    JxError code -7 when the step does not finish in time (the communicator
    is left to the caller to abort).  With `heartbeat` (a
    jxai_b200.liveness.Heartbeat) every rank first announces `step` and waits
    up to liveness_timeout_s for the others: a rank that left raises JxError
    code -7 here, before anything of the step is queued.
    """
    if heartbeat is not None:
        heartbeat.check(step, liveness_timeout_s)
    arr, keep = _layer_array(layers)
    a, keep2 = _step_args(cache, layers, q, k, v, out, pos, n_heads, n_kv_heads, scale, softcap,
                          sliding_window, yarn_scale, neox, seq_ids, 0)
    check(cache.lib.jx_attn_step_sharded(cache.handle, arr, len(layers), C.byref(a),
                                         C.c_void_p(int(comm)), int(timeout_ms),
                                         _stream_ptr(stream)))


class StepPlan:
    """One attn_step (or attn_step_partial, or attn_step_sharded) call with its
    C arguments built once.

    For callers that repeat the step on the same buffers (a decode loop whose
    inputs are rewritten in place, or a benchmark): run() costs one foreign
    call, and set_positions() moves every sequence to its next position.  The
    library additionally recognises an identical call and relaunches the
    launches it built for it.  With `comm` (an ncclComm_t address) the call is
    jx_attn_step_sharded over that communicator.
    """

    def __init__(self, cache: KVCache, layers: Sequence[Layer], q, k, v, out, pos: Sequence[int],
                 n_heads: int, n_kv_heads: int, scale: Optional[float] = None,
                 softcap: float = 0.0, sliding_window: int = 0, yarn_scale: float = 1.0,
                 neox: bool = True, seq_ids: Optional[Sequence[int]] = None, partials=None,
                 comm=None, timeout_ms: int = 0):
        self.cache = cache
        self.arr, self._keep = _layer_array(layers)
        self.args, self._keep2 = _step_args(cache, layers, q, k, v, out if partials is None else None,
                                            pos, n_heads, n_kv_heads, scale, softcap,
                                            sliding_window, yarn_scale, neox, seq_ids, 0)
        self._tensors = (q, k, v, out, partials)
        self._pos = self._keep2[0]  # the ctypes position array args.pos points at
        self.n_layers = len(layers)
        if comm is not None:
            if partials is not None:
                raise JxError(-1, "a sharded step writes out, not partials")
            self._call = cache.lib.jx_attn_step_sharded
            self._head = (cache.handle, self.arr, self.n_layers, C.byref(self.args),
                          C.c_void_p(int(comm)), int(timeout_ms))
        elif partials is None:
            self._call = cache.lib.jx_attn_step
            self._head = (cache.handle, self.arr, self.n_layers, C.byref(self.args))
        else:
            hd = layers[0].head_dim
            pp = _dev_ptr(partials, "partials", len(pos) * len(layers) * n_heads * (hd + 2))
            self._call = cache.lib.jx_attn_step_partial
            self._head = (cache.handle, self.arr, self.n_layers, C.byref(self.args), pp)

    def set_positions(self, pos: Sequence[int]) -> None:
        """New positions for the next run() (same sequences): a decode loop
        advancing every slot by one token, as forward_token's seq_pos++
        (src/transformer.cpp:2792).  The library then builds that step's plan."""
        if len(pos) != len(self._pos):
            raise JxError(-1, "set_positions: one position per sequence of the plan")
        for i, p in enumerate(pos):
            self._pos[i] = int(p)

    def run(self, stream=None) -> None:
        rc = self._call(*self._head, _stream_ptr(stream))
        if rc:
            check(rc)


def lse_merge(gathered, n_shards: int, n_groups: int, n_heads: int, head_dim: int, out,
              out_stride: Optional[int] = None, stream=None) -> None:
    """Merge n_shards back-to-back partial buffers into out [n_groups, out_stride]."""
    per = n_groups * n_heads * (head_dim + 2)
    g = _dev_ptr(gathered, "gathered", per * n_shards)
    out_stride = out_stride or n_heads * head_dim
    o = _dev_ptr(out, "out", n_groups * out_stride)
    check(load().jx_lse_merge(g, n_shards, per, n_groups, n_heads, head_dim, o, out_stride,
                              _stream_ptr(stream)))


def fill_normal(t, seed: int, stream_id: int, stream=None) -> None:
    """Seeded N(0,1) fill of a float32 CUDA tensor (benchmark inputs)."""
    p = _dev_ptr(t, "t", 0)
    check(load().jx_fill_normal_f32(p, t.numel(), C.c_uint64(seed), stream_id,
                                    _stream_ptr(stream)))
