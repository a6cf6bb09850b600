"""jx_attn_step_noalloc: the decode step for callers that cannot allocate GPU memory.

Engines that hand all of HBM to their own arena, or serving loops that must
not run into cudaMalloc/cudaFree (and the device synchronisation they can
imply) in the middle of a token, call this entry point with caller-owned cache
buffers; its scratch lives in one fixed array per GPU.  These tests call it
through the C ABI, twice in a row (the shared scratch keeps the previous
call's contents, so the second call shows that everything that must start at
zero is cleared), and check each call against

  * the CPU oracle (src/transformer.cpp:2497-2566): appended K and V rows
    bit-exact, attention within the 1e-4 every GPU parity test uses;
  * jx_attn_step, the handle-based entry point, on the same inputs.

A kernel error inside a no-allocation step (a bounded wait that runs out) is
read back with jx_noalloc_check_device_error.  This file is collected last so
that a failure here cannot hide any other test's result.
"""
import ctypes as C
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-4  # the attention tolerance every GPU parity test uses
DTYPES = ("f32", "bf16", "f16")


def _case(dtype_name, seed, H=32, HK=8, hd=64, L=3, lengths=(700, 333), window=0, swa=(),
          seq_ids=None, n_cache_seqs=None):
    import torch

    import jxai_b200 as jx
    from jxai_b200 import _lib
    from oracle.oracle import BF16, F16T, F32
    from tests.helpers import random_cache

    dt = {"f32": (F32, _lib.JX_F32), "bf16": (BF16, _lib.JX_BF16),
          "f16": (F16T, _lib.JX_F16_TRUNC)}[dtype_name]
    rng = np.random.default_rng(seed)
    n_step = len(lengths)
    n_seqs = n_cache_seqs or n_step
    cap, rs = max(lengths) + 4, HK * hd
    kc = random_cache(rng, (n_seqs, L, cap, rs), dt[0])
    vc = random_cache(rng, (n_seqs, L, cap, rs), dt[0])
    q = rng.standard_normal((n_step, L, H * hd)).astype(np.float32)
    k = rng.standard_normal((n_step, L, HK * hd)).astype(np.float32)
    v = rng.standard_normal((n_step, L, HK * hd)).astype(np.float32)
    layers = [jx.Layer(hd, hd, 5e5 if l % 2 else 1e6, l, is_swa=l in swa) for l in range(L)]
    return dict(torch=torch, jx=jx, lib=_lib, dt=dt, n_seqs=n_seqs, L=L, H=H, HK=HK, hd=hd,
                cap=cap, rs=rs, kc=kc, vc=vc, q=q, k=k, v=v, layers=layers,
                pos=[t - 1 for t in lengths], window=window, seq_ids=seq_ids)


def _oracle(s):
    """Oracle output and caches after the step (host copies of the inputs)."""
    from oracle.oracle import Oracle
    from tests.helpers import layer_dicts
    ko, vo = s["kc"].copy(), s["vc"].copy()
    sids = s["seq_ids"] or list(range(len(s["pos"])))
    out = np.zeros_like(s["q"])
    # the oracle steps sequences 0..n-1 of its cache arrays: gather the listed ones
    for i, sid in enumerate(sids):
        kk, vv = ko[sid:sid + 1].copy(), vo[sid:sid + 1].copy()
        out[i:i + 1] = Oracle("port").step(
            kk, vv, s["dt"][0], [s["pos"][i]], layer_dicts(s["layers"]), s["q"][i:i + 1],
            s["k"][i:i + 1], s["v"][i:i + 1], s["H"], s["HK"], s["hd"], 1 / math.sqrt(s["hd"]),
            0.0, s["window"], 1.0, True)
        ko[sid], vo[sid] = kk[0], vv[0]
    return out, ko, vo


def _noalloc(s, kbuf, vbuf, out, stream):
    from jxai_b200.attention import _layer_array, _step_args
    desc = s["lib"].KvDesc(s["n_seqs"], s["L"], s["cap"], s["rs"], s["dt"][1], 0, 0)
    arr, keep = _layer_array(s["layers"])
    torch = s["torch"]
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (s["q"], s["k"], s["v"]))
    args, keep2 = _step_args(None, s["layers"], qd, kd, vd, out, s["pos"], s["H"], s["HK"], None,
                             0.0, s["window"], 1.0, True, s["seq_ids"], 0)
    native = s["jx"].load_library()
    rc = native.jx_attn_step_noalloc(C.byref(desc), kbuf.data_ptr(), vbuf.data_ptr(), arr,
                                     s["L"], C.byref(args), stream)
    assert rc == 0, native.jx_last_error_string()
    return qd, kd, vd  # the caller keeps the inputs alive until the step has run


def _check_error(stream):
    import jxai_b200 as jx
    native = jx.load_library()
    code = C.c_int(-99)
    rc = native.jx_noalloc_check_device_error(0, C.byref(code), stream)
    return rc, code.value, native.jx_last_error_string()


def _device_caches(s):
    torch = s["torch"]
    as_t = (lambda a: a.view(np.int16)) if s["dt"][1] != s["lib"].JX_F32 else (lambda a: a)
    return (torch.from_numpy(as_t(s["kc"]).copy()).cuda(),
            torch.from_numpy(as_t(s["vc"]).copy()).cuda())


@pytest.mark.parametrize("dtype_name", DTYPES)
def test_noalloc_matches_oracle_and_jx_attn_step_on_two_calls(dtype_name):
    s = _case(dtype_name, seed={"f32": 17, "bf16": 18, "f16": 19}[dtype_name])
    torch, jx = s["torch"], s["jx"]
    ref, ko, vo = _oracle(s)

    # the existing entry point, on a library-owned cache
    cache = jx.KVCache(s["n_seqs"], s["L"], s["cap"], s["rs"], dtype_name)
    try:
        for q_ in range(s["n_seqs"]):
            for l in range(s["L"]):
                cache.write_rows(q_, l, 0, 0, s["kc"][q_, l])
                cache.write_rows(q_, l, 1, 0, s["vc"][q_, l])
        qd, kd, vd = (torch.from_numpy(x).cuda() for x in (s["q"], s["k"], s["v"]))
        step_out = torch.zeros_like(qd)
        jx.attn_step(cache, s["layers"], qd, kd, vd, step_out, s["pos"], s["H"], s["HK"],
                     neox=True)
        torch.cuda.synchronize()
        step_out = step_out.cpu().numpy()
    finally:
        cache.close()

    # the no-allocation entry point, on caller-owned cache buffers
    kbuf, vbuf = _device_caches(s)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full((len(s["pos"]), s["L"], s["H"] * s["hd"]), float("nan"), device="cuda")
        keep = _noalloc(s, kbuf, vbuf, out, stream)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}"
        assert np.abs(got - ref).max() <= TOL, f"call {call}: vs oracle"
        assert np.abs(got - step_out).max() <= TOL, f"call {call}: vs jx_attn_step"
        kh, vh = kbuf.cpu().numpy(), vbuf.cpu().numpy()
        assert np.array_equal(kh.view(np.uint8), ko.view(np.uint8)), f"call {call}: K rows"
        assert np.array_equal(vh.view(np.uint8), vo.view(np.uint8)), f"call {call}: V rows"
        rc, code, msg = _check_error(stream)
        assert rc == 0 and code == 0, msg


@pytest.mark.parametrize("dtype_name", ("f32", "f16"))
def test_noalloc_window_and_sequence_ids(dtype_name):
    # sliding-window layers and a step over some of the cache's sequences, in
    # another order: this path builds its own plan rows and RoPE table
    s = _case(dtype_name, seed=23, H=8, HK=2, hd=128, L=3, lengths=(900, 70, 513), window=256,
              swa=(0, 2), seq_ids=[3, 0, 2], n_cache_seqs=4)
    torch = s["torch"]
    ref, ko, vo = _oracle(s)
    kbuf, vbuf = _device_caches(s)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full((3, s["L"], s["H"] * s["hd"]), float("nan"), device="cuda")
        keep = _noalloc(s, kbuf, vbuf, out, stream)
        torch.cuda.synchronize()
        assert np.abs(out.cpu().numpy() - ref).max() <= TOL, f"call {call}"
        assert np.array_equal(kbuf.cpu().numpy().view(np.uint8), ko.view(np.uint8))
        assert np.array_equal(vbuf.cpu().numpy().view(np.uint8), vo.view(np.uint8))


def test_noalloc_reports_a_bounded_wait_that_ran_out():
    # Test hook of the error path: CTA 0 waits once on a barrier nothing
    # arrives at, bounded to ~2 ms.  The kernel gives up, finishes and sets the
    # error word; the check reads it, clears it, and the next step is correct.
    s = _case("f32", seed=29, lengths=(400, 120))
    torch, lib = s["torch"], s["jx"].load_library()
    ref, ko, vo = _oracle(s)
    kbuf, vbuf = _device_caches(s)
    stream = torch.cuda.current_stream().cuda_stream
    out = torch.zeros((2, s["L"], s["H"] * s["hd"]), device="cuda")
    assert _check_error(stream)[1] == 0  # nothing pending from earlier tests
    try:
        assert lib.jx_noalloc_set_option(b"wait_limit_ms", 2) == 0
        assert lib.jx_noalloc_set_option(b"test_wait_cta", 1) == 0
        keep = _noalloc(s, kbuf, vbuf, out, stream)
    finally:
        lib.jx_noalloc_set_option(b"test_wait_cta", 0)
        lib.jx_noalloc_set_option(b"wait_limit_ms", 0)
    torch.cuda.synchronize()
    rc, code, msg = _check_error(stream)
    assert rc == s["lib"].JX_ERR_DEVICE and code == 1, (rc, code, msg)
    assert b"bounded wait ran out" in msg and b"block 0" in msg, msg
    assert _check_error(stream)[1] == 0  # read and cleared
    # the failed step may have left a wrong row at pos (its output is
    # invalid); the next step on the same buffers writes that row again and
    # its output is correct
    keep = _noalloc(s, kbuf, vbuf, out, stream)
    torch.cuda.synchronize()
    assert np.abs(out.cpu().numpy() - ref).max() <= TOL
    assert np.array_equal(kbuf.cpu().numpy().view(np.uint8), ko.view(np.uint8))
    assert _check_error(stream)[1] == 0


def test_noalloc_rejects_steps_beyond_its_scratch():
    import torch

    import jxai_b200 as jx
    from jxai_b200 import _lib
    from jxai_b200.attention import _layer_array, _step_args

    n_seqs, L, H, HK, hd, cap = 64, 16, 32, 8, 64, 128
    q = torch.zeros(n_seqs, L, H * hd, device="cuda")
    k = torch.zeros(n_seqs, L, HK * hd, device="cuda")
    v = torch.zeros_like(k)
    out = torch.zeros_like(q)
    small = torch.zeros(1024, device="cuda")  # never touched: the call is refused first
    layers = [jx.Layer(hd, hd, 5e5, l) for l in range(L)]
    desc = _lib.KvDesc(n_seqs, L, cap, HK * hd, _lib.JX_F32, 0, 0)
    arr, keep = _layer_array(layers)
    args, keep2 = _step_args(None, layers, q, k, v, out, [100] * n_seqs, H, HK, None, 0.0, 0,
                             1.0, False, None, 0)
    native = jx.load_library()
    rc = native.jx_attn_step_noalloc(C.byref(desc), small.data_ptr(), small.data_ptr(), arr, L,
                                     C.byref(args), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.JX_ERR_RANGE
    assert b"scratch" in native.jx_last_error_string()


def test_noalloc_refuses_pageable_and_host_cache_pointers():
    # the same pointer rules as jx_attn_step: a kernel given pageable host
    # memory would fault, so such calls are refused on the host
    import torch

    import jxai_b200 as jx
    from jxai_b200 import _lib
    from jxai_b200.attention import _layer_array

    H, HK, hd, L, cap = 8, 2, 64, 1, 64
    layers = [jx.Layer(hd, hd, 5e5, 0)]
    desc = _lib.KvDesc(1, L, cap, HK * hd, _lib.JX_F32, 0, 0)
    arr, keep = _layer_array(layers)
    cache = torch.zeros(2, cap * HK * hd, device="cuda")
    dev_in = torch.zeros(3, H * hd, device="cuda")
    pageable = np.zeros(H * hd, np.float32)
    pos = (C.c_int32 * 1)(10)
    native = jx.load_library()

    def call(q_ptr, k_cache_ptr):
        a = _lib.StepArgs()
        a.n_heads, a.n_kv_heads, a.n_seqs = H, HK, 1
        a.pos = C.cast(pos, C.POINTER(C.c_int32))
        a.q = q_ptr
        a.k = dev_in[1].data_ptr()
        a.v = dev_in[2].data_ptr()
        a.out = dev_in[0].data_ptr()
        a.q_stride, a.kv_stride = H * hd, HK * hd
        a.scale, a.yarn_scale, a.rope_neox = 0.125, 1.0, 1
        return native.jx_attn_step_noalloc(C.byref(desc), k_cache_ptr, cache[1].data_ptr(), arr,
                                           L, C.byref(a), torch.cuda.current_stream().cuda_stream)

    assert call(pageable.ctypes.data, cache[0].data_ptr()) == _lib.JX_ERR_INVALID
    assert b"q" in native.jx_last_error_string()
    assert call(dev_in[0].data_ptr(), pageable.ctypes.data) == _lib.JX_ERR_INVALID
    assert b"k_cache" in native.jx_last_error_string()
    torch.cuda.synchronize()


def test_noalloc_refuses_stream_capture():
    # a captured plan copy would replay from a host slot that later calls
    # reuse, so the call is refused while its stream is capturing
    import torch

    import jxai_b200 as jx
    from jxai_b200 import _lib
    from jxai_b200.attention import _layer_array

    H, HK, hd, L, cap = 8, 2, 64, 1, 64
    layers = [jx.Layer(hd, hd, 5e5, 0)]
    desc = _lib.KvDesc(1, L, cap, HK * hd, _lib.JX_F32, 0, 0)
    arr, keep = _layer_array(layers)
    cache = torch.zeros(2, cap * HK * hd, device="cuda")
    io = torch.zeros(4, H * hd, device="cuda")
    pos = (C.c_int32 * 1)(10)
    native = jx.load_library()
    a = _lib.StepArgs()
    a.n_heads, a.n_kv_heads, a.n_seqs = H, HK, 1
    a.pos = C.cast(pos, C.POINTER(C.c_int32))
    a.q, a.k, a.v, a.out = (io[i].data_ptr() for i in range(4))
    a.q_stride, a.kv_stride = H * hd, HK * hd
    a.scale, a.yarn_scale, a.rope_neox = 0.125, 1.0, 1
    # one ordinary call first (the device's set-up), then one under capture
    s = torch.cuda.Stream()
    assert native.jx_attn_step_noalloc(C.byref(desc), cache[0].data_ptr(), cache[1].data_ptr(),
                                       arr, L, C.byref(a), s.cuda_stream) == _lib.JX_OK
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    rc = None
    with torch.cuda.stream(s):
        g.capture_begin()
        try:
            rc = native.jx_attn_step_noalloc(C.byref(desc), cache[0].data_ptr(),
                                             cache[1].data_ptr(), arr, L, C.byref(a),
                                             s.cuda_stream)
        finally:
            g.capture_end()
    assert rc == _lib.JX_ERR_UNSUPPORTED
    assert b"captured" in native.jx_last_error_string()
    code = C.c_int(-1)
    assert native.jx_noalloc_check_device_error(0, C.byref(code), s.cuda_stream) == _lib.JX_OK
    assert code.value == 0
    del g
