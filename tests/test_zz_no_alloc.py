"""jx_attn_step_noalloc: the decode step for callers that cannot allocate GPU memory.

Engines that hand all of HBM to their own arena, or serving loops that must
not run into cudaMalloc/cudaFree (and the device synchronisation they can
imply) in the middle of a token, call this entry point with caller-owned cache
buffers; its scratch lives in one fixed array per GPU.  These tests call it
through the C ABI and check it against jx_attn_step on the same inputs, twice
in a row (the shared scratch keeps the previous call's contents, so the second
call shows that everything that must start at zero is cleared).  This file is
collected last so that a failure here cannot hide any other test's result.
"""
import ctypes as C
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-4  # the attention tolerance every GPU parity test uses


def _setup(dtype_name, seed):
    import torch

    import jxai_b200 as jx
    from jxai_b200 import _lib
    from tests.helpers import random_cache
    from oracle.oracle import BF16, F32

    dt = {"f32": (F32, _lib.JX_F32), "bf16": (BF16, _lib.JX_BF16)}[dtype_name]
    rng = np.random.default_rng(seed)
    n_seqs, L, H, HK, hd = 2, 3, 32, 8, 64
    lengths = [700, 333]
    cap, rs = 704, HK * hd
    kc = random_cache(rng, (n_seqs, L, cap, rs), dt[0])
    vc = random_cache(rng, (n_seqs, L, cap, rs), dt[0])
    q = torch.from_numpy(rng.standard_normal((n_seqs, L, H * hd)).astype(np.float32)).cuda()
    k = torch.from_numpy(rng.standard_normal((n_seqs, L, HK * hd)).astype(np.float32)).cuda()
    v = torch.from_numpy(rng.standard_normal((n_seqs, L, HK * hd)).astype(np.float32)).cuda()
    layers = [jx.Layer(hd, hd, 5e5 if l % 2 else 1e6, l) for l in range(L)]
    pos = [t - 1 for t in lengths]
    return dict(torch=torch, jx=jx, lib=_lib, dt=dt, n_seqs=n_seqs, L=L, H=H, HK=HK, hd=hd,
                cap=cap, rs=rs, kc=kc, vc=vc, q=q, k=k, v=v, layers=layers, pos=pos)


@pytest.mark.parametrize("dtype_name", ["f32", "bf16"])
def test_noalloc_matches_jx_attn_step_on_two_calls(dtype_name):
    s = _setup(dtype_name, seed=17 if dtype_name == "f32" else 18)
    torch, jx, lib = s["torch"], s["jx"], s["lib"]
    from jxai_b200.attention import _layer_array, _step_args

    # the existing entry point, on a library-owned cache
    cache = jx.KVCache(s["n_seqs"], s["L"], s["cap"], s["rs"], dtype_name)
    for q_ in range(s["n_seqs"]):
        for l in range(s["L"]):
            cache.write_rows(q_, l, 0, 0, s["kc"][q_, l])
            cache.write_rows(q_, l, 1, 0, s["vc"][q_, l])
    ref = torch.zeros_like(s["q"])
    jx.attn_step(cache, s["layers"], s["q"], s["k"], s["v"], ref, s["pos"], s["H"], s["HK"],
                 neox=True)
    torch.cuda.synchronize()
    ref_k = [[cache.read_rows(q_, l, 0, 0, s["cap"]) for l in range(s["L"])]
             for q_ in range(s["n_seqs"])]

    # the no-allocation entry point, on caller-owned cache buffers
    kbuf = torch.from_numpy(s["kc"].view(np.int16) if dtype_name == "bf16" else s["kc"]).cuda()
    vbuf = torch.from_numpy(s["vc"].view(np.int16) if dtype_name == "bf16" else s["vc"]).cuda()
    desc = lib.KvDesc(s["n_seqs"], s["L"], s["cap"], s["rs"], s["dt"][1], 0, 0)
    arr, keep = _layer_array(s["layers"])
    native = jx.load_library()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full_like(s["q"], float("nan"))
        args, keep2 = _step_args(None, s["layers"], s["q"], s["k"], s["v"], out, s["pos"],
                                 s["H"], s["HK"], None, 0.0, 0, 1.0, True, None, 0)
        rc = native.jx_attn_step_noalloc(C.byref(desc), kbuf.data_ptr(), vbuf.data_ptr(), arr,
                                         s["L"], C.byref(args), stream)
        assert rc == 0, native.jx_last_error_string()
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}"
        err = np.abs(got - ref.cpu().numpy()).max()
        assert err <= TOL, f"call {call}: max-abs {err}"
        kh = kbuf.cpu().numpy()
        for q_ in range(s["n_seqs"]):
            for l in range(s["L"]):
                assert np.array_equal(kh[q_, l].view(np.uint8), ref_k[q_][l].view(np.uint8))
    cache.close()


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
