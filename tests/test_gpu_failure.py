"""Failure detection on the GPU without a fault (the survey's plan for the
device side): every pipeline wait of the decode kernel is bounded, and a wait
that runs out makes the kernel give up, finish and report through the device
error word, leaving the context usable.

The error is made with the library's test hook: one CTA waits once on a
barrier nothing arrives at, under a ~2 ms bound ("wait_limit_ms",
"test_wait_cta").  Nothing traps or faults; the reference has no counterpart
(it has no device code).
"""
import math

import numpy as np
import pytest

from oracle.oracle import BF16, F32
from tests.helpers import oracle_step, random_cache

pytestmark = pytest.mark.gpu

TOL = 1e-4


def _case(dtype, seed):
    import torch
    import jxai_b200 as jx
    rng = np.random.default_rng(seed)
    H, HK, hd, L = 32, 8, 64, 2
    lengths = [900, 300]
    cap, rs = 904, HK * hd
    kc = random_cache(rng, (2, L, cap, rs), dtype)
    vc = random_cache(rng, (2, L, cap, rs), dtype)
    q = rng.standard_normal((2, L, H * hd)).astype(np.float32)
    k = rng.standard_normal((2, L, HK * hd)).astype(np.float32)
    v = rng.standard_normal((2, L, HK * hd)).astype(np.float32)
    layers = [jx.Layer(hd, hd, 5e5, l) for l in range(L)]
    cache = jx.KVCache(2, L, cap, rs, dtype)
    for s in range(2):
        for l in range(L):
            cache.write_rows(s, l, 0, 0, kc[s, l])
            cache.write_rows(s, l, 1, 0, vc[s, l])
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
    pos = [t - 1 for t in lengths]
    ko, vo = kc.copy(), vc.copy()
    ref = oracle_step(ko, vo, dtype, pos, layers, q, k, v, H, HK, hd, 1 / math.sqrt(hd),
                      neox=False)
    return torch, jx, cache, layers, (qd, kd, vd), pos, ref, ko, H, HK


@pytest.mark.parametrize("dtype", [F32, BF16])
@pytest.mark.parametrize("cta", [1, 5])
def test_bounded_wait_runs_out_and_is_reported(dtype, cta):
    torch, jx, cache, layers, (qd, kd, vd), pos, ref, ko, H, HK = _case(dtype, 11 + cta)
    try:
        out = torch.zeros_like(qd)
        cache.set_option("wait_limit_ms", 2)
        cache.set_option("test_wait_cta", cta)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        jx.attn_step(cache, layers, qd, kd, vd, out, pos, H, HK, neox=False)
        t1.record()
        torch.cuda.synchronize()  # the kernel returned: the wait gave up
        assert t0.elapsed_time(t1) < 1000.0
        assert cache.check_device_error() == 1
        msg = jx.load_library().jx_last_error_string()
        assert b"bounded wait ran out" in msg and f"block {cta - 1} ".encode() in msg, msg
        assert cache.check_device_error() == 0  # read and cleared
        # back to the default bound, no hook: the same step (it writes row pos
        # again) is correct on the same context
        cache.set_option("test_wait_cta", 0)
        cache.set_option("wait_limit_ms", 0)
        out.fill_(float("nan"))
        jx.attn_step(cache, layers, qd, kd, vd, out, pos, H, HK, neox=False)
        torch.cuda.synchronize()
        assert cache.check_device_error() == 0
        assert np.abs(out.cpu().numpy() - ref).max() <= TOL
        for s in range(2):
            for l in range(len(layers)):
                assert np.array_equal(cache.read_rows(s, l, 0, 0, cache.capacity).view(np.uint8),
                                      ko[s, l].view(np.uint8))
    finally:
        cache.close()
