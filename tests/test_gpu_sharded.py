"""jx_attn_step_sharded on two GPUs: one context sharded by position over an
NCCL communicator (partial step, ncclAllGather, log-sum-exp merge in one call).

* parity: both ranks receive the full output, within 1e-4 of the unsharded CPU
  oracle, and only the rank holding `pos` appends (bit-exact).

Runs as two spawned processes, one per GPU, NVLS off; skipped with fewer than
two GPUs.
"""
import math
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-4
H, HK, HD, L, T = 8, 2, 64, 2, 700


def _case():
    rng = np.random.default_rng(77)
    rs = HK * HD
    kc = rng.standard_normal((1, L, T, rs)).astype(np.float32)
    vc = rng.standard_normal((1, L, T, rs)).astype(np.float32)
    q = rng.standard_normal((1, L, H * HD)).astype(np.float32)
    k = rng.standard_normal((1, L, HK * HD)).astype(np.float32)
    v = rng.standard_normal((1, L, HK * HD)).astype(np.float32)
    return kc, vc, q, k, v


def _worker(rank, world, q_uid, q_res):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    torch.cuda.set_device(rank)
    import jxai_b200 as jx
    from jxai_b200.nccl import NcclComm
    from oracle.oracle import F32
    from tests.helpers import oracle_step

    result = {"rank": rank}
    try:
        if rank == 0:
            uid = NcclComm.unique_id()
            for _ in range(world - 1):
                q_uid.put(uid)
        else:
            uid = q_uid.get(timeout=120)
        # non-blocking creation with a deadline (the all-gather may then report
        # ncclInProgress while the communicator connects; the library waits)
        comm = NcclComm(world, rank, uid, timeout_s=120)
        kc, vc, q, k, v = _case()
        rs = HK * HD
        b, e = T * rank // world, T * (rank + 1) // world
        layers = [jx.Layer(HD, HD, 1e6, 0), jx.Layer(HD, HD, 1e4, 1)]
        cache = jx.KVCache(1, L, e - b, rs, "f32", device=rank, pos_base=b)
        for l in range(L):
            cache.write_rows(0, l, 0, 0, kc[0, l, b:e])
            cache.write_rows(0, l, 1, 0, vc[0, l, b:e])
        dev = torch.device("cuda", rank)
        qd, kd, vd = (torch.from_numpy(x).to(dev) for x in (q, k, v))
        out = torch.full_like(qd, float("nan"))
        pos = T - 1
        jx.attn_step_sharded(cache, layers, qd, kd, vd, out, [pos], H, HK, comm.handle,
                             timeout_ms=30000, neox=False)
        torch.cuda.synchronize()
        ko, vo = kc.copy(), vc.copy()
        ref = oracle_step(ko, vo, F32, [pos], layers, q, k, v, H, HK, HD,
                          1 / math.sqrt(HD), neox=False)
        result["err"] = float(np.abs(out.cpu().numpy() - ref).max())
        result["dev_err"] = cache.check_device_error()
        ok = True
        for l in range(L):
            got = cache.read_rows(0, l, 0, 0, e - b)
            ok &= bool(np.array_equal(got, ko[0, l, b:e]))
            got = cache.read_rows(0, l, 1, 0, e - b)
            ok &= bool(np.array_equal(got, vo[0, l, b:e]))
        result["append_ok"] = ok
        comm.destroy()
        cache.close()
    except Exception as ex:  # reported to the parent
        result["exc"] = repr(ex)
    q_res.put(result)


def _run():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q_uid, q_res = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, q_uid, q_res))
             for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(2):
        r = q_res.get(timeout=300)
        results[r["rank"]] = r
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in results.values():
        assert "exc" not in r, r
    return results


def test_sharded_step_matches_unsharded_oracle():
    res = _run()
    for r in res.values():
        assert r["dev_err"] == 0
        assert r["err"] <= TOL, r
        assert r["append_ok"], r


def _lonely_rank(q_res):
    # rank 0 of a 2-rank communicator whose rank 1 never exists: the
    # non-blocking creation must give up at its deadline (host side: NCCL's
    # bootstrap waits for the peer; no kernel runs)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import time
    import torch
    torch.cuda.set_device(0)
    from jxai_b200.nccl import NcclComm, NcclTimeout
    res = {}
    t0 = time.monotonic()
    try:
        NcclComm(2, 0, NcclComm.unique_id(), timeout_s=3.0)
        res["raised"] = None
    except NcclTimeout as e:
        res["raised"] = "timeout"
        res["msg"] = str(e)
    except Exception as e:
        res["raised"] = repr(e)
    res["elapsed"] = time.monotonic() - t0
    q_res.put(res)


def test_nonblocking_init_gives_up_when_a_rank_never_joins():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 1:
        pytest.skip("needs a GPU")
    ctx = mp.get_context("spawn")
    q_res = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(q_res,))
    p.start()
    try:
        res = q_res.get(timeout=180)
    finally:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res["raised"] == "timeout", res
    assert 2.9 <= res["elapsed"] < 60.0, res
