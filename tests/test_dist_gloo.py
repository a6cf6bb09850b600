"""Two CPU ranks (gloo) run the multi-GPU host logic of the sharded configs.

* sequence partition (c3/c5): ranks take LPT shares; together they cover every
  sequence once;
* position sharding (c4): each rank computes (m, l, o) partials over its
  contiguous position shard, all-gathers them, and the log-sum-exp merge
  reproduces the oracle's full attention.
The partial/merge arithmetic here is numpy; on GPUs the same steps run as
jx_attn_step_partial + NCCL all-gather + jx_lse_merge.
"""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from jxai_b200 import workloads as W


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _partials(qrot, K, V, lo, hi, H, HK, hd, scale):
    G = H // HK
    out = np.zeros((H, hd + 2))
    for h in range(H):
        kvh = h // G
        if hi <= lo:
            out[h, hd] = -np.inf
            continue
        s = (K[lo:hi, kvh * hd:(kvh + 1) * hd].astype(np.float64) @ qrot[h * hd:(h + 1) * hd]) * scale
        m = s.max()
        p = np.exp(s - m)
        out[h, :hd] = p @ V[lo:hi, kvh * hd:(kvh + 1) * hd]
        out[h, hd], out[h, hd + 1] = m, p.sum()
    return out


def _merge(parts):
    M = np.max(parts[:, :, -2], axis=0)
    f = np.where(np.isinf(parts[:, :, -2]), 0.0, np.exp(parts[:, :, -2] - M))
    L = (parts[:, :, -1] * f).sum(0)
    O = (parts[:, :, :-2] * f[:, :, None]).sum(0)
    return O / L[:, None]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # -- sequence partition
        T = W.c3_lengths()
        mine = W.lpt_partition(T, world)[rank]
        got = [None] * world
        dist.all_gather_object(got, mine)
        flat = sorted(i for p in got for i in p)
        ok_seq = flat == list(range(len(T)))
        # -- position sharding of one sequence
        from oracle.oracle import F32, Oracle
        rng = np.random.default_rng(11)
        H, HK, hd, T1 = 8, 2, 64, 203
        cap = T1
        kc = rng.standard_normal((1, 1, cap, HK * hd)).astype(np.float32)
        vc = rng.standard_normal((1, 1, cap, HK * hd)).astype(np.float32)
        qv = rng.standard_normal((1, 1, H * hd)).astype(np.float32)
        kv = rng.standard_normal((1, 1, HK * hd)).astype(np.float32)
        vv = rng.standard_normal((1, 1, HK * hd)).astype(np.float32)
        orc = Oracle("port")
        ko, vo = kc.copy(), vc.copy()
        full = orc.step(ko, vo, F32, [T1 - 1], [dict(rope_dim=hd, rope_base=1e6)], qv, kv, vv,
                        H, HK, hd, 1 / math.sqrt(hd), 0.0, 0, 1.0, False)[0, 0]
        qrot, _ = orc.apply_rope(qv[0, 0], None, H, 0, hd, hd, T1 - 1, 1e6, 1.0, False)
        lo, hi = W.position_shards(T1, world)[rank]
        mine_p = torch.from_numpy(_partials(qrot, ko[0, 0], vo[0, 0], lo, hi, H, HK, hd,
                                            1 / math.sqrt(hd)))
        gathered = [torch.zeros_like(mine_p) for _ in range(world)]
        dist.all_gather(gathered, mine_p)
        merged = _merge(torch.stack(gathered).numpy()).reshape(-1)
        err = float(np.abs(merged - full).max())
        q.put((rank, ok_seq, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_host_logic_two_ranks(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_seq, err in res:
        assert ok_seq
        assert err < 1e-5, err


def _liveness_worker(rank, world, port, q):
    # rank 1 runs step 0 and then leaves (its process ends between steps);
    # rank 0's next liveness check must raise JX_ERR_TIMEOUT before anything
    # of step 1 is queued
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=timedelta(seconds=30))
    from jxai_b200 import JxError
    from jxai_b200._lib import JX_ERR_TIMEOUT
    from jxai_b200.liveness import Heartbeat
    hb = Heartbeat(store, rank, world)
    queued = []
    res = {"rank": rank}
    try:
        hb.check(0, timeout_s=20.0)  # both ranks are alive for step 0
        queued.append(0)             # stands for the sharded step's launch
        if rank == 1:
            q.put(res)
            return                   # leaves between steps
        import time
        t0 = time.monotonic()
        try:
            hb.check(1, timeout_s=1.0)
            queued.append(1)
            res["raised"] = None
        except JxError as e:
            res["raised"] = e.code
            res["msg"] = str(e)
        res["elapsed"] = time.monotonic() - t0
        res["queued"] = queued
        res["code"] = JX_ERR_TIMEOUT
    except Exception as ex:  # reported to the parent
        res["exc"] = repr(ex)
    q.put(res)
    if rank == 0:
        import time
        time.sleep(0.5)  # the store server outlives the other rank's last read


def test_liveness_check_reports_a_rank_that_left():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_liveness_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r = q.get(timeout=120)
        res[r["rank"]] = r
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert "exc" not in res[0] and "exc" not in res[1], res
    r0 = res[0]
    assert r0["raised"] == r0["code"], r0
    assert "[1]" in r0["msg"] and "step 1" in r0["msg"]
    assert r0["queued"] == [0]          # step 1 queued nothing
    assert 0.9 <= r0["elapsed"] < 10.0  # the deadline, not the store's 30 s timeout
