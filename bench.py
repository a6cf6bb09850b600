#!/usr/bin/env python
"""Decode-attention benchmark: KV-read HBM GB/s and steps/s of the fused B200 step.

One step = RoPE + KV append + grouped-query decode attention on every layer of
every sequence of the workload (jxai src/transformer.cpp:2497-2566).  The
default workload is c4, the long-context config the scaling target names:
Mistral-7B shape (32 layers, 32/8 heads, head_dim 128) with one fp32 cache of
131071 rows, appending row 131071 -- on one GPU the whole step, on N GPUs
sharded by position.  --config c2 is BASELINE configs[1] (Llama-3.2-1B,
T = 4096).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1..c5] [--dtype f32|bf16]
    python bench.py --impl reference ...   # the reference's CPU implementation

Multi-GPU (launched by torchrun, one rank per GPU): c1/c2 run one replica per
GPU; c3/c5 partition the sequences (greedy LPT on length); c4 shards the one
long sequence by position and merges per-shard (m, l, o) partials after one
NCCL all-gather.  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

if int(os.environ.get("WORLD_SIZE", "1")) > 1:
    # NCCL's communicator lines (rank, nRanks, transports) in the run's
    # output (on stderr: main() keeps stdout for the JSON line).  Set before
    # torch (and its NCCL) is loaded, which reads them once; a level below
    # INFO (an environment's VERSION or WARN) is raised, INFO / TRACE kept.
    if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
        os.environ["NCCL_DEBUG"] = "INFO"
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")

from jxai_b200 import workloads as W  # noqa: E402

METRIC = "decode-attn KV-read HBM GB/s"
FALLBACK_HBM_GBS = 6650.0
_JSON_FD = None  # the process's original stdout when fd 1 was sent to stderr


def emit(line: dict) -> None:
    """Prints the run's one JSON line on the original standard output."""
    text = json.dumps(line) + "\n"
    if _JSON_FD is None:
        sys.stdout.write(text)
        sys.stdout.flush()
    else:
        sys.stdout.flush()
        os.write(_JSON_FD, text.encode())


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None,
                   help="timed steps (default: 2000 for c1/c2, 200 for the larger configs)")
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--config", default=None,
                   help="workload c1..c5 (default: c4 for decode steps; c2, the shape the\n"
                        "reference's prompt loop is measured on, for --prefill / --engine)")
    p.add_argument("--dtype", default=None, help="KV cache type (f32 | bf16 | f16)")
    p.add_argument("--cpu-sample-s", type=float, default=8.0,
                   help="seconds of CPU work for the cpu_baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--clock-probe-s", type=float, default=1.0,
                   help="untimed seconds of steps before warm-up so clocks leave idle")
    p.add_argument("--seqs", type=int, default=0,
                   help="keep only the first N sequences of the workload (small profiling cases)")
    p.add_argument("--len", type=int, default=0, dest="length",
                   help="attended length T of every sequence instead of the config's\n"
                        "(small profiling cases of the long configs)")
    p.add_argument("--sustained-s", type=float, default=1.0,
                   help="after the K timed steps, repeat them for about this many seconds and "
                        "report that figure as 'sustained' beside the burst (0: off; skipped "
                        "when the K steps already take half of it)")
    p.add_argument("--no-graph", action="store_true",
                   help="time K eager launches instead of one CUDA graph of K launches")
    p.add_argument("--set", action="append", default=[], metavar="KEY=VALUE",
                   help="library option (jx_kv_set_option) for the run's cache; repeatable")
    p.add_argument("--engine", action="store_true",
                   help="per-token latency through the C++ engine drop-in (include/jx_engine.hpp):\n"
                        "one synchronous block call per layer on host vectors, as forward_token\n"
                        "makes it; single-sequence full-attention configs (c1, c2, c4)")
    p.add_argument("--tokens", type=int, default=200, help="timed tokens of --engine")
    p.add_argument("--prefill", type=int, default=0, metavar="N",
                   help="prompt throughput: one prompt of N tokens per jx_attn_prefill call\n"
                        "(full-attention configs), the reference's token-serial loop beside it")
    a = p.parse_args()
    if a.config is None:
        a.config = "c2" if (a.prefill or a.engine) else "c4"
    if a.steps is None:
        a.steps = 2000 if a.config.lower() in ("c1", "c2", "qwen2.5-0.5b", "llama-3.2-1b") else 200
    return a


def make_workload(args) -> W.Workload:
    """The config's workload, cut to --seqs sequences / --len rows if asked."""
    w = W.make(args.config, args.dtype)
    if args.seqs > 0:
        w.lengths = w.lengths[:args.seqs]
    if args.length > 0:
        w.lengths = [args.length] * len(w.lengths)
    return w


# ----------------------------------------------------------------------------- helpers

def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            d = json.load(fh)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, STREAM-style copy)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback 6.65 TB/s (earlier measurement on this pool)"


def tensor_peak():
    """Dense bf16 tensor peak for a kernel timed alone (burst figure)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            d = json.load(fh)
        return float(d["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, cuBLAS burst)"
    except Exception:
        return 1590.0, "fallback 1.59 PFLOP/s (earlier measurement on this pool)"


def ncu_traffic(key: str):
    """DRAM bytes per launch of a kernel from the committed ncu summaries (the
    decode kernel per workload, the tensor-core prefill per prompt)."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(path) as fh:
            d = json.load(fh)
        e = d.get(key)
        return None if e is None else float(e["dram_bytes_per_launch"])
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 100 ms on one GPU."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.dev)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append((time.time(), ln.strip()))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            if self.t:
                self.t.join(timeout=2)

    def summary(self, t0: float, t1: float, min_samples: int = 1):
        rows = []
        for ts, ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((ts, float(parts[1]), float(parts[2]), parts[4:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        window = [r for r in rows if t0 <= r[0] <= t1]
        extended = False
        if len(window) < min_samples:
            # a timed region shorter than a few sample periods: the samples
            # from its start on (the same steps go on repeating after it)
            later = [r for r in rows if r[0] >= t0][:min_samples]
            if len(later) > len(window):
                window, extended = later, True
        window = window or rows[-5:]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in window:
            for nm, v in zip(names, r[3][1:]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        out = {"sm_mhz": statistics.median(r[1] for r in window),
               "sm_max_mhz": max(r[2] for r in window), "reasons": sorted(reasons),
               "samples": len(window)}
        if extended:
            out["window"] = "from the timed region's start into the repeats that follow it"
        return out


# ----------------------------------------------------------------------------- our arm

class Runner:
    """One rank's share of a workload, driven through the public Python API.

    extra_rows: cache rows beyond the workload's lengths, for steps that go on
    decoding (each appends one more row); in a position-sharded run they go to
    the last shard, which holds the newest positions."""

    def __init__(self, w: W.Workload, rank: int, world: int, device: int, options=(),
                 extra_rows: int = 0):
        import torch
        import jxai_b200 as jx
        self.torch, self.jx, self.w = torch, jx, w
        self.rank, self.world, self.device = rank, world, device
        self.mode = w.sharding if world > 1 else "replica"
        T = w.lengths
        if self.mode == "sequences":
            self.local = [T[i] for i in W.lpt_partition(T, world)[rank]]
        else:
            self.local = list(T)
        self.pos_base = 0
        if self.mode == "positions":
            (b, e) = W.position_shards(T[0], world)[rank]
            self.shard = (b, e)
            self.pos_base, cap = b, e - b + (extra_rows if rank == world - 1 else 0)
            rows = [max(0, min(e, T[0] - 1) - b)]
        else:
            cap = max(self.local) + extra_rows
            rows = [t - 1 for t in self.local]
        n = len(self.local)
        self.n = n
        self.cache = jx.KVCache(n, w.n_layers, cap, w.kv_dim, w.dtype, device, self.pos_base)
        for opt in options:
            key, _, val = opt.partition("=")
            self.cache.set_option(key, int(val))
        self.cache.fill_normal(rows, W.SEED + rank)
        dev = torch.device("cuda", device)
        self.q = torch.empty(n, w.n_layers, w.q_dim, device=dev)
        self.k = torch.empty(n, w.n_layers, w.kv_dim, device=dev)
        self.v = torch.empty_like(self.k)
        self.out = torch.empty_like(self.q)
        jx.fill_normal(self.q, W.SEED, 3)
        jx.fill_normal(self.k, W.SEED, 4)
        jx.fill_normal(self.v, W.SEED, 5)
        self.pos = [t - 1 for t in self.local]
        if self.mode == "positions":
            hd2 = w.head_dim + 2
            self.partials = torch.empty(n * w.n_layers * w.n_heads * hd2, device=dev)
            self.gathered = torch.empty(world * self.partials.numel(), device=dev)
        self.kv_bytes = self.kv_bytes_at(0)  # KV bytes this rank reads per step
        self.alg_bytes = self.kv_bytes + w.other_bytes(n)
        self._plan = self.plan()

    def kv_bytes_at(self, shift: int = 0) -> int:
        """KV bytes this rank reads in a step `shift` tokens after the first."""
        return W.rank_kv_bytes(self.w, self.mode, self.rank, self.world, shift)

    def plan(self, q=None, k=None, v=None, out=None, comm=None):
        """The step's C call with its arguments built once (jx.StepPlan); with
        `comm` (an ncclComm_t) the library's whole sharded step."""
        q = self.q if q is None else q
        k = self.k if k is None else k
        v = self.v if v is None else v
        out = self.out if out is None else out
        w = self.w
        partials = self.partials if (self.mode == "positions" and comm is None) else None
        return self.jx.StepPlan(self.cache, w.layers, q, k, v, out, self.pos, w.n_heads,
                                w.n_kv_heads, scale=w.scale, sliding_window=w.window,
                                neox=w.neox, partials=partials, comm=comm)

    def kernel(self, plan=None):
        (plan or self._plan).run()

    def finish(self, out=None):
        """Collective tail of a sharded step (all-gather + log-sum-exp merge)."""
        if self.mode != "positions":
            return
        import torch.distributed as dist
        out = self.out if out is None else out
        if self.world > 1:
            dist.all_gather_into_tensor(self.gathered, self.partials)
            g = self.gathered
        else:
            g = self.partials
        self.jx.lse_merge(g, self.world, self.n * self.w.n_layers, self.w.n_heads,
                          self.w.head_dim, out, self.w.q_dim)

    def step(self):
        self.kernel()
        self.finish()

    def launches_per_step(self):
        return self.cache.last_launch_count() + (1 if self.mode == "positions" else 0)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    w = make_workload(args)
    # the end-to-end leg decodes warmup + K further tokens: room for their rows
    extra = 0 if args.no_e2e else args.warmup + args.steps + 16
    r = Runner(w, rank, world, local_rank, args.set, extra_rows=extra)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    sampler = ClockSampler(local_rank)
    sampler.start()
    # untimed clock probe so clocks leave idle before warm-up.  Every rank runs
    # the same number of steps (a sharded step holds a collective): time five
    # steps, size the probe from the slowest rank, then run it.
    n_probe = 0
    if args.clock_probe_s > 0:
        t0 = time.time()
        for _ in range(5):
            r.step()
        torch.cuda.synchronize()
        per_step = max_over_ranks((time.time() - t0) / 5)
        n_probe = int(min(100000, max(0.0, args.clock_probe_s / max(per_step, 1e-6))))
        for _ in range(n_probe):
            r.step()
        torch.cuda.synchronize()
        n_probe += 5
    for _ in range(args.warmup):
        r.step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()

    K = args.steps
    e_start = torch.cuda.Event(enable_timing=True)
    e_stop = torch.cuda.Event(enable_timing=True)
    # The K timed steps run as one CUDA graph of K launches (the way a serving
    # loop issues them: no per-launch CPU cost between steps) unless the step
    # holds a collective (sharded positions) or --no-graph is given; then they
    # are K eager launches, each bracketed by events.
    use_graph = not args.no_graph and r.mode != "positions"
    if use_graph:
        gstream = torch.cuda.Stream()
        gstream.wait_stream(stream)
        with torch.cuda.stream(gstream):
            for _ in range(3):
                r.kernel()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=gstream):
            for _ in range(K):
                r.kernel()
        with torch.cuda.stream(gstream):
            graph.replay()  # untimed: uploads the graph
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        t_wall0 = time.time()
        with torch.cuda.stream(gstream):  # replay() launches on the current stream
            e_start.record(gstream)
            graph.replay()
            e_stop.record(gstream)
        torch.cuda.synchronize()
        t_wall1 = time.time()
        barrier()
        elapsed_ms = e_start.elapsed_time(e_stop)
        kernel_ms = elapsed_ms / K  # launch period: the kernel plus the gap to the next
        timing = "CUDA graph of K launches; kernel_ms = graph time / K (launch period)"
    else:
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(K)]
        t_wall0 = time.time()
        e_start.record(stream)
        for i in range(K):
            ev[i][0].record(stream)
            r.kernel()
            ev[i][1].record(stream)
            r.finish()
        e_stop.record(stream)
        torch.cuda.synchronize()
        t_wall1 = time.time()
        barrier()
        elapsed_ms = e_start.elapsed_time(e_stop)
        kernel_ms = sum(a.elapsed_time(b) for a, b in ev) / K
        timing = "K eager launches; kernel_ms = mean of per-launch CUDA events"
    err = r.cache.check_device_error()
    if err:
        raise RuntimeError(f"device error {err} during the timed region")
    elapsed_ms = max_over_ranks(elapsed_ms)
    total_kv = sum_over_ranks(r.kv_bytes)

    # ---- sustained: the same K steps repeated for about --sustained-s seconds
    # (a short burst runs at boost clocks; a long one meets the power cap).
    # The repeat count comes from the slowest rank, so every rank takes the
    # same steps (a sharded step holds a collective).
    sustained = None
    if args.sustained_s > 0 and elapsed_ms < 0.5 * args.sustained_s * 1e3:
        reps = int(min(1000000 // max(K, 1), math.ceil(args.sustained_s * 1e3 / elapsed_ms)))
        barrier()
        torch.cuda.synchronize()
        s_wall0 = time.time()
        if use_graph:
            with torch.cuda.stream(gstream):
                e_start.record(gstream)
                for _ in range(reps):
                    graph.replay()
                e_stop.record(gstream)
        else:
            e_start.record(stream)
            for _ in range(reps * K):
                r.kernel()
                r.finish()
            e_stop.record(stream)
        torch.cuda.synchronize()
        s_wall1 = time.time()
        barrier()
        if r.cache.check_device_error():
            raise RuntimeError("device error during the sustained steps")
        s_ms = max_over_ranks(e_start.elapsed_time(e_stop)) / (reps * K)
        peak_s, _ = peaks()
        sustained = {"steps": reps * K, "seconds": round(s_ms * reps * K * 1e-3, 3),
                     "ms_per_step": round(s_ms, 5),
                     "value": round(total_kv / (s_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                     "frac": round(r.alg_bytes / (s_ms * 1e-3) / 1e9 / peak_s, 4),
                     "clocks": sampler.summary(s_wall0, s_wall1)}
    if use_graph:
        del graph
    # the timed region's clocks; when it spans under 5 samples (100 ms
    # each), the samples from its start into the sustained repeats after it
    clocks = sampler.summary(t_wall0, t_wall1, min_samples=5)
    sampler.stop()

    # ---- end to end through the public API with host buffers, decoding on:
    # every step is the next token of every sequence (pos + 1, as forward_token
    # advances seq_pos, src/transformer.cpp:2792), so each call builds a new
    # plan and RoPE rows and appends a new row, and attends one row more.
    e2e = None
    comm = None
    if not args.no_e2e:
        # q, k, v and the output in pinned host memory.  Sharded-position
        # steps stage them: one H2D copy of q|k|v and one D2H copy of the
        # output per step around jx_attn_step_sharded (partial step, NCCL
        # all-gather, merge).  Otherwise the C ABI call takes the host buffers
        # themselves: the library copies q/k/v into device memory with one
        # staging kernel and the decode kernel writes attn_out over PCIe.
        nq, nk = r.q.numel(), r.k.numel()
        inh = torch.empty(nq + 2 * nk, pin_memory=True)
        inh[:nq].copy_(r.q.reshape(-1).cpu())
        inh[nq:nq + nk].copy_(r.k.reshape(-1).cpu())
        inh[nq + nk:].copy_(r.v.reshape(-1).cpu())
        oh = torch.empty(r.out.shape, pin_memory=True)
        qh, kh, vh = inh[:nq], inh[nq:nq + nk], inh[nq + nk:]
        zero_copy = r.mode != "positions"
        if zero_copy:
            e2e_plan = r.plan(qh.view(r.q.shape), kh.view(r.k.shape), vh.view(r.v.shape), oh)

            def e2e_step(i):
                e2e_plan.set_positions([p + i for p in r.pos])
                e2e_plan.run()
        else:
            from jxai_b200.nccl import NcclComm
            uid = [NcclComm.unique_id() if rank == 0 else None]
            dist.broadcast_object_list(uid, src=0)
            comm = NcclComm(world, rank, uid[0])
            ind = torch.empty(nq + 2 * nk, device=r.q.device)
            qd = ind[:nq].view(r.q.shape)
            kd = ind[nq:nq + nk].view(r.k.shape)
            vd = ind[nq + nk:].view(r.v.shape)
            od = torch.empty_like(r.out)
            e2e_plan = r.plan(qd, kd, vd, od, comm=comm.handle)

            def e2e_step(i):
                ind.copy_(inh, non_blocking=True)
                e2e_plan.set_positions([p + i for p in r.pos])
                e2e_plan.run()
                oh.copy_(od, non_blocking=True)

        for i in range(args.warmup):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        h0 = time.perf_counter()
        for i in range(args.warmup, args.warmup + K):
            e2e_step(i)
        host_ms = (time.perf_counter() - h0) * 1e3 / K
        b.record(stream)
        torch.cuda.synchronize()
        barrier()
        if r.cache.check_device_error():
            raise RuntimeError("device error during the end-to-end steps")
        e2e_ms = max_over_ranks(a.elapsed_time(b))
        # The host's own cost of a call, without back-pressure: in the loop
        # above the host runs ahead until the library's plan copies (four in
        # flight) wait for the GPU, so host_issue equals the step whenever the
        # GPU is the slower side.  Here: bursts of three calls, each burst
        # issued on an idle GPU, median over five bursts.
        bursts = []
        i0 = args.warmup + K
        for bi in range(5):
            torch.cuda.synchronize()
            barrier()
            h1 = time.perf_counter()
            for jj in range(3):
                e2e_step(i0 + 3 * bi + jj)
            bursts.append((time.perf_counter() - h1) * 1e3 / 3)
        torch.cuda.synchronize()
        barrier()
        host_call_ms = max_over_ranks(statistics.median(bursts))
        e2e_kv = sum_over_ranks(sum(r.kv_bytes_at(i) for i in range(args.warmup,
                                                                     args.warmup + K)))
        h2d = sum_over_ranks((qh.numel() + kh.numel() + vh.numel()) * 4)
        d2h = sum_over_ranks(oh.numel() * 4)
        e2e = {"value": round(e2e_kv / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
               "ms_per_step": round(e2e_ms / K, 5), "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h),
               "host_issue_ms_per_step": round(host_ms, 5),
               "host_call_ms": round(host_call_ms, 5),
               "positions": f"advancing: step i appends row T-1+i and attends T+i rows "
                            f"(i = {args.warmup}..{args.warmup + K - 1} timed)",
               "path": ("pinned host q|k|v and attn_out passed to jx_attn_step (C ABI); the "
                        "library copies q|k|v to device memory with one staging kernel and "
                        "the decode kernel writes attn_out over PCIe" if zero_copy else
                        "pinned host q|k|v -> one H2D -> jx_attn_step_sharded (C ABI: partial "
                        "step, ncclAllGather, merge) -> one D2H attn_out")}
        if comm is not None:
            comm.destroy()

    # ---- CPU baseline (rank 0, N=1)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, args.cpu_sample_s)

    if rank != 0:
        return
    peak, peak_src = peaks()
    achieved = r.alg_bytes / (kernel_ms * 1e-3) / 1e9
    traffic = ncu_traffic(f"{w.name}/{w.dtype}") if world == 1 else None
    steps_per_s = K / (elapsed_ms * 1e-3)
    value = total_kv * K / (elapsed_ms * 1e-3) / 1e9
    parallel = ("one GPU" if world == 1 else
                {"replica": f"replicas x{world}",
                 "sequences": f"sequences split over {world} GPUs (LPT)",
                 "positions": f"positions sharded over {world} GPUs + NCCL all-gather"}[r.mode])
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(elapsed_ms / K, 5),
        "steps_per_s": round(steps_per_s, 2), "higher_is_better": True,
        "scaling": "weak" if w.sharding == "replica" else "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1), device-side)",
        "config": dict(w.describe(), parallelism=parallel,
                       l2=("inputs larger than L2: %.0f MB of KV per step per GPU > 126 MB" %
                           (r.kv_bytes / 1e6)) if r.kv_bytes > 126e6 else
                       "KV per step fits in L2 (latency-bound case)",
                       kv_bytes_per_step=int(total_kv), clock_probe_steps=n_probe),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": "jx::decode_kernel", "kernel_ms": round(kernel_ms, 5),
                     "timing": timing,
                     "alg_bytes_per_launch": int(r.alg_bytes), "peak_source": peak_src},
        "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks,
        "gpu_launches": int(r.launches_per_step() * K),
        "sustained": sustained,
    }
    emit(line)


# ----------------------------------------------------------------------------- CPU side

def _host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0)) or 1
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def _cpu_oracle(all_threads: bool = False):
    """(Oracle, kind): the reference build when present, else the C restatement.

    all_threads: use every host thread this process may run on, even where a
    launcher (torchrun sets OMP_NUM_THREADS=1 per rank) asked for fewer -- the
    reference arm's rank 0 is the only rank that works.
    """
    if all_threads:
        os.environ["OMP_NUM_THREADS"] = str(_host_threads())
    else:
        os.environ.setdefault("OMP_NUM_THREADS", str(_host_threads()))
    from oracle.oracle import Oracle, ref_available
    if ref_available():
        return Oracle("ref"), "reference"
    return Oracle("port"), "port"


def _cpu_case(w: W.Workload, n_seqs: int, n_layers: int, rng):
    """Host inputs for n_seqs sequences x n_layers layers of the workload."""
    from oracle.oracle import BF16, F16T, F32
    dt = {"f32": F32, "bf16": BF16, "f16": F16T}[w.dtype]
    lengths = w.lengths[:n_seqs]
    cap = max(lengths)
    shape = (n_seqs, n_layers, cap, w.kv_dim)
    if dt == F32:
        kc = rng.standard_normal(shape, dtype=np.float32)
        vc = rng.standard_normal(shape, dtype=np.float32)
    else:
        kc = (rng.standard_normal(shape, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
        vc = (rng.standard_normal(shape, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
    q = rng.standard_normal((n_seqs, n_layers, w.q_dim), dtype=np.float32)
    k = rng.standard_normal((n_seqs, n_layers, w.kv_dim), dtype=np.float32)
    v = rng.standard_normal((n_seqs, n_layers, w.kv_dim), dtype=np.float32)
    layers = [dict(rope_dim=L.rope_dim, rope_base=L.rope_base, is_swa=int(L.is_swa),
                   shares_kv=0, kv_source_layer=i) for i, L in enumerate(w.layers[:n_layers])]
    return dt, kc, vc, q, k, v, layers, [t - 1 for t in lengths], lengths


def _cpu_sample_shape(w: W.Workload):
    """Sequences x layers of a bounded CPU sample, and its KV bytes."""
    n_seqs = min(len(w.lengths), 2 if w.name in ("c3", "c5") else 1)
    n_layers = w.n_layers if w.name in ("c1", "c2") else min(w.n_layers, 6 if w.name == "c5" else 2)
    if w.name == "c4":
        n_layers = 1
    sub = W.Workload(w.name, w.model, n_layers, w.n_heads, w.n_kv_heads, w.head_dim, w.neox,
                     w.lengths[:n_seqs], w.dtype, layers=w.layers[:n_layers], window=w.window)
    return n_seqs, n_layers, sub.kv_read_bytes()


def cpu_baseline(w: W.Workload, sample_s: float):
    orc, kind = _cpu_oracle()
    n_seqs, n_layers, kv_bytes = _cpu_sample_shape(w)
    rng = np.random.default_rng(W.SEED)
    dt, kc, vc, q, k, v, layers, pos, lengths = _cpu_case(w, n_seqs, n_layers, rng)
    times = []
    t_end = time.time() + sample_s
    while True:
        t0 = time.perf_counter()
        orc.step(kc, vc, dt, pos, layers, q, k, v, w.n_heads, w.n_kv_heads, w.head_dim, w.scale,
                 0.0, w.window, 1.0, w.neox)
        times.append(time.perf_counter() - t0)
        if time.time() > t_end or len(times) >= 200:
            break
    t = statistics.median(times)
    return {"value": round(kv_bytes / t / 1e9, 3), "unit": "GB/s", "cores": orc.max_threads(),
            "kind": kind,
            "sample": f"{n_seqs} seq x {n_layers} layers of {w.name} ({kv_bytes/1e6:.1f} MB KV), "
                      f"median of {len(times)} runs, {t*1e3:.2f} ms each"}


def run_reference(args, rank, world):
    """The reference's own CPU implementation of the step on this host's cores."""
    if rank != 0:
        return
    w = make_workload(args)
    orc, kind = _cpu_oracle(all_threads=True)
    n_seqs, n_layers, kv_bytes = _cpu_sample_shape(w)
    rng = np.random.default_rng(W.SEED)
    dt, kc, vc, q, k, v, layers, pos, lengths = _cpu_case(w, n_seqs, n_layers, rng)

    def one():
        orc.step(kc, vc, dt, pos, layers, q, k, v, w.n_heads, w.n_kv_heads, w.head_dim, w.scale,
                 0.0, w.window, 1.0, w.neox)

    for _ in range(args.warmup):
        one()
    # bound the run to about two minutes: drop layers from the sample if one step is slow
    t0 = time.perf_counter()
    one()
    t1 = time.perf_counter() - t0
    budget = 120.0 / max(1, args.steps)
    if t1 > budget and n_layers > 1:
        n_layers = max(1, int(n_layers * budget / t1))
        sub = W.Workload(w.name, w.model, n_layers, w.n_heads, w.n_kv_heads, w.head_dim, w.neox,
                         lengths, w.dtype, layers=w.layers[:n_layers], window=w.window)
        kv_bytes = sub.kv_read_bytes()
        dt, kc, vc, q, k, v, layers, pos, lengths = _cpu_case(w, n_seqs, n_layers, rng)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    el = time.perf_counter() - t0
    value = kv_bytes * args.steps / el / 1e9
    sample = (f"{n_seqs} seq x {n_layers} layers of {w.name} per step "
              f"({kv_bytes/1e6:.1f} MB KV); full step = {w.kv_read_bytes()/1e6:.1f} MB")
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True,
        # the same key as this config's own arm (a fixed workload is strong scaling)
        "scaling": "weak" if w.sharding == "replica" else "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1))", "impl": "reference",
        "config": dict(w.describe(), parallelism="host CPU, OpenMP over heads"),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": orc.max_threads(),
                         "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)


def _engine_driver() -> str:
    """tests/engine/engine_latency.cpp built against the in-tree library."""
    import shutil
    from jxai_b200 import load_library
    load_library()  # builds libjxattn.so when it is missing or stale
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    lib_dir = os.path.join(ROOT, "jxai_b200")
    src = os.path.join(ROOT, "tests", "engine", "engine_latency.cpp")
    exe = os.path.join(lib_dir, "_build", "engine_latency")
    os.makedirs(os.path.dirname(exe), exist_ok=True)
    cmd = [shutil.which("g++") or "g++", "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(cuda, "include"), src, "-o", exe, "-L", lib_dir, "-ljxattn",
           "-L", os.path.join(cuda, "lib64"), "-lcudart", f"-Wl,-rpath,{lib_dir}",
           f"-Wl,-rpath,{os.path.join(cuda, 'lib64')}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def run_engine(args, rank, world):
    """Per-token attention latency through the C++ engine drop-in.

    forward_token (src/transformer.cpp:2497-2567) runs the block once per
    layer between CPU matmuls, so every layer is a synchronous round trip:
    host q/k/v in, attn_out back.  The driver times whole tokens (all layers)
    with a wall clock, as the reference's attention_ms does (:2499, 2567), for
    both staging modes of jx::AttentionBlock; the reference's own CPU block is
    timed beside it on the same shape.
    """
    if rank != 0:
        return
    w = W.make(args.config, args.dtype)
    if len(w.lengths) != 1 or w.window:
        raise SystemExit("--engine runs the single-sequence full-attention configs (c1, c2, c4)")
    exe = _engine_driver()
    dt = {"f32": 0, "bf16": 1, "f16": 2}[w.dtype]
    T = w.lengths[0]
    res = {}
    for mode in ("pinned", "copies"):
        cmd = [exe, str(dt), str(T), str(w.n_layers), str(w.n_heads), str(w.n_kv_heads),
               str(w.head_dim), str(int(w.neox)), repr(float(w.layers[0].rope_base)),
               str(args.tokens), str(max(3, args.warmup)), mode]
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
        if r.returncode != 0:
            raise RuntimeError(f"engine driver failed ({mode}): {r.stderr.strip()}")
        res[mode] = json.loads(r.stdout.strip().splitlines()[-1])
    cpu = None
    if not args.no_cpu_baseline:
        c = cpu_baseline(w, args.cpu_sample_s)
        # the CPU sample's KV GB/s over a whole token's KV bytes: its attention_ms
        c["value"] = round(w.kv_read_bytes() / (c["value"] * 1e9) * 1e3, 4)
        c["unit"] = "ms per token"
        cpu = c
    best = min(res.values(), key=lambda d: d["ms_per_token"])
    line = {
        "metric": "engine attention ms per token", "value": best["ms_per_token"], "unit": "ms",
        "n_gpus": 1, "tokens": args.tokens, "higher_is_better": False, "dtype": "f32",
        "data": "synthetic (seeded N(0,1))",
        "config": dict(w.describe(), path="jx::AttentionBlock::forward once per layer on host "
                       "vectors, synchronised per layer (forward_token's call pattern)"),
        "staging": res, "cpu_baseline": cpu,
        "kv_gbs": round(w.kv_read_bytes() / (best["ms_per_token"] * 1e-3) / 1e9, 2),
    }
    emit(line)


def run_prefill(args, rank, world):
    """Prompt throughput: one prompt of --prefill tokens per jx_attn_prefill call.

    jxai feeds a prompt token by token through forward_token
    (src/transformer.cpp:3092-3095): each token appends its row and attends
    over every earlier one.  jx_attn_prefill takes the whole prompt in one
    call (every row appended, then each token attends causally).  The
    reference's own token-serial CPU loop is timed beside it on the last
    tokens of the same prompt (the cache rows before them filled with seeded
    values) and projected to the whole prompt by the rows it reads.
    """
    if rank != 0:
        return
    import torch
    import jxai_b200 as jx
    w = W.make(args.config, args.dtype)
    if w.window:
        raise SystemExit("--prefill runs the full-attention configs (c1..c4)")
    N = args.prefill
    w.lengths = [N]  # the prompt: positions 0 .. N-1
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    cache = jx.KVCache(1, w.n_layers, N, w.kv_dim, w.dtype, 0)
    for opt in args.set:
        key, _, val = opt.partition("=")
        cache.set_option(key, int(val))
    q = torch.empty(N, w.n_layers, w.q_dim, device=dev)
    k = torch.empty(N, w.n_layers, w.kv_dim, device=dev)
    v = torch.empty_like(k)
    jx.fill_normal(q, W.SEED, 3)
    jx.fill_normal(k, W.SEED, 4)
    jx.fill_normal(v, W.SEED, 5)
    out = torch.empty_like(q)
    pos = list(range(N))

    def call():
        jx.attn_prefill(cache, w.layers, q, k, v, out, pos, w.n_heads, w.n_kv_heads,
                        scale=w.scale, neox=w.neox)

    for _ in range(max(3, args.warmup)):
        call()
    torch.cuda.synchronize()
    K = max(1, min(args.steps, 50))
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(K):
        call()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / K
    if cache.check_device_error():
        raise RuntimeError("device error during the prefill timing")
    launches = cache.last_launch_count() + 1  # the append launch is not counted there
    opts = dict(o.partition("=")[::2] for o in args.set)
    tc = (w.dtype in ("bf16", "f16") and w.head_dim in (64, 128)
          and int(opts.get("prefill_tc", "1")) != 0 and w.n_heads // w.n_kv_heads in (1, 2, 4, 8))
    roof = None
    if tc:
        # causal attention from position 0: token t reads t+1 rows; QK^T and
        # PV are 2*head_dim flops per (row, head) each
        rows = N * (N + 1) // 2
        flops = 4.0 * w.head_dim * rows * w.n_heads * w.n_layers
        achieved = flops / (ms * 1e-3) / 1e12
        peak, src = tensor_peak()
        roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                "traffic": ncu_traffic(f"prefill/{w.name}/{w.dtype}/{N}"),
                "kernel": "jx::prefill_tc_kernel", "kernel_ms": round(ms, 4),
                "alg_flops_per_call": flops,
                "issued_tflops": round(2 * achieved, 2),
                "note": "achieved counts the causal attention's own flops; q and p go through "
                        "the tensor pipe as two 16-bit parts each, so the pipe issues twice "
                        "that (issued_tflops), plus the masked halves of diagonal tiles. "
                        "kernel_ms is the whole call: the append launch before the attention "
                        "launch is 7.5% of it in the ncu launch list of the head_dim-128 shape.",
                "peak_source": src}

    cpu = None
    if not args.no_cpu_baseline:
        from oracle.oracle import BF16, F16T, F32
        orc, kind = _cpu_oracle()
        dt = {"f32": F32, "bf16": BF16, "f16": F16T}[w.dtype]
        rng = np.random.default_rng(W.SEED)
        shape = (1, w.n_layers, N, w.kv_dim)
        if dt == F32:
            kc = rng.standard_normal(shape, dtype=np.float32)
            vc = rng.standard_normal(shape, dtype=np.float32)
        else:
            kc = (rng.standard_normal(shape, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
            vc = (rng.standard_normal(shape, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
        qh = rng.standard_normal((N, w.n_layers, w.q_dim), dtype=np.float32)
        kh = rng.standard_normal((N, w.n_layers, w.kv_dim), dtype=np.float32)
        vh = rng.standard_normal((N, w.n_layers, w.kv_dim), dtype=np.float32)
        layers = [dict(rope_dim=L.rope_dim, rope_base=L.rope_base, is_swa=0, shares_kv=0,
                       kv_source_layer=i) for i, L in enumerate(w.layers)]

        def token(t):
            orc.step(kc, vc, dt, [t], layers, qh[t][None], kh[t][None], vh[t][None], w.n_heads,
                     w.n_kv_heads, w.head_dim, w.scale, 0.0, 0, 1.0, w.neox)

        token(N - 1)  # warm-up (thread pool, pages)
        t0 = time.perf_counter()
        token(N - 1)
        one = time.perf_counter() - t0
        n_s = int(min(N, max(1, args.cpu_sample_s / max(one, 1e-6))))
        t0 = time.perf_counter()
        for t in range(N - n_s, N):
            token(t)
        el = time.perf_counter() - t0
        rows_sample = sum(t + 1 for t in range(N - n_s, N))
        rows_full = N * (N + 1) // 2
        cpu_ms = el * 1e3 * rows_full / rows_sample
        cpu = {"value": round(N / (cpu_ms * 1e-3), 2), "unit": "tokens/s",
               "ms_per_prompt": round(cpu_ms, 2), "cores": orc.max_threads(), "kind": kind,
               "sample": f"token-serial loop over the last {n_s} of {N} positions "
                         f"({el:.2f} s), projected to the whole prompt by rows read"}
    line = {
        "metric": "prefill tokens/s", "value": round(N / (ms * 1e-3), 1), "unit": "tokens/s",
        "n_gpus": 1, "steps": K, "warmup": max(3, args.warmup), "ms_per_prompt": round(ms, 4),
        "higher_is_better": True, "dtype": "f32", "data": "synthetic (seeded N(0,1), device-side)",
        "config": dict(w.describe(), prompt_tokens=N,
                       path=("jx_attn_prefill: the whole prompt per call (append launch, then "
                             "causal attention on the tensor cores: 128/G tokens x G heads per "
                             "tile, tcgen05 MMAs with TMEM accumulators, K/V tiles shared by "
                             "the tile)") if tc else
                            ("jx_attn_prefill: the whole prompt per call (append launch, then "
                             "causal attention; 8/G consecutive tokens share a pass over their "
                             "rows)")),
        "gpu_launches": launches * K, "cpu_baseline": cpu, "roofline": roof,
    }
    emit(line)


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.engine:
        run_engine(args, rank, world)
        return
    if args.prefill > 0:
        run_prefill(args, rank, world)
        return
    import torch
    import torch.distributed as dist
    if world > 1:
        # stdout must hold the one JSON line: file descriptor 1 goes to
        # stderr for the whole run (NCCL's communicator lines, libraries and
        # prints alike) and the JSON line is written to the saved stdout
        global _JSON_FD
        sys.stdout.flush()
        _JSON_FD = os.dup(1)
        os.dup2(2, 1)
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
