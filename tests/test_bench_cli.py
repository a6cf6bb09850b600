"""bench.py's reference arm on the CPU: the JSON line the driver reads.

`bench.py --impl reference` times the reference's own CPU implementation of
the step (oracle/_ref when built, else the C restatement) and prints one JSON
line with the same metric, unit and config as the GPU arm.  Under torchrun
only rank 0 works and prints; the other ranks exit 0.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _check_line(d, n_gpus, workload):
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["metric"] == "decode-attn KV-read HBM GB/s" and d["unit"] == "GB/s"
    assert d["value"] > 0 and d["higher_is_better"] is True and d["n_gpus"] == n_gpus
    assert d["config"]["workload"] == workload
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("reference", "port") and cb["cores"] >= 1
    assert cb["sample"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def _json_lines(out):
    return [json.loads(ln) for ln in out.splitlines() if ln.startswith("{")]


def test_reference_arm_prints_one_json_line():
    # the default workload: c4, one layer of the 131072-row context per step
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--steps", "2", "--warmup", "3"],
                       capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    _check_line(lines[0], 1, "c4")


def test_reference_arm_under_torchrun_rank0_only():
    # torchrun sets OMP_NUM_THREADS=1 per rank; the reference arm's rank 0 uses
    # every host thread all the same
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", "29561",
           os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "2",
           "--warmup", "3", "--config", "c2"]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=ROOT)
    except subprocess.TimeoutExpired:
        pytest.fail("torchrun reference arm did not finish")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    _check_line(lines[0], 2, "c2")
    assert lines[0]["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))
