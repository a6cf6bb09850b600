"""The C++ engine drop-in (include/jx_engine.hpp) driven like forward_token.

tests/engine/drop_in_driver.cpp is built with g++ against libjxattn.so and runs
a token stream through jx::KVCacheSlot + jx::AttentionBlock on host vectors:
per token the slot compacts on overflow (transformer.cpp:2373-2375), every
layer runs the attention block (:2497-2567), seq_pos advances (:2792); a prefix
reuse rolls the slot back (:3071-3089).  The batched forms run several slots
per layer call (forward_batch) and a whole prompt per layer call
(forward_prompt).  The test replays the same script through the CPU oracle,
one token at a time per slot (fp16-truncated cache, the reference's native
type), and compares every layer's attn_out, then each slot's final seq_pos and
compaction count.  The compile-only check runs without a GPU.
"""
import math
import os
import shutil
import subprocess
import tempfile

import numpy as np
import pytest

from oracle.oracle import F16T, Oracle
from tests.helpers import layer_dicts

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DRIVER = os.path.join(ROOT, "tests", "engine", "drop_in_driver.cpp")
LATENCY = os.path.join(ROOT, "tests", "engine", "engine_latency.cpp")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")

# the toy GGUF's shape (models/qwen_run.gguf in the reference): 4 layers,
# 4 query heads, 2 kv heads, head_dim 32, Neox RoPE
L, H, HK, HD, CAP, THETA = 4, 4, 2, 32, 64, 1e6
TOL = 1e-4


def _compile(out_path, syntax_only=False, src=DRIVER):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("g++ not available")
    cmd = [cxx, "-std=c++17", "-O2", "-Wall", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA_HOME, "include"), src]
    if syntax_only:
        cmd += ["-fsyntax-only"]
    else:
        lib_dir = os.path.join(ROOT, "jxai_b200")
        cmd += ["-o", out_path, "-L", lib_dir, "-ljxattn",
                "-L", os.path.join(CUDA_HOME, "lib64"), "-lcudart",
                f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{os.path.join(CUDA_HOME, 'lib64')}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)


def test_engine_header_and_driver_compile():
    if not os.path.exists(os.path.join(CUDA_HOME, "include", "cuda_runtime.h")):
        pytest.skip("CUDA headers not available")
    _compile(None, syntax_only=True)
    _compile(None, syntax_only=True, src=LATENCY)


@pytest.mark.gpu
@pytest.mark.parametrize("staging", ["pinned", "copies"])
def test_engine_latency_driver_runs(staging):
    # the per-token latency driver bench.py --engine uses: a few tokens of a
    # small shape, both staging modes; it checks the device error word itself
    import json
    import jxai_b200 as jx
    jx.load_library()
    with tempfile.TemporaryDirectory() as td:
        exe = os.path.join(td, "latency")
        _compile(exe, src=LATENCY)
        r = subprocess.run([exe, "2", "300", "3", "8", "2", "64", "1", "10000", "4", "2", staging],
                           capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["tokens"] == 4 and d["staging"] == staging and d["ms_per_token"] > 0


def _tok(rng, n=None):
    """q, k, v for one token (n None) or n rows of one layer-major op."""
    shape = (L,) if n is None else (L, n)
    return (rng.standard_normal(shape + (H * HD,)).astype(np.float32),
            rng.standard_normal(shape + (HK * HD,)).astype(np.float32),
            rng.standard_normal(shape + (HK * HD,)).astype(np.float32))


def _write_script(path, n_slots, ops):
    """ops: ("tok", slot, (q, k, v)) | ("lcp", slot, lcp) |
    ("batch", [slots], (q, k, v) of [L][m][..]) | ("prompt", slot, (q, k, v) of [L][n][..])"""
    with open(path, "wb") as f:
        np.array([L, H, HK, HD, CAP, 1, F16T, n_slots, len(ops)], dtype=np.int32).tofile(f)
        np.array([THETA], dtype=np.float32).tofile(f)
        for op in ops:
            kind = op[0]
            if kind == "lcp":
                np.array([2, op[1], op[2]], dtype=np.int32).tofile(f)
                continue
            if kind == "tok":
                np.array([1, op[1]], dtype=np.int32).tofile(f)
            elif kind == "batch":
                np.array([3, len(op[1])] + list(op[1]), dtype=np.int32).tofile(f)
            else:
                np.array([4, op[1], op[2][0].shape[1]], dtype=np.int32).tofile(f)
            q, k, v = op[2]
            for l in range(L):
                q[l].tofile(f)
                k[l].tofile(f)
                v[l].tofile(f)


def _run_driver(n_slots, ops, staging="pinned"):
    import jxai_b200 as jx
    jx.load_library()  # builds the library if needed
    with tempfile.TemporaryDirectory() as td:
        exe = os.path.join(td, "driver")
        _compile(exe)
        script, outp = os.path.join(td, "script.bin"), os.path.join(td, "out.bin")
        _write_script(script, n_slots, ops)
        r = subprocess.run([exe, script, outp, staging], capture_output=True, text=True,
                           timeout=300)
        assert r.returncode == 0, r.stderr
        got = np.fromfile(outp, dtype=np.uint8)
    tail = got[len(got) - 8 * n_slots:].view(np.int32).reshape(n_slots, 2)
    return got[: len(got) - 8 * n_slots].view(np.float32), tail


def _replay(n_slots, ops):
    """The same ops through the oracle, one token at a time per slot, with
    forward_token's compaction on overflow; returns the attn_out rows in the
    driver's output order and per-slot (seq_pos, compactions)."""
    import jxai_b200 as jx
    orc = Oracle("port")
    rs = HK * HD
    kc = np.zeros((n_slots, L, CAP, rs), dtype=np.uint16)
    vc = np.zeros((n_slots, L, CAP, rs), dtype=np.uint16)
    layers = layer_dicts([jx.Layer(HD, HD, THETA, l) for l in range(L)])
    seq_pos = [0] * n_slots
    comp = [0] * n_slots
    scale = 1 / math.sqrt(HD)

    def one(s, q, k, v):   # q [L][H*HD]: one token of slot s through all layers
        if seq_pos[s] >= CAP:
            new = orc.compact(kc[s], vc[s], F16T, seq_pos[s], CAP // 2)
            comp[s] += int(new != seq_pos[s])
            seq_pos[s] = new
        o = orc.step(kc[s:s + 1], vc[s:s + 1], F16T, [seq_pos[s]], layers, q[None], k[None],
                     v[None], H, HK, HD, scale, neox=True)[0]
        seq_pos[s] += 1
        return o             # [L][H*HD]

    chunks = []
    for op in ops:
        kind = op[0]
        if kind == "lcp":
            seq_pos[op[1]] = min(seq_pos[op[1]], op[2])
        elif kind == "tok":
            chunks.append(one(op[1], *op[2]).reshape(-1))
        else:
            slots = op[1] if kind == "batch" else [op[1]] * op[2][0].shape[1]
            q, k, v = op[2]
            outs = np.stack([one(s, q[:, i], k[:, i], v[:, i]) for i, s in enumerate(slots)],
                            axis=1)   # [L][rows][H*HD]
            chunks.append(outs.reshape(-1))
    return np.concatenate(chunks), np.array(list(zip(seq_pos, comp)), dtype=np.int32)


@pytest.mark.gpu
@pytest.mark.parametrize("staging", ["pinned", "copies"])
def test_engine_drop_in_matches_oracle_over_a_token_stream(staging):
    # 50 tokens, prefix reuse back to 30, 60 more tokens (crosses the 64-row
    # capacity: one compaction); slot 1 of 2, so the slot id reaches the library.
    # Both staging modes of the block: pinned host rows read/written by the
    # library, and device copies through cudaMemcpyAsync.
    rng = np.random.default_rng(2024)
    ops = [("tok", 1, _tok(rng)) for _ in range(50)] + [("lcp", 1, 30)]
    ops += [("tok", 1, _tok(rng)) for _ in range(60)]
    got, tail = _run_driver(2, ops, staging)
    ref, ref_tail = _replay(2, ops)
    assert np.abs(got - ref).max() <= TOL
    assert (tail == ref_tail).all() and tail[1, 1] == 1


@pytest.mark.gpu
@pytest.mark.parametrize("staging", ["pinned", "copies"])
def test_engine_batched_slots_and_prompts_match_oracle(staging):
    # four slots: prompts of different lengths (forward_prompt), then batched
    # decode over changing subsets of slots (forward_batch), a rollback, and
    # enough batched tokens that two slots compact on overflow
    rng = np.random.default_rng(77)
    ops = [("prompt", 0, _tok(rng, 21)), ("prompt", 2, _tok(rng, 40)),
           ("tok", 3, _tok(rng)), ("prompt", 3, _tok(rng, 9))]
    for i in range(30):
        ids = [0, 1, 2, 3] if i % 3 else [2, 0]
        ops.append(("batch", ids, _tok(rng, len(ids))))
    ops.append(("lcp", 0, 12))
    ops.append(("prompt", 0, _tok(rng, 6)))
    for _ in range(8):
        ops.append(("batch", [3, 2, 1, 0], _tok(rng, 4)))
    got, tail = _run_driver(4, ops, staging)
    ref, ref_tail = _replay(4, ops)
    assert got.shape == ref.shape
    assert np.abs(got - ref).max() <= TOL
    assert (tail == ref_tail).all()
    assert tail[:, 1].sum() >= 1   # at least one slot compacted inside a batch
