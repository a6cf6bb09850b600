"""The C++ engine drop-in (include/jx_engine.hpp) driven like forward_token.

tests/engine/drop_in_driver.cpp is built with g++ against libjxattn.so and runs
a token stream through jx::KVCacheSlot + jx::AttentionBlock on host vectors:
per token the slot compacts on overflow (transformer.cpp:2373-2375), every
layer runs the attention block (:2497-2567), seq_pos advances (:2792); a prefix
reuse rolls the slot back (:3071-3089).  The test replays the same script
through the CPU oracle (fp16-truncated cache, the reference's native type) and
compares every layer's attn_out, then the final seq_pos and compaction count.
The compile-only check runs without a GPU.
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
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")

# the toy GGUF's shape (models/qwen_run.gguf in the reference): 4 layers,
# 4 query heads, 2 kv heads, head_dim 32, Neox RoPE
L, H, HK, HD, CAP, THETA = 4, 4, 2, 32, 64, 1e6
TOL = 1e-4


def _compile(out_path, syntax_only=False):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("g++ not available")
    cmd = [cxx, "-std=c++17", "-O2", "-Wall", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA_HOME, "include"), DRIVER]
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


def _script(rng):
    """Ops: 50 tokens, prefix reuse back to 30, 60 more tokens (crosses the
    64-row capacity: one compaction)."""
    ops = [("tok",)] * 50 + [("lcp", 30)] + [("tok",)] * 60
    tokens = []
    for op in ops:
        if op[0] == "tok":
            tokens.append((rng.standard_normal((L, H * HD)).astype(np.float32),
                           rng.standard_normal((L, HK * HD)).astype(np.float32),
                           rng.standard_normal((L, HK * HD)).astype(np.float32)))
    return ops, tokens


def _write_script(path, ops, tokens):
    with open(path, "wb") as f:
        np.array([L, H, HK, HD, CAP, 1, F16T, len(ops)], dtype=np.int32).tofile(f)
        np.array([THETA], dtype=np.float32).tofile(f)
        it = iter(tokens)
        for op in ops:
            if op[0] == "lcp":
                np.array([2, op[1]], dtype=np.int32).tofile(f)
                continue
            q, k, v = next(it)
            np.array([1], dtype=np.int32).tofile(f)
            for l in range(L):
                q[l].tofile(f)
                k[l].tofile(f)
                v[l].tofile(f)


@pytest.mark.gpu
def test_engine_drop_in_matches_oracle_over_a_token_stream():
    import jxai_b200 as jx
    jx.load_library()  # builds the library if needed
    rng = np.random.default_rng(2024)
    ops, tokens = _script(rng)
    with tempfile.TemporaryDirectory() as td:
        exe = os.path.join(td, "driver")
        _compile(exe)
        script, outp = os.path.join(td, "script.bin"), os.path.join(td, "out.bin")
        _write_script(script, ops, tokens)
        r = subprocess.run([exe, script, outp], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr
        got = np.fromfile(outp, dtype=np.uint8)
    n_tok = len(tokens)
    body = got[: n_tok * L * H * HD * 4].view(np.float32).reshape(n_tok, L, H * HD)
    seq_pos_dev, compactions_dev = got[n_tok * L * H * HD * 4:].view(np.int32)

    # replay through the oracle
    orc = Oracle("port")
    rs = HK * HD
    kc = np.zeros((1, L, CAP, rs), dtype=np.uint16)
    vc = np.zeros((1, L, CAP, rs), dtype=np.uint16)
    layers = [jx.Layer(HD, HD, THETA, l) for l in range(L)]
    seq_pos, compactions, t = 0, 0, 0
    worst = 0.0
    for op in ops:
        if op[0] == "lcp":
            seq_pos = min(seq_pos, op[1])
            continue
        if seq_pos >= CAP:
            new = orc.compact(kc[0], vc[0], F16T, seq_pos, CAP // 2)
            compactions += int(new != seq_pos)
            seq_pos = new
        q, k, v = tokens[t]
        ref = orc.step(kc, vc, F16T, [seq_pos], layer_dicts(layers), q[None], k[None], v[None],
                       H, HK, HD, 1 / math.sqrt(HD), neox=True)
        worst = max(worst, float(np.abs(body[t] - ref[0]).max()))
        seq_pos += 1
        t += 1
    assert worst <= TOL, worst
    assert seq_pos_dev == seq_pos and compactions_dev == compactions == 1
