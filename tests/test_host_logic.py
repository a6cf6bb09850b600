"""Host-side logic: workload definitions, byte accounting, partitioning, the
slice planner, and sanitizer (ASan + UBSan) runs of the planner and the CPU oracle."""
import numpy as np
import pytest

from jxai_b200 import workloads as W


def test_workload_shapes_and_kv_bytes():
    # algorithmic KV bytes per step of the benchmark configs (fp32 cache)
    assert W.make("c1").kv_read_bytes() == 24 * 512 * 128 * 2 * 4
    assert W.make("c2").kv_read_bytes() == 16 * 4096 * 512 * 8 == 268435456
    assert W.make("c4").kv_read_bytes() == 32 * 131072 * 1024 * 8
    c5 = W.make("c5")
    assert c5.kv_read_bytes() == 64 * (4 * 16384 + 22 * 512) * 256 * 8
    assert [l for l in range(26) if not c5.layers[l].is_swa] == [5, 11, 17, 23]
    assert W.make("c3", "bf16").kv_read_bytes() * 2 == W.make("c3").kv_read_bytes()


def test_rope_styles_follow_the_reference_arch_table():
    # src/transformer.cpp:140-179: qwen2/gemma3 Neox, llama (Llama-3.2, Mistral) interleaved
    assert W.make("c1").neox and W.make("c5").neox
    assert not W.make("c2").neox and not W.make("c3").neox and not W.make("c4").neox


def test_c3_lengths_are_seeded_and_in_range():
    a, b = W.c3_lengths(), W.c3_lengths()
    assert a == b and len(a) == 256
    assert min(a) >= 128 and max(a) <= 8192
    assert abs(np.mean(a) - 4160) < 400


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_lpt_partition_balances_ragged_sequences(n):
    T = W.c3_lengths()
    parts = W.lpt_partition(T, n)
    assert sorted(i for p in parts for i in p) == list(range(256))
    loads = [sum(T[i] for i in p) for p in parts]
    assert max(loads) / (sum(T) / n) < 1.01


@pytest.mark.parametrize("n", [1, 2, 3, 8])
def test_position_shards_cover_the_sequence(n):
    sh = W.position_shards(131072, n)
    assert sh[0][0] == 0 and sh[-1][1] == 131072
    assert all(a[1] == b[0] for a, b in zip(sh, sh[1:]))
    assert max(e - b for b, e in sh) - min(e - b for b, e in sh) <= 1


@pytest.mark.parametrize("name,mode", [("c4", "positions"), ("c3", "sequences"),
                                       ("c5", "sequences"), ("c2", "replica")])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_rank_kv_bytes_add_up_to_the_step(name, mode, world):
    # the ranks' shares of a step (the bench's value and its e2e leg, whose
    # steps advance by one row each) add up to the whole step's KV bytes
    w = W.make(name)
    for shift in (0, 1, 7, 220):
        total = sum(W.rank_kv_bytes(w, mode, r, world, shift) for r in range(world))
        whole = w.kv_read_bytes([t + shift for t in w.lengths])
        assert total == (whole * world if mode == "replica" else whole), (shift, total, whole)


def test_slice_planner_boundaries_and_layout_forms(tmp_path):
    # jx::balanced_split (jxai_b200/csrc/jx_plan.h) sizes the persistent CTAs'
    # slices of a step; built with g++ alone and checked on seeded random
    # layouts (tests/host/plan_check.cpp)
    import os
    import shutil
    import subprocess
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("g++ not available")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    exe = str(tmp_path / "plan_check")
    subprocess.run([cxx, "-std=c++17", "-O2", "-Wall", "-I", os.path.join(root, "jxai_b200", "csrc"),
                    os.path.join(root, "tests", "host", "plan_check.cpp"), "-o", exe],
                   check=True, capture_output=True, text=True)
    r = subprocess.run([exe, "20000"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("ok ")


def _san_flags():
    return ["-g", "-O1", "-fsanitize=address,undefined,float-cast-overflow",
            "-fno-sanitize-recover=all"]


def test_oracle_under_sanitizers(tmp_path):
    # the CPU oracle built with AddressSanitizer + UndefinedBehaviorSanitizer
    # (OpenMP on) and run over every exported function (tests/host/oracle_san.c)
    import os
    import shutil
    import subprocess
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("gcc not available")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    exe = str(tmp_path / "oracle_san")
    subprocess.run([cc, "-std=c11", "-ffp-contract=off", "-fopenmp", *_san_flags(),
                    os.path.join(root, "oracle", "jx_oracle.c"),
                    os.path.join(root, "tests", "host", "oracle_san.c"), "-o", exe, "-lm"],
                   check=True, capture_output=True, text=True)
    env = dict(os.environ, OMP_NUM_THREADS="4")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout + r.stderr[-3000:]
    assert r.stdout.startswith("ok ")


def test_slice_planner_under_sanitizers(tmp_path):
    import os
    import shutil
    import subprocess
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("g++ not available")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    exe = str(tmp_path / "plan_check_san")
    subprocess.run([cxx, "-std=c++17", *_san_flags(), "-I", os.path.join(root, "jxai_b200", "csrc"),
                    os.path.join(root, "tests", "host", "plan_check.cpp"), "-o", exe],
                   check=True, capture_output=True, text=True)
    r = subprocess.run([exe, "3000"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr[-3000:]
    assert r.stdout.startswith("ok ")
