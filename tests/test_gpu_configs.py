"""Oracle parity on the five benchmark workloads at their stated sizes.

Each case builds the workload exactly as ``bench.py`` does (its ``Runner``:
device-side seeded fill of the cache, q, k and v; one plan of the whole step),
runs one decode step on cuda:0, copies back the checked subset -- every cache
row a checked (sequence, layer) attends, after the step -- and runs the CPU
oracle on those exact bytes.  The step writes only row pos = T-1 of each
(sequence, layer), so the rows before it are the seeded fill; the oracle
appends row T-1 itself from the same q/k/v and attends over it.

Bars (src/transformer.cpp:2512-2566):
  * the appended K and V rows are bit-exact with the oracle's append;
  * attention within max-abs 1e-4 of the oracle on the same stored cache
    values (fp32 and bf16 caches alike);
  * bf16 cache: within 2e-2 of the fp32 attention over the unrounded values
    (rebuilt on the host from the fill's generator).

Sizes: c1 whole step; c2 all 16 layers x 4096 rows; c3 (fp32 and bf16, 256
ragged sequences up to 8192 rows, 137 / 69 GB of cache) every layer of the 3
longest and 3 shortest sequences plus 2 layers of all 256; c4 (one 131072-row
sequence, 32 layers, 34 GB) 3 layers; c5 (64 x 16384 rows, 26 layers with the
5:1 sliding-window pattern, 56 GB) all layers of 4 sequences.
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-4
TOL_BF16_VS_F32 = 2e-2


def _oracle():
    from oracle.oracle import Oracle, ref_available
    # the reference's own build where it travelled with the tree, else the restatement
    return Oracle("ref") if ref_available() else Oracle("port")


def _run_step(name, dtype):
    import torch
    import bench
    from jxai_b200 import workloads as W
    torch.cuda.set_device(0)
    w = W.make(name, dtype)
    r = bench.Runner(w, 0, 1, 0)
    try:
        r.out.fill_(float("nan"))
        r.step()
        torch.cuda.synchronize()
        assert r.cache.check_device_error() == 0
        host = dict(q=r.q.cpu().numpy(), k=r.k.cpu().numpy(), v=r.v.cpu().numpy(),
                    out=r.out.cpu().numpy())
        assert np.isfinite(host["out"]).all()
    except BaseException:
        r.cache.close()  # a failed case must not keep tens of GB for the next one
        raise
    return w, r, host


def _check_pairs(w, r, host, checks, orc, f32_ref=False):
    """checks: list of (sequence index, [layers]).  Returns the worst errors."""
    from oracle.oracle import BF16, F16T, F32
    from tests.helpers import normal_at
    from jxai_b200 import workloads as W
    dt = {"f32": F32, "bf16": BF16, "f16": F16T}[w.dtype]
    worst, worst_f32 = 0.0, 0.0
    cap = r.cache.capacity
    for s, layer_list in checks:
        T = w.lengths[s]
        pos = T - 1
        for l in layer_list:
            kc = r.cache.read_rows(s, l, 0, 0, T)[None, None]
            vc = r.cache.read_rows(s, l, 1, 0, T)[None, None]
            ko, vo = kc.copy(), vc.copy()
            L = w.layers[l]
            lay = [dict(rope_dim=L.rope_dim, rope_base=L.rope_base, is_swa=int(L.is_swa),
                        shares_kv=0, kv_source_layer=0)]
            q = host["q"][s:s + 1, l:l + 1]
            k = host["k"][s:s + 1, l:l + 1]
            v = host["v"][s:s + 1, l:l + 1]
            ref = orc.step(ko, vo, dt, [pos], lay, q, k, v, w.n_heads, w.n_kv_heads, w.head_dim,
                           w.scale, 0.0, w.window, 1.0, w.neox)
            # the appended row (and, trivially, every row before it) bit-exact
            assert np.array_equal(ko.view(np.uint8), kc.view(np.uint8)), (w.name, s, l, "K")
            assert np.array_equal(vo.view(np.uint8), vc.view(np.uint8)), (w.name, s, l, "V")
            got = host["out"][s, l]
            err = float(np.abs(got - ref[0, 0]).max())
            assert err <= TOL, f"{w.name}/{w.dtype} seq {s} layer {l}: max-abs {err}"
            worst = max(worst, err)
            if f32_ref:
                # the fp32 values the fill rounded into the bf16 cache (the
                # flat element index of row t is ((s*layers + l)*cap + t)*rs + c)
                rs = w.kv_dim
                base = ((s * w.n_layers + l) * cap) * rs
                idx = base + np.arange((T - 1) * rs, dtype=np.uint64)
                kf = np.zeros((1, 1, T, rs), np.float32)
                vf = np.zeros((1, 1, T, rs), np.float32)
                kf[0, 0, :T - 1] = normal_at(W.SEED, 1, idx).reshape(T - 1, rs)
                vf[0, 0, :T - 1] = normal_at(W.SEED, 2, idx).reshape(T - 1, rs)
                ref32 = orc.step(kf, vf, F32, [pos], lay, q, k, v, w.n_heads, w.n_kv_heads,
                                 w.head_dim, w.scale, 0.0, w.window, 1.0, w.neox)
                e32 = float(np.abs(got - ref32[0, 0]).max())
                assert e32 <= TOL_BF16_VS_F32, f"{w.name} bf16 vs fp32 seq {s} layer {l}: {e32}"
                worst_f32 = max(worst_f32, e32)
    return worst, worst_f32


def test_c1_whole_step():
    w, r, host = _run_step("c1", None)
    try:
        _check_pairs(w, r, host, [(0, list(range(w.n_layers)))], _oracle())
    finally:
        r.cache.close()


def test_c2_all_layers_4096():
    w, r, host = _run_step("c2", None)
    try:
        _check_pairs(w, r, host, [(0, list(range(w.n_layers)))], _oracle())
    finally:
        r.cache.close()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_c3_ragged_256_sequences(dtype):
    w, r, host = _run_step("c3", dtype)
    try:
        order = sorted(range(len(w.lengths)), key=lambda i: (w.lengths[i], i))
        every_layer = order[:3] + order[-3:]
        checks = [(s, list(range(w.n_layers))) for s in every_layer]
        checks += [(s, [0, w.n_layers - 1]) for s in range(len(w.lengths)) if s not in every_layer]
        orc = _oracle()
        _check_pairs(w, r, host, checks, orc)
        if dtype == "bf16":
            # fp32 reference of the unrounded values: the longest and the shortest sequence
            _check_pairs(w, r, host, [(order[-1], [0, 7]), (order[0], [15])], orc, f32_ref=True)
    finally:
        r.cache.close()


def test_c4_131072_positions():
    w, r, host = _run_step("c4", None)
    try:
        _check_pairs(w, r, host, [(0, [0, 13, w.n_layers - 1])], _oracle())
    finally:
        r.cache.close()


def test_c5_mixed_window_64_sequences():
    w, r, host = _run_step("c5", None)
    try:
        assert w.window == 512 and len(w.layers) == 26
        assert [l for l, L in enumerate(w.layers) if not L.is_swa] == [5, 11, 17, 23]
        _check_pairs(w, r, host, [(s, list(range(w.n_layers))) for s in (0, 21, 42, 63)], _oracle())
    finally:
        r.cache.close()
