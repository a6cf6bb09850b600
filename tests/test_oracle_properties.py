"""Properties of the CPU oracle's attention step that hold whatever the inputs.

The golden fixtures pin the C restatement (oracle/jx_oracle.c) to the
reference's own outputs; these checks pin what the attention block of
forward_token (src/transformer.cpp:2522-2566) must satisfy by construction,
on random shapes: softmax weights sum to one (every V row equal to c gives c
for every head), equal scores weigh every attended row alike (all-zero keys
give the mean of the attended V rows, windows included), and the step writes
exactly one row per layer.
"""
import numpy as np
import pytest
from hypothesis import given, settings, strategies as st

from oracle.oracle import BF16, F16T, F32, Oracle

DTYPES = (F32, BF16, F16T)


def _enc(x, dtype):
    """float32 values -> the cache's storage (exact for the values used here)."""
    if dtype == F32:
        return x.astype(np.float32)
    if dtype == BF16:
        return (x.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    return x.astype(np.float16).view(np.uint16)


def _layers(n_layers, hd, swa_first):
    return [dict(rope_dim=hd, rope_base=1e4 if l == 0 else 1e6, is_swa=int(swa_first and l == 0),
                 shares_kv=0, kv_source_layer=l) for l in range(n_layers)]


shapes = st.tuples(st.sampled_from([(4, 2), (8, 2), (7, 1), (4, 4), (6, 3)]),
                   st.sampled_from([32, 64, 128]),
                   st.integers(min_value=1, max_value=70),      # T (attended rows)
                   st.sampled_from(DTYPES),
                   st.booleans(),                               # Neox
                   st.sampled_from([0, 1, 16]))                 # sliding window


@settings(max_examples=60, deadline=None)
@given(shapes, st.integers(0, 2**31 - 1))
def test_constant_values_give_that_value(shape, seed):
    (H, HK), hd, T, dtype, neox, window = shape
    rng = np.random.default_rng(seed)
    L, cap = 2, T + 2
    # one constant vector per (layer, kv head), stored in every row and as the new v
    c = np.round(rng.standard_normal((L, HK, hd)) * 4) / 4   # exact in every cache type
    kc = _enc(rng.standard_normal((1, L, cap, HK * hd)), dtype)
    vrow = c.reshape(L, HK * hd)
    vc = _enc(np.broadcast_to(vrow[None, :, None, :], (1, L, cap, HK * hd)).copy(), dtype)
    q = rng.standard_normal((1, L, H * hd)).astype(np.float32)
    k = rng.standard_normal((1, L, HK * hd)).astype(np.float32)
    v = vrow[None].astype(np.float32)
    out = Oracle("port").step(kc, vc, dtype, [T - 1], _layers(L, hd, window > 0), q, k, v, H, HK,
                              hd, 1.0 / np.sqrt(hd), 0.0, window, 1.0, neox)
    G = H // HK
    want = np.repeat(c, G, axis=1).reshape(L, H * hd)
    assert np.abs(out[0] - want).max() <= 1e-5 * max(1.0, np.abs(want).max())


@settings(max_examples=60, deadline=None)
@given(shapes, st.integers(0, 2**31 - 1))
def test_zero_keys_give_the_mean_of_the_attended_rows(shape, seed):
    (H, HK), hd, T, dtype, neox, window = shape
    rng = np.random.default_rng(seed)
    L, cap = 2, T + 2
    kc = _enc(np.zeros((1, L, cap, HK * hd)), dtype)
    vals = np.round(rng.standard_normal((1, L, cap, HK * hd)) * 8) / 8
    vc = _enc(vals, dtype)
    q = rng.standard_normal((1, L, H * hd)).astype(np.float32)
    k = np.zeros((1, L, HK * hd), dtype=np.float32)               # rotated zero stays zero
    v = (np.round(rng.standard_normal((1, L, HK * hd)) * 8) / 8).astype(np.float32)
    layers = _layers(L, hd, window > 0)
    out = Oracle("port").step(kc, vc, dtype, [T - 1], layers, q, k, v, H, HK, hd,
                              1.0 / np.sqrt(hd), 0.0, window, 1.0, neox)
    rows = vals[0].copy()
    rows[:, T - 1] = v[0]                                         # the appended row
    G = H // HK
    for l in range(L):
        lo = T - window if (layers[l]["is_swa"] and window and T - 1 >= window) else 0
        mean = rows[l, lo:T].mean(axis=0).reshape(HK, hd)
        want = np.repeat(mean, G, axis=0).reshape(H * hd)
        assert np.abs(out[0, l] - want).max() <= 1e-5 * max(1.0, np.abs(want).max()), l


@pytest.mark.parametrize("dtype", DTYPES)
def test_step_writes_only_the_new_row(dtype):
    rng = np.random.default_rng(3)
    H, HK, hd, L, T, cap = 8, 2, 64, 3, 20, 24
    kc = _enc(rng.standard_normal((2, L, cap, HK * hd)), dtype)
    vc = _enc(rng.standard_normal((2, L, cap, HK * hd)), dtype)
    k0, v0 = kc.copy(), vc.copy()
    q = rng.standard_normal((2, L, H * hd)).astype(np.float32)
    k = rng.standard_normal((2, L, HK * hd)).astype(np.float32)
    # exact in every cache type, so the cache's own conversion stores them as is
    v = (np.round(rng.standard_normal((2, L, HK * hd)) * 8) / 8).astype(np.float32)
    pos = [T - 1, 5]
    Oracle("port").step(kc, vc, dtype, pos, _layers(L, hd, False), q, k, v, H, HK, hd,
                        1.0 / np.sqrt(hd))
    for s in range(2):
        mask = np.ones(cap, dtype=bool)
        mask[pos[s]] = False
        assert np.array_equal(kc[s][:, mask], k0[s][:, mask])
        assert np.array_equal(vc[s][:, mask], v0[s][:, mask])
        assert np.array_equal(vc[s][:, pos[s]], _enc(v[s], dtype))
