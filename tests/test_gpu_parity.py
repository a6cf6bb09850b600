"""GPU parity: the fused sm_100a step against the CPU oracle on identical seeded inputs.

Bars: KV append bit-exact for every cache type; attention
output within max-abs 1e-4 of the reference's fp32 CPU attention on an fp32
cache, and within 2e-2 of it when the cache is bf16.  On identical stored
bytes the GPU must also agree with the oracle of the same cache type to 1e-4.
"""
import math

import numpy as np
import pytest

from oracle.oracle import BF16, F16T, F32
from tests.helpers import np_dtype, oracle_step, random_cache

pytestmark = pytest.mark.gpu

TOL = 1e-4


def _torch():
    import torch
    return torch


def run_case(dtype, n_heads, n_kv, hd, lengths, neox=True, n_layers=2, softcap=0.0, window=0,
             swa_layers=(), grid=0, seed=0, capacity=None, row_pad=0, rope_dim=None,
             yarn=1.0, rope_freqs=None, check_fp32_ref=False, q_scale=1.0, poison_tail=False,
             options=None):
    import jxai_b200 as jx
    torch = _torch()
    rng = np.random.default_rng(seed)
    n_seqs = len(lengths)
    cap = capacity or max(lengths) + 3
    rs = n_kv * hd + row_pad
    rdim = rope_dim or hd
    layers = [jx.Layer(hd, rdim, 1e6 if l % 2 else 5e5, l, is_swa=l in swa_layers,
                       rope_freqs=rope_freqs) for l in range(n_layers)]
    kc = random_cache(rng, (n_seqs, n_layers, cap, rs), dtype)
    vc = random_cache(rng, (n_seqs, n_layers, cap, rs), dtype)
    q = (rng.standard_normal((n_seqs, n_layers, n_heads * hd)) * q_scale).astype(np.float32)
    k = rng.standard_normal((n_seqs, n_layers, n_kv * hd)).astype(np.float32)
    v = rng.standard_normal((n_seqs, n_layers, n_kv * hd)).astype(np.float32)
    pos = [T - 1 for T in lengths]
    if poison_tail:
        # rows past each sequence's position are never attended; make them Inf
        inf = {F32: np.float32(np.inf), BF16: np.uint16(0x7F80), F16T: np.uint16(0x7C00)}[dtype]
        for s_, T in enumerate(lengths):
            kc[s_, :, T:] = inf
            vc[s_, :, T:] = inf
    scale = 1.0 / math.sqrt(hd)

    cache = jx.KVCache(n_seqs, n_layers, cap, rs, dtype)
    if grid:
        cache.set_option("grid", grid)
    for key, val in (options or {}).items():
        cache.set_option(key, val)
    for s in range(n_seqs):
        for l in range(n_layers):
            cache.write_rows(s, l, 0, 0, kc[s, l])
            cache.write_rows(s, l, 1, 0, vc[s, l])
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
    out = torch.full_like(qd, float("nan"))
    jx.attn_step(cache, layers, qd, kd, vd, out, pos, n_heads, n_kv, scale=scale,
                 softcap=softcap, sliding_window=window, yarn_scale=yarn, neox=neox)
    torch.cuda.synchronize()
    assert cache.check_device_error() == 0
    got = out.cpu().numpy()

    ko, vo = kc.copy(), vc.copy()
    ref = oracle_step(ko, vo, dtype, pos, layers, q, k, v, n_heads, n_kv, hd, scale, softcap,
                      window, yarn, neox, rope_freqs)
    # appended rows: bit-exact, every other row untouched
    for s in range(n_seqs):
        for l in range(n_layers):
            gk = cache.read_rows(s, l, 0, 0, cap)
            gv = cache.read_rows(s, l, 1, 0, cap)
            assert np.array_equal(gk.view(np.uint8), ko[s, l].view(np.uint8)), (s, l, "K")
            assert np.array_equal(gv.view(np.uint8), vo[s, l].view(np.uint8)), (s, l, "V")
    err = np.abs(got - ref).max()
    assert np.isfinite(got).all()
    assert err <= TOL, f"max-abs {err}"
    if check_fp32_ref:
        # the same step on an fp32 cache holding the unrounded values (north-star bf16 bar)
        kf = kc.astype(np.uint32) << 16 if dtype == BF16 else kc
        return got, kf
    cache.close()
    return got, ref


@pytest.mark.parametrize("dtype", [F32, BF16, F16T])
@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("shape", [(14, 2, 64), (32, 8, 64), (32, 8, 128), (4, 1, 256)])
def test_step_matches_oracle(dtype, neox, shape):
    H, HK, hd = shape
    run_case(dtype, H, HK, hd, [1, 33, 200], neox=neox)


@pytest.mark.parametrize("grid", [1, 3, 7, 64])
@pytest.mark.parametrize("penalty", [None, 0, 40])
def test_split_pieces_merge(grid, penalty):
    # forcing few/many CTAs puts segment boundaries everywhere: multi-piece
    # merges; slices balanced by the default per-piece cost, uniform (0) or a
    # large cost (40 us: several short or empty slices)
    opts = {} if penalty is None else {"split_penalty_us": penalty}
    run_case(F32, 32, 8, 64, [5, 97, 300, 1], grid=grid, n_layers=3, options=opts)
    run_case(BF16, 32, 8, 64, [5, 97, 300, 1], grid=grid, n_layers=3, options=opts)


@pytest.mark.parametrize("pdl", [0, 1])
def test_programmatic_launch_off_and_on(pdl):
    run_case(F32, 32, 8, 64, [200, 33], grid=7, options={"pdl": pdl})


@pytest.mark.parametrize("T", [1, 2, 31, 32, 33, 63, 64, 65, 511, 512])
def test_lengths_tile_edges(T):
    run_case(F32, 14, 2, 64, [T], n_layers=2)


def test_head_dim_32_and_group_8():
    run_case(F16T, 4, 2, 32, [40, 7])           # toy-model shape (fp16 trunc, native)
    run_case(BF16, 8, 1, 64, [70])              # group 8
    run_case(F32, 7, 1, 64, [70])               # group 7 padded to 8


@pytest.mark.parametrize("dtype", [BF16, F16T])
@pytest.mark.parametrize("shape", [(8, 8, 64), (16, 8, 64), (16, 2, 64), (8, 8, 32), (6, 3, 64),
                                   (16, 4, 128), (8, 1, 256), (12, 4, 64), (6, 3, 32),
                                   (3, 1, 32)])
def test_16bit_tensor_core_path(dtype, shape):
    # 16-bit caches run QK and PV on the tensor cores, two kv heads per tile row
    # when the heads pair up (head_dim 32/64, even kv heads, unpadded group);
    # otherwise at head_dim 32 one 64-byte row per tile row (64-byte swizzle);
    # grid=5 splits segments into pieces merged across CTAs
    H, HK, hd = shape
    run_case(dtype, H, HK, hd, [1, 17, 32, 33, 300], grid=5, n_layers=2)


@pytest.mark.parametrize("dtype", [BF16, F16T])
def test_16bit_softcap_window_and_q_range(dtype):
    run_case(dtype, 8, 2, 64, [600, 100], softcap=50.0, window=64, swa_layers=(0,), n_layers=3)
    run_case(dtype, 8, 2, 64, [300, 5], q_scale=3e4)     # |q| beyond the fp16 range
    run_case(dtype, 8, 2, 64, [300, 5], q_scale=1e-6)    # |q| in the fp16 subnormals
    run_case(dtype, 4, 2, 128, [300, 5], q_scale=3e4)


@pytest.mark.parametrize("dtype", [F32, BF16, F16T])
def test_unattended_rows_holding_inf(dtype):
    # the tail tile of a segment reaches rows past pos; Inf there must not leak
    run_case(dtype, 32, 8, 64, [33, 47, 5], capacity=96, poison_tail=True, grid=3)
    run_case(dtype, 4, 1, 256, [40], capacity=64, poison_tail=True)


def test_softcap_and_window():
    run_case(F32, 4, 1, 256, [600, 100], softcap=50.0, window=64, swa_layers=(0,), n_layers=3)


def test_partial_rope_and_padding():
    run_case(F32, 8, 2, 128, [50], rope_dim=64, row_pad=32, yarn=2.0)
    rf = np.linspace(1.0, 8.0, 64).astype(np.float32)
    run_case(F32, 8, 2, 128, [50], rope_freqs=rf)


def test_bf16_cache_within_2e2_of_fp32_reference():
    import jxai_b200 as jx
    torch = _torch()
    rng = np.random.default_rng(5)
    H, HK, hd, T, L = 32, 8, 64, 700, 2
    rs = HK * hd
    kf = rng.standard_normal((1, L, T + 1, rs)).astype(np.float32)
    vf = rng.standard_normal((1, L, T + 1, rs)).astype(np.float32)
    q = rng.standard_normal((1, L, H * hd)).astype(np.float32)
    k = rng.standard_normal((1, L, HK * hd)).astype(np.float32)
    v = rng.standard_normal((1, L, HK * hd)).astype(np.float32)
    layers = [jx.Layer(hd, hd, 5e5, l) for l in range(L)]
    from oracle.oracle import Oracle
    o = Oracle("port")
    kb = o.convert_array(kf[0, :, :T - 1], BF16)
    vb = o.convert_array(vf[0, :, :T - 1], BF16)
    cache = jx.KVCache(1, L, T + 1, rs, "bf16")
    for l in range(L):
        cache.write_rows(0, l, 0, 0, kb[l])
        cache.write_rows(0, l, 1, 0, vb[l])
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
    out = torch.zeros_like(qd)
    jx.attn_step(cache, layers, qd, kd, vd, out, [T - 1], H, HK, neox=False)
    torch.cuda.synchronize()
    ref = oracle_step(kf.copy(), vf.copy(), F32, [T - 1], layers, q, k, v, H, HK, hd,
                      1 / math.sqrt(hd), neox=False)
    assert np.abs(out.cpu().numpy() - ref).max() <= 2e-2


@pytest.mark.parametrize("stages", [2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("grid", [1, 3])
def test_every_ring_size_on_long_pieces(stages, grid):
    # one or three CTAs walk thousands of rows: every stage is reused many
    # times, so a consumer that could wait on the wrong phase would show up
    import jxai_b200 as jx
    torch = _torch()
    rng = np.random.default_rng(stages * 10 + grid)
    H, HK, hd, T = 8, 2, 64, 3000
    rs = HK * hd
    kc = rng.standard_normal((1, 1, T + 1, rs)).astype(np.float32)
    vc = rng.standard_normal((1, 1, T + 1, rs)).astype(np.float32)
    q = rng.standard_normal((1, 1, H * hd)).astype(np.float32)
    k = rng.standard_normal((1, 1, HK * hd)).astype(np.float32)
    v = rng.standard_normal((1, 1, HK * hd)).astype(np.float32)
    layers = [jx.Layer(hd, hd, 5e5, 0)]
    cache = jx.KVCache(1, 1, T + 1, rs, "f32")
    cache.set_option("stages", stages)
    cache.set_option("grid", grid)
    cache.write_rows(0, 0, 0, 0, kc[0, 0])
    cache.write_rows(0, 0, 1, 0, vc[0, 0])
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
    ref = oracle_step(kc.copy(), vc.copy(), F32, [T - 1], layers, q, k, v, H, HK, hd,
                      1 / math.sqrt(hd), neox=False)
    for _ in range(3):
        out = torch.full_like(qd, float("nan"))
        jx.attn_step(cache, layers, qd, kd, vd, out, [T - 1], H, HK, neox=False)
        torch.cuda.synchronize()
        assert cache.check_device_error() == 0
        assert np.abs(out.cpu().numpy() - ref).max() <= TOL
    cache.close()


@pytest.mark.parametrize("hd,stages", [(128, 2), (128, 3), (128, 4), (256, 2), (256, 3)])
def test_wide_heads_long_pieces(hd, stages):
    import jxai_b200 as jx
    torch = _torch()
    rng = np.random.default_rng(hd + stages)
    H, HK, T = 8, 2, 1500
    rs = HK * hd
    kc = rng.standard_normal((1, 1, T + 1, rs)).astype(np.float32)
    vc = rng.standard_normal((1, 1, T + 1, rs)).astype(np.float32)
    q = rng.standard_normal((1, 1, H * hd)).astype(np.float32)
    k = rng.standard_normal((1, 1, HK * hd)).astype(np.float32)
    v = rng.standard_normal((1, 1, HK * hd)).astype(np.float32)
    layers = [jx.Layer(hd, hd, 1e6, 0)]
    cache = jx.KVCache(1, 1, T + 1, rs, "f32")
    cache.set_option("stages", stages)
    cache.set_option("grid", 2)
    cache.write_rows(0, 0, 0, 0, kc[0, 0])
    cache.write_rows(0, 0, 1, 0, vc[0, 0])
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
    out = torch.zeros_like(qd)
    jx.attn_step(cache, layers, qd, kd, vd, out, [T - 1], H, HK, neox=True)
    torch.cuda.synchronize()
    assert cache.check_device_error() == 0
    ref = oracle_step(kc.copy(), vc.copy(), F32, [T - 1], layers, q, k, v, H, HK, hd,
                      1 / math.sqrt(hd), neox=True)
    assert np.abs(out.cpu().numpy() - ref).max() <= TOL
    cache.close()


def test_repeated_and_alternating_calls():
    # an identical call relaunches the launches built for it; a call with other
    # positions rebuilds the plan; going back must not reuse stale launches
    import jxai_b200 as jx
    torch = _torch()
    rng = np.random.default_rng(23)
    H, HK, hd, L = 8, 2, 64, 2
    cap, rs = 400, HK * hd
    kc = rng.standard_normal((2, L, cap, rs)).astype(np.float32)
    vc = rng.standard_normal((2, L, cap, rs)).astype(np.float32)
    q = rng.standard_normal((2, L, H * hd)).astype(np.float32)
    k = rng.standard_normal((2, L, HK * hd)).astype(np.float32)
    v = rng.standard_normal((2, L, HK * hd)).astype(np.float32)
    layers = [jx.Layer(hd, hd, 1e6, l) for l in range(L)]
    cache = jx.KVCache(2, L, cap, rs, "f32")
    for s in range(2):
        for l in range(L):
            cache.write_rows(s, l, 0, 0, kc[s, l])
            cache.write_rows(s, l, 1, 0, vc[s, l])
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
    ko, vo = kc.copy(), vc.copy()
    refs = {}
    # b appends rows (350, 399), outside a's attended rows (<= 300, <= 120); b attends
    # over a's appended rows, so its reference is taken after a's step
    for pos in ([300, 120], [350, 399]):
        refs[tuple(pos)] = oracle_step(ko, vo, F32, pos, layers, q, k, v, H, HK, hd,
                                       1 / math.sqrt(hd))
    out = torch.zeros_like(qd)
    plan_a = jx.StepPlan(cache, layers, qd, kd, vd, out, [300, 120], H, HK)
    plan_b = jx.StepPlan(cache, layers, qd, kd, vd, out, [350, 399], H, HK)
    for seq in ("a", "a", "b", "a", "b", "b", "a"):
        out.fill_(float("nan"))
        (plan_a if seq == "a" else plan_b).run()
        torch.cuda.synchronize()
        ref = refs[(300, 120)] if seq == "a" else refs[(350, 399)]
        assert np.abs(out.cpu().numpy() - ref).max() <= TOL, seq
    assert cache.check_device_error() == 0
    cache.close()


def _mixed_case(layers, cache_layers, n_heads, n_kv, lengths, dtype, seed, hd_max, options=None):
    """One jx_attn_step over `layers` (a mix of head dims and shares-KV layers)
    against the oracle run layer by layer in call order, as forward_token runs
    them (src/transformer.cpp:2442, 2512): a sharing layer reads its source
    layer's cache after that layer appended this step's row."""
    import jxai_b200 as jx
    torch = _torch()
    from oracle.oracle import Oracle
    from tests.helpers import layer_dicts
    rng = np.random.default_rng(seed)
    n_seqs, L = len(lengths), len(layers)
    cap = max(lengths) + 2
    rs = n_kv * hd_max
    qs, ks = n_heads * hd_max, n_kv * hd_max
    kc = random_cache(rng, (n_seqs, cache_layers, cap, rs), dtype)
    vc = random_cache(rng, (n_seqs, cache_layers, cap, rs), dtype)
    q = rng.standard_normal((n_seqs, L, qs)).astype(np.float32)
    k = rng.standard_normal((n_seqs, L, ks)).astype(np.float32)
    v = rng.standard_normal((n_seqs, L, ks)).astype(np.float32)
    pos = [T - 1 for T in lengths]
    cache = jx.KVCache(n_seqs, cache_layers, cap, rs, dtype)
    for key, val in (options or {}).items():
        cache.set_option(key, val)
    for s in range(n_seqs):
        for l in range(cache_layers):
            cache.write_rows(s, l, 0, 0, kc[s, l])
            cache.write_rows(s, l, 1, 0, vc[s, l])
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
    out = torch.full_like(qd, float("nan"))
    # scale 1/sqrt(64) for every layer (the step takes one scale)
    jx.attn_step(cache, layers, qd, kd, vd, out, pos, n_heads, n_kv, scale=0.125, neox=True)
    torch.cuda.synchronize()
    assert cache.check_device_error() == 0
    launches = cache.last_launch_count()
    got = out.cpu().numpy()
    ko, vo = kc.copy(), vc.copy()
    orc = Oracle("port")
    ref = np.zeros_like(got)
    for l, Ld in enumerate(layers):
        ref[:, l:l + 1] = orc.step(ko, vo, dtype, pos, layer_dicts([Ld]), q[:, l:l + 1],
                                   k[:, l:l + 1], v[:, l:l + 1], n_heads, n_kv, Ld.head_dim,
                                   0.125, 0.0, 0, 1.0, True)
    for s in range(n_seqs):
        for l in range(cache_layers):
            gk = cache.read_rows(s, l, 0, 0, cap)
            gv = cache.read_rows(s, l, 1, 0, cap)
            assert np.array_equal(gk.view(np.uint8), ko[s, l].view(np.uint8)), (s, l, "K")
            assert np.array_equal(gv.view(np.uint8), vo[s, l].view(np.uint8)), (s, l, "V")
    for l, Ld in enumerate(layers):
        w = n_heads * Ld.head_dim
        err = np.abs(got[:, l, :w] - ref[:, l, :w]).max()
        assert np.isfinite(got[:, l, :w]).all(), l
        assert err <= TOL, f"layer {l}: max-abs {err}"
    cache.close()
    return launches


@pytest.mark.parametrize("dtype", [F32, BF16, F16T])
@pytest.mark.parametrize("pdl", [0, 1])
def test_shared_kv_layers(dtype, pdl):
    # Gemma-3n/4 style shared-KV layers (src/transformer.cpp:2127-2137): a
    # sharing layer appends nothing and reads its source layer's cache.  Layers
    # 2 and 4 read cache layers 0 and 1, appended by layers 0 and 1 of the same
    # call (a second launch that must see those appends); layer 3 reads cache
    # layer 5, which no layer of the call appends (first launch).  Cache layers
    # 2, 3 and 4 stay untouched.
    import jxai_b200 as jx
    hd = 64
    layers = [jx.Layer(hd, hd, 1e6, 0), jx.Layer(hd, hd, 1e4, 1),
              jx.Layer(hd, hd, 1e6, 0, shares_kv=True),
              jx.Layer(hd, hd, 1e6, 5, shares_kv=True),
              jx.Layer(hd, hd, 1e4, 1, shares_kv=True), jx.Layer(hd, hd, 1e6, 6)]
    n = _mixed_case(layers, 7, 8, 2, [300, 41, 7], dtype, seed=31 + dtype, hd_max=hd,
                    options={"pdl": pdl, "grid": 9})
    assert n == 2


@pytest.mark.parametrize("dtype", [F32, BF16])
def test_mixed_head_dims_in_one_call(dtype):
    # layers of different head_dim (as Gemma-3n's per-layer head sizes): one
    # launch per head_dim in one call, all sharing the q / kv strides
    import jxai_b200 as jx
    layers = [jx.Layer(64, 64, 1e6, 0), jx.Layer(128, 128, 1e4, 1), jx.Layer(64, 64, 1e6, 2),
              jx.Layer(128, 128, 1e6, 3, shares_kv=True), jx.Layer(128, 128, 1e6, 1,
                                                                    shares_kv=True)]
    n = _mixed_case(layers, 4, 8, 2, [257, 66], dtype, seed=41 + dtype, hd_max=128)
    assert n == 3  # hd 64, hd 128 (incl. the sharer of layer 3), then the sharer of layer 1
