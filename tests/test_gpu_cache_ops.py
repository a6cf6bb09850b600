"""GPU parity of the cache operations and the sequence-sharded step.

* KVCacheSlot::compact / rollback / clear (src/transformer.cpp:25-66) on the
  device cache against the CPU oracle and the reference's semantics;
* the append's fp16-truncating and bf16 conversions on special values
  (NaN, Inf, overflow, subnormals, rounding ties), bit for bit;
* one long sequence split over several shards (jx_attn_step_partial on each,
  jx_lse_merge of the gathered partials) against the unsharded oracle.
"""
import math

import numpy as np
import pytest

from oracle.oracle import BF16, F16T, F32, Oracle
from tests.helpers import oracle_step, random_cache

pytestmark = pytest.mark.gpu

TOL = 1e-4


def _torch():
    import torch
    return torch


@pytest.mark.parametrize("dtype", [F16T, F32])
@pytest.mark.parametrize("seq_pos,keep", [(64, 32), (40, 8), (10, 6), (37, 0), (64, 59), (61, 40)])
def test_compact_matches_reference(dtype, seq_pos, keep):
    import jxai_b200 as jx
    rng = np.random.default_rng(seq_pos * 7 + keep)
    L, cap, rs = 3, 64, 32
    k = random_cache(rng, (L, cap, rs), dtype)
    v = random_cache(rng, (L, cap, rs), dtype)
    cache = jx.KVCache(2, L, cap, rs, dtype)
    for l in range(L):
        cache.write_rows(1, l, 0, 0, k[l])
        cache.write_rows(1, l, 1, 0, v[l])
    slot = jx.KVCacheSlot(cache, 1)
    slot.seq_pos = seq_pos
    slot.token_history = list(range(seq_pos))
    ko, vo = k.copy(), v.copy()
    want_pos = Oracle("port").compact(ko, vo, dtype, seq_pos, keep)
    slot.compact(keep)
    assert slot.seq_pos == want_pos
    assert len(slot.token_history) == min(seq_pos, want_pos)
    assert slot.compactions == (1 if want_pos != seq_pos else 0)
    for l in range(L):
        assert np.array_equal(cache.read_rows(1, l, 0, 0, cap).view(np.uint8), ko[l].view(np.uint8))
        assert np.array_equal(cache.read_rows(1, l, 1, 0, cap).view(np.uint8), vo[l].view(np.uint8))
    # the other sequence is untouched (all zeros, as created)
    assert not cache.read_rows(0, 0, 0, 0, cap).view(np.uint8).any()
    cache.close()


def test_rollback_and_clear():
    import jxai_b200 as jx
    rng = np.random.default_rng(4)
    cache = jx.KVCache(2, 2, 32, 32, "bf16")
    slot = jx.KVCacheSlot(cache, 0)
    rows = random_cache(rng, (32, 32), BF16)
    cache.write_rows(0, 1, 0, 0, rows)
    slot.seq_pos = 20
    slot.token_history = list(range(20))
    slot.rollback(25)                  # never moves forward (transformer.cpp:32-39)
    assert slot.seq_pos == 20
    slot.rollback(12)
    assert slot.seq_pos == 12 and slot.token_history == list(range(12))
    assert np.array_equal(cache.read_rows(0, 1, 0, 0, 32), rows)   # rows kept
    slot.clear()                        # zero rows, seq_pos 0 (transformer.cpp:25-30)
    assert slot.seq_pos == 0 and slot.token_history == []
    assert not cache.read_rows(0, 1, 0, 0, 32).any()
    cache.close()


SPECIAL = np.array(
    [0.0, -0.0, np.inf, -np.inf, np.nan, 1.0, -1.0, 65504.0, 65519.99, 65520.0, 1e9, -1e9,
     6.1e-5, 6.0e-5, 5.96e-8, 2.0 ** -24, 2.0 ** -25, 1e-30, -1e-30, 1.00390625, 1.01171875,
     3.0e38, 1.17549435e-38, 1.0009765625, 0.33333334, -2.7182817],
    dtype=np.float32)


@pytest.mark.parametrize("dtype", [F16T, BF16, F32])
def test_append_conversions_bit_exact_on_special_values(dtype):
    # rope_dim 0: no rotation, so the stored rows are the conversions of k and v
    import jxai_b200 as jx
    torch = _torch()
    rng = np.random.default_rng(9)
    H, HK, hd = 4, 2, 64
    n = HK * hd
    vals = np.concatenate([SPECIAL, rng.standard_normal(2 * n - SPECIAL.size).astype(np.float32)
                           * np.float32(10.0) ** rng.integers(-8, 6, 2 * n - SPECIAL.size).astype(np.float32)])
    vals = vals.astype(np.float32)
    k = vals[:n].reshape(1, 1, n).copy()
    v = vals[n:2 * n].reshape(1, 1, n).copy()
    q = rng.standard_normal((1, 1, H * hd)).astype(np.float32)
    cache = jx.KVCache(1, 1, 8, n, dtype)
    layers = [jx.Layer(hd, 0, 1e4, 0)]
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
    out = torch.zeros_like(qd)
    jx.attn_step(cache, layers, qd, kd, vd, out, [3], H, HK)
    torch.cuda.synchronize()
    orc = Oracle("port")
    want_k, want_v = orc.convert_array(k[0, 0], dtype), orc.convert_array(v[0, 0], dtype)
    got_k = cache.read_rows(0, 0, 0, 3, 1)[0]
    got_v = cache.read_rows(0, 0, 1, 3, 1)[0]
    assert np.array_equal(got_k.view(np.uint8), want_k.view(np.uint8))
    assert np.array_equal(got_v.view(np.uint8), want_v.view(np.uint8))
    cache.close()


@pytest.mark.parametrize("n_shards", [1, 2, 3, 5])
@pytest.mark.parametrize("window", [0, 100])
def test_sharded_partials_merge_to_full_attention(n_shards, window):
    import jxai_b200 as jx
    torch = _torch()
    rng = np.random.default_rng(n_shards * 10 + window)
    H, HK, hd, L, T = 8, 2, 64, 2, 700
    rs = HK * hd
    kc = rng.standard_normal((1, L, T, rs)).astype(np.float32)
    vc = rng.standard_normal((1, L, T, rs)).astype(np.float32)
    q = rng.standard_normal((1, L, H * hd)).astype(np.float32)
    k = rng.standard_normal((1, L, HK * hd)).astype(np.float32)
    v = rng.standard_normal((1, L, HK * hd)).astype(np.float32)
    # layer 0 full attention, layer 1 sliding window (when window > 0)
    layers = [jx.Layer(hd, hd, 1e6, 0), jx.Layer(hd, hd, 1e4, 1, is_swa=window > 0)]
    pos = T - 1
    ko, vo = kc.copy(), vc.copy()
    ref = oracle_step(ko, vo, F32, [pos], layers, q, k, v, H, HK, hd, 1 / math.sqrt(hd),
                      window=window, neox=False)
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
    hd2 = hd + 2
    per = L * H * hd2
    gathered = torch.empty(n_shards * per, device="cuda")
    bounds = [(T * r // n_shards, T * (r + 1) // n_shards) for r in range(n_shards)]
    caches = []
    for r, (b, e) in enumerate(bounds):
        c = jx.KVCache(1, L, e - b, rs, "f32", pos_base=b)
        for l in range(L):
            c.write_rows(0, l, 0, 0, kc[0, l, b:e])
            c.write_rows(0, l, 1, 0, vc[0, l, b:e])
        jx.attn_step_partial(c, layers, qd, kd, vd, gathered[r * per:(r + 1) * per], [pos], H,
                             HK, sliding_window=window, neox=False)
        caches.append(c)
    out = torch.full_like(qd, float("nan"))
    jx.lse_merge(gathered, n_shards, L, H, hd, out, H * hd)
    torch.cuda.synchronize()
    for c in caches:
        assert c.check_device_error() == 0
    assert np.abs(out.cpu().numpy() - ref).max() <= TOL
    # only the shard holding `pos` appended, bit-exact
    last = caches[-1]
    b = bounds[-1][0]
    for l in range(L):
        assert np.array_equal(last.read_rows(0, l, 0, pos - b, 1)[0], ko[0, l, pos])
        assert np.array_equal(last.read_rows(0, l, 1, pos - b, 1)[0], vo[0, l, pos])
    for c in caches[:-1]:
        for l in range(L):
            bb, ee = bounds[caches.index(c)]
            assert np.array_equal(c.read_rows(0, l, 0, 0, ee - bb), kc[0, l, bb:ee])
    for c in caches:
        c.close()


def test_unsharded_step_refuses_positions_outside_the_cache():
    import jxai_b200 as jx
    torch = _torch()
    cache = jx.KVCache(1, 1, 16, 128, "f32", pos_base=32)
    layers = [jx.Layer(64, 64, 1e4, 0)]
    q = torch.zeros(1, 1, 4 * 64, device="cuda")
    k = torch.zeros(1, 1, 128, device="cuda")
    with pytest.raises(jx.JxError) as e:
        jx.attn_step(cache, layers, q, k, k, q.clone(), [40], 4, 2)
    assert e.value.code == -5
    with pytest.raises(jx.JxError) as e:
        jx.attn_step(jx.KVCache(1, 1, 16, 128, "f32"), layers, q, k, k, q.clone(), [16], 4, 2)
    assert e.value.code == -5
    cache.close()


def test_step_timer_reports_device_time():
    # the counterpart of forward_token's attention_ms (transformer.cpp:2499, 2567)
    import jxai_b200 as jx
    torch = _torch()
    cache = jx.KVCache(1, 2, 512, 128, "f32")
    layers = [jx.Layer(64, 64, 1e4, 0), jx.Layer(64, 64, 1e4, 1)]
    q = torch.zeros(1, 2, 4 * 64, device="cuda")
    k = torch.zeros(1, 2, 128, device="cuda")
    with pytest.raises(jx.JxError):
        cache.last_step_ms()           # nothing timed yet
    cache.set_option("timing", 1)
    jx.attn_step(cache, layers, q, k, k, q.clone(), [300], 4, 2)
    ms = cache.last_step_ms()
    assert 0.0 < ms < 1000.0
    cache.close()


def test_step_on_pinned_host_buffers():
    # q/k/v/out in pinned host memory: the kernel reads and writes them over PCIe
    import jxai_b200 as jx
    torch = _torch()
    rng = np.random.default_rng(21)
    H, HK, hd, L, T = 8, 2, 64, 2, 300
    rs = HK * hd
    kc = random_cache(rng, (1, L, T, rs), F32)
    vc = random_cache(rng, (1, L, T, rs), F32)
    q = rng.standard_normal((1, L, H * hd)).astype(np.float32)
    k = rng.standard_normal((1, L, rs)).astype(np.float32)
    v = rng.standard_normal((1, L, rs)).astype(np.float32)
    layers = [jx.Layer(hd, hd, 5e5, 0), jx.Layer(hd, hd, 1e6, 1)]
    cache = jx.KVCache(1, L, T, rs, "f32")
    for l in range(L):
        cache.write_rows(0, l, 0, 0, kc[0, l])
        cache.write_rows(0, l, 1, 0, vc[0, l])
    qh, kh, vh = (torch.from_numpy(x).pin_memory() for x in (q, k, v))
    oh = torch.full(qh.shape, float("nan")).pin_memory()
    jx.attn_step(cache, layers, qh, kh, vh, oh, [T - 1], H, HK, neox=False)
    torch.cuda.synchronize()
    assert cache.check_device_error() == 0
    ko, vo = kc.copy(), vc.copy()
    ref = oracle_step(ko, vo, F32, [T - 1], layers, q, k, v, H, HK, hd, 1 / math.sqrt(hd),
                      neox=False)
    assert np.abs(oh.numpy() - ref).max() <= TOL
    for l in range(L):
        assert np.array_equal(cache.read_rows(0, l, 0, T - 1, 1)[0], ko[0, l, T - 1])
    cache.close()


def test_pageable_host_pointer_is_refused_before_any_launch():
    # head_dim 48 is unsupported too: should the pointer check ever let a
    # pageable buffer through, the call still ends on the host (-4), not in a kernel
    import ctypes as C
    import jxai_b200 as jx
    from jxai_b200 import _lib
    cache = jx.KVCache(1, 1, 64, 96, "f32")
    lib = jx.load_library()
    buf = np.zeros(4096, dtype=np.float32)          # pageable host memory
    p = buf.ctypes.data
    layer = _lib.LayerDesc(48, 48, 1e4, 0, 0, 0, None)
    pos = (C.c_int32 * 1)(10)
    a = _lib.StepArgs()
    a.n_heads, a.n_kv_heads, a.n_seqs = 2, 2, 1
    a.seq_ids, a.pos = None, C.cast(pos, C.POINTER(C.c_int32))
    a.q = a.k = a.v = a.out = p
    a.q_stride, a.kv_stride = 96, 96
    a.scale, a.softcap, a.sliding_window, a.yarn_scale, a.rope_neox = 0.14, 0.0, 0, 1.0, 1
    rc = lib.jx_attn_step(cache.handle, C.byref(layer), 1, C.byref(a), None)
    assert rc == _lib.JX_ERR_INVALID, rc
    assert b"pinned" in lib.jx_last_error_string()
    cache.close()
