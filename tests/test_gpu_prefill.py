"""Multi-token prefill (jx_attn_prefill) against the oracle run token by token.

The reference feeds a prompt through forward_token one token at a time
(transformer.cpp:3092-3095): each token appends its row, then attends over the
rows up to its position.  One prefill call must give every row's output and the
same cache contents as that token-serial run -- here for two sequences at once
(one continuing a 37-row prefix, one from position 0), a sliding-window layer
and a full layer, all three cache types, both RoPE styles.
"""
import math

import numpy as np
import pytest

from oracle.oracle import BF16, F16T, F32
from tests.helpers import oracle_step, random_cache

pytestmark = pytest.mark.gpu

TOL = 1e-4


@pytest.mark.parametrize("dtype", [F32, BF16, F16T])
@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("shape", [(8, 2, 64), (4, 1, 128), (4, 2, 32)])
@pytest.mark.parametrize("order", ["shuffled", "sorted"])
def test_prefill_matches_token_serial_oracle(dtype, neox, shape, order):
    # rows in position order per sequence form blocks of 8/G tokens that share
    # one pass over their rows; shuffled rows run one token per pass
    import torch
    import jxai_b200 as jx
    H, HK, HD = shape
    L, cap, window = 2, 128, 16
    rs = HK * HD
    rng = np.random.default_rng(hash((dtype, neox, shape)) % 2**32)
    start = [37, 0]       # rows already in each sequence
    n_new = [29, 45]      # prompt tokens fed by the call
    kc = random_cache(rng, (2, L, cap, rs), dtype)
    vc = random_cache(rng, (2, L, cap, rs), dtype)
    layers = [jx.Layer(HD, HD, 1e4, 0, is_swa=True), jx.Layer(HD, HD, 1e6, 1)]
    rows = [(s, start[s] + t) for s in range(2) for t in range(n_new[s])]
    if order == "shuffled":
        rng.shuffle(rows)     # any row order
    n = len(rows)
    q = rng.standard_normal((n, L, H * HD)).astype(np.float32)
    k = rng.standard_normal((n, L, rs)).astype(np.float32)
    v = rng.standard_normal((n, L, rs)).astype(np.float32)

    cache = jx.KVCache(2, L, cap, rs, dtype)
    for s in range(2):
        for l in range(L):
            cache.write_rows(s, l, 0, 0, kc[s, l])
            cache.write_rows(s, l, 1, 0, vc[s, l])
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
    out = torch.full_like(qd, float("nan"))
    jx.attn_prefill(cache, layers, qd, kd, vd, out, [p for _, p in rows], H, HK,
                    seq_ids=[s for s, _ in rows], sliding_window=window, neox=neox)
    torch.cuda.synchronize()
    assert cache.check_device_error() == 0
    got = out.cpu().numpy()

    # token-serial oracle, per sequence in position order
    ko, vo = kc.copy(), vc.copy()
    ref = np.zeros_like(got)
    order = sorted(range(n), key=lambda i: (rows[i][0], rows[i][1]))
    for i in order:
        s, p = rows[i]
        ks, vs = ko[s:s + 1].copy(), vo[s:s + 1].copy()
        ref[i] = oracle_step(ks, vs, dtype, [p], layers, q[i:i + 1], k[i:i + 1], v[i:i + 1],
                             H, HK, HD, 1 / math.sqrt(HD), window=window, neox=neox)[0]
        ko[s:s + 1], vo[s:s + 1] = ks, vs
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= TOL
    for s in range(2):
        for l in range(L):
            assert np.array_equal(cache.read_rows(s, l, 0, 0, cap).view(np.uint8),
                                  ko[s, l].view(np.uint8)), (s, l, "K")
            assert np.array_equal(cache.read_rows(s, l, 1, 0, cap).view(np.uint8),
                                  vo[s, l].view(np.uint8)), (s, l, "V")
    cache.close()


@pytest.mark.parametrize("dtype", [F32, BF16])
@pytest.mark.parametrize("group", [1, 2, 4])
def test_prefill_blocks_across_groups(dtype, group):
    # blocks of 8/G tokens for groups 1, 2, 4; lengths not multiples of the block
    import torch
    import jxai_b200 as jx
    HK, HD, L, cap, window = 2, 64, 2, 96, 24
    H = HK * group
    rs = HK * HD
    rng = np.random.default_rng(100 + group)
    start, n_new = [5, 0, 60], [19, 37, 11]
    kc = random_cache(rng, (3, L, cap, rs), dtype)
    vc = random_cache(rng, (3, L, cap, rs), dtype)
    layers = [jx.Layer(HD, HD, 1e4, 0, is_swa=True), jx.Layer(HD, HD, 1e6, 1)]
    rows = [(s, start[s] + t) for s in range(3) for t in range(n_new[s])]
    n = len(rows)
    q = rng.standard_normal((n, L, H * HD)).astype(np.float32)
    k = rng.standard_normal((n, L, rs)).astype(np.float32)
    v = rng.standard_normal((n, L, rs)).astype(np.float32)
    cache = jx.KVCache(3, L, cap, rs, dtype)
    for s in range(3):
        for l in range(L):
            cache.write_rows(s, l, 0, 0, kc[s, l])
            cache.write_rows(s, l, 1, 0, vc[s, l])
    qd, kd, vd = (torch.from_numpy(x).cuda() for x in (q, k, v))
    out = torch.full_like(qd, float("nan"))
    jx.attn_prefill(cache, layers, qd, kd, vd, out, [p for _, p in rows], H, HK,
                    seq_ids=[s for s, _ in rows], sliding_window=window, neox=True)
    torch.cuda.synchronize()
    assert cache.check_device_error() == 0
    got = out.cpu().numpy()
    ko, vo = kc.copy(), vc.copy()
    ref = np.zeros_like(got)
    for i, (s, p) in enumerate(rows):   # rows are already in position order
        ks, vs = ko[s:s + 1].copy(), vo[s:s + 1].copy()
        ref[i] = oracle_step(ks, vs, dtype, [p], layers, q[i:i + 1], k[i:i + 1], v[i:i + 1],
                             H, HK, HD, 1 / math.sqrt(HD), window=window, neox=True)[0]
        ko[s:s + 1], vo[s:s + 1] = ks, vs
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= TOL
    for s in range(3):
        for l in range(L):
            assert np.array_equal(cache.read_rows(s, l, 0, 0, cap).view(np.uint8),
                                  ko[s, l].view(np.uint8))
    cache.close()


def test_prefill_rejects_a_position_listed_twice():
    import torch
    import jxai_b200 as jx
    cache = jx.KVCache(1, 1, 64, 128, "f32")
    layers = [jx.Layer(64, 64, 1e4, 0)]
    q = torch.zeros(3, 1, 4 * 64, device="cuda")
    k = torch.zeros(3, 1, 128, device="cuda")
    with pytest.raises(jx.JxError) as e:
        jx.attn_prefill(cache, layers, q, k, k, q.clone(), [5, 6, 5], 4, 2)
    assert e.value.code == -1
    cache.close()
