"""K2a accumulated decode-query attention scores and the full eviction pipeline (config 2 shape,
scaled down) vs the oracle."""

import numpy as np
import pytest
import torch

import oracle as O
from kvref import np32, unpack, token_meta, channel_meta, gather_rows

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("pool", [0, 5])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_query_scores(cuda_dev, pool, dtype):
    import kvb
    gen = torch.Generator().manual_seed(21 + pool)
    B, Hkv, rep, nq, T, d = 2, 2, 4, 16, 3001, 128
    q = torch.randn(B, Hkv * rep, nq, d, generator=gen).to(dtype)
    k = torch.randn(B, Hkv, T, d, generator=gen).to(dtype)
    n_cand = T - 128
    got = kvb.query_scores(q.to(cuda_dev), k.to(cuda_dev), d ** -0.5, n_cand, pool).cpu().numpy()
    ref = O.query_scores(np32(q), np32(k), d ** -0.5, n_cand, pool)
    np.testing.assert_allclose(got, ref, rtol=2e-4, atol=1e-9)


def test_eviction_pipeline(cuda_dev):
    """Scores -> top-k + window -> KIVI 4-bit g64 of kept tokens.  Kept sets are exact given the same
    score tensor; codes / scales of the kept tokens are exact."""
    import kvb
    gen = torch.Generator().manual_seed(33)
    B, Hkv, rep, nq, T, d = 1, 2, 4, 64, 4096, 128
    budget, window = 500, 128
    q = torch.randn(B, Hkv * rep, nq, d, generator=gen).to(torch.bfloat16)
    K = torch.randn(B, Hkv, T, d, generator=gen).to(torch.bfloat16)
    V = torch.randn(B, Hkv, T, d, generator=gen).to(torch.bfloat16)
    cache, kept, sc = kvb.cache.build_eviction(q.to(cuda_dev), K.to(cuda_dev), V.to(cuda_dev), d ** -0.5, budget,
                                               window, bits=4, group=64)
    kept_np = kept.cpu().numpy()
    # (i) identical score tensor -> identical kept set
    np.testing.assert_array_equal(kept_np, O.topk_kept(sc.cpu().numpy(), budget, window))
    # (ii) end to end from the oracle's own scores: equal except near-ties at the k-th score
    ref_sc = O.query_scores(np32(q), np32(K), d ** -0.5, T - window)
    ref_kept = O.topk_kept(ref_sc, budget, window)
    for h in range(Hkv):
        diff = set(kept_np[0, h]) ^ set(ref_kept[0, h])
        if diff:
            kth = np.sort(ref_sc[0, h])[::-1][budget - 1]
            for j in diff:
                assert abs(ref_sc[0, h, j] - kth) <= 1e-6 * max(kth, 1e-30) + 1e-12
    # codes of the kept tokens
    s = cache.strata[0]
    n = budget + window
    gk = gather_rows(np32(K), kept_np)
    gv = gather_rows(np32(V), kept_np)
    rk, rv = O.kivi_quant(gk, 4, 64, True, 0), O.kivi_quant(gv, 4, 64, False, 0)
    np.testing.assert_array_equal(unpack(s["kc"], 4, n), rk["codes"])
    np.testing.assert_array_equal(unpack(s["vc"], 4, n), rv["codes"])
    lo, scl = channel_meta(s["km"], n, 64)
    np.testing.assert_array_equal(lo, rk["lo"])
    np.testing.assert_array_equal(scl, rk["scale"])
    lo, scl = token_meta(s["vm"], n)
    np.testing.assert_array_equal(lo, rv["lo"])
    np.testing.assert_array_equal(scl, rv["scale"])
    # decode over the kept cache vs dequantise-then-attend in fp32
    qd = torch.randn(B, Hkv * rep, 1, d, generator=gen).to(torch.bfloat16)
    out = kvb.decode(cache, qd.to(cuda_dev), d ** -0.5, out_dtype=torch.float32).cpu().numpy()
    ref = O.chunked_attention(np32(qd), d ** -0.5, np.array([T]), rk["xhat"], rv["xhat"], np.arange(n),
                              np.full(n, O.attention.BIG), None, 256)
    assert np.abs(out - ref).max() <= 2e-3


@pytest.mark.parametrize("case", ["a", "b"])
def test_snapkv_scores_golden(cuda_dev, golden, case):
    """kvb_snapkv_scores (causal observation window) against the reference's own snapkv_scores
    (STRATA_KV.py:932-954, fixture generated from it): scores within float32 accumulation tolerance,
    and the top-40 kept set of the GPU scores equals the reference's wherever the reference's
    boundary margin exceeds the score error."""
    import kvb
    g = golden("snapkv128")
    B, Hkv, rep, H, w, kern = (int(x) for x in g[f"{case}_cfg"])
    qw = torch.from_numpy(g[f"{case}_qw"]).half().to(cuda_dev)
    k = torch.from_numpy(g[f"{case}_k"]).half().to(cuda_dev)
    got = kvb.snapkv_scores(qw, k, 128 ** -0.5, pool=kern)
    assert kvb.device_status() == 0
    ref = g[f"{case}_scores"][..., :H - w]
    gn = got.cpu().numpy()
    np.testing.assert_allclose(gn, ref, rtol=2e-4, atol=1e-9)
    top = kvb.rank_split(got, [40], want=[0])[0].cpu().numpy()
    err = np.abs(gn - ref).max()
    for b in range(B):
        for h in range(Hkv):
            if g[f"{case}_gap40"][b, h] > 4 * err:
                np.testing.assert_array_equal(top[b, h], g[f"{case}_top40"][b, h])
