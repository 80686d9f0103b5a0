"""kvb_coverage_stats (STRATA's coverage statistics, STRATA_KV.py:1226-1298) on the GPU:

* for four cases in the three input dtypes: the float64 oracle on the same inputs with the tolerances
  of the oracle's own pin (tests/test_oracle_coverage.py), and the reference's own float32 outputs
  (coverage.npz) with the median bound doubled: the reference's result is itself up to 6e-5 (median,
  case b) from the float64 value, and the kernels' float32 sums (FMA for float32 inputs, split-TF32
  tensor-core tiles for 16-bit ones) round in another order than its sequential ones;
* the float64 oracle at config 1's layer shape (32 query heads, 8 KV heads, d 128): the window group
  alone at 32768 positions, and every group at 8192;
* at 32768 positions with every group (65): two calls bit-identical, finite and non-negative sums.
"""

import numpy as np
import pytest
import torch

from oracle.coverage import coverage_groups as oracle_groups, coverage_stats as oracle_stats
from test_oracle_coverage import case, check_close

pytestmark = pytest.mark.gpu

KEYS = ("A", "W", "DD", "S", "Mbar")


def run(c, dtype, dev):
    import kvb
    from kvb.coverage import CoverageConfig
    cfg = CoverageConfig(N_SINK=c["n_sink"], W_OBS=c["w_obs"], STRATA_SEGMENT=c["segment"],
                         STRATA_QUERIES=c["queries"], STRATA_LOCAL=c["local"], STRATA_FLOOR=c["floor"])
    q = torch.from_numpy(c["q"])[None].to(dev, dtype)
    k = torch.from_numpy(c["k"])[None].to(dev, dtype)
    v = torch.from_numpy(c["v"])[None].to(dev, dtype)
    M = torch.from_numpy(np.ascontiguousarray(c["M"])).to(dev)
    return kvb.coverage_stats(q, k, v, c["scaling"], c["H"], c["rs"], c["re"], M, cfg, c["wonly"])


@pytest.mark.parametrize("name", list("abcd"))
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_coverage_matches_reference(golden, cuda_dev, name, dtype):
    g = golden("coverage")
    c = case(g, name)
    st = run(c, dtype, cuda_dev)
    assert len(st["groups"]) == len(c["groups"])
    for a, b in zip(st["groups"], c["groups"]):
        np.testing.assert_array_equal(a, b)
    ref = oracle_stats(c["q"], c["k"], c["v"], c["scaling"], c["rs"], c["re"], c["M"], c["groups"], c["local"],
                       c["floor"])
    for key in KEYS:
        check_close(st[key].cpu().numpy(), ref[key], key)
        check_close(st[key].cpu().numpy(), g[f"{name}_{key}"], key, median_tol=2e-4)


def layer(H, seed, dev):
    """One layer of config 1's shape: bf16 queries, keys (a decaying spectrum plus an offset, as the
    reference's self-test draws them) and values; metrics W_aᵀ W_a."""
    gen = torch.Generator().manual_seed(seed)
    Hkv, rep, d = 8, 4, 128
    spec = torch.exp(-torch.arange(d) / 25.0)
    q = (torch.randn(1, Hkv * rep, H, d, generator=gen) * spec.sqrt() * 3).bfloat16()
    k = (torch.randn(1, Hkv, H, d, generator=gen) * spec.sqrt() * 3 + 1.0).bfloat16()
    v = torch.randn(1, Hkv, H, d, generator=gen).bfloat16()
    Wa = torch.randn(Hkv * rep, 192, d, generator=gen) / d ** 0.5
    M = (Wa.transpose(-1, -2) @ Wa).float()
    return q, k, v, M


def oracle_of(q, k, v, M, H, groups):
    return oracle_stats(q[0].float().numpy(), k[0].float().numpy(), v[0].float().numpy(), 128 ** -0.5, 4, H - 32,
                        M.numpy(), groups, 64, 1e-3)


@pytest.mark.parametrize("H,wonly", [(32768, True), (8192, False)])
def test_coverage_full_shape_against_oracle(cuda_dev, H, wonly):
    import kvb
    q, k, v, M = layer(H, 11 + H, cuda_dev)
    st = kvb.coverage_stats(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), 128 ** -0.5, H, 4, H - 32,
                            M.to(cuda_dev), None, wonly)
    groups = oracle_groups(H)
    if wonly:
        groups = groups[-1:]
    ref = oracle_of(q, k, v, M, H, groups)
    for key in KEYS:
        check_close(st[key].cpu().numpy(), ref[key], key)


def test_coverage_32k_every_group_deterministic(cuda_dev):
    import kvb
    H = 32768
    q, k, v, M = (t.to(cuda_dev) for t in layer(H, 7, cuda_dev))
    a = kvb.coverage_stats(q, k, v, 128 ** -0.5, H, 4, H - 32, M)
    b = kvb.coverage_stats(q, k, v, 128 ** -0.5, H, 4, H - 32, M)
    assert len(a["groups"]) == 65
    for key in KEYS:
        assert torch.equal(a[key], b[key]), key
        assert torch.isfinite(a[key]).all(), key
    for key in ("A", "W", "DD"):
        assert (a[key] > 0).all(), key              # the floor keeps every token's price positive
    # S[h] is a normalised second moment: symmetric, positive semi-definite up to round-off
    S = a["S"].double()
    assert torch.allclose(S, S.transpose(-1, -2), rtol=1e-4, atol=1e-6 * S.abs().max().item())
    assert torch.linalg.eigvalsh((S + S.transpose(-1, -2)) / 2).min() > -1e-4 * S.abs().max()
    assert kvb.device_status() == 0


def test_coverage_batches_of_groups_bit_identical(cuda_dev):
    """A score cap of 1 MiB splits the 17 groups of an 8192-position layer into many passes (one group
    per pass for most): the same results, bit for bit, as one pass."""
    import kvb
    H = 8192
    q, k, v, M = (t.to(cuda_dev) for t in layer(H, 21, cuda_dev))
    one = kvb.coverage_stats(q, k, v, 128 ** -0.5, H, 4, H - 32, M)
    many = kvb.coverage_stats(q, k, v, 128 ** -0.5, H, 4, H - 32, M, score_cap=1 << 20)
    for key in KEYS:
        assert torch.equal(one[key], many[key]), key


def test_coverage_rejects_bad_arguments(cuda_dev):
    import kvb
    q, k, v, M = (t.to(cuda_dev) for t in layer(256, 3, cuda_dev))
    with pytest.raises(ValueError):
        kvb.coverage_stats(q, k, v, 0.1, 256, 10, 5, M)                 # re <= rs
    with pytest.raises(ValueError):
        kvb.coverage_stats(q.float(), k, v, 0.1, 256, 4, 224, M)        # mixed dtypes
    with pytest.raises(NotImplementedError):
        kvb.coverage_stats(q[..., :96].contiguous(), k[..., :96].contiguous(), v[..., :96].contiguous(),
                           0.1, 256, 4, 224, M[:, :96, :96].contiguous())   # d = 96
