"""STRATA's coverage statistics (coverage_groups / coverage_stats, STRATA_KV.py:1206-1298) in the oracle
against the reference's own outputs (coverage.npz): the sampled observation positions exactly, and
A, W, DD, S, Mbar within float32 round-off of the reference (the oracle computes in float64).  CPU
only."""

import numpy as np
import pytest

from oracle.coverage import coverage_groups, coverage_stats


def bf16(bits):
    return (np.asarray(bits, np.uint32) << 16).view(np.float32)


def case(g, name):
    Hkv, rep, d, H, rs, re, local, wonly, n_sink, w_obs, seg, nqs = (int(x) for x in g[f"{name}_shape"])
    qpos = g[f"{name}_qpos"]
    q = np.zeros((Hkv * rep, H, d), np.float32)
    q[:, qpos] = bf16(g[f"{name}_q"])
    pos, off = g[f"{name}_pos"], g[f"{name}_goff"]
    groups = [pos[off[i]:off[i + 1]] for i in range(len(off) - 1)]
    return dict(q=q, k=bf16(g[f"{name}_k"]), v=bf16(g[f"{name}_v"]), M=g[f"{name}_M"], H=H, rs=rs, re=re,
                local=local, wonly=bool(wonly), n_sink=n_sink, w_obs=w_obs, segment=seg, queries=nqs,
                groups=groups, scaling=float(g[f"{name}_scaling"]), floor=float(g[f"{name}_floor"]))


@pytest.mark.parametrize("name", list("abcd"))
def test_coverage_groups_golden(golden, name):
    c = case(golden("coverage"), name)
    got = coverage_groups(c["H"], c["n_sink"], c["local"], c["w_obs"], c["segment"], c["queries"])
    if c["wonly"]:
        got = got[-1:]
    assert len(got) == len(c["groups"])
    for a, b in zip(got, c["groups"]):
        np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("name", list("abcd"))
def test_coverage_stats_golden(golden, name):
    g = golden("coverage")
    c = case(g, name)
    st = coverage_stats(c["q"], c["k"], c["v"], c["scaling"], c["rs"], c["re"], c["M"], c["groups"],
                        c["local"], c["floor"])
    for key in ("A", "W", "DD", "S", "Mbar"):
        check_close(st[key], g[f"{name}_{key}"], key)


# Tolerances of a float32 computation of the same sums, relative to each array's largest entry.  DD
# carries (pR / (1 - pR))^2: where one key holds nearly all of a query's probability, float32 keeps
# few digits of 1 - pR (one unit in the last place of 1.0 is 6e-8, so 1 - pR = 1e-5 is known to
# ~1e-2 and its square to ~2e-2), in the reference as here.  Those few entries get the loose maximum;
# 99.9 % of DD's entries and every entry of the other arrays are held tightly.  Every group's weight
# 1 / N inherits DD's error through N = sum DD, so A, W and S move together by N's relative error
# (~6e-5 in case b).
SCALE_TOL = {"A": 3e-4, "W": 3e-4, "DD": 3e-2, "S": 3e-4, "Mbar": 3e-4}
Q999_TOL = 1e-3


def check_close(x, ref, key, median_tol=1e-4):
    x, ref = np.asarray(x, np.float64), np.asarray(ref, np.float64)
    assert x.shape == ref.shape, key
    assert np.all(np.isfinite(x)), key
    scale = np.abs(ref).max()
    err = np.abs(x - ref)
    assert err.max() <= SCALE_TOL[key] * scale, (key, err.max() / scale)
    assert np.quantile(err, 0.999) <= Q999_TOL * scale, (key, np.quantile(err, 0.999) / scale)
    if key != "S":      # S's small off-diagonal entries are sums that cancel: no relative bound
        assert np.median(err / np.maximum(np.abs(ref), 1e-30)) <= median_tol, key


def test_coverage_groups_edges():
    # no position can see a compressible key at long range: no group at all
    assert coverage_groups(50) == []
    # too short for a segment: the window group alone, starting at n_sink + local
    gs = coverage_groups(90)
    assert len(gs) == 1
    np.testing.assert_array_equal(gs[0], np.arange(68, 90))
    # segments: sorted, unique, inside their segment, at most `queries` each
    gs = coverage_groups(5000)
    for s, grp in zip(range(68, 5000 - 32, 512), gs[:-1]):
        assert np.all(np.diff(grp) > 0) and grp[0] >= s and grp[-1] < min(s + 512, 5000 - 32)
        assert len(grp) == min(16, min(s + 512, 5000 - 32) - s)
    np.testing.assert_array_equal(gs[-1], np.arange(5000 - 32, 5000))


def test_coverage_stats_edges():
    """Every group skipped (no group reads a coded token: te <= rs): zero sensitivities, Mbar the plain
    mean of the head's metrics (STRATA_KV.py:1293-1294); a context with only the window group."""
    rng = np.random.default_rng(3)
    Hkv, rep, d, H = 2, 2, 16, 200
    q = rng.standard_normal((Hkv * rep, H, d)).astype(np.float32)
    k = rng.standard_normal((Hkv, H, d)).astype(np.float32)
    v = rng.standard_normal((Hkv, H, d)).astype(np.float32)
    Wa = rng.standard_normal((Hkv * rep, 24, d)).astype(np.float32)
    M = np.einsum("axd,axe->ade", Wa, Wa)
    st = coverage_stats(q, k, v, 0.25, 150, 190, M, [np.arange(100, 120)], 4, 1e-3)
    for key in ("A", "W", "DD", "S"):
        np.testing.assert_array_equal(st[key], 0.0)
    np.testing.assert_allclose(st["Mbar"], M.astype(np.float64).reshape(Hkv, rep, d, d).mean(1), rtol=1e-12)
    gs = coverage_groups(90, w_obs=32)                 # 90 < n_sink + local + w_obs: no segment group
    assert len(gs) == 1 and gs[0][0] == 68
    st = coverage_stats(q, k, v, 0.25, 4, 90 - 32, M, gs, 64, 1e-3)
    assert np.all(st["A"] > 0) and np.all(np.isfinite(st["S"]))
