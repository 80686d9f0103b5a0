"""STRATA's coverage statistics (numpy, CPU).  TEST INFRASTRUCTURE ONLY (see package docstring).

Restates ``coverage_groups`` (STRATA_KV.py:1206-1222) and ``coverage_stats`` (:1226-1298).  Observation
groups: one per context segment of ``segment`` positions from ``n_sink + local`` up to ``H - w_obs``
(``queries`` positions sampled without replacement by numpy's generator seeded with
[SEED, crc32("cover_group"), crc32(str(H)), crc32(str(segment start))], :306-307), then the last
``w_obs`` positions (the window group).  For group g (positions P, nq = |P|, mmax = max P + 1,
te = min(re, mmax), nt = te - rs; skipped when te <= rs), per KV head h and query row (r, i) of query
head a = h rep + r at position P_i:

    qa = q[a, P_i] * scaling;  p = softmax over keys j <= P_i of qa . k_j;  o = sum_j p_j v_j
    pR_j = p_j where rs <= j < te and j <= P_i - local (local = 1 for the window group), else 0
    u2_j = max(vMv[a, j] - 2 (o M_a) . v_j + (o M_a) . o, 0),   vMv[a, j] = v_j M_a v_j
    dd_j = sum_(r,i) (pR / max(1 - pR, 1e-6))^2 u2 / nq,   a_(r,i,j) = pR^2 u2
    N = sum_(h,j) dd;  wgt = 1 / max(N, 1e-30) if N > 0 else 0
    A += sum_(r,i) a / nq wgt;  DD += dd wgt;  WVa[h, r] += sum_i pR^2 / nq wgt
    S[h] += sum_(r,i) (sum_j a / nq) qa qaᵀ wgt;  live += (N > 0)

then A, DD, WVa, S over max(live, 1); S[h] /= max(sum_j A[h, j], 1e-30); omega = sum_j WVa;
Mbar[h] = sum_r omega_r M_(h rep + r) / max(sum_r omega_r, 1e-30), or the mean of the M_a of the head
when sum_r omega_r = 0; W = sum_r WVa; A, W, DD each plus 1e-3-style floor ``eta`` times their mean.
Float64 throughout (the reference computes in float32).
"""

from __future__ import annotations

import zlib

import numpy as np

SEED = 42           # STRATA_KV.py:271


def _rng(*keys) -> np.random.Generator:
    """STRATA_KV.py:306-307."""
    return np.random.default_rng([SEED] + [zlib.crc32(str(k).encode()) for k in keys])


def coverage_groups(H: int, n_sink: int = 4, local: int = 64, w_obs: int = 32, segment: int = 512,
                    queries: int = 16) -> list:
    """STRATA_KV.py:1206-1222."""
    lo = n_sink + local
    win = max(lo, H - w_obs)
    groups = []
    for s in range(lo, win, segment):
        seg = np.arange(s, min(s + segment, win))
        n = min(len(seg), queries)
        groups.append(np.sort(_rng("cover_group", H, s).choice(seg, n, replace=False)))
    groups.append(np.arange(win, H))
    return [g for g in groups if len(g)]


def coverage_stats(q, k, v, scaling: float, rs: int, re: int, M, groups, local: int, floor: float):
    """STRATA_KV.py:1226-1298 for one batch row.  q (Hq, H, d) (only the rows at the groups'
    positions are read), k and v (Hkv, H, d), M (Hq, d, d); ``groups`` as from coverage_groups
    (the caller passes the window group alone for window_only)."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    M = np.asarray(M, np.float64)
    Hkv, d = k.shape[0], k.shape[-1]
    rep = q.shape[0] // Hkv
    n = re - rs
    A = np.zeros((Hkv, n))
    DD = np.zeros((Hkv, n))
    WVa = np.zeros((Hkv, rep, n))
    S = np.zeros((Hkv, d, d))
    live = 0.0
    Mg = M.reshape(Hkv, rep, d, d)
    VR = v[:, rs:re]
    vMv = np.stack([((VR @ Mg[:, r]) * VR).sum(-1) for r in range(rep)], 1)
    for gi, P in enumerate(groups):
        P = np.asarray(P, np.int64)
        nq, mmax = len(P), int(P.max()) + 1
        te = min(re, mmax)
        if te <= rs:
            continue
        nt = te - rs
        qa = q[:, P].reshape(Hkv, rep, nq, d) * scaling
        sc = qa @ k[:, None, :mmax].swapaxes(-1, -2)
        sc = np.where(np.arange(mmax)[None, None, None, :] > P[None, None, :, None], -np.inf, sc)
        mx = sc.max(-1, keepdims=True)
        e = np.exp(sc - mx)
        p = e / e.sum(-1, keepdims=True)
        o = p @ v[:, None, :mmax]
        loc = 1 if gi == len(groups) - 1 else local
        far = np.arange(rs, te)[None, :] <= (P[:, None] - loc)
        pR = p[..., rs:te] * far
        oM = o @ Mg
        u2 = np.maximum(vMv[:, :, None, :nt] - 2 * (oM @ VR[:, None, :nt].swapaxes(-1, -2))
                        + (oM * o).sum(-1)[..., None], 0.0)
        dd = ((pR / np.maximum(1 - pR, 1e-6)) ** 2 * u2).sum((1, 2)) / nq
        a = pR ** 2 * u2
        N = dd.sum()
        wgt = 1.0 / max(N, 1e-30) if N > 0 else 0.0
        A[:, :nt] += a.sum((1, 2)) / nq * wgt
        DD[:, :nt] += dd * wgt
        WVa[:, :, :nt] += (pR ** 2).sum(2) / nq * wgt
        alpha = a.sum(-1) / nq
        qw = (alpha[..., None] * qa).reshape(Hkv, rep * nq, d)
        S += (qw.swapaxes(-1, -2) @ qa.reshape(Hkv, rep * nq, d)) * wgt
        live += float(N > 0)
    live = max(live, 1.0)
    A, DD, WVa, S = A / live, DD / live, WVa / live, S / live
    S = S / np.maximum(A.sum(-1), 1e-30)[:, None, None]
    omega = WVa.sum(-1)
    Mbar = np.einsum("hr,hrde->hde", omega, Mg) / np.maximum(omega.sum(-1), 1e-30)[:, None, None]
    Mbar = np.where(omega.sum(-1)[:, None, None] > 0, Mbar, Mg.mean(1))
    W = WVa.sum(1)
    return {"A": A + floor * A.mean(), "W": W + floor * W.mean(), "DD": DD + floor * DD.mean(), "S": S,
            "Mbar": Mbar}
