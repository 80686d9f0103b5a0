"""STRATA's head-synchronous rate allocation (numpy, CPU).  TEST INFRASTRUCTURE ONLY (see package
docstring).

Restates ``head_sync_allocate`` (STRATA_KV.py:1307-1351): Lagrangian relaxation over one multiplier
mu (Everett, 1963).  For each mu every rank position j takes the option l minimising
Dsort[j, l] + mu cost[l] among drop (l = 0), exact (l = nlev - 1) and the coded levels 1 .. c allowed
by a cap c (the deepest coded level of the layer, which also fixes the layer's bits fixed[c]); c
minimises the layer total.  The smallest feasible mu is bracketed by `rounds` rounds of `grid`
multipliers on a log scale from e^-80 to e^25.

Arithmetic follows the reference's float32 operations where they decide the result: mu = exp(g),
Q = D + mu cost (one rounding each), the drop / exact comparison (ties to drop), the running minimum
over levels (ties move to the later level, as torch.cummin), the cap comparison (strict), the grid
g = lo + (hi - lo) steps with torch.linspace's steps.  The layer totals and the bit sums are taken in
float64 (the reference sums float32 in its device's order); decisions agree except where two totals
are equal to float32 rounding.
"""

from __future__ import annotations

import numpy as np

f32, f64 = np.float32, np.float64


def linspace_torch(n: int) -> np.ndarray:
    """torch.linspace(0, 1, n) in float32: step = 1 / (n - 1); the first half start + step * i, the
    second half end - step * (n - 1 - i), each with one rounding (torch's vectorised kernel fuses the
    multiply-add)."""
    if n == 1:
        return np.zeros(1, f32)
    step = f32(1.0) / f32(n - 1)
    half = n // 2
    out = np.empty(n, f32)
    for i in range(n):
        out[i] = f32(f64(step) * i) if i < half else f32(1.0 - f64(step) * (n - 1 - i))
    return out


def evaluate(Dsort: np.ndarray, cost: np.ndarray, fixed: np.ndarray, log_mu: np.ndarray):
    """One batched evaluation (STRATA_KV.py:1325-1341): (M,) multipliers -> bits (M,) float64,
    choice (M, n) int64, cap (M,) int64."""
    Dsort = np.asarray(Dsort, f32)
    cost = np.asarray(cost, f32)
    fixed = np.asarray(fixed, f32)
    n, nlev = Dsort.shape
    L = nlev - 2
    mu = np.exp(np.asarray(log_mu, f32)).astype(f32)
    Q = (Dsort[None] + (mu[:, None, None] * cost[None, None, :]).astype(f32)).astype(f32)  # (M, n, nlev)
    q0, ql = Q[..., 0], Q[..., -1]
    base = np.minimum(q0, ql)
    bidx = np.where(ql < q0, nlev - 1, 0)
    M = len(mu)
    if L > 0:
        cm = np.empty((M, n, L), f32)
        ci = np.empty((M, n, L), np.int64)
        run, idx = Q[..., 1].copy(), np.zeros((M, n), np.int64)
        for l in range(L):
            if l:
                take = Q[..., 1 + l] <= run
                run = np.where(take, Q[..., 1 + l], run)
                idx = np.where(take, l, idx)
            cm[..., l], ci[..., l] = run, idx
        tot = np.concatenate([base.astype(f64).sum(1)[:, None],
                              np.minimum(base[..., None], cm).astype(f64).sum(1)], 1)
        tot = tot + (mu[:, None] * fixed[None, :]).astype(f32)
        c = tot.argmin(1)
        cc = np.maximum(c - 1, 0)
        cm_c = np.take_along_axis(cm, cc[:, None, None].repeat(n, 1), 2)[..., 0]
        ci_c = np.take_along_axis(ci, cc[:, None, None].repeat(n, 1), 2)[..., 0]
        use = (c > 0)[:, None] & (cm_c < base)
        choice = np.where(use, ci_c + 1, bidx)
    else:
        c = np.zeros(M, np.int64)
        choice = bidx
    bits = cost[choice].astype(f64).sum(1) + fixed[c].astype(f64)
    return bits, choice, c


def head_sync_allocate(Dsort, cost, fixed, budget: float, rounds: int = 4, grid: int = 32):
    """``head_sync_allocate`` STRATA_KV.py:1308-1351 -> (choice (n,) int64, cap int, bits float)."""
    lo, hi = f32(-80.0), f32(25.0)
    steps = linspace_torch(grid)
    for _ in range(rounds):
        g = (lo + ((hi - lo) * steps).astype(f32)).astype(f32)
        ok = evaluate(Dsort, cost, fixed, g)[0] <= budget
        i = int(np.argmax(ok)) if ok.any() else grid - 1
        lo, hi = g[max(i - 1, 0)], g[i]
    bits, choice, c = evaluate(Dsort, cost, fixed, np.array([hi], f32))
    return choice[0], int(c[0]), float(bits[0])
