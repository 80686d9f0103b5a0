"""LCTC's clipped uniform quantiser and its operational rate-distortion table (numpy, CPU).  TEST
INFRASTRUCTURE ONLY (see package docstring).

Restates ``uq_codes`` / ``uq_values`` (LCTC_KV.py:443-455) with float32 rounding at every operation, as
the reference's float32 tensors round (no fused multiply-add):

    levels = 2^bits;  step = 2 clip / levels
    idx = min(max(floor((a + clip) / step), 0), levels - 1)
    value = -clip + (idx + 0.5) step

and ``operational_rd`` (:458-481): per column k of A (rows = calibration tokens), rms = max(sqrt(mean a^2),
1e-20); D[k, 0] = mean a^2; for every bit width b_j (j >= 1) the clip c = m rms over the multipliers m
(in order) with the least mean (a - Q(a))^2, the first on ties (strict <).  The means here are float64
sums of the float32 squares (the reference takes float32 means, then float64).
"""

from __future__ import annotations

import numpy as np

f32 = np.float32


def uq_codes(a, bits, clip):
    a = np.asarray(a, f32)
    levels = np.power(f32(2.0), np.asarray(bits, f32)).astype(f32)
    step = (f32(2.0) * np.asarray(clip, f32) / levels).astype(f32)
    idx = np.floor(((a + clip).astype(f32) / step).astype(f32))
    idx = np.maximum(idx, f32(0.0))
    return np.minimum(idx, levels - f32(1.0)).astype(f32)


def uq_values(idx, bits, clip):
    clip = np.asarray(clip, f32)
    levels = np.power(f32(2.0), np.asarray(bits, f32)).astype(f32)
    step = (f32(2.0) * clip / levels).astype(f32)
    return (-clip + ((np.asarray(idx, f32) + f32(0.5)).astype(f32) * step).astype(f32)).astype(f32)


def operational_rd(A, bits_set, mults):
    """A (N, n) float32; bits_set with bits_set[0] == 0; mults the clip multipliers (float32, the
    reference's torch.logspace(log10 0.5, log10 8, n_mults)).  Returns D (n, nb) float64, C (n, nb)
    float32 and the per-(column, width, multiplier) errors (n, nb - 1, n_mults)."""
    A = np.asarray(A, f32)
    n = A.shape[1]
    ms = (A.astype(np.float64) ** 2).mean(0)
    rms = np.maximum(np.sqrt(ms.astype(f32)), f32(1e-20)).astype(f32)
    nb = len(bits_set)
    D = np.empty((n, nb))
    C = np.zeros((n, nb), f32)
    D[:, 0] = ms
    errs = np.empty((n, nb - 1, len(mults)))
    for j, b in enumerate(bits_set[1:], 1):
        bits = np.full(n, b, f32)
        best = np.full(n, np.inf)
        bestc = np.zeros(n, f32)
        for mi, m in enumerate(mults):
            clip = (f32(m) * rms).astype(f32)
            v = uq_values(uq_codes(A, bits, clip), bits, clip)
            diff = (A - v).astype(f32)
            err = (diff.astype(np.float64) ** 2).mean(0)
            errs[:, j - 1, mi] = err
            better = err < best
            best = np.where(better, err, best)
            bestc = np.where(better, clip, bestc)
        D[:, j], C[:, j] = best, bestc
    return D, C, errs
