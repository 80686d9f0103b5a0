"""QUASAR's coded decode over embedded stage codes (numpy, CPU).  TEST INFRASTRUCTURE ONLY (see package
docstring).

Restates ``QuasarState.coded_scores`` / ``coded_values`` (QUASAR_KV.py:1918-1940) on the flat layout
the reference's kernels read (QUASAR_KV.py:1884-1898): per side, one uint8 buffer holding every
step's (Hkv, n_s, bytes) block of MSB-first packed codes (``pack_rows`` :1185), and a step table of
int32 rows (offset, n_s, bytes per row, band start a, band width w, bits b, level offset), with the
stage level tables concatenated (``stage_codebooks`` :1144).  Step s owns tokens [0, n_s) and
coefficients [a, a + w):

    scores[h, r, j] = sum over steps owning j of  qt[h, r, a:a+w] . level[code_s(h, j, :)]
    values[h, r, a:a+w] += sum over j < n_s of  pv[h, r, j] level[code_s(h, j, :)]

Float64 here; the reference sums float32 per step.
"""

from __future__ import annotations

import numpy as np


def unpack_step(flat: np.ndarray, row, Hkv: int) -> np.ndarray:
    """Level indices (Hkv, n_s, w) of one step: codes of b bits, the first code of a byte in its most
    significant bits."""
    off, n, nb, a, w, b, lo = (int(x) for x in row)
    by = np.asarray(flat[off:off + Hkv * n * nb], np.uint8).reshape(Hkv, n, nb)
    per = 8 // b
    shifts = (per - 1 - np.arange(per)) * b
    codes = (by[..., None] >> shifts) & ((1 << b) - 1)
    return lo + codes.reshape(Hkv, n, nb * per)[..., :w]


def coded_scores(qt: np.ndarray, flat: np.ndarray, table: np.ndarray, levels: np.ndarray, n_c: int) -> np.ndarray:
    """qt (Hkv, rows, R) -> scores (Hkv, rows, n_c)."""
    qt = np.asarray(qt, np.float64)
    Hkv, rows, _ = qt.shape
    lev = np.asarray(levels, np.float64)
    sc = np.zeros((Hkv, rows, n_c))
    for row in table:
        n, a, w = int(row[1]), int(row[3]), int(row[4])
        val = lev[unpack_step(flat, row, Hkv)]                       # (Hkv, n, w)
        sc[:, :, :n] += np.einsum("hrw,hnw->hrn", qt[:, :, a:a + w], val)
    return sc


def coded_values(pv: np.ndarray, flat: np.ndarray, table: np.ndarray, levels: np.ndarray, R: int) -> np.ndarray:
    """pv (Hkv, rows, n_c) -> values (Hkv, rows, R)."""
    pv = np.asarray(pv, np.float64)
    Hkv, rows, _ = pv.shape
    lev = np.asarray(levels, np.float64)
    out = np.zeros((Hkv, rows, R))
    for row in table:
        n, a, w = int(row[1]), int(row[3]), int(row[4])
        val = lev[unpack_step(flat, row, Hkv)]
        out[:, :, a:a + w] += np.einsum("hrn,hnw->hrw", pv[:, :, :n], val)
    return out
