"""Level tables for the non-uniform codes (host-side constants, computed once per width).

Lloyd-Max quantiser of a unit Gaussian (Max, IRE Trans. Inf. Theory 6(1), 1960): reconstruction
levels that are the conditional means of their cells, cell edges halfway between levels, found by
Lloyd's iteration.  The reference computes them the same way for its HEDGE code (HEDGE_KV.py:1055-1070:
a 360001-point grid over [-9, 9] weighted by the Gaussian density, cell-centre quantiles as the start,
500 iterations), so the tables here are the reference's float32 levels bit for bit.  They are inputs
of ``ops.hedge_quant`` and ``ops.decode_rows_lut``; no kernel work happens here.
"""

from __future__ import annotations

from functools import lru_cache

import numpy as np
import torch


@lru_cache(maxsize=None)
def _lloyd_max_np(bits: int) -> np.ndarray:
    from scipy.special import ndtri
    n = 1 << bits
    grid = np.linspace(-9.0, 9.0, 360001)
    dens = np.exp(-0.5 * grid * grid)
    dens /= dens.sum()
    lv = ndtri((np.arange(n) + 0.5) / n)
    for _ in range(500):
        cell = np.searchsorted((lv[1:] + lv[:-1]) / 2, grid)
        lv = np.bincount(cell, dens * grid, n) / np.maximum(np.bincount(cell, dens, n), 1e-300)
    return lv.astype(np.float32)


def lloyd_max(bits: int, device=None) -> torch.Tensor:
    """2^bits float32 Lloyd-Max levels of N(0, 1), ascending (bits 1..4 in the HEDGE code)."""
    if not 1 <= bits <= 8:
        raise ValueError("lloyd_max: bits must be in 1..8")
    return torch.from_numpy(_lloyd_max_np(bits).copy()).to(device)
