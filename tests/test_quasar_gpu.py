"""QUASAR's coded decode over embedded stage codes on the GPU (kvb_quasar_scores / kvb_quasar_values)
against the reference's own outputs (quasar.npz: QuasarState.coded_scores / coded_values,
QUASAR_KV.py:1918-1940) and the float64 oracle at a longer context.  Tolerance: 2e-5 of the largest
magnitude (float32 sums in another order than the reference's)."""

import numpy as np
import pytest
import torch

from oracle import quasar as Qo

pytestmark = pytest.mark.gpu


def _close(got, ref, rel=2e-5):
    assert np.abs(got - ref).max() <= rel * np.abs(ref).max(), (np.abs(got - ref).max(), np.abs(ref).max())


@pytest.mark.parametrize("name", ["a", "b"])
def test_coded_scores_values_golden(golden, cuda_dev, name):
    import kvb
    g = golden("quasar")
    Hkv, rows, n_c, R = (int(x) for x in g[f"{name}_shape"])
    f0 = torch.from_numpy(g[f"{name}_flat0"]).to(cuda_dev)
    f1 = torch.from_numpy(g[f"{name}_flat1"]).to(cuda_dev)
    sc = kvb.ops.quasar_scores(torch.from_numpy(g[f"{name}_qt"]).to(cuda_dev), f0, g[f"{name}_table0"],
                               g[f"{name}_levels"], n_c)
    va = kvb.ops.quasar_values(torch.from_numpy(g[f"{name}_pv"]).to(cuda_dev), f1, g[f"{name}_table1"],
                               g[f"{name}_levels"], R)
    _close(sc.cpu().numpy(), g[f"{name}_scores"])
    _close(va.cpu().numpy(), g[f"{name}_values"])
    assert kvb.device_status() == 0


def test_coded_long_context_matches_oracle(cuda_dev):
    """8 KV heads, 4 query rows, 16384 coded tokens, 128 coefficients in three bands at stages (2, 2, 4)."""
    import kvb
    rng = np.random.default_rng(5)
    Hkv, rows, n_c, R = 8, 4, 16384, 128
    levels = np.concatenate([rng.standard_normal(4), 0.3 * rng.standard_normal(4), 0.05 * rng.standard_normal(16)])
    levels = levels.astype(np.float32)
    lvl_off, stage_bits = [0, 4, 8], [2, 2, 4]
    table, chunks, off = [], [], 0
    for a, w, nst in ((0, 32, 3), (32, 32, 2), (64, 64, 1)):
        for t in range(nst):
            n = int(n_c * (1.0 - 0.2 * t - 0.1 * (a // 32)))
            b = stage_bits[t]
            nb = w * b // 8
            by = rng.integers(0, 256, (Hkv, n, nb), dtype=np.uint8)
            table.append([off, n, nb, a, w, b, lvl_off[t]])
            chunks.append(by.reshape(-1))
            off += by.size
    flat = np.concatenate(chunks)
    table = np.array(table, np.int32)
    qt = rng.standard_normal((Hkv, rows, R)).astype(np.float32)
    pv = rng.random((Hkv, rows, n_c)).astype(np.float32)
    pv /= pv.sum(-1, keepdims=True)
    ft = torch.from_numpy(flat).to(cuda_dev)
    for _ in range(2):
        sc = kvb.ops.quasar_scores(torch.from_numpy(qt).to(cuda_dev), ft, table, levels, n_c)
        va = kvb.ops.quasar_values(torch.from_numpy(pv).to(cuda_dev), ft, table, levels, R)
        _close(sc.cpu().numpy(), Qo.coded_scores(qt, flat, table, levels, n_c))
        _close(va.cpu().numpy(), Qo.coded_values(pv, flat, table, levels, R))
    assert kvb.device_status() == 0


def test_coded_rejects_steps_outside_the_buffer(cuda_dev):
    import kvb
    flat = torch.zeros(100, dtype=torch.uint8, device=cuda_dev)
    qt = torch.zeros(1, 4, 32, device=cuda_dev)
    with pytest.raises(ValueError):
        kvb.ops.quasar_scores(qt, flat, [[0, 50, 4, 0, 16, 2, 0]], np.zeros(4, np.float32), 50)   # 200 > 100 bytes
    with pytest.raises(ValueError):
        kvb.ops.quasar_scores(qt, flat, [[0, 10, 4, 24, 16, 2, 0]], np.zeros(4, np.float32), 10)  # band past R
