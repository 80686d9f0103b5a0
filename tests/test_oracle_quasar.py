"""QUASAR's coded decode over embedded stage codes (coded_scores / coded_values, QUASAR_KV.py:1918-1940)
in the oracle against the reference's own outputs (quasar.npz): the restatement is float64, the
reference float32 per step, so they agree to 1e-6 of the largest magnitude.  CPU only."""

import numpy as np
import pytest

from oracle import quasar as Qo


@pytest.mark.parametrize("name", ["a", "b"])
def test_coded_scores_and_values_golden(golden, name):
    g = golden("quasar")
    Hkv, rows, n_c, R = (int(x) for x in g[f"{name}_shape"])
    sc = Qo.coded_scores(g[f"{name}_qt"], g[f"{name}_flat0"], g[f"{name}_table0"], g[f"{name}_levels"], n_c)
    va = Qo.coded_values(g[f"{name}_pv"], g[f"{name}_flat1"], g[f"{name}_table1"], g[f"{name}_levels"], R)
    ref_s, ref_v = g[f"{name}_scores"], g[f"{name}_values"]
    assert np.abs(sc - ref_s).max() <= 1e-6 * np.abs(ref_s).max()
    assert np.abs(va - ref_v).max() <= 1e-6 * np.abs(ref_v).max()
