"""TILT's moment-atom read (atom_read, TILT_KV.py:673-714) in the oracle against the reference's own
outputs (atoms.npz) for every combination of order, tilt, projection and the phase correction,
including a disabled atom (log-mass -inf).  Float64 here, float32 there.  CPU only."""

import numpy as np
import pytest

from oracle.atoms import atom_read

KEYS = ("mu_k", "logn", "U", "lam", "diag", "R", "A", "Bk", "Rv")


def moments(g, name):
    order, tilt, project, phase, rep = (int(x) for x in g[f"{name}_flags"])
    mom = {k: g[k] for k in KEYS}
    mom.update(order=order, tilt=bool(tilt), project=bool(project), phase=bool(phase))
    return mom, rep


@pytest.mark.parametrize("name", list("abcde"))
def test_atom_read_golden(golden, name):
    g = golden("atoms")
    mom, rep = moments(g, name)
    logit, cfac, tB = atom_read(g["qs"], mom, rep)
    ref = g[f"{name}_logit"]
    np.testing.assert_array_equal(np.isneginf(logit), np.isneginf(ref))
    fin = np.isfinite(ref)
    np.testing.assert_allclose(logit[fin], ref[fin], rtol=1e-6, atol=1e-4)
    np.testing.assert_allclose(cfac, g[f"{name}_cfac"], rtol=1e-5, atol=1e-6)
    if mom["tilt"]:
        np.testing.assert_allclose(tB, g[f"{name}_tB"], rtol=1e-5, atol=1e-5)
    else:
        assert tB is None and f"{name}_tB" not in g
