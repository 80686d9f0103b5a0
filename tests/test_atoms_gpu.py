"""TILT's moment-atom read on the GPU (kvb_atom_read) against the reference's own atom_read outputs
(atoms.npz, TILT_KV.py:673-714) for every combination of order, tilt, projection and phase, and the
float64 oracle at rank 8 with longer query blocks.  Float32 dot products in another order than the
reference's: logits within 2e-4, factors and tilt coordinates within 1e-4 relative."""

import numpy as np
import pytest
import torch

from oracle.atoms import atom_read as oracle_read

pytestmark = pytest.mark.gpu
KEYS = ("mu_k", "logn", "U", "lam", "diag", "R", "A", "Bk", "Rv")


def _check(got, ref):
    logit, cfac, tB = got
    lg = logit.cpu().numpy()
    np.testing.assert_array_equal(np.isneginf(lg), np.isneginf(ref[0]))
    fin = np.isfinite(ref[0])
    np.testing.assert_allclose(lg[fin], ref[0][fin], rtol=1e-5, atol=2e-4)
    np.testing.assert_allclose(cfac.cpu().numpy(), ref[1], rtol=1e-4, atol=1e-5)
    if ref[2] is None:
        assert tB is None
    else:
        np.testing.assert_allclose(tB.cpu().numpy(), ref[2], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("name", list("abcde"))
def test_atom_read_golden(golden, cuda_dev, name):
    import kvb
    g = golden("atoms")
    order, tilt, project, phase, rep = (int(x) for x in g[f"{name}_flags"])
    mom = {k: torch.from_numpy(g[k]).to(cuda_dev) for k in KEYS}
    mom.update(order=order, tilt=bool(tilt), project=bool(project), phase=bool(phase))
    got = kvb.ops.atom_read(torch.from_numpy(g["qs"]).to(cuda_dev), mom, rep)
    _check(got, (g[f"{name}_logit"], g[f"{name}_cfac"], g.get(f"{name}_tB")))
    assert kvb.device_status() == 0


def test_atom_read_rank8_matches_oracle(cuda_dev):
    import kvb
    rng = np.random.default_rng(8)
    B, H, rep, c, NA, d, r = 1, 8, 4, 32, 4, 128, 8
    f = lambda *s: rng.standard_normal(s).astype(np.float32)
    mom = {"mu_k": 0.3 * f(B, H, NA, d), "logn": np.log(rng.integers(16, 512, (B, H, NA))).astype(np.float32),
           "U": f(B, H, NA, d, r) / 11.3, "lam": (2 * rng.random((B, H, NA, r))).astype(np.float32),
           "diag": (0.05 * rng.random((B, H, NA, d))).astype(np.float32), "R": (2 + 3 * rng.random((B, H, NA))).astype(np.float32),
           "A": f(B, H, NA, d, r) / 11.3, "Bk": f(B, H, NA, d, r) / 11.3, "Rv": (0.2 + rng.random((B, H, NA))).astype(np.float32)}
    qs = f(B, H * rep, c, d) * 1.5
    flags = dict(order=2, tilt=True, project=True, phase=True)
    ref = oracle_read(qs, dict(mom, **flags), rep)
    got = kvb.ops.atom_read(torch.from_numpy(qs).to(cuda_dev),
                            dict({k: torch.from_numpy(v).to(cuda_dev) for k, v in mom.items()}, **flags), rep)
    _check(got, ref)
