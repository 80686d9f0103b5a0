"""LCTC's clipped uniform quantiser (uq_codes / uq_values, LCTC_KV.py:443-455) and operational
rate-distortion table (operational_rd, :458-481) in the oracle against the reference's own outputs
(lctc.npz).  Codes and values bit-exact; D within float32 round-off of the reference's float32 means;
the chosen clips equal wherever the two best multipliers of a (column, width) are not within that
round-off of each other.  CPU only."""

import numpy as np
import pytest

from oracle.lctc import operational_rd, uq_codes, uq_values


def test_uq_codes_values_golden(golden):
    g = golden("lctc")
    idx = uq_codes(g["uq_a"], g["uq_bits"], g["uq_clip"])
    np.testing.assert_array_equal(idx.astype(np.uint8), g["uq_idx"])
    np.testing.assert_array_equal(uq_values(idx, g["uq_bits"], g["uq_clip"]), g["uq_values"])


def check_rd(D, C, errs, ref_D, ref_C):
    """D within 2e-5 relative (the reference's float32 means over a few hundred to a few thousand rows
    carry ~1e-6 to 1e-5 of round-off; float64 sums here); clips within 1e-6 relative (the column rms
    from a float32 mean there, a float64 one here: an ulp apart at most) except at near-ties, where a
    different multiplier (12 % apart at 24 multipliers) may win."""
    # (a dead column's errors are float32 subnormals there, ~1e-42: compared absolutely)
    np.testing.assert_allclose(D, ref_D, rtol=2e-5, atol=1e-35)
    same = np.isclose(C, ref_C, rtol=1e-6, atol=0)
    if not same.all():
        # every differing choice is a near-tie: the reference's pick is within round-off of the best
        k, j = np.nonzero(~same)
        assert (j > 0).all()
        e = errs[k, j - 1]
        srt = np.sort(e, axis=-1)
        assert np.all(srt[:, 1] - srt[:, 0] <= 4e-5 * srt[:, 0]), (k, j)
    return int((~same).sum())


@pytest.mark.parametrize("name", ["rd24", "rd12"])
def test_operational_rd_golden(golden, name):
    g = golden("lctc")
    D, C, errs = operational_rd(g[f"{name}_A"], list(g[f"{name}_bits"]), g[f"{name}_mults"])
    assert check_rd(D, C, errs, g[f"{name}_D"], g[f"{name}_C"]) <= 2
    # the dead column: rms at its floor 1e-20, errors of the order of its clip squared
    assert np.all(g[f"{name}_D"][4] <= 1e-35) and np.all(D[4] <= 1e-35)
    np.testing.assert_allclose(C[4, 1:], g[f"{name}_mults"][0] * np.float32(1e-20), rtol=1e-6)


def test_uq_edges():
    bits = np.array([1, 2, 8, 8], np.float32)
    clip = np.array([1.0, 0.5, 3.0, 1e-3], np.float32)
    a = np.array([[-5.0, 0.5, 3.0, 0.0], [5.0, -0.5, -3.0, 1.0], [0.0, 0.25, 2.999, -1e-3]], np.float32)
    idx = uq_codes(a, bits, clip)
    assert idx.min() >= 0 and np.all(idx <= 2.0 ** bits - 1)
    np.testing.assert_array_equal(idx[0], [0, 3, 255, 128])     # clipped from below / above, and the middle
    np.testing.assert_array_equal(idx[1], [1, 0, 0, 255])
