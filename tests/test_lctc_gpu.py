"""kvb_uq_codes / kvb_uq_values / kvb_operational_rd (LCTC's quantiser and rate-distortion table,
LCTC_KV.py:443-481) on the GPU: codes and values bit-identical to the reference's own (lctc.npz); the
RD table against the reference within its float32 round-off (clips equal but at near-ties) and against
the oracle run with the same clip multipliers (clips equal, D to 1e-12); the LCTC calibration shape
(8192 rows); bad widths."""

import numpy as np
import pytest
import torch

from oracle.lctc import operational_rd as oracle_rd
from test_oracle_lctc import check_rd

pytestmark = pytest.mark.gpu


def test_uq_codes_values_match_reference(golden, cuda_dev):
    from kvb import lctc
    g = golden("lctc")
    a = torch.from_numpy(g["uq_a"]).to(cuda_dev)
    bits, clip = torch.from_numpy(g["uq_bits"]).to(cuda_dev), torch.from_numpy(g["uq_clip"]).to(cuda_dev)
    codes, values = lctc.uq_quantize(a, bits, clip)
    np.testing.assert_array_equal(codes.cpu().numpy(), g["uq_idx"])
    np.testing.assert_array_equal(values.cpu().numpy(), g["uq_values"])
    np.testing.assert_array_equal(lctc.uq_codes(a, bits, clip).cpu().numpy(), g["uq_idx"].astype(np.float32))
    np.testing.assert_array_equal(lctc.uq_values(codes, bits, clip).cpu().numpy(), g["uq_values"])
    # a strided view of the same rows gives the same codes
    wide = torch.zeros(a.shape[0], a.shape[1] + 16, device=cuda_dev)
    wide[:, :a.shape[1]] = a
    c2, _ = lctc.uq_quantize(wide[:, :a.shape[1]], bits, clip)
    assert torch.equal(c2, codes)


@pytest.mark.parametrize("name", ["rd24", "rd12"])
def test_operational_rd_matches_reference(golden, cuda_dev, name):
    from kvb import lctc
    g = golden("lctc")
    A = torch.from_numpy(g[f"{name}_A"]).to(cuda_dev)
    bits = [int(b) for b in g[f"{name}_bits"]]
    M = len(g[f"{name}_mults"])
    D, C = lctc.operational_rd(A, bits, M)
    D, C = D.cpu().numpy(), C.cpu().numpy()
    mults = torch.logspace(np.log10(0.5), np.log10(8.0), M, device=cuda_dev).cpu().numpy()
    oD, oC, errs = oracle_rd(g[f"{name}_A"], bits, mults)
    np.testing.assert_array_equal(C, oC)
    np.testing.assert_allclose(D, oD, rtol=1e-12, atol=1e-40)
    assert check_rd(D, C, errs, g[f"{name}_D"], g[f"{name}_C"]) <= 2


def test_operational_rd_calibration_shape(cuda_dev):
    """RD_ROWS = 8192 calibration rows (LCTC_KV.py:280) of 256 heavy-tailed KLT coefficients."""
    from kvb import lctc
    gen = torch.Generator().manual_seed(5)
    A = torch.randn(8192, 256, generator=gen) * torch.exp(torch.randn(256, generator=gen))
    A = A * (1 + 3 * (torch.rand(8192, 256, generator=gen) < 0.01))          # a few outliers per column
    bits = [0, 1, 2, 3, 4, 5, 6, 8]
    D, C = lctc.operational_rd(A.to(cuda_dev), bits, 24)
    mults = torch.logspace(np.log10(0.5), np.log10(8.0), 24, device=cuda_dev).cpu().numpy()
    oD, oC, _ = oracle_rd(A.numpy(), bits, mults)
    np.testing.assert_array_equal(C.cpu().numpy(), oC)
    np.testing.assert_allclose(D.cpu().numpy(), oD, rtol=1e-12)
    assert (np.diff(oD[:, 1:], axis=1) <= 0).all()          # more bits never cost distortion here


def test_bad_widths(cuda_dev):
    import kvb
    from kvb import lctc
    A = torch.randn(64, 8, device=cuda_dev)
    with pytest.raises(ValueError):
        lctc.operational_rd(A, [1, 2, 4], 8)                   # the first width must be 0
    with pytest.raises(ValueError):
        lctc.operational_rd(A, [0, 2, 9], 8)                   # widths 1..8
    kvb.device_status()
    codes, _ = lctc.uq_quantize(A, torch.full((8,), 2.5, device=cuda_dev), torch.ones(8, device=cuda_dev))
    torch.cuda.synchronize()
    assert kvb.device_status() != 0                            # non-integral width: flagged, nothing written
    assert kvb.device_status() == 0
