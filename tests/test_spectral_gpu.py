"""K4 spectral code (tcgen05 projection + mid-rise code epilogue) and coefficient-domain decode vs the
oracle: float32-grade coefficients, bit-exact codes / scales given those coefficients, attention
within 2e-3 of the oracle's coefficient-domain decode (equal to dequantise-then-attend, Prop. 2)."""

import numpy as np
import pytest
import torch

import oracle as O
from kvref import np32, unpack

pytestmark = pytest.mark.gpu


def _inputs(B, H, T, seed):
    import kvb
    bases = kvb.workloads.qr_bases(H, 128, seed=seed)
    K, V = kvb.workloads.spectral_kv(B, H, T, 128, bases, torch.float16, seed=seed)
    return bases, K, V


@pytest.mark.parametrize("B,H,T,bits", [(1, 2, 256, 4), (2, 3, 1000, 4), (1, 2, 129, 2), (1, 1, 300, 8)])
def test_projection_and_code(cuda_dev, B, H, T, bits):
    import kvb
    bases, K, V = _inputs(B, H, T, seed=T + bits)
    br = bases[:, :, :32].float()
    hilo = kvb.ops.split_basis(br.to(cuda_dev))
    r = kvb.ops.spectral_encode(K.to(cuda_dev), hilo, bits, want_coef=True)
    assert kvb.device_status() == 0
    coef = r["coef"].cpu().numpy()
    ref = np.einsum("bhtd,hdr->bhtr", np32(K).astype(np.float64), br.numpy().astype(np.float64))
    assert np.abs(coef - ref).max() <= 2e-5 * max(1.0, np.abs(ref).max())
    # the code of the GPU's own coefficients is exactly the oracle's
    c, s, _ = O.strata_quantize(coef, bits)
    np.testing.assert_array_equal(unpack(r["codes"], bits, T), c)
    np.testing.assert_array_equal(r["meta"][:, :, :T].float().cpu().numpy(), s)


@pytest.mark.parametrize("rep,Tq", [(4, 1), (4, 2)])
def test_spectral_decode(cuda_dev, rep, Tq):
    import kvb
    B, H, T = 2, 2, 1500
    bases, K, V = _inputs(B, H, T, seed=55)
    cache = kvb.cache.build_spectral(K.to(cuda_dev), V.to(cuda_dev), bases)
    q = kvb.workloads.queries(B, H * rep, Tq, 128, torch.float16, seed=55)
    out = kvb.decode(cache, q.to(cuda_dev), 128 ** -0.5, qpos=[T] * Tq, out_dtype=torch.float32).cpu().numpy()
    s = cache.strata[0]
    br = bases[:, :, :32].float().numpy()
    ref = O.spectral_attend(np32(q), 128 ** -0.5, br, unpack(s["kc"], 4, T), s["km"][:, :, :T].float().cpu().numpy(),
                            unpack(s["vc"], 4, T), s["vm"][:, :, :T].float().cpu().numpy(), bits=4)
    err = np.abs(out - ref).max()
    assert err <= 2e-3, err
