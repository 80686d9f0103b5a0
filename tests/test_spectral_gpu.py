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


@pytest.mark.parametrize("B,H,T,bits,amp", [(1, 2, 256, 4, 1.0), (2, 3, 1000, 4, 1.0), (1, 2, 129, 2, 1.0),
                                             (1, 1, 300, 8, 1.0), (2, 8, 4096, 4, 1.0), (1, 4, 2048, 4, 1e-3),
                                             (1, 4, 2048, 2, 300.0), (1, 4, 1111, 8, 40.0)])
def test_projection_and_code(cuda_dev, B, H, T, bits, amp):
    """Coefficients to float32 accuracy; codes and scales bit-exact given those coefficients (the
    code's division runs through a correctly rounded reciprocal + Markstein correction: millions of
    quotients over several exponent ranges here)."""
    import kvb
    bases, K, V = _inputs(B, H, T, seed=T + bits)
    K = (K.float() * amp).half()
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


def test_projection_strided_input(cuda_dev):
    """x as a (B, H, T, d) view of (B, T, H, d) storage (a model's projection layout): the 4D tensor
    map reads it in place, same codes as the contiguous copy."""
    import kvb
    bases, K, V = _inputs(2, 4, 700, seed=5)
    hilo = kvb.ops.split_basis(bases[:, :, :32].float().to(cuda_dev))
    Kc = K.to(cuda_dev).contiguous()
    Ks = Kc.transpose(1, 2).contiguous().transpose(1, 2)
    assert not Ks.is_contiguous()
    a = kvb.ops.spectral_encode(Kc, hilo, 4, want_coef=True)
    b = kvb.ops.spectral_encode(Ks, hilo, 4, want_coef=True)
    assert torch.equal(a["codes"], b["codes"]) and torch.equal(a["meta"], b["meta"])
    assert torch.equal(a["coef"], b["coef"])


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
