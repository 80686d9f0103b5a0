"""Pins the coefficient-domain decode restatement (oracle.spectral_attend) to the golden-pinned
dequantise-then-attend oracle (oracle.chunked_attention, checked against the reference's own
outputs in test_oracle_golden.py).

By Prop. 2 of the reference (STRATA_KV.py:90-93), attention in the coefficient domain equals
attention over the reconstructed vectors x_hat = ((c - h) s) B_r^T: the logits q . x_hat =
(q B_r) . ((c - h) s) because B_r has orthonormal columns, and the attended value lifts back by
B_r^T.  So the two oracles must agree to float32 rounding on any codes, scales and basis; the
config-3 decode's 2e-3 check against spectral_attend thereby rests on the pinned chunked_attention.
"""

import numpy as np
import pytest

import oracle as O


@pytest.mark.parametrize("B,Hkv,rep,Tq,T,bits,r", [(1, 2, 4, 1, 300, 4, 32), (2, 3, 4, 2, 129, 4, 32),
                                                   (1, 1, 8, 1, 1000, 2, 16), (2, 2, 2, 3, 64, 8, 128)])
def test_spectral_attend_equals_dequantise_then_attend(B, Hkv, rep, Tq, T, bits, r):
    d = 128
    g = np.random.default_rng([B, Hkv, rep, T, bits, r])
    basis = np.stack([O.seeded_qr_basis(d, 45, h) for h in range(Hkv)])          # (Hkv, d, d) float64
    br = basis[:, :, :r].astype(np.float32)
    kc = g.integers(0, 2 ** bits, (B, Hkv, T, r), dtype=np.uint8)
    vc = g.integers(0, 2 ** bits, (B, Hkv, T, r), dtype=np.uint8)
    ks = (np.abs(g.standard_normal((B, Hkv, T))) * 0.3 + 0.01).astype(np.float16).astype(np.float32)
    vs = (np.abs(g.standard_normal((B, Hkv, T))) * 0.3 + 0.01).astype(np.float16).astype(np.float32)
    q = g.standard_normal((B, Hkv * rep, Tq, d)).astype(np.float32)
    out = O.spectral_attend(q, d ** -0.5, br, kc, ks, vc, vs, bits=bits)
    half = (2 ** bits - 1) / 2.0
    # reconstructions in model space (float64 to keep the comparison about the oracle, not rounding)
    kh = np.einsum("bhtk,hdk->bhtd", (kc - half) * ks[..., None].astype(np.float64), br.astype(np.float64))
    vh = np.einsum("bhtk,hdk->bhtd", (vc - half) * vs[..., None].astype(np.float64), br.astype(np.float64))
    ref = O.chunked_attention(q, d ** -0.5, np.full(Tq, T), kh.astype(np.float32), vh.astype(np.float32),
                              np.arange(T), np.full(T, O.attention.BIG), None, 256)
    assert out.shape == ref.shape
    np.testing.assert_allclose(out, ref, rtol=0, atol=2e-5 * max(1.0, float(np.abs(ref).max())))


def test_spectral_attend_full_rank_is_plain_attention():
    """r = d: the basis drops out entirely (B B^T = I), so coefficient-domain attention over the
    coded coefficients of x equals plain attention over the reconstructions in model space."""
    d, T, Hkv, rep = 128, 200, 2, 4
    g = np.random.default_rng(7)
    basis = np.stack([O.seeded_qr_basis(d, 3, h) for h in range(Hkv)]).astype(np.float32)
    X = g.standard_normal((1, Hkv, T, d)).astype(np.float32)
    C, codes, s, _ = O.spectral_encode(X, basis, bits=8)
    q = g.standard_normal((1, Hkv * rep, 1, d)).astype(np.float32)
    out = O.spectral_attend(q, d ** -0.5, basis, codes, s, codes, s, bits=8)
    xh = np.einsum("bhtk,hdk->bhtd", (codes - 127.5) * s[..., None], basis)
    ref = O.chunked_attention(q, d ** -0.5, np.array([T]), xh, xh, np.arange(T), np.full(T, O.attention.BIG))
    np.testing.assert_allclose(out, ref, rtol=0, atol=2e-5)
