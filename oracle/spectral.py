"""Spectral (basis-projection) code restatements (numpy, CPU).  TEST INFRASTRUCTURE ONLY.

Per KV head an orthonormal basis B (d x d); a vector x is stored as its leading r coefficients
c = x B[:, :r], coded with the STRATA per-token uniform code (one fp16 scale, b bits, mid-rise);
attention runs in the coefficient domain: q~ = scaling q B[:, :r], logit s_j (q~ . c_j) - s_j h
sum(q~), value sum lifted back by B[:, :r]^T.  The coefficient-domain decode follows
``QuasarState.attend`` QUASAR_KV.py:1942-1967 (one stage, one band); the code follows
``strata_quantize`` STRATA_KV.py:1158-1168; the QR basis follows the non-power-of-two branch of
``rotation_matrix`` STRATA_KV.py:1126-1127.
"""

from __future__ import annotations

import math
import zlib

import numpy as np

from .codecs import strata_quantize, pack_planar
from .attention import _softmax

SEED = 42


def rotation_matrix(d: int, key: str) -> np.ndarray:
    """Seeded orthogonal matrix: randomised Hadamard H diag(+-1) / sqrt(d) when d is a power of two,
    else the sign-fixed Q factor of a seeded Gaussian.  Restates ``rotation_matrix``
    STRATA_KV.py:1110-1128 with its seeding (``_rng`` STRATA_KV.py:304-305: numpy default_rng
    over [42, crc32("rotation"), crc32(key)])."""
    g = np.random.default_rng([SEED] + [zlib.crc32(str(s).encode()) for s in ("rotation", key)])
    if d & (d - 1) == 0:
        Hm = np.array([[1.0]])
        while Hm.shape[0] < d:
            Hm = np.block([[Hm, Hm], [Hm, -Hm]])
        R = Hm / math.sqrt(d) * g.choice([-1.0, 1.0], d)[None, :]
    else:
        Q, Rr = np.linalg.qr(g.standard_normal((d, d)))
        R = Q * np.sign(np.diag(Rr))[None, :]
    return R.astype(np.float32)


def seeded_qr_basis(d: int, seed: int, head: int) -> np.ndarray:
    """Orthonormal (d, d) basis of one KV head: Q of the QR factorisation of a Gaussian matrix drawn
    from numpy default_rng([seed, head]), columns sign-fixed so diag(R) > 0 (the QR branch of
    STRATA_KV.py:1126-1127, seeded per head).  float64."""
    g = np.random.default_rng([seed, head])
    Q, Rr = np.linalg.qr(g.standard_normal((d, d)))
    return Q * np.sign(np.diag(Rr))[None, :]


def spectral_encode(X, basis_r, bits=4):
    """X (B, Hkv, T, d), basis_r (Hkv, d, r) -> coefficients C (float32, B, Hkv, T, r), codes (uint8),
    scales s (float32 holding fp16 values, B, Hkv, T), planar-packed codes (B, Hkv, T, r * bits / 8)."""
    X = np.asarray(X, np.float32)
    Br = np.asarray(basis_r, np.float32)
    C = np.einsum("bhtd,hdr->bhtr", X, Br, optimize=True).astype(np.float32)
    codes, s, _ = strata_quantize(C, bits)
    return C, codes, s, pack_planar(codes, bits)


def spectral_attend(q, scaling, basis_r, kcodes, ks, vcodes, vs, bits=4):
    """Coefficient-domain decode attention (float32).  q (B, Hq, Tq, d); codes (B, Hkv, T, r) uint8;
    scales (B, Hkv, T).  Returns out (B, Tq, Hq, d).  Equal, by Prop. 2 of the reference
    (STRATA_KV.py:90-93), to dequantise-then-attend over x_hat = ((c - h) s) B_r^T."""
    q = np.asarray(q, np.float32)
    B, Hq, Tq, d = q.shape
    Hkv = kcodes.shape[1]
    rep = Hq // Hkv
    Br = np.asarray(basis_r, np.float32)
    half = np.float32((2 ** bits - 1) / 2.0)
    qt = np.einsum("bhrd,hdk->bhrk", q.reshape(B, Hkv, rep * Tq, d), Br, optimize=True) * np.float32(scaling)
    kh = (kcodes.astype(np.float32) - half) * np.asarray(ks, np.float32)[..., None]
    vh = (vcodes.astype(np.float32) - half) * np.asarray(vs, np.float32)[..., None]
    p = _softmax(np.einsum("bhrk,bhtk->bhrt", qt, kh, optimize=True))
    acc = np.einsum("bhrt,bhtk->bhrk", p, vh, optimize=True)
    o = np.einsum("bhrk,hdk->bhrd", acc, Br, optimize=True)
    return np.ascontiguousarray(o.reshape(B, Hq, Tq, d).transpose(0, 2, 1, 3))
