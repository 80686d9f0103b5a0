"""Seeded synthetic inputs with the shapes and value distributions of the five benchmark configs.

The reference measures on real models and long-context datasets that are not available here;
these generators stand in for them with the distributions the configs name (no dataset items are
reproduced).  Seeds follow the reference's SEED = 42 (STRATA_KV.py:271): config c uses 42 + c.
Small cases are generated on the CPU (bit-identical for the oracle); full-size cases are generated
directly on the GPU with a seeded CUDA generator.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

SEED = 42


@dataclass(frozen=True)
class Shape:
    layers: int
    B: int
    Hq: int
    Hkv: int
    d: int
    T: int
    dtype: torch.dtype


C0 = Shape(1, 1, 32, 8, 128, 4096, torch.float16)
C1 = Shape(32, 8, 32, 8, 128, 32768, torch.bfloat16)
C2 = Shape(32, 4, 32, 8, 128, 32768, torch.bfloat16)
C3 = Shape(1, 16, 32, 8, 128, 16384, torch.float16)
C4 = Shape(80, 32, 64, 8, 128, 131072, torch.bfloat16)


def gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def outlier_kv(B, Hkv, T, d, dtype, device="cpu", seed=SEED, n_outlier=4, factor=8.0):
    """Config 0 / 4: K, V ~ N(0, 1); per KV head 4 seeded channels scaled x8 (outliers)."""
    g = gen(device, seed)
    K = torch.randn(B, Hkv, T, d, generator=g, device=device)
    V = torch.randn(B, Hkv, T, d, generator=g, device=device)
    gc = gen("cpu", seed + 1000)
    scale = torch.ones(Hkv, d)
    for h in range(Hkv):
        scale[h, torch.randperm(d, generator=gc)[:n_outlier]] = factor
    K = K * scale.to(device)[None, :, None, :]
    return K.to(dtype), V.to(dtype)


def lognormal_kv(B, Hkv, T, d, dtype, device="cpu", seed=SEED + 1, layer=0):
    """Config 1: keys N(0, 1) x a per-channel lognormal(0, 0.5) scale (one draw per layer and KV
    head), values N(0, 1)."""
    gc = gen("cpu", seed * 1000 + layer)
    chs = torch.exp(0.5 * torch.randn(Hkv, d, generator=gc))
    g = gen(device, seed * 1000 + layer + 1)
    K = torch.randn(B, Hkv, T, d, generator=g, device=device) * chs.to(device)[None, :, None, :]
    V = torch.randn(B, Hkv, T, d, generator=g, device=device)
    return K.to(dtype), V.to(dtype)


def queries(B, Hq, Tq, d, dtype, device="cpu", seed=SEED):
    g = gen(device, seed + 7)
    return torch.randn(B, Hq, Tq, d, generator=g, device=device).to(dtype)


def spectral_kv(B, Hkv, T, d, basis, dtype, device="cpu", seed=SEED + 3):
    """Config 3: coordinate i in the head's basis ~ N(0, (1 / (1 + i))^2): X = Z diag(1/(1+i)) B^T."""
    g = gen(device, seed)
    decay = (1.0 / (1.0 + torch.arange(d, dtype=torch.float32))).to(device)
    Bm = basis.to(device=device, dtype=torch.float32)                      # (Hkv, d, d)
    K = torch.einsum("bhtk,hdk->bhtd", torch.randn(B, Hkv, T, d, generator=g, device=device) * decay, Bm)
    V = torch.einsum("bhtk,hdk->bhtd", torch.randn(B, Hkv, T, d, generator=g, device=device) * decay, Bm)
    return K.to(dtype), V.to(dtype)


def qr_bases(Hkv: int, d: int, seed: int = SEED + 3) -> torch.Tensor:
    """Per KV head, the sign-fixed Q factor of a seeded Gaussian (QR branch of rotation_matrix,
    STRATA_KV.py:1126-1127): (Hkv, d, d) float64, orthonormal columns."""
    import numpy as np
    out = np.empty((Hkv, d, d))
    for h in range(Hkv):
        rng = np.random.default_rng([seed, h])
        Q, R = np.linalg.qr(rng.standard_normal((d, d)))
        out[h] = Q * np.sign(np.diag(R))[None, :]
    return torch.from_numpy(out)


def coverage_layer(Hq, Hkv, T, d, dtype, device="cpu", seed=SEED + 1, o_dim=None):
    """One layer's prefill for STRATA's coverage statistics (config 1's shape, batch row 1): queries and
    keys with a decaying per-channel spectrum (keys offset by 1, as the reference's own self-test draws
    them, STRATA_KV.py:1963-1967), values N(0, 1), and output metrics M_a = W_aᵀ W_a from seeded
    Gaussian output projections W_a ((3/2) d x d, scaled 1 / sqrt(d))."""
    g = gen(device, seed)
    spec = torch.exp(-torch.arange(d, device=device) / (d / 5.0)).sqrt()
    q = (torch.randn(1, Hq, T, d, generator=g, device=device) * spec * 3).to(dtype)
    k = (torch.randn(1, Hkv, T, d, generator=g, device=device) * spec * 3 + 1.0).to(dtype)
    v = torch.randn(1, Hkv, T, d, generator=g, device=device).to(dtype)
    Wa = torch.randn(Hq, o_dim or (3 * d // 2), d, generator=g, device=device) / d ** 0.5
    M = (Wa.transpose(-1, -2) @ Wa).float().contiguous()
    return q, k, v, M
