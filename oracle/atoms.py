"""TILT's moment-atom read (numpy, CPU).  TEST INFRASTRUCTURE ONLY (see package docstring).

Restates ``atom_read`` (TILT_KV.py:673-714): for scaled queries qs (B, Hq, c, d) and the atoms of KV
head h = hq // rep (HF repeat_kv order), per atom a

    logit = qs . mu_k + log n
    order 2:  v2 = sum_d qs_d^2 diag_d + sum_r (qs . U_r)^2 lam_r
              phase (Prop. 6): L = max(log n, 0), sigma = sqrt(max(v2, 0)), sigma_c = sqrt(2 L);
                g = v2 / 2 and cfac = 1 while sigma <= sigma_c, else g = sigma sigma_c - L and
                cfac = sigma_c / sigma;  without phase g = v2 / 2
              project (Prop. 4): m = |qs| R; where g > m: cfac = m / v2, g = m
              logit += g
    tilt:     tB_r = qs . Bk_r;  |cfac A tB| through the Gram matrix A^T A; cfac *= min(Rv / |...|, 1)

Returns logit, cfac (B, Hq, c, NA) and tB (B, Hq, c, NA, r) or None.  Float64.
"""

from __future__ import annotations

import numpy as np


def atom_read(qs, mom: dict, rep: int):
    qs = np.asarray(qs, np.float64)
    f = {k: (np.repeat(np.asarray(v, np.float64), rep, axis=1) if isinstance(v, np.ndarray) else v)
         for k, v in mom.items()}
    logit = np.einsum("bhcd,bhad->bhca", qs, f["mu_k"]) + f["logn"][:, :, None]
    cfac = np.ones_like(logit)
    if mom["order"] == 2:
        proj = np.einsum("bhcd,bhadr->bhcar", qs, f["U"])
        v2 = np.einsum("bhcd,bhad->bhca", qs ** 2, f["diag"]) + (proj ** 2 * f["lam"][:, :, None]).sum(-1)
        if mom.get("phase", True):
            L = np.maximum(f["logn"][:, :, None], 0.0)
            sig = np.sqrt(np.maximum(v2, 0.0))
            sc = np.sqrt(2 * L)
            hot = sig <= sc
            g = np.where(hot, 0.5 * v2, sig * sc - L)
            cfac = np.where(hot, cfac, sc / np.maximum(sig, 1e-30))
        else:
            g = 0.5 * v2
        if mom["project"]:
            mb = np.linalg.norm(qs, axis=-1, keepdims=True) * f["R"][:, :, None]
            cfac = np.where(g <= mb, cfac, mb / np.maximum(v2, 1e-30))
            g = np.minimum(g, mb)
        logit = logit + g
    tB = None
    if mom["tilt"]:
        tB = np.einsum("bhcd,bhadr->bhcar", qs, f["Bk"])
        gram = np.einsum("bhadr,bhads->bhars", f["A"], f["A"])
        nrm = cfac * np.sqrt(np.maximum(np.einsum("bhcar,bhars,bhcas->bhca", tB, gram, tB), 0.0))
        with np.errstate(divide="ignore"):
            cfac = cfac * np.minimum(f["Rv"][:, :, None] / np.maximum(nrm, 1e-30), 1.0)
    return logit, cfac, tB
