"""Attention restatements (numpy, float32, CPU).  TEST INFRASTRUCTURE ONLY.

``chunked_attention`` is the reference's dequantise-then-attend harness: the numerical reference
every CUDA decode path is checked against (max-abs 2e-3 in fp32).  ``strata_attend`` restates
STRATA's compressed-domain decode (exact-row partial + per-stratum flash partials merged by
log-sum-exp, rotation applied to the query).
"""

from __future__ import annotations

import numpy as np

from .codecs import unpack_planar

BIG = 1 << 40                                   # "never hidden" (STRATA_KV.py:297)


def _softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    m = np.max(x, axis=axis, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    e = np.exp(x - m)
    return e / e.sum(axis=axis, keepdims=True)


def chunked_attention(q, scaling, q_pos, K, V, kv_pos, hide_at, tok=None, chunk=256):
    """One softmax over exact rows (readable by query m iff kv_pos <= m < hide_at) and token
    entries (logit q.k + b, value v, visible iff tau <= m).  ``hide_at`` is (Tk,) or (B, Hkv, Tk).
    q (B, Hq, Tq, d) -> float32 out (B, Tq, Hq, d) (the reference casts to q's dtype afterwards;
    parity is judged before that cast).  GQA: KV head h serves query heads h*rep..h*rep+rep-1.
    Follows ``chunked_attention`` STRATA_KV.py:641-675."""
    q = np.asarray(q, np.float32)
    K = np.asarray(K, np.float32)
    V = np.asarray(V, np.float32)
    B, Hq, Tq, d = q.shape
    Hkv = K.shape[1]
    rep = Hq // Hkv
    q_pos = np.asarray(q_pos, np.int64)
    kv_pos = np.asarray(kv_pos, np.int64)
    hide_at = np.asarray(hide_at, np.int64)
    if tok is not None:
        tk = np.asarray(tok["k"], np.float32)
        tv = np.asarray(tok["v"], np.float32)
        tb = np.asarray(tok["b"], np.float32)
        ttau = np.asarray(tok["tau"], np.int64)
    out = np.empty((B, Hq, Tq, d), np.float32)
    qg = q.reshape(B, Hkv, rep, Tq, d)
    for s in range(0, Tq, chunk):
        qs = qg[:, :, :, s:s + chunk] * np.float32(scaling)                  # (B,Hkv,rep,t,d)
        qp = q_pos[s:s + chunk]
        if hide_at.ndim == 3:
            readable = (kv_pos[None, None, None, None, :] <= qp[None, None, None, :, None]) & \
                       (qp[None, None, None, :, None] < hide_at[:, :, None, None, :])
        else:
            readable = ((kv_pos[None, :] <= qp[:, None]) & (qp[:, None] < hide_at[None, :]))[None, None, None]
        blocks = [np.where(readable, np.einsum("bhrtd,bhnd->bhrtn", qs, K, optimize=True), -np.inf)]
        if tok is not None:
            vis = (ttau[None, :] <= qp[:, None])[None, None, None]
            lt = np.einsum("bhrtd,bhnd->bhrtn", qs, tk, optimize=True) + tb[:, :, None, None, :]
            blocks.append(np.where(vis, lt, -np.inf))
        p = _softmax(np.concatenate(blocks, -1).astype(np.float32))
        T0 = K.shape[2]
        o = np.einsum("bhrtn,bhnd->bhrtd", p[..., :T0], V, optimize=True)
        if tok is not None:
            o = o + np.einsum("bhrtn,bhnd->bhrtd", p[..., T0:], tv, optimize=True)
        out[:, :, s:s + chunk] = o.reshape(B, Hq, -1, d)
    return np.ascontiguousarray(out.transpose(0, 2, 1, 3))


def lse_merge(parts):
    """Exact merge of flash-decoding partials [(m, l, acc)], each m, l (..., rows), acc (..., rows, d):
    returns (M, L, ACC) with ACC / L the merged attention output (STRATA_KV.py:1784-1792)."""
    ms = np.stack([p[0] for p in parts], 0)
    M = ms.max(0)
    Mf = np.where(np.isfinite(M), M, 0.0)
    L = np.zeros_like(M)
    ACC = np.zeros_like(parts[0][2])
    for m, l, acc in parts:
        w = np.where(np.isfinite(m), np.exp(m - Mf), 0.0)
        L = L + w * l
        ACC = ACC + w[..., None] * acc
    return M, L, ACC


def tier_reference(qr, qb, bits, kc, vc, ks, vs):
    """Flash partials of one STRATA stratum: keys / values ``(c - h) * s`` from planar codes.
    qr (Hkv, rows, d) rotated + scaled query, qb (Hkv, rows) logit of the mean key.
    Returns m, l (Hkv, rows), acc (Hkv, rows, d) in the rotated value basis.
    Follows ``StrataState.tier_reference`` STRATA_KV.py:1751-1760."""
    half = np.float32((2 ** bits - 1) / 2.0)
    kh = (unpack_planar(kc, bits).astype(np.float32) - half) * np.asarray(ks, np.float32)[..., None]
    vh = (unpack_planar(vc, bits).astype(np.float32) - half) * np.asarray(vs, np.float32)[..., None]
    s = np.einsum("hrd,hnd->hrn", qr, kh, optimize=True) + qb[..., None]
    m = s.max(-1)
    e = np.exp(s - m[..., None])
    return m, e.sum(-1), np.einsum("hrn,hnd->hrd", e, vh, optimize=True)


def strata_attend(q, scaling, qpos, Kx, Vx, n0, H, tiers, mu_k, mu_v, R):
    """STRATA's compressed-domain decode in float32 (batch 1): exact rows Kx, Vx (1, Hkv, n, d)
    (the last n - n0 appended rows causal w.r.t. qpos), packed strata ``tiers`` (dicts with bits,
    kc, vc, ks, vs), fp16 means mu_k, mu_v (Hkv, d), rotation R (d, d).  The query is rotated once
    (q_r = scaling q R^T); stratum logits s_j (q_r . c_j) - s_j h sum(q_r) + scaling q . mu_K;
    partials merged exactly; coded sum lifted by R, plus (sum p) mu_V.
    Follows ``StrataState.attend`` STRATA_KV.py:1762-1796 (with dtype = float32)."""
    q = np.asarray(q, np.float32)
    B, Hq, Tq, d = q.shape
    Hkv = Kx.shape[1]
    rep = Hq // Hkv
    qg = q.reshape(Hkv, rep * Tq, d)
    n = Kx.shape[2]
    s_ex = np.einsum("hrd,hnd->hrn", qg, np.asarray(Kx[0], np.float32), optimize=True) * np.float32(scaling)
    if n > n0:
        row_pos = H + np.arange(n - n0)
        bad = row_pos[None, :] > np.asarray(qpos)[:, None]
        s_ex[..., n0:] = np.where(np.tile(bad, (rep, 1))[None], -np.inf, s_ex[..., n0:])
    m_e = s_ex.max(-1)
    e_ex = np.exp(s_ex - m_e[..., None])
    l_e = e_ex.sum(-1)
    o = np.einsum("hrn,hnd->hrd", e_ex, np.asarray(Vx[0], np.float32), optimize=True)
    if tiers:
        R = np.asarray(R, np.float32)
        qr = (qg @ R.T) * np.float32(scaling)
        qb = np.einsum("hrd,hd->hr", qg, np.asarray(mu_k, np.float32)) * np.float32(scaling)
        parts = [tier_reference(qr, qb, t["bits"], t["kc"], t["vc"], t["ks"], t["vs"]) for t in tiers]
        mc = np.stack([p_[0] for p_ in parts], 1)
        M = np.maximum(m_e, mc.max(1))
        we = np.exp(m_e - M)
        accr = np.zeros_like(o)
        wl = np.zeros_like(m_e)
        for m_, l_, a_ in parts:
            w_ = np.exp(m_ - M)
            accr += w_[..., None] * a_
            wl += w_ * l_
        o = (we[..., None] * o + accr @ R + wl[..., None] * np.asarray(mu_v, np.float32)[:, None, :]) / \
            (we * l_e + wl)[..., None]
    else:
        o = o / l_e[..., None]
    return np.ascontiguousarray(o.reshape(B, Hq, Tq, d).transpose(0, 2, 1, 3))
