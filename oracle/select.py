"""Importance scores and budgeted selection (numpy, CPU).  TEST INFRASTRUCTURE ONLY.

Selection contract (index work, bit-exact): larger score first, LOWER index on ties (a stable
descending sort), kept indices returned in ascending position order.  The reference uses
``torch.topk`` whose tie order is unspecified; this rule is the explicit one the CUDA selection
kernel implements, and the golden tests check the reference's sets wherever its scores have no
ties at the k-th position.
"""

from __future__ import annotations

import numpy as np

from .attention import _softmax


def _avg_pool1d(sc: np.ndarray, kernel: int) -> np.ndarray:
    """torch ``avg_pool1d(kernel, stride 1, padding kernel // 2)`` with zero padding counted."""
    pad = kernel // 2
    n = sc.shape[-1]
    z = np.zeros(sc.shape[:-1] + (n + 2 * pad,), np.float32)
    z[..., pad:pad + n] = sc
    acc = np.zeros_like(sc, dtype=np.float32)
    for i in range(kernel):
        acc = acc + z[..., i:i + n]
    return (acc / np.float32(kernel)).astype(np.float32)


def snapkv_scores(q, k, H, scaling, window=64, kernel=5):
    """SnapKV scores: the last ``window`` context queries attend causally to the context (fp32
    softmax), window columns dropped, mean over the window queries, ``avg_pool1d(kernel)``, mean over
    the query heads of each KV group; the window gets (global max + 1).  Returns (B, Hkv, H).
    Follows ``snapkv_scores`` STRATA_KV.py:932-954."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    B, Hkv = k.shape[:2]
    Hq, d = q.shape[1], q.shape[-1]
    rep = Hq // Hkv
    w = window
    qo = q[:, :, H - w:H].reshape(B, Hkv, rep, w, d)
    att = np.einsum("bhrwd,bhnd->bhrwn", qo, k[:, :, :H], optimize=True) * np.float32(scaling)
    i = np.arange(w)[:, None]
    j = np.arange(H)[None, :]
    att = np.where(j - i >= H - w + 1, -np.inf, att)
    att = _softmax(att.astype(np.float32))[..., :H - w]
    sc = att.mean(-2).astype(np.float32).reshape(B, Hq, H - w)
    if kernel and kernel > 1:
        sc = _avg_pool1d(sc, kernel)
    sc = sc.reshape(B, Hkv, rep, H - w).mean(2).astype(np.float32)
    return np.concatenate([sc, np.full((B, Hkv, w), np.float32(sc.max()) + 1, np.float32)], -1)


def query_scores(q, k, scaling, n_cand, kernel=0):
    """Accumulated attention of decode queries that see every key: softmax(q K^T scaling) over all
    T keys (fp32), mean over the queries, restricted to the candidate columns [0, n_cand),
    optional ``avg_pool1d(kernel)``, mean over the query heads of each KV group.  q (B, Hq, nq, d),
    k (B, Hkv, T, d) -> (B, Hkv, n_cand).  The SnapKV accumulation of STRATA_KV.py:932-953 with
    decode-time queries (no causal mask, no observation window inside the context)."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    B, Hkv, T, d = k.shape
    Hq, nq = q.shape[1], q.shape[2]
    rep = Hq // Hkv
    qg = q.reshape(B, Hkv, rep, nq, d)
    out = np.empty((B, Hkv, rep, n_cand), np.float32)
    for b in range(B):
        for h in range(Hkv):
            att = np.einsum("rqd,nd->rqn", qg[b, h], k[b, h], optimize=True) * np.float32(scaling)
            p = _softmax(att.astype(np.float32))
            out[b, h] = p[..., :n_cand].mean(1)
    sc = out.reshape(B, Hq, n_cand)
    if kernel and kernel > 1:
        sc = _avg_pool1d(sc, kernel)
    return sc.reshape(B, Hkv, rep, n_cand).mean(2).astype(np.float32)


def topk_kept(scores: np.ndarray, budget: int, window: int = 0) -> np.ndarray:
    """Per row of ``scores`` (..., n_cand): the ``budget`` largest (ties: lower index first), sorted
    by position, followed by the ``window`` positions n_cand .. n_cand + window - 1 that are always
    kept.  Returns int64 (..., min(budget, n_cand) + window).  The selection of
    ``SnapKVQuantMethod.entries`` STRATA_KV.py:1022-1023 with an explicit tie rule."""
    s = np.asarray(scores, np.float32)
    n = s.shape[-1]
    kk = min(budget, n)
    flat = s.reshape(-1, n)
    out = np.empty((flat.shape[0], kk + window), np.int64)
    idx = np.arange(n)
    for r in range(flat.shape[0]):
        order = np.lexsort((idx, -flat[r].astype(np.float64)))
        out[r, :kk] = np.sort(order[:kk])
        out[r, kk:] = n + np.arange(window)
    return out.reshape(s.shape[:-1] + (kk + window,))


def l2_importance(k) -> np.ndarray:
    """Per-token key energy sum_c k_c^2, accumulated in float64 (exact for bf16 / fp16 keys, so the
    ranking does not depend on summation order).  Ranking by it equals ranking by the L2 norm."""
    k = np.asarray(k, np.float32).astype(np.float64)
    return (k * k).sum(-1)


def strata_counts(T: int, tenths8: int = 1, tenths4: int = 3):
    """Tokens per stratum: floor(0.1 T) at 8 bits, floor(0.3 T) at 4 bits, the rest at 2 bits
    (integer arithmetic, so no rounding of 0.1 / 0.3 can move a boundary)."""
    n8 = (T * tenths8) // 10
    n4 = (T * tenths4) // 10
    return n8, n4, T - n8 - n4


def mixed_strata(importance: np.ndarray, n8: int = None, n4: int = None):
    """Head-synchronous 8 / 4 / 2-bit strata from a per-token importance (B, H, T): the top n8
    tokens of each head go to 8 bits, the next n4 to 4 bits, the rest to 2 bits (ties: lower
    index first); defaults are ``strata_counts(T)``.  Returns {8: idx, 4: idx, 2: idx}, each
    (B, H, n_b) int64 in position order.  Every head stores the same number of tokens per stratum,
    the dense layout of STRATA_KV.py:65-69."""
    imp = np.asarray(importance)
    B, H, T = imp.shape
    if n8 is None or n4 is None:
        n8, n4, _ = strata_counts(T)
    out = {8: np.empty((B, H, n8), np.int64), 4: np.empty((B, H, n4), np.int64),
           2: np.empty((B, H, T - n8 - n4), np.int64)}
    idx = np.arange(T)
    for b in range(B):
        for h in range(H):
            order = np.lexsort((idx, -imp[b, h].astype(np.float64)))
            out[8][b, h] = np.sort(order[:n8])
            out[4][b, h] = np.sort(order[n8:n8 + n4])
            out[2][b, h] = np.sort(order[n8 + n4:])
    return out
