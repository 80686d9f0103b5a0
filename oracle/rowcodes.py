"""Per-vector row codes (numpy, CPU).  TEST INFRASTRUCTURE ONLY (see package docstring).

Restates the token-like stored vectors of the reference's chunk methods and its format variants:

  * absmax codes in two variants: STRATA's (``absmax_quant`` STRATA_KV.py:549-554, fp16 scale
    floored at 2^-24) and TILT's (``fake_quant_tokens`` TILT_KV.py:721-727, float32 scale
    ``max(amax, 1e-8) / qmax``);
  * the HEDGE per-token code (``hedge_quant`` / ``centered_code`` HEDGE_KV.py:1103-1130):
    rotation ``y = (x - mu) R^T``, Lloyd-Max levels of N(0, 1) times the fp16 RMS of y at 1-4
    bits, symmetric absmax int8 (offset 127) at 8 bits, read back as ``(level s) R + mu``;
  * TILT's chunk selection (``finalize_chunk`` TILT_KV.py:745-766, eviction family): share of
    each chunk key under the observed queries, top-m by share, kept positions ascending;
  * byte-LUT decode of MSB-first packed rows (``pack_rows`` / ``byte_lut`` QUASAR_KV.py:1185-1203).

The rotation, its read-back and the RMS of y follow the reference's float32 CPU order
(``codecs.matmul_fma``, ``codecs.rms_f32``), as the CUDA kernel does, so HEDGE codes, scales and
reconstructions are bit-exact.  TILT's share (a float64 einsum here) is compared within tolerance;
its top-m positions are exact.
"""

from __future__ import annotations

from functools import lru_cache

import numpy as np

from .codecs import as_stored, matmul_fma, pack_codes, rms_f32, _gauss_grid, _TINY


def absmax_tilt(x: np.ndarray, bits: int):
    """TILT's per-vector symmetric absmax code: s = max(max|x|, 1e-8) / qmax in float32 (no fp16
    rounding), codes clamp(rint(x / s), -qmax, qmax).  Returns (codes float32, s (..., 1)); the
    stored vector is codes * s.  Follows ``fake_quant_tokens`` TILT_KV.py:721-727."""
    x = np.asarray(x, np.float32)
    qmax = np.float32(2 ** (bits - 1) - 1)
    s = np.maximum(np.abs(x).max(-1, keepdims=True), np.float32(1e-8)) / qmax
    return np.clip(np.rint(x / s), -qmax, qmax).astype(np.float32), s.astype(np.float32)


def absmax_packed(codes: np.ndarray, bits: int) -> np.ndarray:
    """Stored bytes of signed absmax codes: codes + qmax as an MSB-first stream, the form the
    reference charges (``payload_bytes`` STRATA_KV.py:2765-2766)."""
    return pack_codes(np.asarray(codes).astype(np.int64) + 2 ** (bits - 1) - 1, bits)


@lru_cache(maxsize=None)
def lloyd_max_gaussian(bits: int) -> np.ndarray:
    """Lloyd-Max reconstruction levels of N(0, 1) with 2^bits cells: 500 Lloyd iterations on the
    360001-point grid over [-9, 9], started from the cell-centre quantiles.  Restates
    ``lloyd_max_gaussian`` HEDGE_KV.py:1055-1070 (same grid, start and iteration count)."""
    from scipy import stats
    n = 2 ** bits
    x, w = _gauss_grid()
    c = stats.norm.ppf((np.arange(n) + 0.5) / n)
    for _ in range(500):
        cell = np.searchsorted((c[1:] + c[:-1]) / 2, x)
        mass = np.bincount(cell, w, n)
        c = np.bincount(cell, w * x, n) / np.maximum(mass, 1e-300)
    return c.astype(np.float32)


def hedge_codes_from_y(y: np.ndarray, bits: int, levels: np.ndarray = None):
    """The code step of ``hedge_quant`` (HEDGE_KV.py:1114-1121) applied to rotated rows y:
    returns (codes uint8, s (..., 1) float32, yhat = level * s float32)."""
    y = np.asarray(y, np.float32)
    if bits == 8:
        s = np.maximum(as_stored(np.abs(y).max(-1, keepdims=True) / np.float32(127)), _TINY)
        c = np.clip(np.rint(y / s), -127, 127).astype(np.float32)
        return (c + 127).astype(np.uint8), s, c * s
    cb = lloyd_max_gaussian(bits) if levels is None else np.asarray(levels, np.float32)
    s = np.maximum(as_stored(rms_f32(y)), _TINY)
    mids = ((cb[1:] + cb[:-1]) / np.float32(2)).astype(np.float32)
    c = np.searchsorted(mids, y / s, side="left")          # torch.bucketize(right=False)
    return c.astype(np.uint8), s, cb[c] * s


def hedge_quant(x: np.ndarray, R: np.ndarray, bits: int, mu: np.ndarray = None):
    """``centered_code`` (HEDGE_KV.py:1124-1129) / ``hedge_quant`` (:1103-1121): y = (x - mu) R^T,
    code y, read back as (yhat) R + mu.  Returns (xhat, codes, s, y); 16 bits keeps x."""
    x = np.asarray(x, np.float32)
    if bits >= 16:
        return x, None, None, None
    xc = x if mu is None else x - np.asarray(mu, np.float32)
    R = np.asarray(R, np.float32)
    y = matmul_fma(xc, R)
    c, s, yh = hedge_codes_from_y(y, bits)
    xh = matmul_fma(yh, R.T)
    return (xh if mu is None else xh + np.asarray(mu, np.float32)), c, s, y


def chunk_share(k: np.ndarray, qref: np.ndarray) -> np.ndarray:
    """Within-chunk attention share of every key: softmax over the chunk's C keys of the scaled
    observed queries' logits, averaged over the queries.  k (U, H, C, d), qref (U, H, nq, d) ->
    (U, H, C).  ``finalize_chunk`` TILT_KV.py:743-745."""
    s = np.einsum("uhqd,uhcd->uhqc", np.asarray(qref, np.float64), np.asarray(k, np.float64))
    s = s - s.max(-1, keepdims=True)
    e = np.exp(s)
    return (e / e.sum(-1, keepdims=True)).mean(2).astype(np.float32)


def chunk_topm(share: np.ndarray, m: int) -> np.ndarray:
    """Kept positions of a chunk: the m largest shares (ties: lower position first), ascending.
    ``finalize_chunk`` TILT_KV.py:759-760 (argsort descending, first m, sorted)."""
    share = np.asarray(share, np.float32)
    C = share.shape[-1]
    flat = share.reshape(-1, C)
    out = np.empty((flat.shape[0], m), np.int64)
    pos = np.arange(C)
    for r in range(flat.shape[0]):
        order = np.lexsort((pos, -flat[r].astype(np.float64)))
        out[r] = np.sort(order[:m])
    return out.reshape(share.shape[:-1] + (m,))


def unpack_rows(packed: np.ndarray, bits: int, w: int) -> np.ndarray:
    """Inverse of ``pack_rows`` / per-row ``pack_codes``: MSB-first stream of w codes per row."""
    p = np.asarray(packed, np.uint8)
    bitsarr = np.unpackbits(p, axis=-1)[..., :w * bits].reshape(*p.shape[:-1], w, bits)
    weights = (1 << np.arange(bits - 1, -1, -1)).astype(np.int64)
    return (bitsarr.astype(np.int64) * weights).sum(-1)


def byte_lut(levels: np.ndarray, bits: int) -> np.ndarray:
    """(256, 8 / bits) table: one packed byte -> the levels of its codes, first code in the most
    significant bits.  ``byte_lut`` QUASAR_KV.py:1194-1203 for one stage's level table."""
    per = 8 // bits
    byte = np.arange(256)[:, None]
    shifts = np.arange(per - 1, -1, -1)[None, :] * bits
    return np.asarray(levels, np.float32)[(byte >> shifts) & (2 ** bits - 1)]


def decode_rows_lut(packed: np.ndarray, bits: int, levels: np.ndarray, acc: np.ndarray = None) -> np.ndarray:
    """Row decode through the byte table: out = acc + lut[byte] per byte, concatenated (float32
    adds in stage order, as ``embedded_quantize`` accumulates, QUASAR_KV.py:1172-1182)."""
    lut = byte_lut(levels, bits)
    p = np.asarray(packed, np.uint8)
    v = lut[p].reshape(*p.shape[:-1], p.shape[-1] * (8 // bits))
    return v if acc is None else (np.asarray(acc, np.float32) + v).astype(np.float32)
