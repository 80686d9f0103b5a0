"""Codec restatements (numpy, CPU): storage rounding, KIVI group quantiser, STRATA per-token code,
absmax code and the three bit-packing formats.  TEST INFRASTRUCTURE ONLY (see package docstring).

All arithmetic is float32 where the reference computes in float32, in the same operation order, so
integer codes and fp16 scales are reproduced bit for bit (numpy and torch both use IEEE-754
float32 division and round-half-to-even).  Two results of the reference depend on the order of a
float32 reduction inside a third-party library, PyTorch (2.11.0 CPU build, MKL 2024.2, the build the
golden fixtures were made with; the reference pins no version):

* ``Y.pow(2).mean(-1)`` (STRATA_KV.py:1166, HEDGE_KV.py:1119): torch's CPU float32 sum over a
  contiguous last axis (``cascade_sum`` / ``vectorized_inner_sum`` / ``row_sum`` /
  ``multi_row_sum`` in aten/src/ATen/native/cpu/SumKernel.cpp) followed by an IEEE division by n;
  restated in :func:`mean_sq_f32`;
* ``x @ R.T`` on CPU (HEDGE_KV.py:1113, :1121): MKL's sgemm, which for row counts of 7 and more
  returns a float32 fused multiply-add chain over k in ascending order from 0 (checked bit for bit
  against torch's CPU matmul; one to six rows take a gemv path with another order); restated in
  :func:`matmul_fma`.

The CUDA kernels take the same orders, so codes and scales match the reference's CPU results bit for
bit.
"""

from __future__ import annotations

import math
from functools import lru_cache

import numpy as np

FP16_MAX = 65504.0
_TINY = np.float32(2.0 ** -24)            # smallest positive fp16 subnormal


def as_stored(x: np.ndarray) -> np.ndarray:
    """Clamp to +-65504 and round to fp16 (RNE), back to float32.
    Follows ``as_stored`` STRATA_KV.py:539-543."""
    x = np.asarray(x, dtype=np.float32)
    return np.clip(x, -FP16_MAX, FP16_MAX).astype(np.float16).astype(np.float32)


def kivi_quant(x: np.ndarray, bits: int, group: int, along_tokens: bool, n_sink: int) -> dict:
    """Asymmetric min/max quantiser of KIVI.  Keys: per channel over ``group`` consecutive tokens
    (``along_tokens``; a partial last group is padded by repeating its last row, which leaves its
    min / max unchanged).  Values: per token over ``group`` channels (or the whole row when
    ``group`` does not divide d).  Rows before ``n_sink`` stay exact.  fp16 lo and scale (the scale
    floored at 2^-24), codes ``clamp(rint((x - lo) / scale), 0, 2^bits - 1)``.
    Follows ``kivi_quant`` STRATA_KV.py:826-856 (same shapes for lo / scale: (B, H, n_g, 1, d) or
    (B, H, n, d / width, 1))."""
    qmax = 2 ** bits - 1
    y = np.asarray(x, dtype=np.float32)
    body = y[:, :, n_sink:]
    B, H, n, d = body.shape
    if along_tokens:
        n_g = -(-n // group)
        pad = n_g * group - n
        if pad and n:
            body = np.concatenate([body, np.repeat(body[:, :, -1:], pad, axis=2)], axis=2)
        g = body.reshape(B, H, n_g, group, d)
        red = 3
    else:
        width = group if d % group == 0 else d
        g = body.reshape(B, H, n, d // width, width)
        red = 4
    if g.size == 0:
        shp = list(g.shape)
        shp[red] = 1
        lo = np.zeros(shp, np.float32)
        sc = np.full(shp, _TINY, np.float32)
        codes = np.zeros(g.shape, np.float32)
    else:
        lo = as_stored(g.min(axis=red, keepdims=True))
        sc = np.maximum(as_stored((g.max(axis=red, keepdims=True) - lo) / np.float32(qmax)), _TINY)
        codes = np.clip(np.rint((g - lo) / sc), 0, qmax).astype(np.float32)
    deq = (codes * sc + lo).reshape(B, H, -1, d)[:, :, :n]
    return {"xhat": np.concatenate([y[:, :, :n_sink], deq], axis=2).astype(np.float32),
            "codes": codes.reshape(B, H, -1, d)[:, :, :n].astype(np.uint8),
            "lo": lo.astype(np.float32), "scale": sc.astype(np.float32)}


def kivi_dequant(codes: np.ndarray, lo: np.ndarray, scale: np.ndarray, group: int, along_tokens: bool) -> np.ndarray:
    """What a reader of a KIVI code computes: ``codes * scale + lo`` in float32, with lo / scale in
    the shapes ``kivi_quant`` returns (STRATA_KV.py:853)."""
    c = np.asarray(codes, np.float32)
    B, H, n, d = c.shape
    if along_tokens:
        n_g = lo.shape[2]
        cp = np.zeros((B, H, n_g * group, d), np.float32)
        cp[:, :, :n] = c
        out = cp.reshape(B, H, n_g, group, d) * scale + lo
        return out.reshape(B, H, -1, d)[:, :, :n]
    width = group if d % group == 0 else d
    return (c.reshape(B, H, n, d // width, width) * scale + lo).reshape(B, H, n, d)


def _gauss_grid():
    x = np.linspace(-9.0, 9.0, 360001)
    w = np.exp(-0.5 * x * x)
    return x, w / w.sum()


@lru_cache(maxsize=None)
def uniform_step(bits: int) -> tuple:
    """Step (in RMS units) of the MSE-optimal mid-rise uniform quantiser of N(0, 1) with 2^bits
    levels, by golden-section search on a 360001-point grid over [-9, 9], and its MSE.
    Restates ``uniform_step`` STRATA_KV.py:1133-1155 (same grid, bracket [1e-4, 4], 200 steps)."""
    x, w = _gauss_grid()
    top = 2 ** bits - 1
    half = top / 2.0

    def distortion(step):
        c = np.clip(np.round(x / step + half), 0, top)
        return float((w * (x - (c - half) * step) ** 2).sum())

    a, b = 1e-4, 4.0
    ratio = (math.sqrt(5) - 1) / 2
    for _ in range(200):
        left, right = b - ratio * (b - a), a + ratio * (b - a)
        if distortion(left) < distortion(right):
            b = right
        else:
            a = left
    step = 0.5 * (a + b)
    return step, distortion(step)


def fma_f32(a, b, c) -> np.ndarray:
    """Correctly rounded float32 fused multiply-add ``a * b + c`` (IEEE fmaf), elementwise.

    ``a * b`` is exact in float64 (48-bit significand); the float64 sum rounds at most once, and its
    exact error comes from Knuth's TwoSum.  Rounding the float64 sum to float32 is then wrong only when
    the sum sits exactly halfway between two float32 values while the exact value does not; the
    error's sign says which neighbour is right."""
    f32, f64 = np.float32, np.float64
    a = np.asarray(a, f32)
    b = np.asarray(b, f32)
    c = np.asarray(c, f32)
    p = a.astype(f64) * b.astype(f64)
    cd = c.astype(f64)
    s = p + cd
    bb = s - p
    e = (p - (s - bb)) + (cd - bb)
    r = s.astype(f32)
    d = s - r.astype(f64)
    with np.errstate(invalid="ignore", over="ignore"):
        up = np.nextafter(r, f32(np.inf))
        dn = np.nextafter(r, f32(-np.inf))
        fix_up = (d == (up.astype(f64) - r.astype(f64)) / 2) & (e > 0)
        fix_dn = (-d == (r.astype(f64) - dn.astype(f64)) / 2) & (e < 0)
    return np.where(fix_up, up, np.where(fix_dn, dn, r)).astype(f32)


def matmul_fma(x: np.ndarray, W: np.ndarray) -> np.ndarray:
    """``x @ W.T`` in float32 as one fused multiply-add chain per output, k ascending from 0: the
    result torch's CPU matmul (MKL sgemm) gives for 7 or more rows.  x (..., K), W (N, K)."""
    x = np.asarray(x, np.float32)
    W = np.asarray(W, np.float32)
    y = np.zeros(x.shape[:-1] + (W.shape[0],), np.float32)
    for k in range(x.shape[-1]):
        y = fma_f32(x[..., k:k + 1], W[:, k], y)
    return y


def sum_f32_torch(x: np.ndarray) -> np.ndarray:
    """Float32 sum over the last axis in the order of torch's CPU reduction of a contiguous row
    (aten/src/ATen/native/cpu/SumKernel.cpp): the row as n // 8 vectors of 8 lanes; vector j adds into
    accumulator j % 4 of the first n // 32 * 4 vectors (lanewise, in j order, from zero), the
    remaining whole vectors into accumulator 0; the accumulators combine as ((a0 + a1) + a2) + a3;
    the n % 8 scalar tail and then the 8 lanes add one by one, in order, into a zero.  Rows of fewer
    than 8 elements take the same four-accumulator scheme on scalars.  Valid while n // 32 < 16 (no second cascade level), i.e. n < 512."""
    f32 = np.float32
    x = np.asarray(x, f32)
    n = x.shape[-1]
    lead = x.shape[:-1]
    if n < 8:                                   # scalar path: the same four accumulators on scalars
        acc = [np.zeros(lead, f32) for _ in range(4)]
        for i in range(n // 4):
            for k in range(4):
                acc[k] = (acc[k] + x[..., 4 * i + k]).astype(f32)
        for j in range(n // 4 * 4, n):
            acc[0] = (acc[0] + x[..., j]).astype(f32)
        return (((acc[0] + acc[1]).astype(f32) + acc[2]).astype(f32) + acc[3]).astype(f32)
    nv = n // 8
    assert nv // 4 < 16, "a second cascade level is not restated"
    V = x[..., :nv * 8].reshape(*lead, nv, 8)
    acc = [np.zeros(lead + (8,), f32) for _ in range(4)]
    for i in range(nv // 4):
        for k in range(4):
            acc[k] = (acc[k] + V[..., 4 * i + k, :]).astype(f32)
    for j in range(nv // 4 * 4, nv):
        acc[0] = (acc[0] + V[..., j, :]).astype(f32)
    p = acc[0]
    for k in range(1, 4):
        p = (p + acc[k]).astype(f32)
    t = np.zeros(lead, f32)
    for i in range(nv * 8, n):
        t = (t + x[..., i]).astype(f32)
    for lane in range(8):
        t = (t + p[..., lane]).astype(f32)
    return t


def mean_sq_f32(Y: np.ndarray) -> np.ndarray:
    """``Y.pow(2).mean(-1, keepdim=True)`` as torch computes it on CPU: float32 squares, the sum of
    :func:`sum_f32_torch`, one IEEE float32 division by n."""
    Y = np.asarray(Y, np.float32)
    sq = (Y * Y).astype(np.float32)
    return (sum_f32_torch(sq) / np.float32(Y.shape[-1])).astype(np.float32)[..., None]


def rms_f32(Y: np.ndarray) -> np.ndarray:
    """sqrt(mean(Y^2)) over the last axis (keepdim), float32, in the reference's order."""
    return np.sqrt(mean_sq_f32(Y))


def strata_quantize(Y: np.ndarray, bits: int):
    """Per-vector mid-rise uniform code: one fp16 scale ``s = fp16(step_b * RMS(y))`` (floored at
    2^-24), codes ``clamp(rint(y / s + (2^b - 1) / 2))``, reconstruction ``(c - h) s``.
    Follows ``strata_quantize`` STRATA_KV.py:1158-1168.  Returns (codes uint8, s (...), yhat)."""
    Y = np.asarray(Y, np.float32)
    top = 2 ** bits - 1
    half = np.float32(top / 2.0)
    s = np.maximum(as_stored(np.float32(uniform_step(bits)[0]) * rms_f32(Y)), _TINY)
    c = np.clip(np.rint(Y / s + half), 0, top).astype(np.float32)
    return c.astype(np.uint8), s[..., 0], (c - half) * s


def absmax_quant(x: np.ndarray, bits: int):
    """Symmetric per-vector absmax code: integer codes in [-qmax, qmax] and the fp16 scale.
    Follows ``absmax_quant`` STRATA_KV.py:549-554."""
    x = np.asarray(x, np.float32)
    qmax = 2 ** (bits - 1) - 1
    s = np.maximum(as_stored(np.abs(x).max(-1, keepdims=True) / np.float32(qmax)), _TINY)
    return np.clip(np.rint(x / s), -qmax, qmax).astype(np.float32), s


def pack_planar(codes: np.ndarray, bits: int) -> np.ndarray:
    """(..., d) codes < 2^bits -> (..., d * bits / 8) bytes, planar: byte i holds coordinate
    ``p * d / P + i`` in bits [p * bits, (p + 1) * bits) for plane p < P = 8 / bits.
    Follows ``pack_planar`` STRATA_KV.py:1171-1182."""
    P = 8 // bits
    c = np.asarray(codes).astype(np.uint32)
    d = c.shape[-1]
    planes = c.reshape(*c.shape[:-1], P, d // P)
    out = np.zeros(planes.shape[:-2] + (d // P,), np.uint32)
    for p in range(P):
        out |= planes[..., p, :] << np.uint32(p * bits)
    return out.astype(np.uint8)


def unpack_planar(packed: np.ndarray, bits: int) -> np.ndarray:
    """Inverse of ``pack_planar`` (STRATA_KV.py:1185-1189): (..., d * bits / 8) -> (..., d) int32."""
    P = 8 // bits
    x = np.asarray(packed).astype(np.int32)
    mask = (1 << bits) - 1
    return np.concatenate([(x >> (p * bits)) & mask for p in range(P)], axis=-1)


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """MSB-first bit stream of the flattened codes (``pack_codes`` STRATA_KV.py:2728-2733)."""
    c = np.asarray(codes).reshape(-1).astype(np.int64)
    planes = ((c[:, None] >> np.arange(bits - 1, -1, -1)) & 1).astype(np.uint8)
    return np.packbits(planes.reshape(-1))


def pack_rows(codes: np.ndarray, bits: int) -> np.ndarray:
    """(..., w) codes -> (..., w * bits / 8) bytes, first code of each byte in the most significant
    bits (``pack_rows`` QUASAR_KV.py:1185-1190)."""
    per = 8 // bits
    c = np.asarray(codes).astype(np.uint32)
    c = c.reshape(*c.shape[:-1], c.shape[-1] // per, per)
    out = np.zeros(c.shape[:-1], np.uint32)
    for i in range(per):
        out |= c[..., i] << np.uint32((per - 1 - i) * bits)
    return out.astype(np.uint8)
