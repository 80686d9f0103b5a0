"""LCTC's clipped uniform quantiser and operational rate-distortion table on the device: the drop-in for
``uq_codes`` / ``uq_values`` / ``operational_rd`` (LCTC_KV.py:443-481), with the reference's signatures and
return values, plus ``uq_quantize`` (codes and values in one kernel, for ``Part.encode`` :532-539).

Everything runs in ``libkvb.so``; without it the calls raise.
"""

from __future__ import annotations

import ctypes as C
import math

import torch

from . import _lib as L
from .ops import _ptr, _stream


def _cols(a: torch.Tensor, bits, clip):
    if not a.is_cuda or a.dtype != torch.float32 or a.dim() != 2 or a.stride(1) != 1:
        raise ValueError("lctc: a must be a (rows, n) float32 CUDA tensor with contiguous columns")
    n = a.shape[1]
    bits = torch.as_tensor(bits, device=a.device).float().reshape(-1).expand(n).contiguous()
    clip = torch.as_tensor(clip, device=a.device).float().reshape(-1).expand(n).contiguous()
    return bits, clip


def uq_quantize(a: torch.Tensor, bits, clip, want_values: bool = True):
    """Codes (rows, n) uint8 and, if asked, the values uq_values(codes) (rows, n) float32."""
    bits, clip = _cols(a, bits, clip)
    rows, n = a.shape
    codes = torch.empty((rows, n), dtype=torch.uint8, device=a.device)
    values = torch.empty((rows, n), dtype=torch.float32, device=a.device) if want_values else None
    L.check(L.lib().kvb_uq_codes(_ptr(a), rows, n, a.stride(0), _ptr(bits), _ptr(clip), _ptr(codes), _ptr(values),
                                 C.c_void_p(_stream(a.device))), "kvb_uq_codes")
    return codes, values


def uq_codes(a: torch.Tensor, bits, clip) -> torch.Tensor:
    """The reference's uq_codes: the code indices as float32."""
    return uq_quantize(a, bits, clip, want_values=False)[0].float()


def uq_values(idx: torch.Tensor, bits, clip) -> torch.Tensor:
    """The reference's uq_values: -clip + (idx + 0.5) step, float32 (idx uint8, or integral floats)."""
    if not idx.is_cuda or idx.dim() != 2:
        raise ValueError("lctc: idx must be a (rows, n) CUDA tensor")
    codes = idx if idx.dtype == torch.uint8 else idx.to(torch.uint8)
    codes = codes.contiguous()
    rows, n = codes.shape
    bits = torch.as_tensor(bits, device=codes.device).float().reshape(-1).expand(n).contiguous()
    clip = torch.as_tensor(clip, device=codes.device).float().reshape(-1).expand(n).contiguous()
    values = torch.empty((rows, n), dtype=torch.float32, device=codes.device)
    L.check(L.lib().kvb_uq_values(_ptr(codes), rows, n, n, _ptr(bits), _ptr(clip), _ptr(values),
                                  C.c_void_p(_stream(codes.device))), "kvb_uq_values")
    return values


def operational_rd(A: torch.Tensor, bits_set, n_mults: int):
    """The reference's operational_rd: D (n, nb) float64 (column dropped, then each width's least mean
    squared error over the clip grid) and the clips C (n, nb) float32."""
    if not A.is_cuda or A.dtype != torch.float32 or A.dim() != 2 or A.stride(1) != 1:
        raise ValueError("operational_rd: A must be a (rows, n) float32 CUDA tensor with contiguous columns")
    rows, n = A.shape
    bs = (C.c_int32 * len(bits_set))(*[int(b) for b in bits_set])
    nb = len(bits_set)
    mults = torch.logspace(math.log10(0.5), math.log10(8.0), n_mults, device=A.device, dtype=A.dtype)
    lib = L.lib()
    need = lib.kvb_operational_rd_workspace(n, nb, n_mults)
    if need == 0:
        raise ValueError("operational_rd: widths (2 to 16, the first 0) / multipliers")
    ws = torch.empty(need, dtype=torch.uint8, device=A.device)
    D = torch.empty((n, nb), dtype=torch.float64, device=A.device)
    Cl = torch.empty((n, nb), dtype=torch.float32, device=A.device)
    L.check(lib.kvb_operational_rd(_ptr(A), rows, n, A.stride(0), C.cast(bs, C.c_void_p), nb, _ptr(mults), n_mults,
                                   _ptr(D), _ptr(Cl), _ptr(ws), need, C.c_void_p(_stream(A.device))),
            "kvb_operational_rd")
    return D, Cl
