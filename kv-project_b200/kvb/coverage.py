"""STRATA's coverage statistics on the device: the drop-in for ``coverage_groups`` / ``coverage_stats``
(STRATA_KV.py:1206-1298), with the reference's signature and return value.

``coverage_groups`` is host logic (the observation positions of a context: numpy's generator seeded as
the reference seeds it, STRATA_KV.py:306-307); ``coverage_stats`` runs ``kvb_coverage_stats`` of
``libkvb.so`` on the layer's CUDA tensors and returns A, W, DD, S, Mbar as float32 CUDA tensors, plus
the groups.  There is no CPU path: without the library the call raises.
"""

from __future__ import annotations

import ctypes as C
import zlib
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib as L
from .ops import _DT, _ptr, _stream

SEED = 42


@dataclass(frozen=True)
class CoverageConfig:
    """The fields of the reference's Config that the coverage statistics read (defaults as there,
    STRATA_KV.py:354-365)."""
    N_SINK: int = 4
    W_OBS: int = 32
    STRATA_SEGMENT: int = 512
    STRATA_QUERIES: int = 16
    STRATA_LOCAL: int = 64
    STRATA_FLOOR: float = 1e-3
    WINDOW: int = 32


def _rng(*keys) -> np.random.Generator:
    return np.random.default_rng([SEED] + [zlib.crc32(str(k).encode()) for k in keys])


def coverage_groups(H: int, cfg=None) -> list:
    """Observation positions, all < H: one group per context segment of STRATA_SEGMENT positions
    (STRATA_QUERIES sampled without replacement, seeded by (H, segment start)), then the last W_OBS
    positions (the window group, always last); positions start at N_SINK + STRATA_LOCAL."""
    cfg = cfg or CoverageConfig()
    lo = cfg.N_SINK + cfg.STRATA_LOCAL
    win = max(lo, H - cfg.W_OBS)
    groups = []
    for s in range(lo, win, cfg.STRATA_SEGMENT):
        seg = np.arange(s, min(s + cfg.STRATA_SEGMENT, win))
        n = min(len(seg), cfg.STRATA_QUERIES)
        groups.append(np.sort(_rng("cover_group", H, s).choice(seg, n, replace=False)))
    groups.append(np.arange(win, H))
    return [g for g in groups if len(g)]


_WS = {}


def _workspace(dev: torch.device, nbytes: int) -> torch.Tensor:
    ws = _WS.get(dev)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
        _WS[dev] = ws
    return ws


def coverage_stats(q, k, v, scaling, H: int, rs: int, re: int, M: torch.Tensor, cfg=None,
                   window_only: bool = False, score_cap: int = 0) -> dict:
    """q (1, Hq, T, d), k and v (1, Hkv, T, d) CUDA tensors of one dtype (f32 / f16 / bf16, d contiguous,
    d in {64, 128}); M (Hq, d, d) the output metrics W_O,aᵀ W_O,a.  Returns {"A", "W", "DD" (Hkv, re - rs),
    "S", "Mbar" (Hkv, d, d), "groups"} as the reference's coverage_stats does.  score_cap: bytes of
    scores held between the two passes over a batch of groups (0: the library's 4 GiB)."""
    cfg = cfg or CoverageConfig()
    for t in (q, k, v, M):
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError("coverage_stats: q, k, v and M must be CUDA tensors")
    if q.dim() != 4 or k.dim() != 4 or v.shape != k.shape or q.shape[0] != 1 or k.shape[0] != 1:
        raise ValueError("coverage_stats: q (1, Hq, T, d), k and v (1, Hkv, T, d)")
    if q.dtype != k.dtype or v.dtype != k.dtype or k.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise ValueError("coverage_stats: q, k and v of one dtype among float32, float16, bfloat16")
    Hq, d, Hkv = q.shape[1], q.shape[-1], k.shape[1]
    if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1 or k.stride() != v.stride():
        raise ValueError("coverage_stats: d must be contiguous and k, v laid out alike")
    groups = coverage_groups(H, cfg)
    if window_only:
        groups = groups[-1:]
    pos = np.ascontiguousarray(np.concatenate(groups) if groups else np.zeros(0), dtype=np.int64)
    goff = np.ascontiguousarray(np.cumsum([0] + [len(g) for g in groups]), dtype=np.int64)
    Mc = M.float().contiguous()
    desc = L.Coverage(_ptr(q), _ptr(k), _ptr(v), _DT[k.dtype], q.stride(1), q.stride(2), k.stride(1), k.stride(2),
                      _ptr(Mc), Hq, Hkv, d, int(H), int(rs), int(re), float(scaling), float(cfg.STRATA_FLOOR),
                      int(cfg.STRATA_LOCAL), int(score_cap))
    lib = L.lib()
    pp, gp = pos.ctypes.data_as(C.c_void_p), goff.ctypes.data_as(C.c_void_p)
    need = lib.kvb_coverage_workspace_size(C.byref(desc), pp, gp, len(groups))
    if need == 0:
        L.check(lib.kvb_coverage_stats(C.byref(desc), pp, gp, len(groups), None, None, None, None, None, None, 0,
                                       None), "kvb_coverage_stats")
    dev = k.device
    n = re - rs
    f32 = dict(dtype=torch.float32, device=dev)
    A, W, DD = (torch.empty((Hkv, n), **f32) for _ in range(3))
    S, Mbar = (torch.empty((Hkv, d, d), **f32) for _ in range(2))
    ws = _workspace(dev, need)
    L.check(lib.kvb_coverage_stats(C.byref(desc), pp, gp, len(groups), _ptr(A), _ptr(W), _ptr(DD), _ptr(S),
                                   _ptr(Mbar), _ptr(ws), ws.numel(), C.c_void_p(_stream(dev))),
            "kvb_coverage_stats")
    return {"A": A, "W": W, "DD": DD, "S": S, "Mbar": Mbar, "groups": groups}
