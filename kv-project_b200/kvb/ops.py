"""Tensor-level wrappers over the C ABI (include/kvb.h).

PyTorch provides device memory and the current stream; every computation runs in libkvb.so.
Each wrapper checks shapes / dtypes / devices, passes raw pointers and raises on a non-zero
status.  No wrapper falls back to another implementation.
"""

from __future__ import annotations

import ctypes as C
import math
import numpy as np

import torch

from . import _lib as L

_DT = {torch.float32: L.KVB_F32, torch.float16: L.KVB_F16, torch.bfloat16: L.KVB_BF16, torch.float64: L.KVB_F64}

# MSE-optimal mid-rise steps of N(0, 1) (uniform_step, STRATA_KV.py:1133), by golden-section search
UNIFORM_STEP = {2: 0.9956803260610909, 3: 0.5860196721213176, 4: 0.33520647283490446, 8: 0.030762719123913013}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise ValueError(f"kvb: unsupported dtype {t.dtype}") from None


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("kvb: tensors must live on a CUDA device")


def round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


# ------------------------------------------------------------------------------------------------
# K1: quantise + pack
# ------------------------------------------------------------------------------------------------
def quant_pack(x: torch.Tensor, bits: int, group: int, *, per_channel: bool = False, midrise: bool = False,
               idx: torch.Tensor = None, first_row: int = 0, n: int = None, n_alloc: int = None,
               want_xhat: bool = False, step: float = None, blocked: bool = False) -> dict:
    """Quantise rows of x (B, H, T, d) and planar-pack them.

    Rows: idx (B, H, n) int64 gathers source rows; otherwise rows first_row .. first_row + n - 1.
    per_channel: KIVI keys (min / max per channel over `group` stored rows); else per-token groups
    of `group` channels (KIVI values / the mixed strata), or, with midrise, the STRATA code.
    blocked: (values, per token, d = 128) codes in the 128-token channel-major block layout the
    tensor-core decode reads, codes (B, H, n_alloc / 128, 128, 16 * bits), n_alloc % 128 == 0.
    Returns codes (B, H, n_alloc, d * bits / 8) uint8, meta (fp16 pairs / scales as documented in
    kvb.h), n, n_alloc, optional xhat (B, H, n, d) float32, layout."""
    if blocked:
        return _quant_pack_blocked(x, bits, group, midrise=midrise, idx=idx, first_row=first_row, n=n,
                                   n_alloc=n_alloc, want_xhat=want_xhat, step=step)
    _cuda(x, idx)
    if x.dim() != 4 or x.stride(-1) != 1:
        raise ValueError("quant_pack: x must be (B, H, T, d) with unit channel stride")
    B, H, T, d = x.shape
    if idx is not None:
        if idx.dtype != torch.int64 or idx.shape[:2] != (B, H):
            raise ValueError("quant_pack: idx must be int64 (B, H, n)")
        idx = idx.contiguous()
        n = idx.shape[2]
    elif n is None:
        n = T - first_row
    align = max(16, group if per_channel else 16)
    n_alloc = round_up(max(n, 1), align) if n_alloc is None else n_alloc
    rb = d * bits // 8
    codes = torch.empty((B, H, n_alloc, rb), dtype=torch.uint8, device=x.device)
    if midrise:
        meta = torch.empty((B, H, n_alloc), dtype=torch.float16, device=x.device)
    elif per_channel:
        meta = torch.empty((B, H, n_alloc // group, d, 2), dtype=torch.float16, device=x.device)
    else:
        width = group if d % group == 0 else d
        meta = torch.empty((B, H, n_alloc, d // width, 2), dtype=torch.float16, device=x.device)
    xhat = torch.empty((B, H, n, d), dtype=torch.float32, device=x.device) if want_xhat else None
    st = UNIFORM_STEP[bits] if (midrise and step is None) else (step or 0.0)
    L.check(L.lib().kvb_quant_pack(
        _ptr(x), dtype_code(x), B, H, T, d, x.stride(0), x.stride(1), x.stride(2),
        _ptr(idx), first_row, n, n_alloc, bits, group if not midrise else d,
        L.KVB_K_PER_CHANNEL if per_channel else L.KVB_K_PER_TOKEN,
        L.KVB_CODE_MIDRISE if midrise else L.KVB_CODE_ASYM, C.c_float(st),
        _ptr(codes), _ptr(meta), _ptr(xhat), C.c_void_p(_stream(x.device))), "kvb_quant_pack")
    return {"codes": codes, "meta": meta, "xhat": xhat, "n": n, "n_alloc": n_alloc, "bits": bits, "group": group,
            "layout": L.KVB_V_TOKEN_MAJOR}


def _quant_pack_blocked(x, bits, group, *, midrise, idx, first_row, n, n_alloc, want_xhat, step):
    _cuda(x, idx)
    if x.dim() != 4 or x.stride(-1) != 1 or x.shape[-1] != 128:
        raise ValueError("quant_pack(blocked): x must be (B, H, T, 128) with unit channel stride")
    B, H, T, d = x.shape
    if idx is not None:
        if idx.dtype != torch.int64 or idx.shape[:2] != (B, H):
            raise ValueError("quant_pack: idx must be int64 (B, H, n)")
        idx = idx.contiguous()
        n = idx.shape[2]
    elif n is None:
        n = T - first_row
    n_alloc = round_up(max(n, 1), 128) if n_alloc is None else n_alloc
    codes = torch.empty((B, H, n_alloc // 128, 128, 16 * bits), dtype=torch.uint8, device=x.device)
    if midrise:
        meta = torch.empty((B, H, n_alloc), dtype=torch.float16, device=x.device)
    else:
        meta = torch.empty((B, H, n_alloc, 128 // group, 2), dtype=torch.float16, device=x.device)
    xhat = torch.empty((B, H, n, d), dtype=torch.float32, device=x.device) if want_xhat else None
    st = UNIFORM_STEP[bits] if (midrise and step is None) else (step or 0.0)
    L.check(L.lib().kvb_quant_pack_blocked(
        _ptr(x), dtype_code(x), B, H, T, d, x.stride(0), x.stride(1), x.stride(2), _ptr(idx), first_row, n, n_alloc,
        bits, d if midrise else group, L.KVB_CODE_MIDRISE if midrise else L.KVB_CODE_ASYM, C.c_float(st),
        _ptr(codes), _ptr(meta), _ptr(xhat), C.c_void_p(_stream(x.device))), "kvb_quant_pack_blocked")
    return {"codes": codes, "meta": meta, "xhat": xhat, "n": n, "n_alloc": n_alloc, "bits": bits, "group": group,
            "layout": L.KVB_V_BLOCK128}


def unblock_codes(codes: torch.Tensor) -> torch.Tensor:
    """Block-layout value codes (B, H, n_alloc / 128, 128, 16 * bits) -> the token-major planar layout
    (B, H, n_alloc, 16 * bits) (torch ops on the device; for inspection and tests)."""
    B, H, nb, d, rb = codes.shape
    bits = rb // 16
    P = 8 // bits
    x = codes.to(torch.int32)
    # unpack along tokens: token pl * 128 / P + k of channel c is in byte k, bits [pl * bits, ...)
    tok = torch.cat([(x >> (pl * bits)) & ((1 << bits) - 1) for pl in range(P)], -1)     # (B, H, nb, d, 128)
    tok = tok.transpose(-1, -2)                                                            # (B, H, nb, 128, d)
    # repack along channels (planar): byte i holds channel pl * d / P + i
    planes = [tok[..., pl * (d // P):(pl + 1) * (d // P)] << (pl * bits) for pl in range(P)]
    out = planes[0]
    for t in planes[1:]:
        out = out | t
    return out.to(torch.uint8).reshape(B, H, nb * 128, rb)


# ------------------------------------------------------------------------------------------------
# K2: importance, rank split, scores
# ------------------------------------------------------------------------------------------------
def key_energy(k: torch.Tensor) -> torch.Tensor:
    """sum_c k_c^2 per token in float64, (B, H, T)."""
    _cuda(k)
    B, H, T, d = k.shape
    if k.stride(-1) != 1:
        raise ValueError("key_energy: unit channel stride required")
    out = torch.empty((B, H, T), dtype=torch.float64, device=k.device)
    L.check(L.lib().kvb_key_energy(_ptr(k), dtype_code(k), B, H, T, d, k.stride(0), k.stride(1), k.stride(2),
                                   _ptr(out), C.c_void_p(_stream(k.device))), "kvb_key_energy")
    return out


def rank_split(keys: torch.Tensor, counts, want=None):
    """keys (..., n) float32 / float64.  Class c gets ranks [sum(counts[:c]), sum(counts[:c+1])) by
    key descending (ties: lower index first); the last class gets the rest.  Returns one int64
    tensor (..., count_c) per class (ascending indices); classes not in `want` are None.  NaN keys
    set bit 2 of the device status word (device_status()); nothing here synchronises."""
    _cuda(keys)
    if keys.dtype not in (torch.float32, torch.float64):
        raise ValueError("rank_split: keys must be float32 or float64")
    lead, n = keys.shape[:-1], keys.shape[-1]
    k2 = keys.reshape(-1, n)
    if k2.stride(-1) != 1:
        k2 = k2.contiguous()
    rows = k2.shape[0]
    counts = [int(c) for c in counts]
    if any(c < 0 for c in counts) or sum(counts) > n:
        raise ValueError("rank_split: counts must be >= 0 and sum to <= n")
    sizes = counts + [n - sum(counts)]
    ncls = len(sizes)
    want = set(range(ncls)) if want is None else set(want)
    outs = [torch.empty((rows, s), dtype=torch.int64, device=keys.device) if (c in want and s > 0) else None
            for c, s in enumerate(sizes)]
    cnt = (C.c_int64 * 4)(*(counts + [0] * (4 - len(counts))))
    ptrs = (C.c_void_p * 4)(*[(o.data_ptr() if o is not None else None) for o in outs] + [None] * (4 - ncls))
    strides = (C.c_int64 * 4)(*[(o.stride(0) if o is not None else 0) for o in outs] + [0] * (4 - ncls))
    L.check(L.lib().kvb_rank_split(_ptr(k2), dtype_code(k2), rows, n, k2.stride(0), ncls, cnt, ptrs, strides,
                                   C.c_void_p(_stream(keys.device))), "kvb_rank_split")
    return [None if o is None else o.reshape(*lead, o.shape[-1]) for o in outs]


def query_scores(q: torch.Tensor, k: torch.Tensor, scaling: float, n_cand: int, pool: int = 0) -> torch.Tensor:
    """Accumulated attention of decode queries (B, Hq, nq, d) over keys (B, Hkv, T, d):
    (B, Hkv, n_cand) float32 = mean over the group's query heads and queries of softmax(q K^T s)."""
    _cuda(q, k)
    if q.dtype != k.dtype or q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("query_scores: q and k must share dtype f16 / bf16")
    q, k = q.contiguous(), k.contiguous()
    B, Hq, nq, d = q.shape
    Hkv, T = k.shape[1], k.shape[2]
    lib = L.lib()
    wsb = lib.kvb_scores_workspace_size(B, Hkv, n_cand)
    ws = torch.empty(wsb, dtype=torch.uint8, device=q.device)
    out = torch.empty((B, Hkv, n_cand), dtype=torch.float32, device=q.device)
    L.check(lib.kvb_query_scores(_ptr(q), _ptr(k), dtype_code(q), B, Hq, Hkv, nq, T, d, C.c_float(scaling),
                                 n_cand, pool, _ptr(out), _ptr(ws), wsb, C.c_void_p(_stream(q.device))),
            "kvb_query_scores")
    return out


def snapkv_scores(q_window: torch.Tensor, k: torch.Tensor, scaling: float, pool: int = 5) -> torch.Tensor:
    """SnapKV scores at the horizon H = k.shape[2] (snapkv_scores STRATA_KV.py:932-954):
    q_window (B, Hq, w, d) = the queries of the last w context positions, causally masked; returns
    the scores of the H - w candidate positions (B, Hkv, H - w) float32.  The window itself is
    always kept by the caller (the reference pads its columns with max + 1)."""
    _cuda(q_window, k)
    if q_window.dtype != k.dtype or k.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("snapkv_scores: q and k must share dtype f16 / bf16")
    q, k = q_window.contiguous(), k.contiguous()
    B, Hq, w, d = q.shape
    Hkv, H = k.shape[1], k.shape[2]
    lib = L.lib()
    wsb = lib.kvb_scores_workspace_size(B, Hkv, H - w)
    ws = torch.empty(max(wsb, 256), dtype=torch.uint8, device=q.device)
    out = torch.empty((B, Hkv, H - w), dtype=torch.float32, device=q.device)
    L.check(lib.kvb_snapkv_scores(_ptr(q), _ptr(k), dtype_code(q), B, Hq, Hkv, w, H, d, C.c_float(scaling), pool,
                                  _ptr(out), _ptr(ws), wsb, C.c_void_p(_stream(q.device))), "kvb_snapkv_scores")
    return out


def device_diag(clear: bool = True, device=None) -> int:
    """Where the first bounded wait gave up (0 if none); see kvb_device_diag in kvb.h."""
    v = C.c_uint(0)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    L.check(L.lib().kvb_device_diag(C.byref(v), int(clear), C.c_void_p(_stream(dev))), "kvb_device_diag")
    return v.value


def device_status(clear: bool = True, device=None) -> int:
    v = C.c_uint(0)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    L.check(L.lib().kvb_device_status(C.byref(v), int(clear), C.c_void_p(_stream(dev))), "kvb_device_status")
    return v.value


# ------------------------------------------------------------------------------------------------
# K3: decode over a packed cache
# ------------------------------------------------------------------------------------------------
class PackedCache:
    """A head-synchronous packed cache of one layer: up to 4 strata of codes (+ optional exact rows,
    query map / lift for rotated or spectral codes).  Holds the device tensors and builds the
    kvb_cache descriptor."""

    def __init__(self, B, Hkv, d, *, d_code=None, midrise=False, per_channel=False, k_group=None, v_group=None):
        self.B, self.Hkv, self.d = B, Hkv, d
        self.d_code = d if d_code is None else d_code
        self.midrise, self.per_channel = midrise, per_channel
        self.k_group = self.d_code if midrise else k_group
        self.v_group = self.d_code if midrise else v_group
        self.strata = []
        self.k_exact = self.v_exact = None
        self.n_exact = self.n0 = self.pos0 = 0
        self.qmap = self.lift = self.mu_k = self.mu_v = None
        self._ws = {}

    def __setattr__(self, name, value):
        # any attribute change (exact rows appended, a new query map ...) drops the cached descriptor
        object.__setattr__(self, name, value)
        if name != "_c":
            object.__setattr__(self, "_c", None)

    def add_stratum(self, kq: dict, vq: dict):
        if kq["n"] != vq["n"] or kq["n_alloc"] != vq["n_alloc"]:
            raise ValueError("key and value codes of a stratum must hold the same tokens")
        self.strata.append({"kbits": kq["bits"], "vbits": vq["bits"], "n": kq["n"], "n_alloc": kq["n_alloc"],
                            "kc": kq["codes"], "vc": vq["codes"], "km": kq["meta"], "vm": vq["meta"],
                            "v_layout": vq.get("layout", L.KVB_V_TOKEN_MAJOR)})
        self._c = None
        return self

    def set_exact(self, K, V, n_exact=None, n0=None, pos0=0):
        self.k_exact, self.v_exact = K.contiguous(), V.contiguous()
        self.n_exact = K.shape[2] if n_exact is None else n_exact
        self.n0 = self.n_exact if n0 is None else n0
        self.pos0 = pos0
        return self

    def struct(self) -> L.Cache:
        """The kvb_cache descriptor, built once and reused until an attribute of the cache changes
        (the strata and their tensors are not edited in place after add_stratum)."""
        if self._c is not None:
            return self._c
        c = L.Cache()
        c.B, c.Hkv, c.d, c.d_code = self.B, self.Hkv, self.d, self.d_code
        c.code_kind = L.KVB_CODE_MIDRISE if self.midrise else L.KVB_CODE_ASYM
        c.k_mode = L.KVB_K_PER_CHANNEL if self.per_channel else L.KVB_K_PER_TOKEN
        c.k_group = int(self.k_group or self.d_code)
        c.v_group = int(self.v_group or self.d_code)
        c.n_strata = len(self.strata)
        for i, s in enumerate(self.strata):
            c.strata[i].kbits, c.strata[i].vbits = s["kbits"], s["vbits"]
            c.strata[i].v_layout = s.get("v_layout", L.KVB_V_TOKEN_MAJOR)
            c.strata[i].n, c.strata[i].n_alloc = s["n"], s["n_alloc"]
            c.strata[i].kc, c.strata[i].vc = s["kc"].data_ptr(), s["vc"].data_ptr()
            c.strata[i].kmeta, c.strata[i].vmeta = s["km"].data_ptr(), s["vm"].data_ptr()
        if self.k_exact is not None and self.n_exact > 0:
            c.k_exact, c.v_exact = self.k_exact.data_ptr(), self.v_exact.data_ptr()
            c.exact_dtype = dtype_code(self.k_exact)
            c.exact_cap = self.k_exact.shape[2]
            c.n_exact, c.n0, c.pos0 = self.n_exact, self.n0, self.pos0
        for name in ("qmap", "lift", "mu_k", "mu_v"):
            t = getattr(self, name)
            setattr(c, name, None if t is None else t.data_ptr())
        self._c = c
        return c

    def stored_bytes(self) -> int:
        """Bytes of every stored tensor a decode step reads (codes + metadata + exact rows)."""
        tot = 0
        for s in self.strata:
            n = s["n"]
            tot += n * (self.d_code * (s["kbits"] + s["vbits"]) // 8) * self.B * self.Hkv
            for m in ("km", "vm"):
                t = s[m]
                if t.dim() == 5 and m == "km" and self.per_channel:
                    tot += self.B * self.Hkv * (-(-n // self.k_group)) * t.shape[3] * 4
                else:
                    tot += t[:, :, :n].numel() * t.element_size()
        if self.n_exact:
            tot += 2 * self.B * self.Hkv * self.n_exact * self.d * self.k_exact.element_size()
        return tot

    def workspace(self, Hq, Tq, n_ctas=0):
        key = (Hq, Tq, n_ctas)
        if key not in self._ws:
            c = self.struct()
            size = L.lib().kvb_decode_workspace_size(C.byref(c), Hq, Tq, n_ctas)
            if size == 0:
                L.check(L.KVB_EINVAL, "kvb_decode_workspace_size")
            dev = self.strata[0]["kc"].device if self.strata else self.k_exact.device
            # zero-filled once: the in-kernel merge's counters start at zero and every call leaves them so
            self._ws[key] = torch.zeros(size, dtype=torch.uint8, device=dev)
        return self._ws[key]


class overlap_previous:
    """Context manager: decode calls inside it may start copying their packed cache while the kernel
    launched before them on the stream finishes (kvb_set_decode_flags(KVB_DECODE_OVERLAP)).  Use it
    only where no kernel right before a decode call writes that call's packed strata, e.g. around the
    decode calls of consecutive layers."""

    def __enter__(self):
        self._old = L.lib().kvb_set_decode_flags(1)
        return self

    def __exit__(self, *exc):
        L.lib().kvb_set_decode_flags(self._old)
        return False


def decode(cache: PackedCache, q: torch.Tensor, scaling: float, qpos=None, out=None, out_dtype=None,
           n_ctas: int = 0, events=None) -> torch.Tensor:
    """Decode attention of q (B, Hq, Tq, d) over the packed cache -> (B, Tq, Hq, d).
    events: optional (begin, end) torch.cuda.Event pair (already created, e.g. recorded once)
    recorded around the main split-K kernel on the current stream."""
    _cuda(q)
    q = q.contiguous()
    B, Hq, Tq, d = q.shape
    if B != cache.B or d != cache.d:
        raise ValueError("decode: q shape does not match the cache")
    odt = out_dtype or q.dtype
    if out is None:
        out = torch.empty((B, Tq, Hq, d), dtype=odt, device=q.device)
    ws = cache.workspace(Hq, Tq, n_ctas)
    c = cache.struct()
    qp = None
    if qpos is not None:
        qp = (C.c_int64 * Tq)(*[int(v) for v in qpos])
    if events is None:
        L.check(L.lib().kvb_decode(C.byref(c), _ptr(q), dtype_code(q), Hq, Tq, C.c_float(scaling), qp, _ptr(out),
                                   dtype_code(out), n_ctas, _ptr(ws), ws.numel(), C.c_void_p(_stream(q.device))),
                "kvb_decode")
    else:
        e0, e1 = (C.c_void_p(e.cuda_event) for e in events)
        L.check(L.lib().kvb_decode_events(C.byref(c), _ptr(q), dtype_code(q), Hq, Tq, C.c_float(scaling), qp,
                                          _ptr(out), dtype_code(out), n_ctas, _ptr(ws), ws.numel(),
                                          C.c_void_p(_stream(q.device)), e0, e1), "kvb_decode_events")
    return out


def decode_lse(cache: PackedCache, q: torch.Tensor, scaling: float, out: torch.Tensor, lse: torch.Tensor,
               qpos=None, n_ctas: int = 0):
    """decode() that also writes lse (B, Tq, Hq) float32 (natural log of the attended mass); `out`
    (B, Tq, Hq, d) and `lse` are caller-provided (views of one exchange buffer in a sequence split)."""
    _cuda(q, out, lse)
    q = q.contiguous()
    B, Hq, Tq, d = q.shape
    if (B != cache.B or d != cache.d or tuple(out.shape) != (B, Tq, Hq, d) or tuple(lse.shape) != (B, Tq, Hq)
            or lse.dtype != torch.float32 or not out.is_contiguous() or not lse.is_contiguous()):
        raise ValueError("decode_lse: q / out / lse shapes do not match the cache")
    ws = cache.workspace(Hq, Tq, n_ctas)
    c = cache.struct()
    qp = None if qpos is None else (C.c_int64 * Tq)(*[int(v) for v in qpos])
    L.check(L.lib().kvb_decode_lse(C.byref(c), _ptr(q), dtype_code(q), Hq, Tq, C.c_float(scaling), qp, _ptr(out),
                                   dtype_code(out), _ptr(lse), n_ctas, _ptr(ws), ws.numel(),
                                   C.c_void_p(_stream(q.device))), "kvb_decode_lse")
    return out, lse


def lse_merge(parts: torch.Tensor, lse: torch.Tensor, out: torch.Tensor = None, out_dtype=None) -> torch.Tensor:
    """parts (P, rows..., d) float32, lse (P, rows...) float32 -> merged (rows..., d).  Strided views
    are accepted along P (e.g. the two regions of a gathered exchange buffer)."""
    _cuda(parts, lse)
    P, d = parts.shape[0], parts.shape[-1]
    rows = lse[0].numel()
    if parts.dtype != torch.float32 or lse.dtype != torch.float32 or parts[0].numel() != rows * d:
        raise ValueError("lse_merge: parts (P, ..., d) and lse (P, ...) float32 with matching rows")
    if not (parts[0].is_contiguous() and lse[0].is_contiguous()):
        raise ValueError("lse_merge: each part must be contiguous")
    if out is None:
        out = torch.empty(parts.shape[1:], dtype=out_dtype or torch.float32, device=parts.device)
    L.check(L.lib().kvb_lse_merge(_ptr(parts), parts.stride(0), _ptr(lse), lse.stride(0), P, rows, d, _ptr(out),
                                  dtype_code(out), C.c_void_p(_stream(parts.device))), "kvb_lse_merge")
    return out


def decode_noalloc(cache: PackedCache, q: torch.Tensor, scaling: float, out: torch.Tensor, qpos=None,
                   n_ctas: int = 0) -> torch.Tensor:
    """Decode attention for callers that cannot allocate device memory (an engine whose planner owns
    every byte of the GPU, an allocator-less plugin host):
    `q` must be contiguous and `out` (B, Tq, Hq, d) is supplied by the caller; the split-K scratch is
    the library's built-in 8 MiB device array, so neither this wrapper nor the library allocates (a
    strided `q` is refused rather than copied).  The call runs with q's device current, because the
    library looks up the array's address on the current device.  Calls share that array: do not run
    two of them concurrently.  Raises ValueError when a request needs more scratch than the array
    holds (use `decode` with a workspace for those)."""
    _cuda(q, out)
    if not q.is_contiguous():
        raise ValueError("decode_noalloc: q must be contiguous (copying it would allocate)")
    B, Hq, Tq, d = q.shape
    if B != cache.B or d != cache.d or tuple(out.shape) != (B, Tq, Hq, d) or not out.is_contiguous():
        raise ValueError("decode_noalloc: q / out shapes do not match the cache")
    if out.device != q.device:
        raise ValueError("decode_noalloc: q and out must be on one device")
    c = cache.struct()
    qp = None if qpos is None else (C.c_int64 * Tq)(*[int(v) for v in qpos])
    with torch.cuda.device(q.device):
        L.check(L.lib().kvb_decode_noalloc(C.byref(c), _ptr(q), dtype_code(q), Hq, Tq, C.c_float(scaling), qp,
                                           _ptr(out), dtype_code(out), n_ctas, C.c_void_p(_stream(q.device))),
                "kvb_decode_noalloc")
    return out


def decode_plan(cache: PackedCache, n_ctas: int):
    """The split-K plan (host computation): dict with cta_begin, pieces (head, stratum, lo, hi) in CTA
    order, slots (index of each piece's partial, head-major) and head_begin (indexes slots)."""
    c = cache.struct()
    lib = L.lib()
    need = lib.kvb_decode_plan(C.byref(c), n_ctas, None, 0)
    buf = (C.c_int32 * need)()
    lib.kvb_decode_plan(C.byref(c), n_ctas, buf, need)
    v = list(buf)
    nc, npc, nh = v[0], v[1], v[2]
    o = 3
    cta_begin = v[o:o + nc + 1]
    o += nc + 1
    pieces = [tuple(v[o + 5 * i:o + 5 * i + 4]) for i in range(npc)]
    slots = [v[o + 5 * i + 4] for i in range(npc)]
    o += 5 * npc
    head_begin = v[o:o + nh + 1]
    return {"n_ctas": nc, "cta_begin": cta_begin, "pieces": pieces, "slots": slots, "head_begin": head_begin}


# ------------------------------------------------------------------------------------------------
# K4: spectral code
# ------------------------------------------------------------------------------------------------
SPECTRAL_R = 32


# ------------------------------------------------------------------------------------------------
# K5: per-vector row codes
# ------------------------------------------------------------------------------------------------
def _rows(x, idx, first_row, n):
    _cuda(x, idx)
    if x.dim() != 4 or x.stride(-1) != 1:
        raise ValueError("kvb: x must be (B, H, T, d) with unit channel stride")
    B, H, T, d = x.shape
    if idx is not None:
        if idx.dtype != torch.int64 or idx.dim() != 3 or tuple(idx.shape[:2]) != (B, H):
            raise ValueError("kvb: idx must be int64 (B, H, n)")
        idx = idx.contiguous()
        n = idx.shape[2]
    elif n is None:
        n = T - first_row
    return B, H, T, d, idx, n


def absmax_quant(x: torch.Tensor, bits: int, *, variant: str = "strata", idx: torch.Tensor = None,
                 first_row: int = 0, n: int = None, want_xhat: bool = False) -> dict:
    """Per-vector symmetric absmax code of rows of x (B, H, T, d), optionally gathered by idx (B, H, n).
    variant "strata": fp16 scale (absmax_quant STRATA_KV.py:549); "tilt": float32 scale
    (fake_quant_tokens TILT_KV.py:721).  Returns packed (B, H, n, d * bits / 8) MSB-first codes + qmax,
    scale (B, H, n) float32, optional xhat (B, H, n, d) float32 = codes * scale."""
    B, H, T, d, idx, n = _rows(x, idx, first_row, n)
    var = {"strata": L.KVB_ABSMAX_STRATA, "tilt": L.KVB_ABSMAX_TILT}[variant]
    packed = torch.empty((B, H, n, d * bits // 8), dtype=torch.uint8, device=x.device)
    scale = torch.empty((B, H, n), dtype=torch.float32, device=x.device)
    xhat = torch.empty((B, H, n, d), dtype=torch.float32, device=x.device) if want_xhat else None
    L.check(L.lib().kvb_absmax_quant(_ptr(x), dtype_code(x), B, H, T, d, x.stride(0), x.stride(1), x.stride(2),
                                     _ptr(idx), first_row, n, bits, var, _ptr(packed), _ptr(scale), _ptr(xhat),
                                     C.c_void_p(_stream(x.device))), "kvb_absmax_quant")
    return {"packed": packed, "scale": scale, "xhat": xhat, "bits": bits, "n": n}


def pack_rows(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """(..., w) uint8 codes < 2^bits -> (..., w * bits / 8) MSB-first bytes (pack_rows QUASAR_KV.py:1185)."""
    _cuda(codes)
    if codes.dtype != torch.uint8:
        raise ValueError("pack_rows: codes must be uint8")
    codes = codes.contiguous()
    w = codes.shape[-1]
    rows = codes.numel() // w if w else 0
    out = torch.empty(codes.shape[:-1] + (w * bits // 8,), dtype=torch.uint8, device=codes.device)
    L.check(L.lib().kvb_pack_rows(_ptr(codes), rows, w, bits, _ptr(out), C.c_void_p(_stream(codes.device))),
            "kvb_pack_rows")
    return out


def decode_rows_lut(packed: torch.Tensor, bits: int, levels: torch.Tensor, *, row_scale: torch.Tensor = None,
                    out: torch.Tensor = None) -> torch.Tensor:
    """Table decode of MSB-first rows (..., w * bits / 8) -> (..., w) float32 = levels[code] (* row_scale);
    with `out` given the stage is added to it (byte_lut QUASAR_KV.py:1194, stages summed in order)."""
    _cuda(packed, levels, row_scale, out)
    if packed.dtype != torch.uint8 or levels.dtype != torch.float32 or levels.numel() != 1 << bits:
        raise ValueError("decode_rows_lut: packed uint8, levels float32 of 2^bits entries")
    packed = packed.contiguous()
    rb = packed.shape[-1]
    w = rb * 8 // bits
    rows = packed.numel() // rb if rb else 0
    acc = out is not None
    if out is None:
        out = torch.empty(packed.shape[:-1] + (w,), dtype=torch.float32, device=packed.device)
    elif out.dtype != torch.float32 or not out.is_contiguous() or tuple(out.shape) != tuple(packed.shape[:-1]) + (w,):
        raise ValueError("decode_rows_lut: out must be contiguous float32 (..., w)")
    if row_scale is not None:
        row_scale = row_scale.contiguous().float()
        if row_scale.numel() != rows:
            raise ValueError("decode_rows_lut: row_scale needs one value per row")
    L.check(L.lib().kvb_decode_rows_lut(_ptr(packed), rows, w, bits, _ptr(levels.contiguous()), _ptr(row_scale),
                                        int(acc), _ptr(out), C.c_void_p(_stream(packed.device))),
            "kvb_decode_rows_lut")
    return out


def hedge_quant(x: torch.Tensor, R: torch.Tensor, bits: int, levels: torch.Tensor = None, *, mu: torch.Tensor = None,
                idx: torch.Tensor = None, first_row: int = 0, n: int = None, want_y: bool = False,
                want_xhat: bool = False) -> dict:
    """HEDGE per-token code of rows of x (B, H, T, 128) (hedge_quant / centered_code HEDGE_KV.py:1103-1130):
    y = (x - mu) R^T, Lloyd-Max levels (bits 1-4; `levels` float32 2^bits, see codebooks.lloyd_max) or
    int8 absmax (bits 8).  mu: (H, 128) or None.  Returns packed (B, H, n, 16 * bits) MSB-first, scale
    (B, H, n) float32, optional y and xhat = (level * s) R + mu, (B, H, n, 128) float32."""
    B, H, T, d, idx, n = _rows(x, idx, first_row, n)
    if d != 128:
        raise NotImplementedError("hedge_quant: head dim 128 only")
    _cuda(R, levels, mu)
    R = R.float().contiguous()
    if tuple(R.shape) != (128, 128):
        raise ValueError("hedge_quant: R must be (128, 128)")
    if mu is not None:
        mu = mu.float().reshape(H, 128).contiguous()
    if bits <= 4:
        if levels is None or levels.numel() != 1 << bits:
            raise ValueError("hedge_quant: 2^bits levels needed at 1-4 bits")
        levels = levels.float().contiguous()
    dev = x.device
    packed = torch.empty((B, H, n, 16 * bits), dtype=torch.uint8, device=dev)
    scale = torch.empty((B, H, n), dtype=torch.float32, device=dev)
    y = torch.empty((B, H, n, 128), dtype=torch.float32, device=dev) if want_y else None
    xhat = torch.empty((B, H, n, 128), dtype=torch.float32, device=dev) if want_xhat else None
    L.check(L.lib().kvb_hedge_quant(_ptr(x), dtype_code(x), B, H, T, x.stride(0), x.stride(1), x.stride(2), _ptr(idx),
                                    first_row, n, _ptr(mu), _ptr(R), bits, _ptr(levels if bits <= 4 else None),
                                    _ptr(packed), _ptr(scale), _ptr(y), _ptr(xhat), C.c_void_p(_stream(dev))),
            "kvb_hedge_quant")
    return {"packed": packed, "scale": scale, "y": y, "xhat": xhat, "bits": bits, "n": n}


def chunk_select(k: torch.Tensor, qref: torch.Tensor, m: int, want_share: bool = False):
    """TILT chunk selection (finalize_chunk TILT_KV.py:743-760): k (U, H, C, 128) with C <= 128, qref
    (U, H, nq, 128) scaled observed queries.  Returns idx (U, H, m) int64 (the m largest shares, ties
    to the lower position, ascending) and, optionally, share (U, H, C) float32."""
    _cuda(k, qref)
    if k.dim() != 4 or k.shape[-1] != 128 or k.stride(-1) != 1:
        raise ValueError("chunk_select: k must be (U, H, C, 128) with unit channel stride")
    U, H, Cn, _ = k.shape
    qref = qref.float().contiguous()
    if qref.dim() != 4 or tuple(qref.shape[:2]) != (U, H) or qref.shape[-1] != 128:
        raise ValueError("chunk_select: qref must be (U, H, nq, 128)")
    idx = torch.empty((U, H, m), dtype=torch.int64, device=k.device)
    share = torch.empty((U, H, Cn), dtype=torch.float32, device=k.device) if want_share else None
    L.check(L.lib().kvb_chunk_select(_ptr(k), dtype_code(k), U, H, Cn, k.stride(0), k.stride(1), k.stride(2),
                                     _ptr(qref), qref.shape[2], m, _ptr(idx), _ptr(share),
                                     C.c_void_p(_stream(k.device))), "kvb_chunk_select")
    return idx, share


def chunk_tails(k: torch.Tensor, v: torch.Tensor, qref: torch.Tensor, m: int, keep_bits: int = 8) -> dict:
    """The token part of TILT's finalize_chunk for the eviction family (TILT_KV.py:758-766): the m
    top-share keys of every chunk and their values, each stored as an absmax code with a float32
    scale (fake_quant_tokens TILT_KV.py:721).  Two kernels: chunk_select, then absmax_quant over the
    gathered rows of k and of v.  Returns idx and the k / v codes, scales and reconstructions."""
    idx, _ = chunk_select(k, qref, m)
    kq = absmax_quant(k, keep_bits, variant="tilt", idx=idx, want_xhat=True)
    vq = absmax_quant(v, keep_bits, variant="tilt", idx=idx, want_xhat=True)
    return {"idx": idx, "k": kq, "v": vq}


def split_basis(basis_r: torch.Tensor) -> torch.Tensor:
    """basis_r (H, d, r) float -> (2, H, r, d) fp16: transposed basis split as hi + lo (exact to ~22
    bits), the operand layout kvb_spectral_encode expects."""
    bt = basis_r.transpose(1, 2).contiguous().float()
    hi = bt.to(torch.float16)
    lo = (bt - hi.float()).to(torch.float16)
    return torch.stack([hi, lo]).contiguous()


def spectral_encode(x: torch.Tensor, basis_hilo: torch.Tensor, bits: int = 4, want_coef: bool = False,
                    n_alloc: int = None, n_ctas: int = 0) -> dict:
    """Project x (B, H, T, 128) fp16 onto each head's leading 32 basis columns on the tensor cores and
    code each token's coefficients with the mid-rise code.  Returns a stratum dict (codes, meta =
    fp16 scales, n, n_alloc, bits) and optionally the float32 coefficients."""
    _cuda(x, basis_hilo)
    if x.dtype != torch.float16 or x.dim() != 4 or x.shape[-1] != 128:
        raise ValueError("spectral_encode: x must be fp16 (B, H, T, 128)")
    if x.stride(-1) != 1 or any(s_ % 8 for s_ in x.stride()[:3]):
        x = x.contiguous()                  # the tensor map needs 16-byte strides; other layouts are copied
    B, H, T, d = x.shape
    if basis_hilo.dtype != torch.float16 or tuple(basis_hilo.shape) != (2, H, SPECTRAL_R, d):
        raise ValueError("spectral_encode: basis must be fp16 (2, H, 32, 128) (see split_basis)")
    basis_hilo = basis_hilo.contiguous()
    n_alloc = round_up(T, 16) if n_alloc is None else n_alloc
    codes = torch.empty((B, H, n_alloc, SPECTRAL_R * bits // 8), dtype=torch.uint8, device=x.device)
    scales = torch.zeros((B, H, n_alloc), dtype=torch.float16, device=x.device)
    if n_alloc > T:
        codes[:, :, T:].zero_()
    coef = torch.empty((B, H, T, SPECTRAL_R), dtype=torch.float32, device=x.device) if want_coef else None
    L.check(L.lib().kvb_spectral_encode(_ptr(x), B, H, T, x.stride(0), x.stride(1), x.stride(2), _ptr(basis_hilo),
                                        bits, C.c_float(UNIFORM_STEP[bits]),
                                        _ptr(codes), _ptr(scales), n_alloc, _ptr(coef), n_ctas,
                                        C.c_void_p(_stream(x.device))), "kvb_spectral_encode")
    return {"codes": codes, "meta": scales, "n": T, "n_alloc": n_alloc, "bits": bits, "group": SPECTRAL_R,
            "coef": coef}


# ------------------------------------------------------------------------------------------------
# STRATA rate allocation (head_sync_allocate, STRATA_KV.py:1308-1351)
# ------------------------------------------------------------------------------------------------
def head_sync_allocate(Dsort: torch.Tensor, cost, fixed, budget: float, rounds: int = 4, grid: int = 32):
    """Device allocation of rank positions to options (drop | coded levels | exact) under a bit budget.
    Dsort (n, nlev) float32 CUDA; cost (nlev) and fixed (nlev - 1) sequences of floats.  Returns
    {"choice": (n,) int32, "cap": () int32, "bits": () float64} on Dsort's device (no synchronisation)."""
    _cuda(Dsort)
    if Dsort.dtype != torch.float32 or Dsort.dim() != 2:
        raise ValueError("head_sync_allocate: Dsort (n, nlev) float32")
    Dsort = Dsort.contiguous()
    n, nlev = Dsort.shape
    cost = [float(x) for x in cost]
    fixed = [float(x) for x in fixed]
    if len(cost) != nlev or len(fixed) != nlev - 1:
        raise ValueError("head_sync_allocate: cost has nlev entries, fixed nlev - 1")
    lib = L.lib()
    dev = Dsort.device
    key = ("alloc_ws", dev)
    ws = _ALLOC_WS.get(key)
    if ws is None:
        ws = _ALLOC_WS[key] = torch.zeros(lib.kvb_head_sync_allocate_workspace(), dtype=torch.uint8, device=dev)
    choice = torch.empty(n, dtype=torch.int32, device=dev)
    cap = torch.empty((), dtype=torch.int32, device=dev)
    bits = torch.empty((), dtype=torch.float64, device=dev)
    L.check(lib.kvb_head_sync_allocate(_ptr(Dsort), n, nlev, (C.c_float * nlev)(*cost), (C.c_float * (nlev - 1))(*fixed),
                                       C.c_double(budget), rounds, grid, _ptr(choice), _ptr(cap), _ptr(bits), _ptr(ws),
                                       ws.numel(), C.c_void_p(_stream(dev))), "kvb_head_sync_allocate")
    return {"choice": choice, "cap": cap, "bits": bits}


_ALLOC_WS = {}


# ------------------------------------------------------------------------------------------------
# QUASAR coded decode over embedded stage codes (coded_scores / coded_values, QUASAR_KV.py:1918-1940)
# ------------------------------------------------------------------------------------------------
def _quasar_tables(table, levels):
    t = np.ascontiguousarray(np.asarray(table, np.int32).reshape(-1, 7))
    lv = np.ascontiguousarray(np.asarray(levels, np.float32).reshape(-1))
    return t, lv


def quasar_scores(qt: torch.Tensor, flat: torch.Tensor, table, levels, n_c: int) -> torch.Tensor:
    """qt (Hkv, rows, R) float32 CUDA, flat uint8 CUDA, table (n_steps, 7) and levels on the host ->
    scores (Hkv, rows, n_c) float32."""
    _cuda(qt, flat)
    qt = qt.float().contiguous()
    Hkv, rows, R = qt.shape
    t, lv = _quasar_tables(table, levels)
    out = torch.empty((Hkv, rows, n_c), dtype=torch.float32, device=qt.device)
    L.check(L.lib().kvb_quasar_scores(_ptr(qt), Hkv, rows, R, _ptr(flat), flat.numel(), t.ctypes.data, len(t),
                                      lv.ctypes.data, len(lv), n_c, _ptr(out), C.c_void_p(_stream(qt.device))),
            "kvb_quasar_scores")
    return out


def quasar_values(pv: torch.Tensor, flat: torch.Tensor, table, levels, R: int) -> torch.Tensor:
    """pv (Hkv, rows, n_c) float32 CUDA -> values (Hkv, rows, R) float32."""
    _cuda(pv, flat)
    pv = pv.float().contiguous()
    Hkv, rows, n_c = pv.shape
    t, lv = _quasar_tables(table, levels)
    lib = L.lib()
    ws = torch.empty(max(16, lib.kvb_quasar_values_workspace(Hkv, rows, n_c, R)), dtype=torch.uint8, device=pv.device)
    out = torch.empty((Hkv, rows, R), dtype=torch.float32, device=pv.device)
    L.check(lib.kvb_quasar_values(_ptr(pv), Hkv, rows, n_c, _ptr(flat), flat.numel(), t.ctypes.data, len(t),
                                  lv.ctypes.data, len(lv), R, _ptr(out), _ptr(ws), ws.numel(),
                                  C.c_void_p(_stream(pv.device))), "kvb_quasar_values")
    return out


# ------------------------------------------------------------------------------------------------
# TILT moment-atom read (atom_read, TILT_KV.py:673-714)
# ------------------------------------------------------------------------------------------------
def atom_read(qs: torch.Tensor, mom: dict, rep: int):
    """qs (B, Hq, c, d) float32 CUDA; mom: the atoms' float32 CUDA tensors (mu_k, logn, U, lam, diag,
    R, A, Bk, Rv; those the flags leave unused may be missing) and the flags order, tilt, project,
    phase.  Returns (logit, cfac, tB or None) like the reference's atom_read."""
    _cuda(qs)
    qs = qs.float().contiguous()
    B, Hq, c, d = qs.shape
    mu = mom["mu_k"]
    Bm, Hkv, NA, dm = mu.shape
    if Bm != B or dm != d or Hq != Hkv * rep:
        raise ValueError("atom_read: qs does not match the atoms")
    order, tilt = int(mom["order"]), bool(mom["tilt"])
    r = mom["U"].shape[-1] if order == 2 else (mom["Bk"].shape[-1] if tilt else 1)
    keep = []

    def ptr(name):
        t = mom.get(name)
        if t is None:
            return None
        t = t.float().contiguous()
        keep.append(t)
        return _ptr(t)

    m = L.Atoms(*(ptr(n) for n in ("mu_k", "logn", "U", "lam", "diag", "R", "A", "Bk", "Rv")),
                B, Hkv, NA, d, r, order, int(tilt), int(bool(mom["project"])), int(bool(mom.get("phase", True))))
    logit = torch.empty((B, Hq, c, NA), dtype=torch.float32, device=qs.device)
    cfac = torch.empty_like(logit)
    tB = torch.empty((B, Hq, c, NA, r), dtype=torch.float32, device=qs.device) if tilt else None
    L.check(L.lib().kvb_atom_read(C.byref(m), _ptr(qs), Hq, c, _ptr(logit), _ptr(cfac),
                                  _ptr(tB) if tB is not None else None, C.c_void_p(_stream(qs.device))),
            "kvb_atom_read")
    return logit, cfac, tB
