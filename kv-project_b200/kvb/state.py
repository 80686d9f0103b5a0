"""Decoder state objects with the reference's decode protocol, backed by kvb's packed cache.

The reference decodes through per-layer state objects driven by ``DecodeCtl.attend``
(STRATA_KV.py:2826-2834): ``state.append(k, v, pos)`` then ``state.attend(q, scaling, qpos,
chunk)``, with attributes ``n`` / ``n0`` / ``shared`` and ``context_bytes()`` / ``check_kernel()``.
The classes here keep that protocol (same constructor arguments, same exceptions, same output
layout (B, Tq, Hq, d) in q's dtype) and run every attend as one ``kvb_decode`` call over the exact
rows and all packed strata.  There is no PyTorch path that produces outputs: ``check_kernel`` only
compares the CUDA result against a float32 restatement of the reference formula and raises when
they disagree (the reference would fall back instead, STRATA_KV.py:1814).

  KvbStrataState   replaces StrataState (STRATA_KV.py:1710-1830) over the reference's own packed
                   strata (``StrataMethod.pack`` STRATA_KV.py:1611-1627).
  KvbCodedState    a decoder state over any PackedCache built by ``kvb.cache`` (KIVI, eviction,
                   mixed strata, spectral): replaces LayerState (STRATA_KV.py:682-720) for methods
                   whose token entries are codes rather than reconstructions.
"""

from __future__ import annotations

import torch

from . import ops

BIG = 1 << 40


def _tensor_bytes(ts) -> int:
    """Sum of numel * element_size over nested lists of tensors (``tensor_bytes`` of the reference)."""
    if isinstance(ts, torch.Tensor):
        return ts.numel() * ts.element_size()
    return sum(_tensor_bytes(t) for t in ts)


def tier_as_kvb(t: dict, side: str, device=None) -> dict:
    """One side ("k" or "v") of a reference stratum tier -> a kvb stratum half.

    Reference tier (STRATA_KV.py:1618-1622): ``bits``, ``n``, ``{k,v}c`` planar codes (Hkv, n,
    d * bits / 8) uint8, ``{k,v}s`` fp16 scales (Hkv, n).  kvb wants a batch dimension and a row
    capacity that is a multiple of 16: codes (1, Hkv, n_alloc, RB), scales (1, Hkv, n_alloc) fp16,
    the padding rows zero (never read: every stratum carries its own n)."""
    codes, scales = t[f"{side}c"], t[f"{side}s"]
    dev = codes.device if device is None else torch.device(device)
    Hkv, n, rb = codes.shape
    n_alloc = max(16, ops.round_up(n, 16))
    c = torch.zeros((1, Hkv, n_alloc, rb), dtype=torch.uint8, device=dev)
    s = torch.zeros((1, Hkv, n_alloc), dtype=torch.float16, device=dev)
    c[0, :, :n] = codes.to(dev)
    s[0, :, :n] = scales.to(dev, torch.float16)
    return {"codes": c, "meta": s, "n": int(n), "n_alloc": n_alloc, "bits": int(t["bits"])}


class _KvbState:
    """Exact-row buffer + append protocol shared by the kvb decoder states."""

    def _init_rows(self, Ke: torch.Tensor, Ve: torch.Tensor, extra: int, H: int):
        B, Hkv, n0, d = Ke.shape
        self.K = Ke.new_zeros((B, Hkv, n0 + extra, d))
        self.V = Ve.new_zeros((B, Hkv, n0 + extra, d))
        self.K[:, :, :n0], self.V[:, :, :n0] = Ke, Ve
        self.n0 = self.n = n0
        self.dtype = Ke.dtype
        self.H, self.shared = H, None
        self.use_kernel = True

    def append(self, k, v, pos):
        """Append t exact rows (positions H + n - n0 ...); raises when the buffer is full."""
        t = k.shape[2]
        if self.n + t > self.K.shape[2]:
            raise RuntimeError("decode buffer exhausted")
        self.K[:, :, self.n:self.n + t], self.V[:, :, self.n:self.n + t] = k, v
        self.n += t

    def attend(self, q, scaling, qpos, chunk=None):
        """Attention of q (B, Hq, Tq, d) over exact rows (appended ones causal w.r.t. qpos) and the
        packed strata -> (B, Tq, Hq, d) in q's dtype.  ``chunk`` is accepted for protocol
        compatibility (the split-K plan is chosen by the library)."""
        qp = [int(x) for x in (qpos.tolist() if isinstance(qpos, torch.Tensor) else qpos)]
        c = self.cache
        if self.n > 0:
            c.set_exact(self.K, self.V, n_exact=self.n, n0=self.n0, pos0=self.H)
        out = ops.decode(c, q.to(self.dtype), float(scaling), qpos=qp)   # exact rows and q share a dtype
        return out if out.dtype == q.dtype else out.to(q.dtype)


class KvbStrataState(_KvbState):
    """STRATA decoder state over the reference's packed strata (same constructor as StrataState,
    STRATA_KV.py:1723): exact rows Ke, Ve (1, Hkv, n0, d) in the model dtype; ``packed`` =
    ``StrataMethod.pack`` output (tiers, counts, n_c, fp16 mu_k / mu_v) or None; ``extra`` rows of
    room for appended tokens at positions H, H + 1, ...; rotation R (d, d).

    The stored strata are used as they are (planar codes, fp16 scales): the query rotation q R^T
    and the mean-key bias scaling q . mu_K run in the library's prologue, the coded value sum is
    rotated back by R and gets (sum p) mu_V in its merge (StrataState.attend STRATA_KV.py:1762-1796).
    """

    def __init__(self, Ke, Ve, packed, extra: int, H: int, R: torch.Tensor):
        self._init_rows(Ke, Ve, extra, H)
        B, Hkv, _, d = Ke.shape
        if packed is not None and packed["n_c"]:
            packed = {**packed, "mu_k": packed["mu_k"].to(self.dtype), "mu_v": packed["mu_v"].to(self.dtype)}
        self.p, self.R = packed, R
        dev = Ke.device
        self.cache = ops.PackedCache(B, Hkv, d, midrise=True)
        if packed is not None and packed["n_c"]:
            tiers = [t for t in packed["tiers"] if t["n"] > 0]
            if len(tiers) > 4:
                raise ValueError("KvbStrataState: at most 4 strata")
            for t in tiers:
                self.cache.add_stratum(tier_as_kvb(t, "k", dev), tier_as_kvb(t, "v", dev))
            Rf = R.to(dev, torch.float32)
            self.cache.qmap = Rf.t().expand(Hkv, d, d).contiguous()
            self.cache.lift = Rf.expand(Hkv, d, d).contiguous()
            self.cache.mu_k = packed["mu_k"].to(dev, torch.float32).contiguous()
            self.cache.mu_v = packed["mu_v"].to(dev, torch.float32).contiguous()

    def context_bytes(self) -> int:
        """Bytes of the stored context: exact rows + the packed strata as the reference stores them
        (StrataState.context_bytes STRATA_KV.py:1736-1741; the 16-row padding is not counted)."""
        p = self.p
        coded = 0 if p is None else _tensor_bytes(
            [[[t[x] for x in ("kc", "vc", "ks", "vs")] for t in p["tiers"]], p["counts"]] +
            [p[x] for x in ("mu_k", "mu_v") if x in p])
        return _tensor_bytes([self.K[:, :, :self.n0], self.V[:, :, :self.n0]]) + coded

    @torch.no_grad()
    def reference_attend(self, q, scaling, qpos) -> torch.Tensor:
        """The reference formula in float32 on q's device (dequantise every stratum, rotate back, add
        the means, attend over exact rows + coded tokens).  Used only by check_kernel."""
        B, Hq, Tq, d = q.shape
        Hkv = self.K.shape[1]
        rep = Hq // Hkv
        qg = q.float().reshape(Hkv, rep * Tq, d)
        n = self.n
        s = qg @ self.K[0, :, :n].float().transpose(-1, -2) * scaling
        if n > self.n0:
            row_pos = self.H + torch.arange(n - self.n0, device=q.device)
            qp = torch.as_tensor(qpos, device=q.device).reshape(-1)
            bad = row_pos[None, :] > qp[:, None]
            s[..., self.n0:] = s[..., self.n0:].masked_fill(bad.repeat(rep, 1), float("-inf"))
        Vs = [self.V[0, :, :n].float()]
        if self.p is not None and self.p["n_c"]:
            R = self.R.float().to(q.device)
            mk, mv = self.p["mu_k"].float().to(q.device), self.p["mu_v"].float().to(q.device)
            for t in self.p["tiers"]:
                if t["n"] == 0:
                    continue
                half = (2 ** t["bits"] - 1) / 2.0
                kh = (_unpack_planar(t["kc"].to(q.device), t["bits"]) - half) * t["ks"].float().to(q.device)[..., None]
                vh = (_unpack_planar(t["vc"].to(q.device), t["bits"]) - half) * t["vs"].float().to(q.device)[..., None]
                s = torch.cat([s, qg @ (kh @ R + mk[:, None, :]).transpose(-1, -2) * scaling], -1)
                Vs.append(vh @ R + mv[:, None, :])
        o = s.softmax(-1) @ torch.cat(Vs, 1)
        return o.reshape(B, Hq, Tq, d).transpose(1, 2)

    @torch.no_grad()
    def check_kernel(self, tol: float = 2e-2) -> dict:
        """Parity gate of StrataState.check_kernel (STRATA_KV.py:1798-1822): random queries (seed 42,
        4 query heads per KV head, positions H and H + 1), kvb's output against the float32
        reference formula.  Raises RuntimeError when the relative max error exceeds tol (there is no
        other path to fall back to)."""
        g = torch.Generator(device="cpu").manual_seed(42)
        Hq = self.K.shape[1] * 4
        q = torch.randn(1, Hq, 2, self.K.shape[-1], generator=g).to(self.K.device, self.dtype)
        qpos = [self.H, self.H + 1]
        scaling = self.K.shape[-1] ** -0.5
        ref = self.reference_attend(q, scaling, qpos)
        out = self.attend(q, scaling, qpos).float()
        err = float((out - ref).abs().max() / ref.abs().max().clamp_min(1e-30))
        if not err <= tol:
            raise RuntimeError(f"kvb decode disagrees with the reference formula (rel err {err:.3g} > {tol})")
        return {"kernel": True, "kernel_rel_err": err}


class KvbCodedState(_KvbState):
    """Decoder state over a kvb PackedCache (codes never reconstructed), LayerState's protocol:
    the cache's own exact rows (sinks) are the first n0 rows; appended rows follow, causal at
    positions H, H + 1, ...  ``cache`` comes from ``kvb.cache.build_kivi`` / ``build_eviction`` /
    ``build_mixed`` / ``build_spectral``."""

    def __init__(self, cache: "ops.PackedCache", extra: int, H: int, dtype=None, K_sink=None, V_sink=None):
        dev = cache.strata[0]["kc"].device if cache.strata else K_sink.device
        if K_sink is None:
            K_sink = cache.k_exact[:, :, :cache.n_exact] if cache.k_exact is not None else \
                torch.zeros((cache.B, cache.Hkv, 0, cache.d), dtype=dtype or torch.bfloat16, device=dev)
            V_sink = cache.v_exact[:, :, :cache.n_exact] if cache.v_exact is not None else torch.zeros_like(K_sink)
        self._init_rows(K_sink.to(dtype or K_sink.dtype), V_sink.to(dtype or V_sink.dtype), extra, H)
        self.cache = cache

    def context_bytes(self) -> int:
        """Exact rows + every stored code and metadata byte of the packed cache."""
        c = self.cache
        tot = _tensor_bytes([self.K[:, :, :self.n0], self.V[:, :, :self.n0]])
        for s in c.strata:
            tot += _tensor_bytes([s["kc"][:, :, :s["n"]], s["vc"][:, :, :s["n"]]])
            for m in ("km", "vm"):
                tot += _tensor_bytes(s[m])
        return tot


def _unpack_planar(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """(…, d * bits / 8) planar bytes -> (…, d) float codes (byte i holds channel p * d / P + i in
    bits [p * bits, (p + 1) * bits)), as unpack_planar STRATA_KV.py:1185-1189."""
    P = 8 // bits
    x = codes.to(torch.int32)
    planes = [(x >> (p * bits)) & ((1 << bits) - 1) for p in range(P)]
    return torch.cat(planes, -1).float()
