"""Sequence split of a layer's packed cache over ranks (config 4 with batch <= 4).

Each rank holds a contiguous, group-aligned token range of every (batch, KV head) and decodes it
with ``kvb_decode_lse``: a normalised float32 output and the natural-log mass of its range per
(batch, query position, query head).  Both live in one exchange buffer, gathered from every rank
with a single all-gather (NCCL over NVLink on the GPUs; any torch.distributed backend works), and
``kvb_lse_merge`` combines the parts exactly (the LSE merge of StrataState.attend,
STRATA_KV.py:1784-1792, across ranks instead of across strata).  Exact rows (sinks, appended
tokens) belong to one rank, the owner of the last range.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops


def token_ranges(T: int, world: int, align: int = 128):
    """[lo, hi) per rank: contiguous ranges covering [0, T), every boundary a multiple of `align` (so
    per-channel key groups of `align` tokens never straddle two ranks), sizes within one `align`."""
    if T <= 0 or world <= 0 or align <= 0:
        raise ValueError("token_ranges: T, world and align must be positive")
    units = -(-T // align)
    return [((units * r // world) * align, min(T, (units * (r + 1) // world) * align)) for r in range(world)]


def exchange_views(buf: torch.Tensor, B: int, Tq: int, Hq: int, d: int):
    """The two regions of one exchange buffer (B*Tq*Hq*(d+1) float32): out (B, Tq, Hq, d), lse (B, Tq, Hq)."""
    rows = B * Tq * Hq
    return buf[:rows * d].view(B, Tq, Hq, d), buf[rows * d:rows * (d + 1)].view(B, Tq, Hq)


def gathered_views(g: torch.Tensor, B: int, Tq: int, Hq: int, d: int):
    """Per-rank views of the gathered buffer (P, B*Tq*Hq*(d+1)): parts (P, B, Tq, Hq, d), lse (P, B, Tq, Hq)."""
    rows = B * Tq * Hq
    P = g.shape[0]
    return g[:, :rows * d].view(P, B, Tq, Hq, d), g[:, rows * d:rows * (d + 1)].view(P, B, Tq, Hq)


def all_gather_into(out: torch.Tensor, buf: torch.Tensor, group=None) -> torch.Tensor:
    """out (P, n) <- every rank's `buf` (n,) in rank order, one collective (all_gather_into_tensor on
    NCCL; the list form on backends without it, e.g. gloo)."""
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, buf, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), buf, group=group)
    return out


class SeqSplitDecoder:
    """Decode of a sequence-split layer: this rank's PackedCache holds its token range; attend()
    returns the full attention output on every rank.  Buffers are kept per shape, so repeated calls
    allocate nothing (and can be captured in a CUDA graph together with the NCCL all-gather)."""

    def __init__(self, group=None):
        self.group = group
        self._bufs = {}

    def _buffers(self, B, Tq, Hq, d, device):
        key = (B, Tq, Hq, d, device)
        if key not in self._bufs:
            world = dist.get_world_size(self.group)
            n = B * Tq * Hq * (d + 1)
            self._bufs[key] = (torch.empty(n, dtype=torch.float32, device=device),
                               torch.empty((world, n), dtype=torch.float32, device=device))
        return self._bufs[key]

    def attend(self, cache: "ops.PackedCache", q: torch.Tensor, scaling: float, qpos=None, out=None,
               out_dtype=None) -> torch.Tensor:
        B, Hq, Tq, d = q.shape
        buf, gath = self._buffers(B, Tq, Hq, d, q.device)
        o, lse = exchange_views(buf, B, Tq, Hq, d)
        ops.decode_lse(cache, q, scaling, o, lse, qpos=qpos)
        all_gather_into(gath, buf, self.group)
        parts, lses = gathered_views(gath, B, Tq, Hq, d)
        return ops.lse_merge(parts, lses, out=out, out_dtype=out_dtype or q.dtype)


def shard_cache(build, K: torch.Tensor, V: torch.Tensor, rank: int, world: int, align: int = 128):
    """Build this rank's cache over its token range with `build(K_slice, V_slice)` (e.g. a
    functools.partial of kvb.cache.build_kivi)."""
    lo, hi = token_ranges(K.shape[2], world, align)[rank]
    return build(K[:, :, lo:hi], V[:, :, lo:hi])
