"""Sequence split of a layer's packed cache over ranks (config 4 with batch <= 4).

Each rank holds a contiguous, group-aligned token range of every (batch, KV head) and decodes it
with ``kvb_decode_lse``: a normalised float32 output and the natural-log mass of its range per
(batch, query position, query head).  Two ways to combine the ranks' parts (the LSE merge of
StrataState.attend, STRATA_KV.py:1784-1792, across ranks instead of across strata):

  SeqSplitDecoder     one exchange buffer per rank, a single all-gather (NCCL over NVLink on the
                      GPUs; any torch.distributed backend works), then ``kvb_lse_merge``;
  P2PSeqSplitDecoder  peer memory (CUDA IPC mappings, plain peer stores over NVLink): by default ONE
                      kernel per call (``kvb_decode_xchg``: each head's in-kernel merge publishes
                      this rank's part to every peer, waits for theirs and merges); or
                      ``kvb_decode_lse`` + ``kvb_xchg_merge`` (fused=False).

Exact rows (sinks, appended tokens) belong to one rank, the owner of the last range.
"""

from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _lib as L
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


class P2PSeqSplitDecoder:
    """Sequence-split decode whose cross-rank step runs over peer memory.  Per shape each rank allocates
    an exchange region in libkvb (zeroed) and the 64-byte CUDA IPC handles are all-gathered once over
    the process group.  fused=True (default): every attend() is ONE ``kvb_decode_xchg`` kernel, whose
    in-kernel head merges publish this rank's part to every peer, wait for theirs and merge; fused=False:
    ``kvb_decode_lse`` + one ``kvb_xchg_merge`` kernel.  All ranks must use the same setting and call
    attend() with the same shapes in the same order, each holding at least one token (as for the
    collective version).  Ranks must share one node with peer access (NVLink / NVSwitch); call close()
    before destroying the process group."""

    def __init__(self, group=None, timeout_s: float = 2.0, fused: bool = True):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout_ns = int(timeout_s * 1e9)
        self.fused = fused
        self._state = {}

    def _setup(self, key, nbytes, rows, d, device):
        if key in self._state:
            return self._state[key]
        lib = L.lib()
        with torch.cuda.device(device):
            if nbytes == 0:
                raise ValueError(f"P2PSeqSplitDecoder: unsupported shape or world size {self.world}")
            own = C.c_void_p()
            handle = (C.c_ubyte * 64)()
            L.check(lib.kvb_xchg_alloc(nbytes, C.byref(own), handle), "kvb_xchg_alloc")
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=self.group)
            regions = (C.c_void_p * self.world)()
            opened = []
            for r in range(self.world):
                if r == self.rank:
                    regions[r] = own.value
                    continue
                ptr = C.c_void_p()
                hb = (C.c_ubyte * 64).from_buffer_copy(handles[r])
                L.check(lib.kvb_xchg_open(hb, C.byref(ptr)), "kvb_xchg_open")
                regions[r] = ptr.value
                opened.append(ptr.value)
        part = lse = None
        if not self.fused:
            part = torch.empty((rows, d), dtype=torch.float32, device=device)
            lse = torch.empty((rows,), dtype=torch.float32, device=device)
        self._state[key] = (own.value, opened, regions, part, lse, nbytes, device)
        return self._state[key]

    def attend(self, cache: "ops.PackedCache", q: torch.Tensor, scaling: float, qpos=None, out=None,
               out_dtype=None) -> torch.Tensor:
        B, Hq, Tq, d = q.shape
        rows = B * Tq * Hq
        odt = out_dtype or q.dtype
        if out is None:
            out = torch.empty((B, Tq, Hq, d), dtype=odt, device=q.device)
        elif tuple(out.shape) != (B, Tq, Hq, d) or not out.is_contiguous():
            raise ValueError("P2PSeqSplitDecoder: out must be contiguous (B, Tq, Hq, d)")
        lib = L.lib()
        if self.fused:
            ops._cuda(q, out)
            q = q.contiguous()
            c = cache.struct()
            nbytes = lib.kvb_decode_xchg_bytes(C.byref(c), Hq, Tq, self.world)
            _, _, regions, _, _, _, _ = self._setup(("fused", B, Tq, Hq, cache.Hkv, d, q.device), nbytes, rows, d,
                                                    q.device)
            ws = cache.workspace(Hq, Tq)
            qp = None if qpos is None else (C.c_int64 * Tq)(*[int(v) for v in qpos])
            L.check(lib.kvb_decode_xchg(C.byref(c), ops._ptr(q), ops.dtype_code(q), Hq, Tq, C.c_float(scaling), qp,
                                        ops._ptr(out), ops.dtype_code(out), self.rank, self.world, regions,
                                        self.timeout_ns, 0, ops._ptr(ws), ws.numel(),
                                        C.c_void_p(ops._stream(q.device))), "kvb_decode_xchg")
            return out
        nbytes = lib.kvb_xchg_bytes(rows, d, self.world)
        _, _, regions, part, lse, _, _ = self._setup(("two-kernel", rows, d, q.device), nbytes, rows, d, q.device)
        ops.decode_lse(cache, q, scaling, part.view(B, Tq, Hq, d), lse.view(B, Tq, Hq), qpos=qpos)
        L.check(lib.kvb_xchg_merge(ops._ptr(part), ops._ptr(lse), rows, d, self.rank, self.world, regions,
                                   ops._ptr(out), ops.dtype_code(out), self.timeout_ns,
                                   C.c_void_p(ops._stream(q.device))), "kvb_xchg_merge")
        return out

    def reset(self):
        """Re-establish the exchange after a timed-out wait (KVB_DEV_TIMEOUT in the device status
        word; no exchange runs until then): every rank clears its status word, the ranks meet, every
        rank zeroes its whole region (flags and call counters restart at 0), and the ranks meet again
        before the next attend().  Returns the status word that was cleared."""
        torch.cuda.synchronize()
        st = ops.device_status(clear=True)
        dist.barrier(group=self.group)
        lib = L.lib()
        for own, _, _, _, _, nbytes, device in self._state.values():
            with torch.cuda.device(device):
                torch.cuda.synchronize()
                L.check(lib.kvb_xchg_zero(C.c_void_p(own), nbytes, C.c_void_p(ops._stream(device))),
                        "kvb_xchg_zero")
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        return st

    def close(self):
        """Unmap the peers' regions and free this rank's (after a barrier: no peer may still write)."""
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        lib = L.lib()
        for own, opened, _, _, _, _, _ in self._state.values():
            for ptr in opened:
                L.check(lib.kvb_xchg_close(C.c_void_p(ptr)), "kvb_xchg_close")
        dist.barrier(group=self.group)
        for own, _, _, _, _, _, _ in self._state.values():
            L.check(lib.kvb_xchg_free(C.c_void_p(own)), "kvb_xchg_free")
        self._state.clear()


def shard_cache(build, K: torch.Tensor, V: torch.Tensor, rank: int, world: int, align: int = 128):
    """Build this rank's cache over its token range with `build(K_slice, V_slice)` (e.g. a
    functools.partial of kvb.cache.build_kivi)."""
    lo, hi = token_ranges(K.shape[2], world, align)[rank]
    return build(K[:, :, lo:hi], V[:, :, lo:hi])
