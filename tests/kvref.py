"""Helpers that turn GPU-packed caches back into arrays the oracle understands (test infrastructure)."""

import numpy as np
import torch

import oracle as O


def np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def unpack(codes: torch.Tensor, bits: int, n: int) -> np.ndarray:
    """(B, H, n_alloc, RB) planar bytes -> (B, H, n, d) integer codes (oracle unpack_planar); block-
    layout value codes (B, H, n_alloc / 128, 128, 16 * bits) are unblocked first."""
    if codes.dim() == 5:
        import kvb
        codes = kvb.ops.unblock_codes(codes)
    return O.unpack_planar(codes[:, :, :n].cpu().numpy(), bits).astype(np.uint8)


def token_meta(meta: torch.Tensor, n: int):
    """(B, H, n_alloc, G, 2) fp16 -> lo, scale shaped like kivi_quant's (B, H, n, G, 1)."""
    m = meta[:, :, :n].float().cpu().numpy()
    return m[..., 0:1], m[..., 1:2]


def channel_meta(meta: torch.Tensor, n: int, group: int):
    """(B, H, n_alloc / g, d, 2) fp16 -> lo, scale shaped like kivi_quant's (B, H, n_g, 1, d)."""
    ng = -(-n // group)
    m = meta[:, :, :ng].float().cpu().numpy()
    return m[:, :, :, None, :, 0], m[:, :, :, None, :, 1]


def gather_rows(x: np.ndarray, idx: np.ndarray) -> np.ndarray:
    return np.take_along_axis(x, idx[..., None].repeat(x.shape[-1], -1), 2)


def scatter_rows(full: np.ndarray, idx: np.ndarray, rows: np.ndarray):
    np.put_along_axis(full, idx[..., None].repeat(full.shape[-1], -1), rows, 2)


def attend_reference(q: np.ndarray, scaling: float, Khat: np.ndarray, Vhat: np.ndarray, qpos=None):
    """Dequantise-then-attend (chunked_attention, STRATA_KV.py:641) over a fully readable cache."""
    B, H, T, d = Khat.shape
    Tq = q.shape[2]
    qpos = np.full(Tq, T) if qpos is None else np.asarray(qpos)
    return O.chunked_attention(q, scaling, qpos, Khat, Vhat, np.arange(T), np.full(T, O.attention.BIG), None, 256)
