"""Cache builders: from model-dtype K / V to packed, head-synchronous caches (all on the GPU).

  build_mixed     config 1: per-token importance = key energy, head-synchronous 8 / 4 / 2-bit
                  strata (10 % / 30 % / 60 %), KIVI per-token groups for keys and values
                  (kivi_quant(..., along_tokens=False) per stratum, STRATA_KV.py:826); tc=True
                  stores the values in the block layout of the tcgen05 decode.
  build_kivi      configs 0 / 4: KIVI keys per channel over token groups, values per token
                  (KIVIMethod.entries, STRATA_KV.py:797-803).
  build_eviction  config 2: SnapKV-style scores of decode queries, top-`budget` heavy hitters +
                  recent window, KIVI codes of the kept tokens (SnapKVQuantMethod.entries,
                  STRATA_KV.py:1010-1033).
"""

from __future__ import annotations

import torch

from . import ops


def strata_counts(T: int, tenths8: int = 1, tenths4: int = 3):
    n8 = (T * tenths8) // 10
    n4 = (T * tenths4) // 10
    return n8, n4, T - n8 - n4


def tc_layout_ok(x: torch.Tensor, group: int) -> bool:
    """Whether values can be stored in the block layout of the tensor-core decode (d = 128, fp16 /
    bf16 rows on 16-byte strides, groups of 32 / 64 / 128 channels)."""
    return (x.shape[-1] == 128 and x.dtype in (torch.float16, torch.bfloat16) and group in (32, 64, 128)
            and x.stride(-1) == 1 and all(s % 8 == 0 for s in x.stride()[:3]))


def build_mixed(K: torch.Tensor, V: torch.Tensor, group: int = 64, tenths=(1, 3), tc: bool = False):
    """tc: store values in the block layout read by the tcgen05 decode (decode_tc; exact to the same
    tolerance, currently slower than the mma.sync decode on these shapes); the default keeps the
    token-major layout of the mma.sync decode (decode_main).  None: the block layout whenever the
    shapes allow it."""
    B, H, T, d = K.shape
    n8, n4, _ = strata_counts(T, *tenths)
    imp = ops.key_energy(K)
    i8, i4, i2 = ops.rank_split(imp, [n8, n4])
    cache = ops.PackedCache(B, H, d, k_group=group, v_group=group)
    blocked = tc_layout_ok(V, group) if tc is None else tc
    sets = {}
    for bits, idx in ((8, i8), (4, i4), (2, i2)):
        if idx is None:
            continue
        vq = ops.quant_pack(V, bits, group, idx=idx, blocked=blocked)
        kq = ops.quant_pack(K, bits, group, idx=idx, n_alloc=vq["n_alloc"])
        cache.add_stratum(kq, vq)
        sets[bits] = idx
    return cache, sets


def build_kivi(K: torch.Tensor, V: torch.Tensor, kbits: int, vbits: int, kgroup: int, vgroup: int,
               n_sink: int = 0):
    """Keys per channel over `kgroup` tokens, values per token over `vgroup` channels; rows before
    n_sink become exact rows of the cache."""
    B, H, T, d = K.shape
    n = T - n_sink
    kq = ops.quant_pack(K, kbits, kgroup, per_channel=True, first_row=n_sink, n=n)
    vq = ops.quant_pack(V, vbits, vgroup, first_row=n_sink, n=n, n_alloc=kq["n_alloc"])
    cache = ops.PackedCache(B, H, d, per_channel=True, k_group=kgroup, v_group=vgroup)
    cache.add_stratum(kq, vq)
    if n_sink:
        cache.set_exact(K[:, :, :n_sink], V[:, :, :n_sink])
    return cache


def build_spectral(K: torch.Tensor, V: torch.Tensor, basis: torch.Tensor, bits: int = 4, r: int = 32):
    """Config 3: per KV head an orthonormal (d, d) basis; keys and values are stored as their leading
    r coefficients, coded per token with the mid-rise code (tcgen05 projection + code epilogue);
    decode runs in the coefficient domain (query mapped by B_r, output lifted by B_r^T).
    basis: (H, d, d) float.  Returns the PackedCache."""
    B, H, T, d = K.shape
    br = basis[:, :, :r].to(device=K.device, dtype=torch.float32).contiguous()          # (H, d, r)
    hilo = ops.split_basis(br)
    kq = ops.spectral_encode(K.to(torch.float16), hilo, bits)
    vq = ops.spectral_encode(V.to(torch.float16), hilo, bits)
    cache = ops.PackedCache(B, H, d, d_code=r, midrise=True)
    cache.add_stratum(kq, vq)
    cache.qmap = br
    cache.lift = br.transpose(1, 2).contiguous()
    return cache


def build_eviction(q_obs: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scaling: float, budget: int,
                   window: int, bits: int = 4, group: int = 64, pool: int = 0):
    """Heavy hitters by accumulated decode-query attention over [0, T - window), plus the window;
    kept tokens (position order) stored with KIVI codes: keys per channel over `group` kept tokens,
    values per token over `group` channels.  Returns (cache, kept idx (B, H, budget + window))."""
    B, H, T, d = K.shape
    n_cand = T - window
    sc = ops.query_scores(q_obs, K, scaling, n_cand, pool)
    top = ops.rank_split(sc, [min(budget, n_cand)], want=[0])[0]
    win = torch.arange(n_cand, T, device=K.device, dtype=torch.int64).expand(B, H, window)
    kept = torch.cat([top, win], -1).contiguous()
    kq = ops.quant_pack(K, bits, group, per_channel=True, idx=kept)
    vq = ops.quant_pack(V, bits, group, idx=kept, n_alloc=kq["n_alloc"])
    cache = ops.PackedCache(B, H, d, per_channel=True, k_group=group, v_group=group)
    cache.add_stratum(kq, vq)
    return cache, kept, sc
