"""kvb - B200-native (sm_100a) packed-KV decode path.

Drop-in native replacement for the decode-time hot path shared by the KV-cache compression
methods of TahirSher/KV-Project: quantise + pack (K1), importance scores + budgeted eviction /
strata assignment (K2), fused split-K flash decoding over packed codes (K3), the spectral code
(K4) and per-vector row codes (K5: absmax tails, HEDGE, TILT chunk selection, MSB-first packing).  All compute runs in ``libkvb.so`` (hand-written CUDA for sm_100a behind the C ABI of
``include/kvb.h``); this package only moves tensors and builds descriptors.
"""

from . import _lib, ops, cache, workloads, state, seqsplit, codebooks, coverage, lctc   # noqa: F401
from .ops import (PackedCache, quant_pack, key_energy, rank_split, query_scores, snapkv_scores, decode, decode_plan,  # noqa: F401
                  device_status, overlap_previous, UNIFORM_STEP)
from .state import KvbStrataState, KvbCodedState, tier_as_kvb  # noqa: F401
from .coverage import coverage_groups, coverage_stats  # noqa: F401

__all__ = ["ops", "cache", "workloads", "state", "seqsplit", "codebooks", "PackedCache", "quant_pack", "key_energy", "rank_split",
           "query_scores", "snapkv_scores", "decode", "decode_plan", "device_status", "overlap_previous", "UNIFORM_STEP",
           "KvbStrataState", "KvbCodedState", "tier_as_kvb", "coverage", "coverage_groups", "coverage_stats", "lctc"]
