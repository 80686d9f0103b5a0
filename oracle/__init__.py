"""CPU oracle for the packed-KV decode path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the reference algorithms of TahirSher/KV-Project that the
CUDA path replaces: the KIVI group quantiser, the STRATA per-token code, planar / MSB-first
bit packing, SnapKV-style score accumulation with budgeted top-k, the dequantise-then-attend
attention used as the numerical reference, STRATA's compressed-domain decode, and the
spectral (basis-projection) code.  Every function cites the reference file:line it follows.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import this package, and only as the checker or as the timed CPU
baseline.  The product path (``kvb``) never calls into it; it fails loudly when its CUDA
library is missing instead of falling back here.

Parity pinning: ``tests/golden/make_golden.py`` runs the reference functions themselves on
seeded inputs and stores their outputs as fixtures; ``tests/test_oracle_golden.py`` checks
every function here against those fixtures.
"""

from .codecs import (FP16_MAX, as_stored, kivi_quant, kivi_dequant, uniform_step, strata_quantize,
                     absmax_quant, pack_planar, unpack_planar, pack_codes, pack_rows)
from .attention import chunked_attention, strata_attend, tier_reference, lse_merge
from .select import snapkv_scores, query_scores, topk_kept, l2_importance, mixed_strata, strata_counts
from .spectral import seeded_qr_basis, rotation_matrix, spectral_encode, spectral_attend
from .alloc import head_sync_allocate

__all__ = [
    "FP16_MAX", "as_stored", "kivi_quant", "kivi_dequant", "uniform_step", "strata_quantize",
    "absmax_quant", "pack_planar", "unpack_planar", "pack_codes", "pack_rows",
    "chunked_attention", "strata_attend", "tier_reference", "lse_merge",
    "snapkv_scores", "query_scores", "topk_kept", "l2_importance", "mixed_strata", "strata_counts",
    "seeded_qr_basis", "rotation_matrix", "spectral_encode", "spectral_attend",
    "head_sync_allocate",
]
