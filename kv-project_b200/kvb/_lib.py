"""ctypes binding of libkvb.so (the C ABI declared in include/kvb.h).

The library is loaded lazily on first use.  There is no fallback: if ``libkvb.so`` is missing or
fails to load, every entry point raises, so a GPU run can never silently take another path.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libkvb.so"

KVB_OK, KVB_EINVAL, KVB_ECUDA, KVB_ETIMEDOUT, KVB_EUNSUPPORTED = 0, 1, 2, 3, 4
KVB_F32, KVB_F16, KVB_BF16, KVB_F64 = 0, 1, 2, 3
KVB_CODE_ASYM, KVB_CODE_MIDRISE = 0, 1
KVB_K_PER_TOKEN, KVB_K_PER_CHANNEL = 0, 1
KVB_ABSMAX_STRATA, KVB_ABSMAX_TILT = 0, 1

# every entry point of include/kvb.h, with its ctypes signature (restype, argtypes)
_i64, _i32, _p, _f32 = C.c_int64, C.c_int, C.c_void_p, C.c_float


KVB_V_TOKEN_MAJOR, KVB_V_BLOCK128 = 0, 1


class Stratum(C.Structure):
    _fields_ = [("kbits", C.c_int), ("vbits", C.c_int), ("v_layout", C.c_int), ("reserved", C.c_int),
                ("n", C.c_int64), ("n_alloc", C.c_int64),
                ("kc", C.c_void_p), ("vc", C.c_void_p), ("kmeta", C.c_void_p), ("vmeta", C.c_void_p)]


class Cache(C.Structure):
    _fields_ = [("B", C.c_int), ("Hkv", C.c_int), ("d", C.c_int), ("d_code", C.c_int),
                ("code_kind", C.c_int), ("k_mode", C.c_int), ("k_group", C.c_int), ("v_group", C.c_int),
                ("n_strata", C.c_int), ("strata", Stratum * 4),
                ("k_exact", C.c_void_p), ("v_exact", C.c_void_p), ("exact_dtype", C.c_int),
                ("exact_cap", C.c_int64), ("n_exact", C.c_int64), ("n0", C.c_int64), ("pos0", C.c_int64),
                ("qmap", C.c_void_p), ("lift", C.c_void_p), ("mu_k", C.c_void_p), ("mu_v", C.c_void_p)]


class Atoms(C.Structure):
    """kvb_atoms of include/kvb.h: TILT moment atoms (device float32 pointers) and their flags."""
    _fields_ = [(n, C.c_void_p) for n in ("mu_k", "logn", "U", "lam", "diag", "R", "A", "Bk", "Rv")] + \
               [(n, C.c_int) for n in ("B", "Hkv", "NA", "d", "r", "order", "tilt", "project", "phase")]


class Coverage(C.Structure):
    """kvb_coverage of include/kvb.h: one layer's queries, keys, values and output metrics for STRATA's
    coverage statistics."""
    _fields_ = [("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("dtype", C.c_int),
                ("q_head_stride", C.c_int64), ("q_pos_stride", C.c_int64), ("kv_head_stride", C.c_int64),
                ("kv_pos_stride", C.c_int64), ("M", C.c_void_p), ("Hq", C.c_int), ("Hkv", C.c_int), ("d", C.c_int),
                ("H", C.c_int64), ("rs", C.c_int64), ("re", C.c_int64), ("scaling", C.c_float), ("floor", C.c_float),
                ("local", C.c_int), ("score_cap", C.c_int64)]


SIGNATURES = {
    "kvb_last_error": (C.c_char_p, []),
    "kvb_version": (C.c_int, []),
    "kvb_device_status": (_i32, [C.POINTER(C.c_uint), _i32, _p]),
    "kvb_device_diag": (_i32, [C.POINTER(C.c_uint), _i32, _p]),
    "kvb_set_decode_flags": (C.c_uint, [C.c_uint]),
    "kvb_quant_pack": (_i32, [_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64,
                              _i32, _i32, _i32, _i32, _f32, _p, _p, _p, _p]),
    "kvb_quant_pack_blocked": (_i32, [_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64,
                                      _i32, _i32, _i32, _f32, _p, _p, _p, _p]),
    "kvb_rank_split": (_i32, [_p, _i32, _i64, _i64, _i64, _i32, C.POINTER(C.c_int64), C.POINTER(C.c_void_p),
                              C.POINTER(C.c_int64), _p]),
    "kvb_key_energy": (_i32, [_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p]),
    "kvb_scores_workspace_size": (C.c_size_t, [_i64, _i64, _i64]),
    "kvb_query_scores": (_i32, [_p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _i64, _i32, _p, _p,
                                C.c_size_t, _p]),
    "kvb_snapkv_scores": (_i32, [_p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _p, _p, C.c_size_t,
                                 _p]),
    "kvb_spectral_encode": (_i32, [_p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i32, _f32, _p, _p, _i64, _p, _i32,
                                   _p]),
    "kvb_absmax_quant": (_i32, [_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i32, _i32,
                                _p, _p, _p, _p]),
    "kvb_pack_rows": (_i32, [_p, _i64, _i64, _i32, _p, _p]),
    "kvb_decode_rows_lut": (_i32, [_p, _i64, _i64, _i32, _p, _p, _i32, _p, _p]),
    "kvb_hedge_quant": (_i32, [_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p, _p, _i32, _p,
                               _p, _p, _p, _p, _p]),
    "kvb_chunk_select": (_i32, [_p, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p, _p, _p]),
    "kvb_xchg_bytes": (C.c_size_t, [_i64, _i32, _i32]),
    "kvb_xchg_alloc": (_i32, [C.c_size_t, C.POINTER(C.c_void_p), _p]),
    "kvb_xchg_open": (_i32, [_p, C.POINTER(C.c_void_p)]),
    "kvb_xchg_close": (_i32, [_p]),
    "kvb_xchg_free": (_i32, [_p]),
    "kvb_xchg_zero": (_i32, [_p, C.c_size_t, _p]),
    "kvb_xchg_merge": (_i32, [_p, _p, _i64, _i32, _i32, _i32, C.POINTER(C.c_void_p), _p, _i32, C.c_uint64, _p]),
    "kvb_decode_workspace_size": (C.c_size_t, [C.POINTER(Cache), _i32, _i32, _i32]),
    "kvb_head_sync_allocate_workspace": (C.c_size_t, []),
    "kvb_atom_read": (_i32, [C.POINTER(Atoms), _p, _i32, _i32, _p, _p, _p, _p]),
    "kvb_coverage_workspace_size": (C.c_size_t, [C.POINTER(Coverage), _p, _p, _i32]),
    "kvb_coverage_stats": (_i32, [C.POINTER(Coverage), _p, _p, _i32, _p, _p, _p, _p, _p, _p, C.c_size_t, _p]),
    "kvb_uq_codes": (_i32, [_p, _i64, _i64, _i64, _p, _p, _p, _p, _p]),
    "kvb_uq_values": (_i32, [_p, _i64, _i64, _i64, _p, _p, _p, _p]),
    "kvb_operational_rd_workspace": (C.c_size_t, [_i64, _i32, _i32]),
    "kvb_operational_rd": (_i32, [_p, _i64, _i64, _i64, _p, _i32, _p, _i32, _p, _p, _p, C.c_size_t, _p]),
    "kvb_quasar_scores": (_i32, [_p, _i32, _i32, _i32, _p, C.c_size_t, _p, _i32, _p, _i32, _i64, _p, _p]),
    "kvb_quasar_values_workspace": (C.c_size_t, [_i32, _i32, _i64, _i32]),
    "kvb_quasar_values": (_i32, [_p, _i32, _i32, _i64, _p, C.c_size_t, _p, _i32, _p, _i32, _i32, _p, _p, C.c_size_t, _p]),
    "kvb_head_sync_allocate": (_i32, [_p, _i64, _i32, C.POINTER(C.c_float), C.POINTER(C.c_float), C.c_double, _i32,
                                      _i32, _p, _p, _p, _p, C.c_size_t, _p]),
    "kvb_decode_xchg_bytes": (C.c_size_t, [C.POINTER(Cache), _i32, _i32, _i32]),
    "kvb_decode_xchg": (_i32, [C.POINTER(Cache), _p, _i32, _i32, _i32, _f32, C.POINTER(C.c_int64), _p, _i32, _i32,
                               _i32, C.POINTER(C.c_void_p), C.c_uint64, _i32, _p, C.c_size_t, _p]),
    "kvb_decode": (_i32, [C.POINTER(Cache), _p, _i32, _i32, _i32, _f32, C.POINTER(C.c_int64), _p, _i32, _i32,
                          _p, C.c_size_t, _p]),
    "kvb_decode_events": (_i32, [C.POINTER(Cache), _p, _i32, _i32, _i32, _f32, C.POINTER(C.c_int64), _p, _i32,
                                 _i32, _p, C.c_size_t, _p, _p, _p]),
    "kvb_decode_lse": (_i32, [C.POINTER(Cache), _p, _i32, _i32, _i32, _f32, C.POINTER(C.c_int64), _p, _i32, _p,
                              _i32, _p, C.c_size_t, _p]),
    "kvb_lse_merge": (_i32, [_p, _i64, _p, _i64, _i32, _i64, _i32, _p, _i32, _p]),
    "kvb_decode_plan": (C.c_int64, [C.POINTER(Cache), _i32, C.POINTER(C.c_int32), C.c_int64]),
    "kvb_decode_noalloc": (_i32, [C.POINTER(Cache), _p, _i32, _i32, _i32, _f32, C.POINTER(C.c_int64), _p, _i32,
                                  _i32, _p]),
}

_lib = None


def lib() -> C.CDLL:
    """The loaded library (raises if it is missing: there is no fallback path)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"kvb: {LIB_PATH} is missing; build it with __graft_entry__.build() "
                               "or `python -m kvb.build` (no CPU fallback exists)")
        h = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def exported_symbols():
    return list(SIGNATURES)


def check(status: int, what: str = "kvb"):
    if status != KVB_OK:
        msg = lib().kvb_last_error().decode(errors="replace")
        kind = {KVB_EINVAL: ValueError, KVB_EUNSUPPORTED: NotImplementedError}.get(status, RuntimeError)
        raise kind(f"{what}: {msg} (status {status})")
