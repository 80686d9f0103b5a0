"""CPU-only checks of the C ABI: the library loads, exports every function include/kvb.h declares,
and the host-side split-K planner covers every chunk exactly once with balanced work."""

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def header_functions():
    text = (ROOT / "include" / "kvb.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kvb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from kvb import _lib
    lib = _lib.lib()
    declared = header_functions()
    assert declared, "no functions parsed from kvb.h"
    for name in declared:
        assert hasattr(lib, name), f"libkvb.so does not export {name}"
    assert set(declared) == set(_lib.exported_symbols())
    assert lib.kvb_version() >= 100


def test_uniform_steps_match_oracle():
    import oracle
    from kvb.ops import UNIFORM_STEP
    for b, v in UNIFORM_STEP.items():
        assert v == oracle.uniform_step(b)[0]


def _fake_cache(B, H, counts, bits=((8, 8), (4, 4), (2, 2)), d=128):
    from kvb import _lib
    c = _lib.Cache()
    c.B, c.Hkv, c.d, c.d_code = B, H, d, d
    c.code_kind, c.k_mode, c.k_group, c.v_group = 0, 0, 64, 64
    c.n_strata = len(counts)
    for i, n in enumerate(counts):
        c.strata[i].kbits, c.strata[i].vbits = bits[i]
        c.strata[i].n = n
        c.strata[i].n_alloc = (n + 15) // 16 * 16
    return c


def _plan(c, n_ctas):
    from kvb import _lib
    lib = _lib.lib()
    need = lib.kvb_decode_plan(C.byref(c), n_ctas, None, 0)
    buf = (C.c_int32 * need)()
    assert lib.kvb_decode_plan(C.byref(c), n_ctas, buf, need) == need
    v = np.array(list(buf))
    nc, npc, nh = v[:3]
    o = 3
    cta_begin = v[o:o + nc + 1]
    o += nc + 1
    rows = v[o:o + 5 * npc].reshape(npc, 5)
    head_begin = v[o + 5 * npc:o + 5 * npc + nh + 1]
    return cta_begin, rows[:, :4], rows[:, 4], head_begin


TOK = {(8, 8): 192, (4, 4): 384, (2, 2): 768, (4, 2): 384}


@pytest.mark.parametrize("B,H,T,n_ctas", [(8, 8, 32768, 148), (1, 8, 4096, 148), (2, 2, 300, 148), (8, 8, 32768, 7)])
def test_plan_covers_every_chunk_once(B, H, T, n_ctas):
    n8, n4 = T // 10, 3 * T // 10
    counts = [n8, n4, T - n8 - n4]
    c = _fake_cache(B, H, counts)
    cta_begin, pieces, slots, head_begin = _plan(c, n_ctas)
    assert cta_begin[0] == 0 and cta_begin[-1] == len(pieces)
    assert np.all(np.diff(cta_begin) >= 0)
    # every (head, stratum) chunk exactly once, in order (head by head, strata in order)
    bits = [(8, 8), (4, 4), (2, 2)]
    expect = [(h, s, k) for h in range(B * H) for s in range(3) for k in range(-(-counts[s] // TOK[bits[s]]))]
    got = [(h, s, k) for h, s, lo, hi in pieces for k in range(lo, hi)]
    assert got == expect
    # partial slots: a permutation, head-major, and head_begin indexes each head's slots
    assert sorted(slots) == list(range(len(pieces)))
    by_slot = pieces[np.argsort(slots)]
    for h in range(B * H):
        ps = by_slot[head_begin[h]:head_begin[h + 1]]
        assert len(ps) and np.all(ps[:, 0] == h)
        assert [tuple(x) for x in ps[:, 1:3]] == sorted(tuple(x) for x in ps[:, 1:3])
    # balance: no CTA gets more than (average + one chunk + one segment's fixed costs) of work: code
    # bytes + 60 per token, plus 98304 byte-equivalents per (head, stratum) segment start (its
    # end-of-piece merge) and 131072 per head start (query prep and the previous head's merge),
    # charged to the CTA holding the start, both doubled below 8 chunks per CTA
    bpt = {s: 128 * (bits[s][0] + bits[s][1]) // 8 + 60 for s in range(3)}
    n_chunks = B * H * sum(-(-counts[s] // TOK[bits[s]]) for s in range(3))
    fx = 2 if n_chunks < 8 * n_ctas else 1
    seg, head = 98304 * fx, 131072 * fx
    w = np.zeros(n_ctas)
    for cta in range(n_ctas):
        for h, s, lo, hi in pieces[cta_begin[cta]:cta_begin[cta + 1]]:
            tok = TOK[bits[s]]
            if lo == 0:
                w[cta] += seg + (head if s == 0 else 0)
            for k in range(lo, hi):
                w[cta] += min(tok, counts[s] - k * tok) * bpt[s]
    max_chunk = max(TOK[bits[s]] * bpt[s] for s in range(3))
    assert w.max() <= w.sum() / n_ctas + max_chunk + seg + head + 1


def test_decode_rejects_bad_requests():
    """Argument checks run on the host before any CUDA call."""
    from kvb import _lib
    lib = _lib.lib()
    c = _fake_cache(1, 8, [100], bits=((2, 2),), d=32)    # d_code * 2 < 128: unsupported
    c.k_group = c.v_group = 32
    st = lib.kvb_decode(C.byref(c), C.c_void_p(16), 2, 32, 1, C.c_float(0.1), None, C.c_void_p(16), 2, 148,
                        C.c_void_p(256), 1 << 20, None)
    assert st == _lib.KVB_EUNSUPPORTED
    assert b"bits" in lib.kvb_last_error()
    c = _fake_cache(1, 8, [100])
    st = lib.kvb_decode(C.byref(c), C.c_void_p(16), 2, 30, 1, C.c_float(0.1), None, C.c_void_p(16), 2, 148,
                        C.c_void_p(256), 1 << 20, None)
    assert st == _lib.KVB_EINVAL                                       # Hq % Hkv != 0
    st = lib.kvb_rank_split(None, 0, 1, 1, 1, 2, None, None, None, None)
    assert st == _lib.KVB_EINVAL
