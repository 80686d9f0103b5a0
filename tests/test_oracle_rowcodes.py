"""The row-code oracle (absmax variants, HEDGE, TILT chunk selection, byte-LUT decode) against
fixtures made by the reference's own functions (``rowcodes.npz``; CPU only).

Bit-exact for codes, packed bytes, indices, fp16 scales and the HEDGE rotation and read-back (the
oracle takes the reference's float32 CPU reduction orders); TILT's float64 share within tolerance.
"""

import numpy as np
import pytest

import oracle as O
from oracle import rowcodes as RC


@pytest.mark.parametrize("b", [2, 3, 4, 5, 8])
def test_absmax_strata(golden, b):
    g = golden("rowcodes")
    c, s = O.absmax_quant(g["am_x"], b)
    np.testing.assert_array_equal(s, g[f"am{b}_s"])
    np.testing.assert_array_equal(c, g[f"am{b}_codes"])
    np.testing.assert_array_equal(RC.absmax_packed(c, b), g[f"am{b}_packed"])
    np.testing.assert_array_equal(RC.unpack_rows(g[f"am{b}_packed"].reshape(40, -1), b, 128) - (2 ** (b - 1) - 1),
                                  c.astype(np.int64))


@pytest.mark.parametrize("b", [2, 3, 4, 5, 8])
def test_absmax_tilt(golden, b):
    g = golden("rowcodes")
    c, s = RC.absmax_tilt(g["am_x"], b)
    np.testing.assert_array_equal(c * s, g[f"tilt{b}_xhat"])


@pytest.mark.parametrize("b", [1, 2, 3, 4])
def test_lloyd_max(golden, b):
    g = golden("rowcodes")
    np.testing.assert_array_equal(RC.lloyd_max_gaussian(b), g[f"lm{b}"])


def test_hedge_rotation(golden):
    g = golden("rowcodes")
    np.testing.assert_allclose(O.rotation_matrix(128, "layer0"), g["hedge_R"], rtol=0, atol=1e-7)


@pytest.mark.parametrize("b", [1, 2, 3, 4, 8])
def test_hedge_codes_given_y(golden, b):
    """Codes, scales and level * scale from the reference's own y, bit for bit."""
    g = golden("rowcodes")
    c, s, _ = RC.hedge_codes_from_y(g["hedge_y"], b)
    np.testing.assert_array_equal(s, g[f"hedge{b}_s"])
    np.testing.assert_array_equal(c, g[f"hedge{b}_codes"])


@pytest.mark.parametrize("b", [1, 2, 3, 4, 8])
def test_hedge_centered_code(golden, b):
    """End to end from x and mu: rotation, codes, scales and the read-back, bit for bit."""
    g = golden("rowcodes")
    xh, c, s, y = RC.hedge_quant(g["hedge_x"], g["hedge_R"], b, mu=g["hedge_mu"])
    np.testing.assert_array_equal(y, g["hedge_y"])
    np.testing.assert_array_equal(c, g[f"hedge{b}_codes"])
    np.testing.assert_array_equal(s, g[f"hedge{b}_s"])
    np.testing.assert_array_equal(xh, g[f"hedge{b}_xhat"])
    # 16 bits keeps the vector bit for bit
    assert RC.hedge_quant(g["hedge_x"], g["hedge_R"], 16, mu=g["hedge_mu"])[0] is not None


def test_tilt_chunk_selection(golden):
    g = golden("rowcodes")
    share = RC.chunk_share(g["tilt_k"], g["tilt_q"])
    np.testing.assert_allclose(share, g["tilt_share"], rtol=2e-5, atol=1e-8)
    m = int(g["tilt_m"])
    idx = RC.chunk_topm(g["tilt_share"], m)
    np.testing.assert_array_equal(idx, g["tilt_idx"])
    np.testing.assert_array_equal(RC.chunk_topm(share, m), g["tilt_idx"])
    gk = np.take_along_axis(g["tilt_k"], idx[..., None], 2)
    gv = np.take_along_axis(g["tilt_v"], idx[..., None], 2)
    for x, ref in ((gk, g["tilt_kq"]), (gv, g["tilt_vq"])):
        c, s = RC.absmax_tilt(x, 8)
        np.testing.assert_array_equal(c * s, ref)


@pytest.mark.parametrize("t", [0, 1, 2])
def test_byte_lut_decode(golden, t):
    g = golden("rowcodes")
    bits = (2, 2, 4)[t]
    np.testing.assert_array_equal(RC.byte_lut(g[f"emb_levels{t}"], bits), g[f"emb_lut{t}"])
    np.testing.assert_array_equal(O.pack_rows(g[f"emb_codes{t}"], bits), g[f"emb_rows{t}"])
    np.testing.assert_array_equal(RC.unpack_rows(g[f"emb_rows{t}"], bits, 32), g[f"emb_codes{t}"])
    acc = None
    for s in range(t + 1):
        acc = RC.decode_rows_lut(g[f"emb_rows{s}"], (2, 2, 4)[s], g[f"emb_levels{s}"], acc)
    np.testing.assert_array_equal(acc, g[f"emb_cum{t}"])
