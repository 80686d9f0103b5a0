"""The numpy oracle against fixtures produced by the reference's own functions (CPU only).

Bit-exact where the reference computes integers, bytes, indices or fp16-rounded scales (the STRATA
RMS included: the oracle restates torch's CPU float32 summation order); float32 outputs within a
few ulps.
"""

import numpy as np
import pytest

import oracle as O


def test_as_stored(golden):
    g = golden("codecs")
    np.testing.assert_array_equal(O.as_stored(g["as_stored_in"]), g["as_stored_out"])


@pytest.mark.parametrize("i", range(8))
def test_kivi_quant_bit_exact(golden, i):
    g = golden("codecs")
    B, H, T, d, bits, group, along, sink, _ = g[f"kivi{i}_case"].tolist()
    r = O.kivi_quant(g[f"kivi{i}_x"], bits, group, bool(along), sink)
    np.testing.assert_array_equal(r["codes"], g[f"kivi{i}_codes"])
    np.testing.assert_array_equal(r["lo"], g[f"kivi{i}_lo"])
    np.testing.assert_array_equal(r["scale"], g[f"kivi{i}_scale"])
    np.testing.assert_array_equal(r["xhat"], g[f"kivi{i}_xhat"])
    # the reader's dequantisation from codes + lo / scale reproduces xhat exactly
    deq = O.kivi_dequant(r["codes"], r["lo"], r["scale"], group, bool(along))
    np.testing.assert_array_equal(deq, g[f"kivi{i}_xhat"][:, :, sink:])


@pytest.mark.parametrize("b", [2, 3, 4, 8])
def test_uniform_step(golden, b):
    g = golden("codecs")
    assert O.uniform_step(b) == tuple(g[f"uniform_step_{b}"].tolist())


@pytest.mark.parametrize("b", [2, 4, 8])
def test_strata_quantize(golden, b):
    g = golden("codecs")
    c, s, yh = O.strata_quantize(g["sq_x"], b)
    # the RMS follows torch's CPU float32 summation order, so scales are bit-exact too
    np.testing.assert_array_equal(s, g[f"sq{b}_s"])
    np.testing.assert_array_equal(c, g[f"sq{b}_codes"])
    np.testing.assert_array_equal(yh, g[f"sq{b}_yhat"])
    np.testing.assert_array_equal(O.pack_planar(g[f"sq{b}_codes"], b), g[f"planar{b}"])
    np.testing.assert_array_equal(O.unpack_planar(g[f"planar{b}"], b), g[f"sq{b}_codes"].astype(np.int32))
    np.testing.assert_array_equal(O.pack_codes(g[f"sq{b}_codes"], b), g[f"codes_msb{b}"])


@pytest.mark.parametrize("b", [4, 8])
def test_absmax(golden, b):
    g = golden("codecs")
    c, s = O.absmax_quant(g["absmax_x"], b)
    np.testing.assert_array_equal(s, g[f"absmax{b}_s"])
    np.testing.assert_array_equal(c, g[f"absmax{b}_codes"])


def test_pack_rows(golden):
    g = golden("codecs")
    np.testing.assert_array_equal(O.pack_rows(g["rows2_in"], 2), g["rows2_out"])
    np.testing.assert_array_equal(O.pack_rows(g["rows4_in"], 4), g["rows4_out"])


def test_rotation_matrix(golden):
    g = golden("codecs")
    np.testing.assert_array_equal(O.rotation_matrix(32, "strata"), g["rot32_strata"])
    np.testing.assert_allclose(O.rotation_matrix(24, "t"), g["rot24_t"], rtol=0, atol=1e-6)


def test_snapkv_scores_and_topk(golden):
    g = golden("select")
    H, w, kern = int(g["H"]), int(g["window"]), int(g["kernel"])
    sc = O.snapkv_scores(g["q"], g["k"], H, g["q"].shape[-1] ** -0.5, w, kern)
    np.testing.assert_allclose(sc, g["scores"], rtol=2e-6, atol=1e-9)
    # identical score tensor -> identical kept set (reference scores as input)
    kept = O.topk_kept(g["scores"][..., :H - w], 20)
    np.testing.assert_array_equal(kept, g["top20"])
    # end to end from the oracle's own scores (no near-ties at the boundary in this case)
    np.testing.assert_array_equal(O.topk_kept(sc[..., :H - w], 20), g["top20"])


def test_snapkv_quant_entries(golden):
    """Selection + gather + KIVI of the kept tokens == SnapKVQuantMethod.entries (STRATA_KV.py:1010)."""
    g = golden("select")
    H, w = int(g["H"]), int(g["window"])
    n_q = int(g["mtlp_n_q"])
    sc = O.snapkv_scores(g["q"], g["k"], H, g["q"].shape[-1] ** -0.5, w, int(g["kernel"]))[..., :H - w]
    idx = O.topk_kept(sc, n_q)
    B, Hkv, _, d = g["k"].shape
    gk = np.take_along_axis(g["k"], idx[..., None].repeat(d, -1), 2)
    gv = np.take_along_axis(g["mtlp_v"], idx[..., None].repeat(d, -1), 2)
    kq = O.kivi_quant(gk, 4, 32, True, 0)
    vq = O.kivi_quant(gv, 4, 32, False, 0)
    for side, r in (("k", kq), ("v", vq)):
        np.testing.assert_array_equal(r["codes"], g[f"mtlp_{side}_codes"])
        np.testing.assert_array_equal(r["lo"], g[f"mtlp_{side}_lo"])
        np.testing.assert_array_equal(r["scale"], g[f"mtlp_{side}_scale"])


def test_chunked_attention(golden):
    g = golden("attention")
    tok = {"k": g["tk"], "v": g["tv"], "b": g["tb"], "tau": g["ttau"]}
    d = g["q"].shape[-1]
    o = O.chunked_attention(g["q"], d ** -0.5, g["qpos"], g["K"], g["V"], np.arange(g["K"].shape[2]),
                            g["hide"], tok, 2)
    np.testing.assert_allclose(o, g["out"], rtol=0, atol=2e-6)


def test_strata_decode(golden):
    g = golden("strata")
    tiers = [{"bits": int(g[f"t{i}_bits"]), "kc": g[f"t{i}_kc"], "vc": g[f"t{i}_vc"], "ks": g[f"t{i}_ks"],
              "vs": g[f"t{i}_vs"]} for i in range(int(g["n_tiers"]))]
    d = g["q"].shape[-1]
    for i, t in enumerate(tiers):
        m, l, acc = O.tier_reference(g["qr"], g["qb"], t["bits"], t["kc"], t["vc"], t["ks"], t["vs"])
        np.testing.assert_allclose(m, g[f"t{i}_m"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(l, g[f"t{i}_l"], rtol=1e-5)
        np.testing.assert_allclose(acc, g[f"t{i}_acc"], rtol=1e-5, atol=1e-5)
    H = int(g["H"])
    o = O.strata_attend(g["q"], d ** -0.5, np.array([H]), g["Ke"], g["Ve"], int(g["n0"]), H, tiers,
                        g["mu_k"], g["mu_v"], g["R"])
    np.testing.assert_allclose(o, g["out_native"], rtol=0, atol=2e-6)
    # the reference's decode identity: compressed-domain == harness reconstruction (<= 1e-4)
    assert np.abs(o - g["out_harness"]).max() <= 1e-4 * max(1.0, np.abs(g["out_harness"]).max())


def test_l2_importance_exact_order_free():
    rng = np.random.default_rng(0)
    import torch
    k = torch.tensor(rng.standard_normal((2, 3, 50, 128)), dtype=torch.bfloat16).float().numpy()
    a = O.l2_importance(k)
    b = O.l2_importance(k[..., ::-1])
    np.testing.assert_array_equal(a, b)


def test_mixed_strata_counts_and_ties():
    imp = np.zeros((1, 1, 20))
    imp[0, 0, [3, 7, 11]] = 5.0
    s = O.mixed_strata(imp)
    n8, n4, n2 = O.strata_counts(20)
    assert (n8, n4, n2) == (2, 6, 12)
    np.testing.assert_array_equal(s[8][0, 0], [3, 7])            # tie at 5.0: lower indices first
    np.testing.assert_array_equal(s[4][0, 0], [0, 1, 2, 4, 5, 11])
    assert O.strata_counts(32768) == (3276, 9830, 19662)


@pytest.mark.parametrize("case", ["a", "b"])
def test_snapkv128_scores_and_topk(golden, case):
    """SnapKV at d = 128 (the GPU kernel's head size): the oracle against the reference's
    snapkv_scores (causal observation window, STRATA_KV.py:932-954) and its top-40 set."""
    g = golden("snapkv128")
    B, Hkv, rep, H, w, kern = (int(x) for x in g[f"{case}_cfg"])
    qw = g[f"{case}_qw"]
    q = np.zeros((B, Hkv * rep, H, qw.shape[-1]), np.float32)
    q[:, :, H - w:] = qw                                   # the reference reads only the window positions
    sc = O.snapkv_scores(q, g[f"{case}_k"], H, qw.shape[-1] ** -0.5, w, kern)
    np.testing.assert_allclose(sc, g[f"{case}_scores"], rtol=2e-6, atol=1e-9)
    np.testing.assert_array_equal(O.topk_kept(g[f"{case}_scores"][..., :H - w], 40), g[f"{case}_top40"])
