"""K3 fused split-K decode on the GPU vs the oracle's float32 dequantise-then-attend result
(chunked_attention, STRATA_KV.py:641) and STRATA's compressed-domain decode (StrataState.attend,
STRATA_KV.py:1762).  Tolerance: max-abs 2e-3 on the attention output (fp32 output)."""

import numpy as np
import pytest
import torch

import oracle as O
from kvref import np32, gather_rows, scatter_rows, attend_reference

pytestmark = pytest.mark.gpu
TOL = 2e-3


def mixed_reference(K, V, sets, group=64):
    """Oracle reconstruction of the mixed cache: per stratum KIVI per-token codes of the gathered
    rows, scattered back to their positions."""
    Kf, Vf = np32(K), np32(V)
    Kh, Vh = np.zeros_like(Kf), np.zeros_like(Vf)
    for b, idx in sets.items():
        scatter_rows(Kh, idx, O.kivi_quant(gather_rows(Kf, idx), b, group, False, 0)["xhat"])
        scatter_rows(Vh, idx, O.kivi_quant(gather_rows(Vf, idx), b, group, False, 0)["xhat"])
    return Kh, Vh


@pytest.mark.parametrize("tc", [True, False])
@pytest.mark.parametrize("B,Hkv,rep,T,Tq", [(2, 2, 4, 1000, 1), (1, 2, 4, 5000, 2), (2, 1, 8, 777, 1),
                                             (1, 8, 4, 20000, 1)])
def test_mixed_strata_decode(cuda_dev, B, Hkv, rep, T, Tq, tc):
    """tc: values in the block layout (tcgen05 decode, decode_tc) or token-major (mma.sync decode)."""
    import kvb
    K, V = kvb.workloads.lognormal_kv(B, Hkv, T, 128, torch.bfloat16, seed=T)
    q = kvb.workloads.queries(B, Hkv * rep, Tq, 128, torch.bfloat16, seed=T)
    cache, sets = kvb.cache.build_mixed(K.to(cuda_dev), V.to(cuda_dev), tc=tc)
    assert all(s["v_layout"] == int(tc) for s in cache.strata)
    # strata sets are exactly the oracle's (energy ranking, ties to the lower index)
    ref_sets = O.mixed_strata(O.l2_importance(np32(K)))
    for b in (8, 4, 2):
        np.testing.assert_array_equal(sets[b].cpu().numpy(), ref_sets[b])
    out = kvb.decode(cache, q.to(cuda_dev), 128 ** -0.5, qpos=[T] * Tq, out_dtype=torch.float32)
    assert kvb.device_status() == 0
    Kh, Vh = mixed_reference(K, V, ref_sets)
    ref = attend_reference(np32(q), 128 ** -0.5, Kh, Vh, qpos=[T] * Tq)
    err = np.abs(out.cpu().numpy() - ref).max()
    assert err <= TOL, err


def test_mixed_decode_bf16_output_and_repeat(cuda_dev):
    """Two calls in a row give identical bits (deterministic split-K), bf16 output == rounded fp32."""
    import kvb
    K, V = kvb.workloads.lognormal_kv(1, 2, 3000, 128, torch.bfloat16, seed=5)
    q = kvb.workloads.queries(1, 8, 1, 128, torch.bfloat16, seed=5).to(cuda_dev)
    cache, _ = kvb.cache.build_mixed(K.to(cuda_dev), V.to(cuda_dev))
    a = kvb.decode(cache, q, 128 ** -0.5, out_dtype=torch.float32)
    b = kvb.decode(cache, q, 128 ** -0.5, out_dtype=torch.float32)
    c = kvb.decode(cache, q, 128 ** -0.5)
    assert torch.equal(a, b)
    assert torch.equal(c, a.to(torch.bfloat16))


@pytest.mark.parametrize("kbits,vbits,kgroup,vgroup,rep,T", [(4, 2, 128, 32, 4, 4096), (4, 4, 128, 128, 8, 3000),
                                                             (4, 4, 64, 64, 4, 2176), (8, 8, 32, 64, 4, 1000),
                                                             (2, 2, 64, 128, 4, 999)])
def test_kivi_decode(cuda_dev, kbits, vbits, kgroup, vgroup, rep, T):
    """Configs 0 / 2 / 4 layouts: keys per channel over token groups, values per token."""
    import kvb
    K, V = kvb.workloads.outlier_kv(1, 2, T, 128, torch.float16, seed=T + kbits)
    q = kvb.workloads.queries(1, 2 * rep, 1, 128, torch.float16, seed=T)
    cache = kvb.cache.build_kivi(K.to(cuda_dev), V.to(cuda_dev), kbits, vbits, kgroup, vgroup)
    out = kvb.decode(cache, q.to(cuda_dev), 128 ** -0.5, out_dtype=torch.float32).cpu().numpy()
    Kh = O.kivi_quant(np32(K), kbits, kgroup, True, 0)["xhat"]
    Vh = O.kivi_quant(np32(V), vbits, vgroup, False, 0)["xhat"]
    ref = attend_reference(np32(q), 128 ** -0.5, Kh, Vh)
    err = np.abs(out - ref).max()
    assert err <= TOL, err


def test_kivi_decode_with_sinks(cuda_dev):
    """Rows before n_sink stay exact (fp16) and are merged with the coded partials."""
    import kvb
    T, n_sink = 1500, 4
    K, V = kvb.workloads.outlier_kv(1, 2, T, 128, torch.float16, seed=9)
    q = kvb.workloads.queries(1, 8, 1, 128, torch.float16, seed=9)
    cache = kvb.cache.build_kivi(K.to(cuda_dev), V.to(cuda_dev), 4, 2, 32, 32, n_sink=n_sink)
    out = kvb.decode(cache, q.to(cuda_dev), 128 ** -0.5, out_dtype=torch.float32).cpu().numpy()
    Kh = O.kivi_quant(np32(K), 4, 32, True, n_sink)["xhat"]
    Vh = O.kivi_quant(np32(V), 2, 32, False, n_sink)["xhat"]
    ref = attend_reference(np32(q), 128 ** -0.5, Kh, Vh)
    assert np.abs(out - ref).max() <= TOL


@pytest.mark.parametrize("tc", [True, False])
@pytest.mark.parametrize("rep,Tq", [(4, 1), (4, 2)])
def test_strata_midrise_decode(cuda_dev, rep, Tq, tc):
    """STRATA: rotated, centred mid-rise strata (2 / 4 / 8 bits) + exact rows incl. appended ones,
    query rotated once, output lifted by R plus (sum p) mu_V (StrataState.attend)."""
    import kvb
    gen = torch.Generator().manual_seed(77)
    Hkv, d, H = 2, 128, 3000
    R = torch.from_numpy(O.rotation_matrix(d, "strata"))
    counts = {8: 300, 4: 700, 2: 1500}
    mu_k = (torch.randn(Hkv, d, generator=gen) * 0.5).half().float()
    mu_v = (torch.randn(Hkv, d, generator=gen) * 0.5).half().float()
    tiers, cache = [], kvb.PackedCache(1, Hkv, d, midrise=True)
    for b, n in counts.items():
        Y = torch.randn(1, Hkv, n, d, generator=gen) * 1.3
        Yv = torch.randn(1, Hkv, n, d, generator=gen)
        dt = torch.float16 if tc else torch.float32      # the block layout takes 16-bit inputs
        vq = kvb.quant_pack(Yv.to(cuda_dev, dt), b, d, midrise=True, blocked=tc)
        kq = kvb.quant_pack(Y.to(cuda_dev, dt), b, d, midrise=True, n_alloc=vq["n_alloc"])
        Y, Yv = Y.to(dt).float(), Yv.to(dt).float()
        cache.add_stratum(kq, vq)
        ck, sk, _ = O.strata_quantize(Y.numpy(), b)
        cv, sv, _ = O.strata_quantize(Yv.numpy(), b)
        tiers.append({"bits": b, "kc": O.pack_planar(ck[0], b), "vc": O.pack_planar(cv[0], b),
                      "ks": sk[0], "vs": sv[0]})
    n0, extra = 40, Tq
    Ke = torch.randn(1, Hkv, n0 + extra, d, generator=gen).half()
    Ve = torch.randn(1, Hkv, n0 + extra, d, generator=gen).half()
    cache.set_exact(Ke.to(cuda_dev), Ve.to(cuda_dev), n_exact=n0 + extra, n0=n0, pos0=H)
    cache.qmap = R.T.contiguous()[None].expand(Hkv, d, d).contiguous().to(cuda_dev)
    cache.lift = R[None].expand(Hkv, d, d).contiguous().to(cuda_dev)
    cache.mu_k, cache.mu_v = mu_k.to(cuda_dev), mu_v.to(cuda_dev)
    q = torch.randn(1, Hkv * rep, Tq, d, generator=gen).half()
    qpos = [H + i for i in range(Tq)]
    out = kvb.decode(cache, q.to(cuda_dev), d ** -0.5, qpos=qpos, out_dtype=torch.float32).cpu().numpy()
    ref = O.strata_attend(np32(q), d ** -0.5, np.array(qpos), np32(Ke), np32(Ve), n0, H, tiers,
                          mu_k.numpy(), mu_v.numpy(), R.numpy())
    err = np.abs(out - ref).max()
    assert err <= TOL, err


def test_long_context_many_pieces(cuda_dev):
    """One head, 150k tokens: a single stratum split across every CTA and merged exactly."""
    import kvb
    T = 150000
    K, V = kvb.workloads.lognormal_kv(1, 1, T, 128, torch.bfloat16, seed=1)
    q = kvb.workloads.queries(1, 4, 1, 128, torch.bfloat16, seed=1)
    kq = kvb.quant_pack(K.to(cuda_dev), 4, 64)
    vq = kvb.quant_pack(V.to(cuda_dev), 4, 64)
    cache = kvb.PackedCache(1, 1, 128, k_group=64, v_group=64).add_stratum(kq, vq)
    plan = kvb.decode_plan(cache, 148)
    assert len(plan["pieces"]) >= 100
    out = kvb.decode(cache, q.to(cuda_dev), 128 ** -0.5, out_dtype=torch.float32).cpu().numpy()
    Kh = O.kivi_quant(np32(K), 4, 64, False, 0)["xhat"]
    Vh = O.kivi_quant(np32(V), 4, 64, False, 0)["xhat"]
    ref = attend_reference(np32(q), 128 ** -0.5, Kh, Vh)
    assert np.abs(out - ref).max() <= TOL


@pytest.mark.parametrize("T", [1, 15, 16, 17])
def test_tiny_contexts(cuda_dev, T):
    """Ragged tails: fewer tokens than one 16-token tile, exactly one tile, one more."""
    import kvb
    K, V = kvb.workloads.lognormal_kv(1, 2, T, 128, torch.bfloat16, seed=T + 100)
    q = kvb.workloads.queries(1, 8, 1, 128, torch.bfloat16, seed=T)
    kq = kvb.quant_pack(K.to(cuda_dev), 2, 64)
    vq = kvb.quant_pack(V.to(cuda_dev), 2, 64)
    cache = kvb.PackedCache(1, 2, 128, k_group=64, v_group=64).add_stratum(kq, vq)
    out = kvb.decode(cache, q.to(cuda_dev), 128 ** -0.5, out_dtype=torch.float32).cpu().numpy()
    Kh = O.kivi_quant(np32(K), 2, 64, False, 0)["xhat"]
    Vh = O.kivi_quant(np32(V), 2, 64, False, 0)["xhat"]
    assert np.abs(out - attend_reference(np32(q), 128 ** -0.5, Kh, Vh)).max() <= TOL


@pytest.mark.parametrize("rep,Tq", [(4, 1), (8, 1), (4, 2)])
def test_tc_matches_mma_decode(cuda_dev, rep, Tq):
    """The same mixed cache in both value layouts: tcgen05 and mma.sync decodes agree closely."""
    import kvb
    K, V = kvb.workloads.lognormal_kv(2, 2, 3000, 128, torch.bfloat16, seed=21)
    q = kvb.workloads.queries(2, 2 * rep, Tq, 128, torch.bfloat16, seed=21).to(cuda_dev)
    a, _ = kvb.cache.build_mixed(K.to(cuda_dev), V.to(cuda_dev), tc=True)
    b, _ = kvb.cache.build_mixed(K.to(cuda_dev), V.to(cuda_dev), tc=False)
    oa = kvb.decode(a, q, 128 ** -0.5, qpos=[3000] * Tq, out_dtype=torch.float32)
    ob = kvb.decode(b, q, 128 ** -0.5, qpos=[3000] * Tq, out_dtype=torch.float32)
    assert kvb.device_status() == 0
    assert (oa - ob).abs().max().item() <= 1e-3


def test_cta_counts_and_plan_reuse(cuda_dev):
    """The split-K plan (and the parameter tables built from it) is reused between calls of one
    cache shape and rebuilt when the shape or the CTA count changes: alternating two caches of
    different shapes and several CTA counts gives, every time, the output of a first call."""
    import kvb
    ka, va = kvb.workloads.lognormal_kv(1, 2, 3000, 128, torch.bfloat16, device=cuda_dev, seed=21)
    kb, vb = kvb.workloads.lognormal_kv(2, 2, 1500, 128, torch.bfloat16, device=cuda_dev, seed=22)
    ca, _ = kvb.cache.build_mixed(ka, va)
    cb = kvb.cache.build_kivi(kb, vb, 4, 2, 128, 32)
    qa = kvb.workloads.queries(1, 8, 1, 128, torch.bfloat16, device=cuda_dev, seed=23)
    qb = kvb.workloads.queries(2, 8, 1, 128, torch.bfloat16, device=cuda_dev, seed=24)
    ref_a = kvb.decode(ca, qa, 128 ** -0.5, out_dtype=torch.float32)
    ref_b = kvb.decode(cb, qb, 128 ** -0.5, out_dtype=torch.float32)
    for _ in range(2):
        for n_ctas in (0, 1, 7, 300):
            oa = kvb.decode(ca, qa, 128 ** -0.5, out_dtype=torch.float32, n_ctas=n_ctas)
            ob = kvb.decode(cb, qb, 128 ** -0.5, out_dtype=torch.float32, n_ctas=n_ctas)
            # other CTA counts split the context elsewhere: each split's running max sets the fp16
            # rounding of its value weights, so outputs move by the kernel's own error (~5e-5)
            tol = 0.0 if n_ctas == 0 else 2e-4
            assert (oa - ref_a).abs().max().item() <= tol
            assert (ob - ref_b).abs().max().item() <= tol
    assert kvb.device_status() == 0
