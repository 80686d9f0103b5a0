"""Drop-in decoder states (kvb.state) against the reference's StrataState.

CPU: construction from the reference's packed strata, the append protocol and its error, the
16-row padding of tier_as_kvb, context_bytes equal to the reference's own figure.
GPU: attend after one and after two appended tokens equals StrataState.attend's outputs stored in
tests/golden/strata_state.npz (max-abs 2e-3), check_kernel passes, a KIVI-coded state decodes like
the oracle with appended causal rows."""

import numpy as np
import pytest
import torch

import oracle as O
from kvref import np32


def _packed(g, dev):
    tiers = []
    for i in range(int(g["n_tiers"])):
        tiers.append({"bits": int(g[f"t{i}_bits"]), "n": int(g[f"t{i}_n"]),
                      "kc": torch.from_numpy(g[f"t{i}_kc"]).to(dev), "vc": torch.from_numpy(g[f"t{i}_vc"]).to(dev),
                      "ks": torch.from_numpy(g[f"t{i}_ks"]).to(dev), "vs": torch.from_numpy(g[f"t{i}_vs"]).to(dev)})
    return {"tiers": tiers, "counts": torch.from_numpy(g["counts"]), "n_c": int(g["n_c"]),
            "mu_k": torch.from_numpy(g["mu_k"]).half().to(dev), "mu_v": torch.from_numpy(g["mu_v"]).half().to(dev)}


def _state(g, dev, dtype=torch.float32):
    import kvb
    Ke = torch.from_numpy(g["Ke"]).to(dev, dtype)
    Ve = torch.from_numpy(g["Ve"]).to(dev, dtype)
    R = torch.from_numpy(g["R"]).to(dev, dtype)
    return kvb.KvbStrataState(Ke, Ve, _packed(g, dev), int(g["extra"]), int(g["H"]), R)


def test_tier_padding(golden):
    import kvb
    g = golden("strata_state")
    t = _packed(g, "cpu")["tiers"][1]
    k = kvb.tier_as_kvb(t, "k")
    n = t["n"]
    assert k["n"] == n and k["n_alloc"] % 16 == 0 and k["n_alloc"] >= n and k["bits"] == t["bits"]
    assert tuple(k["codes"].shape) == (1, t["kc"].shape[0], k["n_alloc"], t["kc"].shape[2])
    assert torch.equal(k["codes"][0, :, :n], t["kc"]) and not k["codes"][0, :, n:].any()
    assert torch.equal(k["meta"][0, :, :n], t["ks"]) and k["meta"].dtype == torch.float16


def test_state_protocol_cpu(golden):
    g = golden("strata_state")
    st = _state(g, "cpu")
    n0, extra = int(g["n0"]), int(g["extra"])
    assert st.n == st.n0 == n0 and st.shared is None and st.K.shape[2] == n0 + extra
    assert st.context_bytes() == int(g["context_bytes"])          # the reference's own figure
    kn = torch.from_numpy(g["kn"])
    st.append(kn[:, :, :1], kn[:, :, :1], torch.tensor([int(g["H"])]))
    assert st.n == n0 + 1 and torch.equal(st.K[:, :, n0], kn[:, :, 0])
    st.append(torch.zeros(1, 2, extra - 1, 128), torch.zeros(1, 2, extra - 1, 128), None)
    with pytest.raises(RuntimeError, match="decode buffer exhausted"):
        st.append(kn[:, :, :1], kn[:, :, :1], None)
    # the 3 strata of the fixture: 8 / 4 / 2 bits, one kvb stratum each
    assert [s["kbits"] for s in st.cache.strata] == [int(g[f"t{i}_bits"]) for i in range(int(g["n_tiers"]))]


@pytest.mark.gpu
def test_strata_state_matches_reference(golden, cuda_dev):
    g = golden("strata_state")
    st = _state(g, cuda_dev)
    H = int(g["H"])
    kn, vn = torch.from_numpy(g["kn"]).to(cuda_dev), torch.from_numpy(g["vn"]).to(cuda_dev)
    st.append(kn[:, :, :1], vn[:, :, :1], torch.tensor([H]))
    o1 = st.attend(torch.from_numpy(g["q1"]).to(cuda_dev), 128 ** -0.5, torch.tensor([H]))
    assert o1.shape == (1, 1, 8, 128) and o1.dtype == torch.float32
    assert np.abs(np32(o1) - g["out1"]).max() <= 2e-3
    st.append(kn[:, :, 1:], vn[:, :, 1:], torch.tensor([H + 1]))
    o2 = st.attend(torch.from_numpy(g["q2"]).to(cuda_dev), 128 ** -0.5, torch.tensor([H, H + 1]))
    assert np.abs(np32(o2) - g["out2"]).max() <= 2e-3
    r = st.check_kernel()
    assert r["kernel"] and r["kernel_rel_err"] <= 2e-3


@pytest.mark.gpu
def test_strata_state_bf16(golden, cuda_dev):
    """Model dtype bf16 (as the reference's decoder holds it): q, exact rows and output in bf16."""
    g = golden("strata_state")
    st = _state(g, cuda_dev, torch.bfloat16)
    H = int(g["H"])
    kn, vn = torch.from_numpy(g["kn"]).to(cuda_dev), torch.from_numpy(g["vn"]).to(cuda_dev)
    st.append(kn[:, :, :1].bfloat16(), vn[:, :, :1].bfloat16(), torch.tensor([H]))
    q = torch.from_numpy(g["q1"]).to(cuda_dev).bfloat16()
    o = st.attend(q, 128 ** -0.5, torch.tensor([H]))
    assert o.dtype == torch.bfloat16
    ref = st.reference_attend(q, 128 ** -0.5, [H])
    assert (o.float() - ref).abs().max().item() <= 1e-2        # bf16 output rounding
    assert st.check_kernel()["kernel"]


@pytest.mark.gpu
def test_coded_state_kivi(cuda_dev):
    """KIVI-coded cache with 4 sink rows; two appended tokens decoded causally."""
    import kvb
    B, Hkv, T, d, rep, H = 1, 2, 700, 128, 4, 700
    K, V = kvb.workloads.outlier_kv(B, Hkv, T, d, torch.float16, seed=9)
    cache = kvb.cache.build_kivi(K.to(cuda_dev), V.to(cuda_dev), 4, 2, 128, 64, n_sink=4)
    st = kvb.KvbCodedState(cache, extra=4, H=H)
    assert st.n0 == 4
    gen = torch.Generator().manual_seed(3)
    kn, vn = (torch.randn(B, Hkv, 2, d, generator=gen).half() for _ in range(2))
    st.append(kn.to(cuda_dev), vn.to(cuda_dev), torch.tensor([H, H + 1]))
    q = kvb.workloads.queries(B, Hkv * rep, 2, d, torch.float16, seed=9)
    out = np32(st.attend(q.to(cuda_dev), d ** -0.5, torch.tensor([H, H + 1])))
    # oracle: dequantised cache + sinks, appended rows causal w.r.t. each query
    kq = O.kivi_quant(np32(K), 4, 128, along_tokens=True, n_sink=4)
    vq = O.kivi_quant(np32(V), 2, 64, along_tokens=False, n_sink=4)
    Kh = np.concatenate([kq["xhat"], np32(kn)], 2)
    Vh = np.concatenate([vq["xhat"], np32(vn)], 2)
    pos = np.concatenate([np.arange(T), [H, H + 1]])
    ref = O.chunked_attention(np32(q), d ** -0.5, np.array([H, H + 1]), Kh, Vh, pos,
                              np.full((T + 2,), 1 << 40), None, 256)
    assert np.abs(out - ref).max() <= 2e-3
