"""K5 row codes on the GPU against the oracle and the reference's own outputs (rowcodes.npz):
absmax tails (STRATA and TILT variants), MSB-first packing, byte-table decode, the HEDGE code and
TILT's chunk selection.  Codes, bytes, indices and fp16 scales bit-exact; float32 products that go
through a different summation order within the stated tolerances."""

import numpy as np
import pytest
import torch

import oracle as O
from oracle import rowcodes as RC

pytestmark = pytest.mark.gpu


def _t(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


@pytest.mark.parametrize("b", [2, 3, 4, 5, 8])
@pytest.mark.parametrize("variant", ["strata", "tilt"])
def test_absmax_golden(golden, cuda_dev, b, variant):
    """The reference's own codes / scales / bytes (absmax_quant, pack_codes, fake_quant_tokens)."""
    import kvb
    g = golden("rowcodes")
    x = _t(g["am_x"], cuda_dev).view(1, 1, 40, 128)
    r = kvb.ops.absmax_quant(x, b, variant=variant, want_xhat=True)
    if variant == "strata":
        np.testing.assert_array_equal(r["packed"].cpu().numpy().reshape(-1), g[f"am{b}_packed"])
        np.testing.assert_array_equal(r["scale"].cpu().numpy().reshape(40, 1), g[f"am{b}_s"])
        np.testing.assert_array_equal(r["xhat"].cpu().numpy()[0, 0], g[f"am{b}_codes"] * g[f"am{b}_s"])
    else:
        np.testing.assert_array_equal(r["xhat"].cpu().numpy()[0, 0], g[f"tilt{b}_xhat"])
    assert kvb.device_status() == 0


@pytest.mark.parametrize("d,dtype", [(64, torch.float32), (128, torch.bfloat16), (256, torch.float16),
                                     (96, torch.float32)])
def test_absmax_gather_random(cuda_dev, d, dtype):
    import kvb
    g = torch.Generator().manual_seed(d)
    B, H, T, n = 2, 3, 200, 57
    x = (torch.randn(B, H, T, d, generator=g) * torch.rand(B, H, T, 1, generator=g) * 5).to(dtype)
    x[0, 1, 7] = 0
    idx = torch.stack([torch.randperm(T, generator=g)[:n] for _ in range(B * H)]).view(B, H, n)
    xs = x.float().numpy()
    for variant, fn in (("strata", O.absmax_quant), ("tilt", RC.absmax_tilt)):
        for b in (2, 4, 6, 8):
            r = kvb.ops.absmax_quant(x.to(cuda_dev), b, variant=variant, idx=idx.to(cuda_dev), want_xhat=True)
            rows = np.take_along_axis(xs, idx.numpy()[..., None], 2)
            c, s = fn(rows, b)
            exp_packed = np.stack([RC.absmax_packed(c[i, j, k], b) for i in range(B) for j in range(H)
                                   for k in range(n)]).reshape(B, H, n, -1)
            np.testing.assert_array_equal(r["packed"].cpu().numpy(), exp_packed)
            np.testing.assert_array_equal(r["scale"].cpu().numpy(), s[..., 0])
            np.testing.assert_array_equal(r["xhat"].cpu().numpy(), c * s)
    assert kvb.device_status() == 0


def test_absmax_bad_index_flagged(cuda_dev):
    import kvb
    x = torch.randn(1, 1, 10, 128, device=cuda_dev)
    idx = torch.tensor([[[0, 3, 10]]], device=cuda_dev)
    kvb.device_status()
    kvb.ops.absmax_quant(x, 8, idx=idx)
    torch.cuda.synchronize()
    assert kvb.device_status() & 2


@pytest.mark.parametrize("bits", [1, 2, 3, 4, 5, 6, 7, 8])
def test_pack_rows_and_lut(golden, cuda_dev, bits):
    import kvb
    g = torch.Generator().manual_seed(bits)
    w = 64 if bits % 2 else 48
    codes = torch.randint(0, 1 << bits, (7, 3, w), generator=g, dtype=torch.uint8)
    out = kvb.ops.pack_rows(codes.to(cuda_dev), bits).cpu().numpy()
    exp = np.stack([O.pack_codes(r, bits) for r in codes.numpy().reshape(-1, w)]).reshape(7, 3, -1)
    np.testing.assert_array_equal(out, exp)
    levels = torch.randn(1 << bits, generator=g)
    sc = torch.rand(7, 3, generator=g)
    dec = kvb.ops.decode_rows_lut(_t(out, cuda_dev), bits, levels.to(cuda_dev), row_scale=sc.to(cuda_dev))
    np.testing.assert_array_equal(dec.cpu().numpy(), levels.numpy()[codes.numpy()] * sc.numpy()[..., None])


def test_pack_rows_golden(golden, cuda_dev):
    import kvb
    gg = golden("codecs")
    for b in (2, 4):
        np.testing.assert_array_equal(kvb.ops.pack_rows(_t(gg[f"rows{b}_in"], cuda_dev), b).cpu().numpy(),
                                      gg[f"rows{b}_out"])


def test_embedded_lut_decode_golden(golden, cuda_dev):
    """QUASAR's (2, 2, 4) embedded code: packed stage rows decoded and summed on the device equal the
    reference's cumulative reconstructions bit for bit."""
    import kvb
    g = golden("rowcodes")
    acc = None
    for t, b in enumerate((2, 2, 4)):
        acc = kvb.ops.decode_rows_lut(_t(g[f"emb_rows{t}"], cuda_dev), b, _t(g[f"emb_levels{t}"], cuda_dev), out=acc)
        np.testing.assert_array_equal(acc.cpu().numpy(), g[f"emb_cum{t}"])


@pytest.mark.parametrize("b", [1, 2, 3, 4, 8])
def test_hedge_golden(golden, cuda_dev, b):
    """centered_code of the reference, bit for bit: rotation y (the reference's CPU FMA order), codes,
    fp16 scales (torch's CPU summation order for the RMS) and the read-back x_hat."""
    import kvb
    g = golden("rowcodes")
    x = _t(g["hedge_x"], cuda_dev).view(1, 2, 24, 128)
    R = _t(g["hedge_R"], cuda_dev)
    mu = _t(g["hedge_mu"], cuda_dev).view(2, 128)
    lv = kvb.codebooks.lloyd_max(b, cuda_dev) if b <= 4 else None
    r = kvb.ops.hedge_quant(x, R, b, lv, mu=mu, want_y=True, want_xhat=True)
    np.testing.assert_array_equal(r["y"].cpu().numpy()[0], g["hedge_y"])
    packed = r["packed"].cpu().numpy()[0]
    np.testing.assert_array_equal(RC.unpack_rows(packed, b, 128), g[f"hedge{b}_codes"].astype(np.int64))
    np.testing.assert_array_equal(r["scale"].cpu().numpy()[0], g[f"hedge{b}_s"][..., 0])
    np.testing.assert_array_equal(r["xhat"].cpu().numpy()[0], g[f"hedge{b}_xhat"])


def test_hedge_gather_bf16(cuda_dev):
    import kvb
    g = torch.Generator().manual_seed(5)
    B, H, T, n = 2, 3, 150, 70
    x = (torch.randn(B, H, T, 128, generator=g) * 2).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(T, generator=g)[:n].sort().values for _ in range(B * H)]).view(B, H, n)
    R = torch.from_numpy(O.rotation_matrix(128, "layer3"))
    for b in (2, 4, 8):
        lv = kvb.codebooks.lloyd_max(b, cuda_dev) if b <= 4 else None
        r = kvb.ops.hedge_quant(x.to(cuda_dev), R.to(cuda_dev), b, lv, idx=idx.to(cuda_dev), want_y=True)
        rows = np.take_along_axis(x.float().numpy(), idx.numpy()[..., None], 2)
        _, c, s, y_ref = RC.hedge_quant(rows, R.numpy(), b)
        y = r["y"].cpu().numpy()
        np.testing.assert_array_equal(y, y_ref)
        np.testing.assert_array_equal(RC.unpack_rows(r["packed"].cpu().numpy(), b, 128), c.astype(np.int64))
        np.testing.assert_array_equal(r["scale"].cpu().numpy(), s[..., 0])
    assert kvb.device_status() == 0


def test_chunk_select_golden(golden, cuda_dev):
    """TILT finalize_chunk (eviction family) of the reference: same kept positions, shares within
    float32 tolerance, 8-bit tails identical."""
    import kvb
    g = golden("rowcodes")
    k, v, q = (_t(g[n_], cuda_dev) for n_ in ("tilt_k", "tilt_v", "tilt_q"))
    m = int(g["tilt_m"])
    idx, share = kvb.ops.chunk_select(k, q, m, want_share=True)
    np.testing.assert_allclose(share.cpu().numpy(), g["tilt_share"], rtol=1e-5, atol=1e-9)
    np.testing.assert_array_equal(idx.cpu().numpy(), RC.chunk_topm(share.cpu().numpy(), m))
    np.testing.assert_array_equal(idx.cpu().numpy(), g["tilt_idx"])
    r = kvb.ops.chunk_tails(k, v, q, m, 8)
    np.testing.assert_array_equal(r["k"]["xhat"].cpu().numpy(), g["tilt_kq"])
    np.testing.assert_array_equal(r["v"]["xhat"].cpu().numpy(), g["tilt_vq"])


@pytest.mark.parametrize("C,nq,m,dtype", [(128, 128, 23, torch.bfloat16), (100, 40, 7, torch.float32),
                                          (128, 33, 0, torch.float16), (64, 32, 64, torch.float32),
                                          (128, 1, 1, torch.float32)])
def test_chunk_select_random(cuda_dev, C, nq, m, dtype):
    import kvb
    g = torch.Generator().manual_seed(C + nq + m)
    U, H = 5, 2
    k = (torch.randn(U, H, C, 128, generator=g) * 1.5).to(dtype)
    q = torch.randn(U, H, nq, 128, generator=g) * 128 ** -0.5
    idx, share = kvb.ops.chunk_select(k.to(cuda_dev), q.to(cuda_dev), m, want_share=True)
    sh = share.cpu().numpy()
    np.testing.assert_allclose(sh, RC.chunk_share(k.float().numpy(), q.numpy()), rtol=2e-5, atol=1e-9)
    np.testing.assert_array_equal(idx.cpu().numpy(), RC.chunk_topm(sh, m))
    assert kvb.device_status() == 0


def test_chunk_select_ties(cuda_dev):
    """Identical keys give identical shares: the lower positions are kept."""
    import kvb
    k = torch.ones(1, 1, 128, 128, device=cuda_dev)
    q = torch.randn(1, 1, 16, 128, device=cuda_dev)
    idx, _ = kvb.ops.chunk_select(k, q, 10)
    assert idx.cpu().tolist() == [[list(range(10))]]
