"""K1 quantise + pack on the GPU vs the oracle / the reference's golden outputs: bit-exact codes,
fp16 zero points and scales, and dequantised values."""

import numpy as np
import pytest
import torch

import oracle as O
from kvref import unpack, token_meta, channel_meta, np32

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("i", range(8))
def test_golden_kivi_cases(golden, cuda_dev, i):
    import kvb
    g = golden("codecs")
    B, H, T, d, bits, group, along, sink, bf = g[f"kivi{i}_case"].tolist()
    if d % 32:
        pytest.skip("head_dim not a multiple of 32 (outside the kernel set; d = 48 has no B200 model)")
    x = torch.from_numpy(g[f"kivi{i}_x"]).to(cuda_dev)
    if bf:
        x = x.to(torch.bfloat16)
    n = T - sink
    r = kvb.quant_pack(x, bits, group, per_channel=bool(along), first_row=sink, n=n, want_xhat=True)
    codes = unpack(r["codes"], bits, n)
    np.testing.assert_array_equal(codes, g[f"kivi{i}_codes"])
    if along:
        lo, sc = channel_meta(r["meta"], n, group)
    else:
        lo, sc = token_meta(r["meta"], n)
    np.testing.assert_array_equal(lo, g[f"kivi{i}_lo"])
    np.testing.assert_array_equal(sc, g[f"kivi{i}_scale"])
    np.testing.assert_array_equal(np32(r["xhat"]), g[f"kivi{i}_xhat"][:, :, sink:])


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_token_groups_with_gather(cuda_dev, bits, dtype):
    """Per-token groups of 64 over gathered rows (one stratum of the mixed cache)."""
    import kvb
    gen = torch.Generator().manual_seed(100 + bits)
    B, H, T, d = 2, 3, 333, 128
    x = (torch.randn(B, H, T, d, generator=gen) * torch.exp(0.5 * torch.randn(1, H, 1, d, generator=gen))).to(dtype)
    idx = torch.stack([torch.randperm(T, generator=gen)[:150].sort().values for _ in range(B * H)]).view(B, H, 150)
    r = kvb.quant_pack(x.to(cuda_dev), bits, 64, idx=idx.to(cuda_dev), want_xhat=True)
    xs = np.take_along_axis(np32(x), idx.numpy()[..., None].repeat(d, -1), 2)
    ref = O.kivi_quant(xs, bits, 64, False, 0)
    np.testing.assert_array_equal(unpack(r["codes"], bits, 150), ref["codes"])
    lo, sc = token_meta(r["meta"], 150)
    np.testing.assert_array_equal(lo, ref["lo"])
    np.testing.assert_array_equal(sc, ref["scale"])
    np.testing.assert_array_equal(np32(r["xhat"]), ref["xhat"])
    # planar bytes exactly as pack_planar lays them out; padding rows zero-filled
    np.testing.assert_array_equal(r["codes"][:, :, :150].cpu().numpy(), O.pack_planar(ref["codes"], bits))
    assert int(r["codes"][:, :, 150:].abs().sum()) == 0


@pytest.mark.parametrize("bits,group,T", [(4, 128, 300), (2, 64, 257), (8, 32, 96), (4, 16, 40)])
def test_channel_groups(cuda_dev, bits, group, T):
    """Keys per channel over token groups, including a partial last group."""
    import kvb
    gen = torch.Generator().manual_seed(7 * bits + group)
    x = torch.randn(1, 4, T, 128, generator=gen).to(torch.float16)
    x[..., 5] *= 8
    r = kvb.quant_pack(x.to(cuda_dev), bits, group, per_channel=True, want_xhat=True)
    ref = O.kivi_quant(np32(x), bits, group, True, 0)
    np.testing.assert_array_equal(unpack(r["codes"], bits, T), ref["codes"])
    lo, sc = channel_meta(r["meta"], T, group)
    np.testing.assert_array_equal(lo, ref["lo"])
    np.testing.assert_array_equal(sc, ref["scale"])
    np.testing.assert_array_equal(np32(r["xhat"]), ref["xhat"])


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("d", [32, 128])
def test_midrise(cuda_dev, bits, d):
    """STRATA per-vector code (strata_quantize, STRATA_KV.py:1158) on float32 rows."""
    import kvb
    gen = torch.Generator().manual_seed(3 * bits + d)
    y = torch.randn(2, 2, 500, d, generator=gen) * torch.linspace(0.2, 3.0, d)
    r = kvb.quant_pack(y.to(cuda_dev), bits, d, midrise=True, want_xhat=True)
    c, s, yh = O.strata_quantize(y.numpy(), bits)
    np.testing.assert_array_equal(unpack(r["codes"], bits, 500), c)
    np.testing.assert_array_equal(r["meta"][:, :, :500].float().cpu().numpy(), s)
    np.testing.assert_array_equal(np32(r["xhat"]), yh)


def test_golden_strata_codes(golden, cuda_dev):
    """Mid-rise codes and scales of the reference's golden rotated 32-vectors, bit for bit (the RMS
    takes torch's CPU summation order)."""
    import kvb
    g = golden("codecs")
    y = torch.from_numpy(g["sq_x"])[None, None].contiguous()
    for b in (2, 4, 8):
        r = kvb.quant_pack(y.to(cuda_dev), b, 32, midrise=True, want_xhat=True)
        np.testing.assert_array_equal(r["meta"][0, 0, :y.shape[2]].float().cpu().numpy(), g[f"sq{b}_s"])
        np.testing.assert_array_equal(unpack(r["codes"], b, y.shape[2])[0, 0], g[f"sq{b}_codes"])
        np.testing.assert_array_equal(np32(r["xhat"])[0, 0], g[f"sq{b}_yhat"])


@pytest.mark.parametrize("tag", ["bf", "h"])
@pytest.mark.parametrize("src", ["float32", "native", "blocked"])
def test_golden_midrise128(golden, cuda_dev, tag, src):
    """d = 128 mid-rise codes and scales of the reference (midrise128.npz) from every kernel layout:
    float32 rows (one row per warp), bf16 / fp16 rows (8 lanes per row, token-major) and the
    128-token block layout (16 lanes per row), bit for bit."""
    import kvb
    g = golden("midrise128")
    y = torch.from_numpy(g[f"{tag}_y"])[None, None].contiguous()
    if src != "float32":
        y = y.to(torch.bfloat16 if tag == "bf" else torch.float16)
    n = y.shape[2]
    for b in (2, 4, 8):
        r = kvb.quant_pack(y.to(cuda_dev), b, 128, midrise=True, want_xhat=True, blocked=src == "blocked")
        codes = kvb.ops.unblock_codes(r["codes"]) if src == "blocked" else r["codes"]
        np.testing.assert_array_equal(r["meta"][0, 0, :n].float().cpu().numpy(), g[f"{tag}{b}_s"])
        np.testing.assert_array_equal(unpack(codes, b, n)[0, 0], g[f"{tag}{b}_codes"])
        if b == 2:
            np.testing.assert_array_equal(np32(r["xhat"])[0, 0], g[f"{tag}{b}_yhat"])
    assert kvb.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_bad_rows_are_rejected_not_read(cuda_dev, dtype):
    """An out-of-range gather index (past T, or negative) sets the device bounds flag instead of
    reading out of bounds; the row is stored as zero codes and zero metadata, the others as usual.
    float32 takes the generic kernel, bf16 the 128-bit-load one."""
    import kvb
    x = torch.randn(1, 1, 10, 128, device=cuda_dev).to(dtype)
    for bad in (11, -1):
        idx = torch.tensor([[[0, 3, bad, 9]]], device=cuda_dev)
        kvb.device_status(clear=True)
        r = kvb.quant_pack(x, 4, 64, idx=idx)
        assert kvb.device_status(clear=True) & 2
        assert int(r["codes"][0, 0, 2].abs().sum()) == 0 and int(r["meta"][0, 0, 2].abs().sum()) == 0
        ok = kvb.quant_pack(x, 4, 64, idx=idx[..., [0, 1, 3]])
        assert kvb.device_status() == 0
        assert torch.equal(r["codes"][0, 0, [0, 1, 3]], ok["codes"][0, 0, :3])


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("group,midrise", [(32, False), (64, False), (128, False), (128, True)])
@pytest.mark.parametrize("gather", [False, True])
def test_blocked_layout_same_codes(cuda_dev, bits, group, midrise, gather):
    """kvb_quant_pack_blocked writes the same codes / metadata / xhat as kvb_quant_pack, in the
    128-token channel-major block layout (unblocked here on the device)."""
    import kvb
    T = 700
    x = kvb.workloads.lognormal_kv(2, 3, T, 128, torch.bfloat16, seed=bits + group)[0].to(cuda_dev)
    idx = None
    if gather:
        g = torch.Generator().manual_seed(bits)
        idx = torch.stack([torch.stack([torch.randperm(T, generator=g)[:333].sort().values for _ in range(3)])
                           for _ in range(2)]).to(cuda_dev)
    a = kvb.quant_pack(x, bits, group, midrise=midrise, idx=idx, want_xhat=True, blocked=True)
    b = kvb.quant_pack(x, bits, group, midrise=midrise, idx=idx, want_xhat=True, n_alloc=a["n_alloc"])
    assert a["n_alloc"] % 128 == 0 and a["codes"].dim() == 5
    assert torch.equal(kvb.ops.unblock_codes(a["codes"]), b["codes"])
    assert torch.equal(a["meta"], b["meta"])
    assert torch.equal(a["xhat"], b["xhat"])
    assert kvb.device_status() == 0


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_extreme_rows(cuda_dev, bits, dtype):
    """Rows the storage format clamps or degenerates on: constant rows (zero range: scale floored at
    2^-24), all-zero rows, magnitudes past the fp16 range (zero point and scale clamped to 65504 by
    as_stored), tiny magnitudes (subnormal fp16 scales).  Bit-exact against the oracle."""
    import kvb
    gen = torch.Generator().manual_seed(7 + bits)
    B, H, T, d = 1, 2, 48, 128
    x = torch.randn(B, H, T, d, generator=gen)
    x[0, 0, 0] = 3.25                      # constant row
    x[0, 0, 1] = 0.0                       # zero row
    x[0, 0, 2] *= 1e6                      # beyond fp16
    x[0, 0, 3, :64] = -7e4                 # one group pinned at -70000
    x[0, 1, 4] *= 1e-6                     # scale in the fp16 subnormal range
    x[0, 1, 5, ::2] = 1e-30                # values below every fp16 step
    x = x.to(dtype)
    for group in (64, 128):
        r = kvb.quant_pack(x.to(cuda_dev), bits, group, want_xhat=True)
        ref = O.kivi_quant(np32(x), bits, group, False, 0)
        np.testing.assert_array_equal(unpack(r["codes"], bits, T), ref["codes"])
        lo, sc = token_meta(r["meta"], T)
        np.testing.assert_array_equal(lo, ref["lo"])
        np.testing.assert_array_equal(sc, ref["scale"])
        np.testing.assert_array_equal(np32(r["xhat"]), ref["xhat"])
    assert kvb.device_status() == 0
