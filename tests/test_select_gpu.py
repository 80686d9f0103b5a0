"""K2 importance + rank split on the GPU vs the oracle: bit-exact energies and index sets,
including ties (lower index first), empty and full classes, and ragged row lengths."""

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def test_key_energy_exact(cuda_dev):
    import kvb
    gen = torch.Generator().manual_seed(11)
    k = (torch.randn(2, 3, 777, 128, generator=gen) * 3).to(torch.bfloat16)
    e = kvb.key_energy(k.to(cuda_dev)).cpu().numpy()
    np.testing.assert_array_equal(e, O.l2_importance(k.float().numpy()))


@pytest.mark.parametrize("T", [20, 1000, 4097, 32768, 45056, 65536])   # 65536: the global-memory kernel
def test_strata_split_matches_oracle(cuda_dev, T):
    import kvb
    gen = torch.Generator().manual_seed(T)
    imp = torch.randint(0, 50, (2, 4, T), generator=gen).double()      # many exact ties
    n8, n4, _ = O.strata_counts(T)
    i8, i4, i2 = kvb.rank_split(imp.to(cuda_dev), [n8, n4])
    ref = O.mixed_strata(imp.numpy())
    for got, b in ((i8, 8), (i4, 4), (i2, 2)):
        if ref[b].shape[-1] == 0:
            assert got is None
        else:
            np.testing.assert_array_equal(got.cpu().numpy(), ref[b])


@pytest.mark.parametrize("n,k", [(1, 1), (100, 0), (100, 100), (32640, 2048), (5000, 4999), (60000, 777)])
def test_topk_float32(cuda_dev, n, k):
    import kvb
    gen = torch.Generator().manual_seed(n + k)
    s = torch.rand(3, n, generator=gen)
    s[:, ::7] = 0.5                                                       # ties
    if n > 2:
        s[0, 1] = -0.0
        s[1, 2] = -1e-30
    top = kvb.rank_split(s.to(cuda_dev), [k], want=[0])[0]
    ref = O.topk_kept(s.numpy(), k)
    if k == 0:
        assert top is None
    else:
        np.testing.assert_array_equal(top.cpu().numpy(), ref)


def test_four_classes(cuda_dev):
    import kvb
    gen = torch.Generator().manual_seed(5)
    s = torch.randn(5, 3000, generator=gen).double()
    outs = kvb.rank_split(s.to(cuda_dev), [10, 100, 1000])
    order = np.lexsort((np.tile(np.arange(3000), (5, 1)), -s.numpy()), axis=-1)
    edges = [0, 10, 110, 1110, 3000]
    for c in range(4):
        np.testing.assert_array_equal(outs[c].cpu().numpy(), np.sort(order[:, edges[c]:edges[c + 1]], -1))


@pytest.mark.parametrize("n", [3000, 40000, 50000])
def test_float64_close_keys(cuda_dev, n):
    """Keys that share their high 32 bits (differ only in the low word of the float64) and exact
    ties among them: the boundary is resolved on the full key, ties by lower index."""
    import kvb
    gen = torch.Generator().manual_seed(n)
    base = 100.0 + torch.randint(0, 3, (4, n), generator=gen).double()
    s = base + torch.randint(0, 5, (4, n), generator=gen).double() * 2.0 ** -40
    outs = kvb.rank_split(s.to(cuda_dev), [n // 7, n // 3])
    order = np.lexsort((np.tile(np.arange(n), (4, 1)), -s.numpy()), axis=-1)
    edges = [0, n // 7, n // 7 + n // 3, n]
    for c in range(3):
        np.testing.assert_array_equal(outs[c].cpu().numpy(), np.sort(order[:, edges[c]:edges[c + 1]], -1))


def test_nan_keys_flagged(cuda_dev):
    """A NaN key sets bit 2 of the device status word (no host synchronisation in rank_split)."""
    import kvb
    kvb.device_status()                               # clear
    s = torch.zeros(1, 10, device=cuda_dev)
    s[0, 3] = float("nan")
    kvb.rank_split(s, [2])
    assert kvb.device_status() & 4
    kvb.rank_split(torch.zeros(1, 10, device=cuda_dev), [2])
    assert kvb.device_status() == 0
