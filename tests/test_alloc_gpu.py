"""STRATA's head-synchronous rate allocation on the GPU (kvb_head_sync_allocate) against the
reference's own allocations (alloc.npz: head_sync_allocate, STRATA_KV.py:1308-1351) and the oracle:
choices, cap and bits exactly, including budgets where everything is dropped or kept exact."""

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", list("abcdef"))
def test_allocation_golden(golden, cuda_dev, name):
    import kvb
    g = golden("alloc")
    r = kvb.ops.head_sync_allocate(torch.from_numpy(g[f"{name}_D"]).to(cuda_dev), g[f"{name}_cost"],
                                   g[f"{name}_fixed"], float(g[f"{name}_budget"]))
    np.testing.assert_array_equal(r["choice"].cpu().numpy(), g[f"{name}_choice"])
    assert int(r["cap"]) == int(g[f"{name}_cap"])
    assert float(r["bits"]) == float(g[f"{name}_bits"])


@pytest.mark.parametrize("rounds,grid", [(4, 32), (0, 32), (6, 16)])
def test_allocation_large_matches_oracle(cuda_dev, rounds, grid):
    """32768 rank positions of a config-1-sized layer (8 KV heads, drop | 2 / 4 / 8 bits | exact)."""
    import kvb
    gen = torch.Generator().manual_seed(rounds * 100 + grid)
    n, Hkv, d, bits = 32768, 8, 128, (2, 4, 8)
    imp = torch.sort(torch.exp(1.5 * torch.randn(n, generator=gen)), descending=True).values
    cols = [imp * (2.0 + torch.rand(n, generator=gen))]
    cols += [imp * 4.0 ** (-b) * (0.5 + torch.rand(n, generator=gen)) for b in bits]
    cols.append(torch.zeros(n))
    D = torch.stack(cols, 1).float()
    cost = np.array([0.0] + [2.0 * (b * d + 16) for b in bits] + [2.0 * d * 16], np.float32) * Hkv
    fixed = np.array([160.0] + [160.0 + Hkv * 2 * d * 16.0] * 3, np.float32)
    budget = 0.25 * n * Hkv * 2 * d * 16.0
    choice, cap, tot = O.head_sync_allocate(D.numpy(), cost, fixed, budget, rounds=rounds, grid=grid)
    for _ in range(2):                                     # calls share the workspace: repeatable
        r = kvb.ops.head_sync_allocate(D.to(cuda_dev), cost, fixed, budget, rounds=rounds, grid=grid)
        np.testing.assert_array_equal(r["choice"].cpu().numpy(), choice)
        assert int(r["cap"]) == cap and float(r["bits"]) == tot
    assert kvb.device_status() == 0


def test_allocation_rejects_bad_arguments(cuda_dev):
    import kvb
    D = torch.zeros(10, 9, device=cuda_dev)
    with pytest.raises(ValueError):
        kvb.ops.head_sync_allocate(D, [0.0] * 9, [0.0] * 8, 1.0)          # nlev 9 > 8
    with pytest.raises(ValueError):
        kvb.ops.head_sync_allocate(torch.zeros(10, 5, device=cuda_dev), [0.0] * 5, [0.0] * 4, 1.0, grid=65)
