"""The head-synchronous rate allocator of the oracle (head_sync_allocate, STRATA_KV.py:1308-1351)
against the reference's own allocations (alloc.npz): choices, cap and bits exactly, at budgets from
"drop everything" to "everything exact", with 3, 2 and no coded levels.  CPU only."""

import numpy as np
import pytest

import oracle as O
from oracle.alloc import linspace_torch


def test_linspace_steps_are_torchs(golden):
    g = golden("alloc")
    np.testing.assert_array_equal(linspace_torch(32).view(np.int32), g["linspace32"].view(np.int32))


@pytest.mark.parametrize("name", list("abcdef"))
def test_head_sync_allocate_golden(golden, name):
    g = golden("alloc")
    choice, cap, bits = O.head_sync_allocate(g[f"{name}_D"], g[f"{name}_cost"], g[f"{name}_fixed"],
                                             float(g[f"{name}_budget"]))
    np.testing.assert_array_equal(choice, g[f"{name}_choice"])
    assert cap == int(g[f"{name}_cap"])
    assert bits == float(g[f"{name}_bits"])
    assert bits <= float(g[f"{name}_budget"]) or np.all(choice == 0)
