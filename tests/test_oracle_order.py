"""The two float32 reduction orders the oracle restates from the reference's third-party library
(PyTorch's CPU float32 row sum behind ``Y.pow(2).mean(-1)``, STRATA_KV.py:1166 / HEDGE_KV.py:1119;
MKL's sgemm behind ``x @ R.T``, HEDGE_KV.py:1113), pinned against torch's own CPU ops on this host,
and the d = 128 mid-rise fixture (``midrise128.npz``, made by the reference's ``strata_quantize``).
CPU only."""

import numpy as np
import pytest
import torch

import oracle as O
from oracle import codecs as C


@pytest.mark.parametrize("n", [1, 3, 5, 7, 8, 12, 32, 40, 64, 100, 128, 256, 480])
def test_row_sum_order_is_torch_cpu(n):
    x = (np.random.default_rng(n).standard_normal((4000, n)).astype(np.float32) ** 2).astype(np.float32)
    got = C.sum_f32_torch(x)
    ref = torch.from_numpy(x).sum(-1).numpy()
    np.testing.assert_array_equal(got.view(np.int32), ref.view(np.int32))


@pytest.mark.parametrize("shape", [(3, 5, 300, 128), (2, 700, 32), (1, 1, 9, 64)])
def test_mean_of_squares_is_torch_cpu(shape):
    y = torch.randn(*shape, generator=torch.Generator().manual_seed(sum(shape)))
    ref = y.pow(2).mean(-1, keepdim=True).numpy()
    np.testing.assert_array_equal(C.mean_sq_f32(y.numpy()).view(np.int32), ref.view(np.int32))


def test_fma_is_correctly_rounded():
    """Crafted cases where rounding a float64 a * b + c to float32 rounds twice the wrong way."""
    a = np.array([64 * (1 + 2 ** -12), -64 * (1 + 2 ** -12), 64 * (1 - 2 ** -12), 3.0], np.float32)
    b = np.array([1 - 2 ** -12 + 2 ** -24, 1 - 2 ** -12 + 2 ** -24, 1 + 2 ** -12 + 2 ** -24, 0.5], np.float32)
    c = np.array([2.0 ** 30, -(2.0 ** 30), 2.0 ** 30, 1.0], np.float32)
    np.testing.assert_array_equal(C.fma_f32(a, b, c) - c, np.array([128, -128, 0, 1.5], np.float32))


@pytest.mark.parametrize("rows", [7, 48, 300])
def test_rotation_order_is_torch_cpu_matmul(rows):
    g = np.random.default_rng(rows)
    x = g.standard_normal((rows, 128)).astype(np.float32)
    R = O.rotation_matrix(128, "layer0").astype(np.float32)
    ref = (torch.from_numpy(x) @ torch.from_numpy(R).T).numpy()
    np.testing.assert_array_equal(C.matmul_fma(x, R).view(np.int32), ref.view(np.int32))


@pytest.mark.parametrize("tag", ["bf", "h"])
@pytest.mark.parametrize("b", [2, 4, 8])
def test_midrise128_golden(golden, tag, b):
    g = golden("midrise128")
    c, s, yh = O.strata_quantize(g[f"{tag}_y"], b)
    np.testing.assert_array_equal(s, g[f"{tag}{b}_s"])
    np.testing.assert_array_equal(c, g[f"{tag}{b}_codes"])
    if b == 2:
        np.testing.assert_array_equal(yh, g[f"{tag}{b}_yhat"])
