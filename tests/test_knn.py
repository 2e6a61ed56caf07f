"""knn_indices on the GPU against the bit-exact oracle
(flow2surf/models/ops/knn.py:35-66, flow2surf/models/ops/cuda/knn_global.cu)."""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from flow2surf_b200 import knn_indices
from flow2surf_b200.synthetic import knn_patches
from oracle import native

pytestmark = pytest.mark.gpu


def run(features: np.ndarray, k: int) -> np.ndarray:
    out = knn_indices(torch.from_numpy(features).cuda(), k)
    return out.cpu().numpy()


@pytest.mark.parametrize("k", [16, 32])
def test_knn_microbench_input_bit_exact(cuda, k):
    """The KNN micro-benchmark input (256 patches x 1024 points: uniform cube
    and noisy ellipsoid surfaces), every index identical to the oracle."""
    xyz, _ = knn_patches(256, 1024, 64, seed=2)
    np.testing.assert_array_equal(run(xyz, k), native.knn(xyz, k))


@pytest.mark.parametrize("n,k", [(2, 1), (2, 5), (3, 2), (5, 8), (31, 30), (33, 32),
                                 (64, 16), (100, 7), (257, 32), (1000, 16), (1025, 32),
                                 (2048, 32)])
def test_knn_sizes(cuda, n, k):
    rng = np.random.default_rng(n * 100 + k)
    xyz = rng.normal(size=(3, 3, n)).astype(np.float32)
    np.testing.assert_array_equal(run(xyz, k), native.knn(xyz, k))


@pytest.mark.parametrize("c", [1, 2, 5, 24])
def test_knn_general_channels(cuda, c):
    rng = np.random.default_rng(c)
    f = rng.normal(size=(2, c, 1000)).astype(np.float32)
    np.testing.assert_array_equal(run(f, 20), native.knn(f, 20))


def test_knn_ties_duplicates_and_quantised(cuda):
    rng = np.random.default_rng(5)
    grid = rng.integers(0, 4, size=(4, 3, 512)).astype(np.float32)   # many exact ties
    np.testing.assert_array_equal(run(grid, 32), native.knn(grid, 32))
    same = np.zeros((1, 3, 64), dtype=np.float32)
    np.testing.assert_array_equal(run(same, 10), native.knn(same, 10))
    signed_zero = np.zeros((1, 3, 40), dtype=np.float32)
    signed_zero[0, :, ::2] = -0.0
    np.testing.assert_array_equal(run(signed_zero, 7), native.knn(signed_zero, 7))


def test_knn_degenerate(cuda):
    one = np.ones((3, 3, 1), dtype=np.float32)
    assert np.all(run(one, 4) == 0) and run(one, 4).shape == (3, 1, 4)
    empty = knn_indices(torch.zeros((0, 3, 16), device="cuda"), 4)
    assert empty.shape == (0, 16, 4)


def test_knn_limits_raise(cuda):
    with pytest.raises(ValueError):
        knn_indices(torch.zeros((1, 3, 16), device="cuda"), 33)
    with pytest.raises(ValueError):
        knn_indices(torch.zeros((1, 3, 4096), device="cuda"), 8)


REF_KNN = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libref_knn.so"


def reference_kernel_knn(features: np.ndarray, k: int) -> np.ndarray:
    """The reference's own global_knn (knn_global.cu, built from its sources by
    oracle/build_ref.py) on the same input."""
    lib = ctypes.CDLL(str(REF_KNN))
    lib.ref_global_knn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_void_p, ctypes.c_int]
    B, C, N = features.shape
    x = torch.from_numpy(np.ascontiguousarray(features)).cuda()
    out = torch.empty((B, N, k), dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    assert lib.ref_global_knn(x.data_ptr(), B, C, N, out.data_ptr(), k) == 0
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.skipif(not REF_KNN.exists(), reason="reference KNN kernel not built (no reference checkout)")
@pytest.mark.parametrize("k", [16, 32])
def test_knn_matches_reference_kernel_microbench(cuda, k):
    """Bit-exact against the reference's own kernel on the KNN micro-benchmark
    input (256 patches x 1024 points: uniform cube and noisy ellipsoid
    surfaces), and the oracle with it."""
    xyz, _ = knn_patches(256, 1024, 64, seed=2)
    want = reference_kernel_knn(xyz, k)
    np.testing.assert_array_equal(run(xyz, k), want)
    np.testing.assert_array_equal(native.knn(xyz, k), want)


@pytest.mark.skipif(not REF_KNN.exists(), reason="reference KNN kernel not built (no reference checkout)")
@pytest.mark.parametrize("b,c,n,k", [(3, 3, 1000, 16), (2, 3, 33, 32), (4, 5, 257, 8),
                                     (2, 3, 2, 1), (1, 24, 600, 20)])
def test_knn_matches_reference_kernel_shapes(cuda, b, c, n, k):
    rng = np.random.default_rng(b * 1000 + n)
    xyz = rng.normal(size=(b, c, n)).astype(np.float32)
    xyz[:, :, 1] = xyz[:, :, 0]           # a duplicate point: a zero distance
    np.testing.assert_array_equal(run(xyz, k), reference_kernel_knn(xyz, k))
