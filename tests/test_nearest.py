"""nearest_squared_distances and Chamfer on the GPU against the bit-exact oracle
(flow2surf/training/cuda/nearest_distance_forward.cu, evaluation.py:24-28).
The Chamfer difference bound is 1e-5."""

import numpy as np
import pytest
import torch

from flow2surf_b200.evaluation import chamfer_distance
from flow2surf_b200.ops import chamfer_distances, nearest_squared_distances
from flow2surf_b200.synthetic import mesh_cloud, sphere_cloud
from oracle import inference as oinf
from oracle import native

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("B,M,N", [(2, 300, 257), (1, 1, 1), (3, 1025, 4097), (1, 5000, 3),
                                   (2, 2049, 20000)])
def test_nearest_bit_exact(cuda, B, M, N):
    rng = np.random.default_rng(M + N)
    first = rng.normal(size=(B, M, 3)).astype(np.float32)
    second = rng.normal(size=(B, N, 3)).astype(np.float32)
    got = [t.cpu().numpy() for t in nearest_squared_distances(dev(first), dev(second))]
    want = native.nearest_squared_distances(first, second)
    for g, w in zip(got, want):
        np.testing.assert_array_equal(g, w)


def test_nearest_ties_and_duplicates(cuda):
    rng = np.random.default_rng(3)
    grid = rng.integers(0, 3, size=(2, 700, 3)).astype(np.float32)   # many equal distances
    other = rng.integers(0, 3, size=(2, 2500, 3)).astype(np.float32)
    got = [t.cpu().numpy() for t in nearest_squared_distances(dev(grid), dev(other))]
    want = native.nearest_squared_distances(grid, other)
    for g, w in zip(got, want):
        np.testing.assert_array_equal(g, w)


def test_nearest_reference_golden(cuda, golden):
    fix = golden("nearest")
    d1, i2, d2, i1 = [t.cpu().numpy() for t in
                      nearest_squared_distances(dev(fix["first"]), dev(fix["second"]))]
    np.testing.assert_allclose(d1, fix["d1"], rtol=0, atol=1e-5)
    np.testing.assert_array_equal(i2, fix["i2"])
    np.testing.assert_allclose(d2, fix["d2"], rtol=0, atol=1e-5)
    np.testing.assert_array_equal(i1, fix["i1"])


def test_chamfer_reference_golden(cuda, golden):
    fix = golden("nearest")
    got = chamfer_distance(fix["pred"], fix["target"])
    assert abs(got - float(fix["chamfer"])) < 1e-5


def test_chamfer_full_size_cloud(cuda):
    """A 100k-point denoised-size cloud against its 100k clean sample."""
    noisy, clean, reference = mesh_cloud(100_000, seed=100, sigma_fraction=0.01,
                                         clean_points=100_000)
    got = chamfer_distances(dev(noisy)[None], dev(reference)[None])[0].item()
    want = oinf.chamfer_distance(noisy, reference)
    assert abs(got - want) < 1e-5
    assert abs(got - want) / want < 1e-5


def test_nearest_errors(cuda):
    with pytest.raises(ValueError, match="first shaped"):
        nearest_squared_distances(torch.zeros(2, 4, 2, device="cuda"),
                                  torch.zeros(2, 4, 3, device="cuda"))
    with pytest.raises(ValueError, match="Batch sizes differ"):
        nearest_squared_distances(torch.zeros(2, 4, 3, device="cuda"),
                                  torch.zeros(3, 4, 3, device="cuda"))
    with pytest.raises(ValueError, match="nonempty"):
        nearest_squared_distances(torch.zeros(2, 0, 3, device="cuda"),
                                  torch.zeros(2, 4, 3, device="cuda"))
