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


def _grid_cases():
    """Point-set pairs of at least 4096 points each, so that the grid search
    runs, with the distributions that stress it."""
    rng = np.random.default_rng(11)

    def sphere(n, r=1.0):
        v = rng.normal(size=(n, 3))
        return (r * v / np.linalg.norm(v, axis=1, keepdims=True)).astype(np.float32)

    cases = {}
    noisy, _, reference = mesh_cloud(12_000, seed=5, sigma_fraction=0.01, clean_points=15_000)
    cases["surface"] = (noisy[None], reference[None])
    scale = np.array([1.0, 1e-3, 50.0]).reshape(3, 1, 1)  # a different box per item
    cases["cube_batch"] = ((rng.random((3, 6000, 3)) * scale).astype(np.float32),
                           ((rng.random((3, 7000, 3)) * 1.4 - 0.2) * scale).astype(np.float32))
    # most points in one tiny cluster: the item falls back to the plain scan
    cluster = np.concatenate([rng.random((6000, 3)) * 1e-4, rng.random((200, 3)) * 10])
    cases["cluster"] = (cluster[None].astype(np.float32), rng.random((1, 5000, 3)).astype(np.float32))
    # an integer lattice: thousands of exact ties, decided by the index
    cases["lattice"] = (rng.integers(0, 8, (1, 9000, 3)).astype(np.float32),
                        (rng.integers(-1, 9, (1, 6000, 3)) + 0.5 * rng.integers(0, 2, (1, 6000, 3)))
                        .astype(np.float32))
    # small extent far from the origin (the cell-index rounding allowance)
    cases["offset"] = ((rng.random((1, 8000, 3)) * 1e-2 + 1000).astype(np.float32),
                       (rng.random((1, 5000, 3)) * 1.2e-2 + 1000 - 1e-3).astype(np.float32))
    cases["plane"] = (np.c_[rng.random((8000, 2)), np.zeros(8000)][None].astype(np.float32),
                      rng.random((1, 5000, 3)).astype(np.float32))
    # NaN and infinite coordinates in both sets: never a nearest point
    a = rng.random((1, 7000, 3))
    a[rng.random(a.shape) < 0.01] = np.nan
    b = rng.random((1, 6000, 3))
    b[rng.random(b.shape) < 0.01] = np.inf
    b[0, :5] = -np.inf
    cases["nonfinite"] = (a.astype(np.float32), b.astype(np.float32))
    # queries far outside the other set's box
    cases["far"] = (sphere(6000)[None], np.concatenate([sphere(4500, 40.0), sphere(1000)])[None])
    return cases


@pytest.mark.parametrize("name", ["surface", "cube_batch", "cluster", "lattice", "offset", "plane",
                                  "nonfinite", "far"])
def test_nearest_grid_bit_exact(cuda, name):
    """Sets of 4096 points or more take the grid search; it must give the
    plain scan's (distance, index) winners bit for bit, ties and non-finite
    points included."""
    first, second = _grid_cases()[name]
    got = [t.cpu().numpy() for t in nearest_squared_distances(dev(first), dev(second))]
    want = native.nearest_squared_distances(first, second)
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


# ---------------------------------------------------------------------------
# point-to-surface (flow2surf/evaluation.py:31-34)
# ---------------------------------------------------------------------------

def _mesh_points(n, seed, sigma=0.02):
    from flow2surf_b200.synthetic import sample_surface, union_mesh

    v, f = union_mesh(seed)
    rng = np.random.default_rng(seed)
    pts = sample_surface(v, f, n, rng).astype(np.float64) + rng.normal(scale=sigma, size=(n, 3))
    return pts.astype(np.float32), v.astype(np.float32), f.astype(np.int32)


@pytest.mark.gpu
def test_point_to_mesh_matches_oracle(cuda):
    from flow2surf_b200.evaluation import point_to_surface
    from flow2surf_b200.ops import point_to_mesh_distances
    from oracle.inference import closest_point_sq_distances

    pts, v, f = _mesh_points(3000, seed=4)
    # points exactly on vertices and far away too
    pts = np.concatenate([pts, v[:50], np.array([[3.0, -2.0, 1.0]], np.float32)])
    d, fi = point_to_mesh_distances(torch.from_numpy(pts).cuda(), torch.from_numpy(v).cuda(),
                                    torch.from_numpy(f).cuda())
    d, fi = d.cpu().numpy(), fi.cpu().numpy()
    want_d, want_f = closest_point_sq_distances(pts.astype(np.float64), v.astype(np.float64), f)
    np.testing.assert_allclose(d, want_d, rtol=1e-5, atol=2e-7)
    assert np.all(d[3000:3050] < 1e-12)          # on a vertex
    # the face index, except where two faces are equally close (shared
    # vertices and edges)
    assert (fi == want_f).mean() > 0.9
    got = point_to_surface(pts, v, f)
    assert abs(got - want_d.mean()) <= 1e-6 * want_d.mean()


@pytest.mark.gpu
def test_point_to_mesh_100k_sample(cuda):
    """The evaluation size: 100,000 noisy points against the 15,896-face
    synthetic mesh, a sample of 500 points against the float64 oracle."""
    from flow2surf_b200.ops import point_to_mesh_distances
    from oracle.inference import closest_point_sq_distances

    pts, v, f = _mesh_points(100_000, seed=5, sigma=0.015)
    d, _ = point_to_mesh_distances(torch.from_numpy(pts).cuda(), torch.from_numpy(v).cuda(),
                                   torch.from_numpy(f).cuda())
    d = d.cpu().numpy()
    pick = np.random.default_rng(0).choice(len(pts), 500, replace=False)
    want, _ = closest_point_sq_distances(pts[pick].astype(np.float64), v.astype(np.float64), f)
    np.testing.assert_allclose(d[pick], want, rtol=1e-5, atol=2e-7)
    assert np.isfinite(d).all()


@pytest.mark.gpu
def test_point_to_mesh_edge_cases(cuda):
    from flow2surf_b200.ops import point_to_mesh_distances

    t = lambda a, dt=torch.float32: torch.tensor(a, dtype=dt, device="cuda")  # noqa: E731
    tri_v = t([[0, 0, 0], [1, 0, 0], [0, 1, 0]])
    tri_f = t([[0, 1, 2]], torch.int32)
    pts = t([[0.25, 0.25, 2.0], [2, 0, 0], [-1, -1, 0], [0.5, 0.5, 0.0], [0.5, -1, 0]])
    d, fi = point_to_mesh_distances(pts, tri_v, tri_f)
    np.testing.assert_allclose(d.cpu().numpy(), [4.0, 1.0, 2.0, 0.0, 1.0], rtol=0, atol=1e-6)
    assert fi.cpu().numpy().tolist() == [0] * 5
    d0, _ = point_to_mesh_distances(t(np.zeros((0, 3))), tri_v, tri_f)
    assert d0.numel() == 0
    with pytest.raises(ValueError, match="face indices"):
        point_to_mesh_distances(pts, tri_v, t([[0, 1, 3]], torch.int32))
    with pytest.raises(ValueError, match="mesh is empty"):
        point_to_mesh_distances(pts, tri_v, t(np.zeros((0, 3)), torch.int32))
