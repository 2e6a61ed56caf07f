"""The point-to-mesh oracle (oracle/inference.py: Ericson's region tests, for
flow2surf/evaluation.py:31-34) against an independent exact formulation: the
plane projection when it falls inside the triangle, else the nearest of the
three edge segments. point_cloud_utils (which the reference calls) is not
installed, so this pins the restatement."""

import numpy as np

from flow2surf_b200.synthetic import union_mesh
from oracle.inference import closest_point_sq_distances, point_to_surface


def segment_sq(p, a, b):
    ab = b - a
    t = np.clip(((p - a) * ab).sum(-1) / (ab * ab).sum(-1), 0.0, 1.0)
    return ((p - (a + t[..., None] * ab)) ** 2).sum(-1)


def reference_sq(points, vertices, faces):
    tri = vertices[faces]
    a, b, c = tri[:, 0], tri[:, 1], tri[:, 2]
    n = np.cross(b - a, c - a)
    n = n / np.linalg.norm(n, axis=1, keepdims=True)
    out = np.empty(len(points))
    for i, p in enumerate(points):
        h = ((p - a) * n).sum(-1)
        proj = p - h[:, None] * n
        # inside test: same-side signs of the three edge cross products
        s0 = (np.cross(b - a, proj - a) * n).sum(-1)
        s1 = (np.cross(c - b, proj - b) * n).sum(-1)
        s2 = (np.cross(a - c, proj - c) * n).sum(-1)
        inside = (s0 >= 0) & (s1 >= 0) & (s2 >= 0)
        edge = np.minimum(np.minimum(segment_sq(p, a, b), segment_sq(p, b, c)), segment_sq(p, c, a))
        out[i] = np.where(inside, h * h, edge).min()
    return out


def test_point_to_mesh_oracle_matches_exact_projection():
    v, f = union_mesh(4)
    rng = np.random.default_rng(0)
    pts = v[rng.choice(len(v), 100)] + rng.normal(scale=0.05, size=(100, 3))
    pts = np.concatenate([pts, rng.uniform(-1.5, 1.5, size=(20, 3))])  # far points too
    d, fi = closest_point_sq_distances(pts, v, f)
    want = reference_sq(pts, v, f)
    np.testing.assert_allclose(d, want, rtol=1e-9, atol=1e-14)
    assert fi.min() >= 0 and fi.max() < len(f)
    assert abs(point_to_surface(pts, v, f) - want.mean()) < 1e-12
