"""ORACLE (test infrastructure): NumPy/SciPy restatement of patch_denoise.

Follows flow2surf/inference.py:12-198 and flow2surf/flow.py:24-52, with the
model call replaced by any callable `model(x (B, 3, M) f32, alpha (B,) f32)
-> (B, M, 3)` (normally oracle.model.OracleNet). FPS uses the bit-exact C
restatement; the patch index uses scipy's cKDTree exactly as the reference.
"""

from __future__ import annotations

import hashlib

import numpy as np
from scipy.spatial import cKDTree

from . import native


def make_rng(seed, *parts):
    """flow2surf/inference.py:12-16."""
    key = "::".join([str(seed), *map(str, parts)]).encode("utf-8")
    digest = hashlib.blake2b(key, digest_size=8).digest()
    return np.random.default_rng(int.from_bytes(digest, "little") % (2**32))


def alpha_schedule(num_steps, clean_power, noisy_power):
    """flow2surf/flow.py:24-52."""
    num_steps = int(num_steps)
    if num_steps < 1:
        raise ValueError("num_steps must be >= 1")
    s = np.arange(1, num_steps + 1, dtype=np.float64) / num_steps
    clean_term = s ** float(clean_power)
    noisy_term = (1.0 - s) ** float(noisy_power)
    alpha = (clean_term / (clean_term + noisy_term)).astype(np.float32)
    if not np.isfinite(alpha).all() or alpha[0] <= 0 or np.any(np.diff(alpha) <= 0):
        raise ValueError("schedule parameters must produce strictly increasing positive "
                         "float32 levels")
    return alpha


def patch_seed_count(num_points, patch_size, seed_k):
    """flow2surf/inference.py:44-59."""
    num_points, patch_size, seed_k = int(num_points), int(patch_size), int(seed_k)
    effective = min(patch_size, num_points)
    return min(num_points, max(1, int(seed_k * num_points / effective)))


def patch_seed_indices(points, patch_size, seed_k, rng):
    """flow2surf/inference.py:62-65 with the C FPS (first index rng.integers(N))."""
    count = patch_seed_count(len(points), patch_size, seed_k)
    first = rng.integers(len(points))
    return native.farthest_point_indices(points, count, first)


def build_patch_index(points, seed_idx, patch_size):
    """flow2surf/inference.py:110-122."""
    tree = cKDTree(points)
    distances, neighbor_idx = tree.query(points[seed_idx], k=patch_size, workers=-1)
    if patch_size == 1:
        distances, neighbor_idx = distances[:, None], neighbor_idx[:, None]
    return neighbor_idx, distances / (distances[:, -1:] + 1e-8)


def build_aggregation(neighbor_idx, radial, beta, num_points):
    """flow2surf/inference.py:124-134."""
    point_idx = neighbor_idx.reshape(-1)
    r = radial.reshape(-1)
    weights = np.exp(-beta * r * r)
    weight_sum = np.bincount(point_idx, weights=weights, minlength=num_points)
    return point_idx, weights, weight_sum, weight_sum == 0


def predict_velocity(model, points, neighbor_idx, seed_idx, alpha_value, chunk_size):
    """flow2surf/inference.py:141-153: per-patch velocities (P, M, 3) f32."""
    patches = points[neighbor_idx]
    votes = np.zeros_like(patches)
    for start in range(0, len(seed_idx), chunk_size):
        batch = patches[start:start + chunk_size]
        centers = points[seed_idx[start:start + len(batch)]][:, None, :]
        x = np.ascontiguousarray((batch - centers).transpose(0, 2, 1), dtype=np.float32)
        alpha = np.full((len(batch),), alpha_value, dtype=np.float32)
        votes[start:start + len(batch)] = model(x, alpha)
    return votes


def aggregate_votes(votes, point_idx, weights, weight_sum, num_points):
    """flow2surf/inference.py:158-171."""
    flat = votes.reshape(-1, 3)
    velocity_sum = np.stack([np.bincount(point_idx, weights=weights * flat[:, c],
                                         minlength=num_points) for c in range(3)], axis=1)
    return (velocity_sum / (weight_sum[:, None] + 1e-8)).astype(np.float32)


def euler_update(current, velocity, alpha_step, uncovered):
    """flow2surf/inference.py:193-196 (float32 array times a Python float)."""
    updated = current - np.float32(alpha_step) * velocity
    if uncovered.any():
        updated[uncovered] = current[uncovered]
    return updated


def patch_denoise(model, pc_noisy, patch_size, seed_k, num_steps, num_chunks, rng=None,
                  patch_seed_idx=None, patch_agg_beta=4.0, alpha_clean_power=1.0,
                  alpha_noisy_power=1.0, trace=None):
    """flow2surf/inference.py:68-198. `trace`, if a list, receives per step
    (alpha, step input, votes, fused velocity, step output)."""
    if rng is None:
        rng = np.random.default_rng(0)
    num_points = pc_noisy.shape[0]
    if num_chunks < 1:
        raise ValueError(f"num_chunks must be >= 1, got {num_chunks}")
    patch_size = min(patch_size, num_points)
    num_patches = patch_seed_count(num_points, patch_size, seed_k)
    if patch_seed_idx is None:
        seed_idx = patch_seed_indices(pc_noisy, patch_size, seed_k, rng)
    else:
        seed_idx = np.asarray(patch_seed_idx, dtype=np.int64)
    chunk_size = (num_patches + num_chunks - 1) // num_chunks
    neighbor_idx, radial = build_patch_index(pc_noisy, seed_idx, patch_size)
    point_idx, weights, weight_sum, uncovered = build_aggregation(
        neighbor_idx, radial, patch_agg_beta, num_points)
    alphas = alpha_schedule(num_steps, alpha_clean_power, alpha_noisy_power)
    current = pc_noisy.copy()
    for step in range(num_steps - 1, -1, -1):
        alpha_current = float(alphas[step])
        alpha_previous = float(alphas[step - 1]) if step > 0 else 0.0
        votes = predict_velocity(model, current, neighbor_idx, seed_idx, alpha_current,
                                 chunk_size)
        velocity = aggregate_votes(votes, point_idx, weights, weight_sum, num_points)
        updated = euler_update(current, velocity, alpha_current - alpha_previous, uncovered)
        if trace is not None:
            trace.append((alpha_current, current, votes, velocity, updated))
        current = updated
    return current.astype(np.float32)


def chamfer_distance(pred, target):
    """flow2surf/evaluation.py:24-28."""
    a, _ = cKDTree(target).query(pred, workers=-1)
    b, _ = cKDTree(pred).query(target, workers=-1)
    return float((a ** 2).mean() + (b ** 2).mean())


def closest_point_sq_distances(points, vertices, faces, chunk=256):
    """Squared distance from each point to a triangle mesh and the closest face
    (ties to the smaller index), float64: the quantity point_cloud_utils'
    closest_points_on_mesh gives for flow2surf/evaluation.py:31-34, restated
    from the region tests of Ericson, Real-Time Collision Detection (2005),
    sec. 5.1.5 (vertex a, vertex b, edge ab, vertex c, edge ac, edge bc, face,
    the first region that holds)."""
    p_all = np.asarray(points, dtype=np.float64)
    tri = np.asarray(vertices, dtype=np.float64)[np.asarray(faces)]
    a, b, c = tri[:, 0], tri[:, 1], tri[:, 2]
    ab, ac = b - a, c - a
    out_d = np.empty(len(p_all))
    out_f = np.empty(len(p_all), dtype=np.int64)
    for s in range(0, len(p_all), chunk):
        p = p_all[s:s + chunk, None, :]                       # (P, 1, 3)
        ap, bp, cp = p - a, p - b, p - c
        d1, d2 = (ab * ap).sum(-1), (ac * ap).sum(-1)
        d3, d4 = (ab * bp).sum(-1), (ac * bp).sum(-1)
        d5, d6 = (ab * cp).sum(-1), (ac * cp).sum(-1)
        vc, vb, va = d1 * d4 - d3 * d2, d5 * d2 - d1 * d6, d3 * d6 - d5 * d4
        with np.errstate(divide="ignore", invalid="ignore"):
            denom = va + vb + vc
            v, w = vb / denom, vc / denom                     # face
            e43, e56 = d4 - d3, d5 - d6
            regions = [                                        # lowest precedence first
                ((va <= 0) & (e43 >= 0) & (e56 >= 0), 1 - e43 / (e43 + e56), e43 / (e43 + e56)),
                ((vb <= 0) & (d2 >= 0) & (d6 <= 0), 0.0, d2 / (d2 - d6)),
                ((d6 >= 0) & (d5 <= d6), 0.0, 1.0),
                ((vc <= 0) & (d1 >= 0) & (d3 <= 0), d1 / (d1 - d3), 0.0),
                ((d3 >= 0) & (d4 <= d3), 1.0, 0.0),
                ((d1 <= 0) & (d2 <= 0), 0.0, 0.0),
            ]
            for cond, rv, rw in regions:
                v = np.where(cond, rv, v)
                w = np.where(cond, rw, w)
        q = a + v[..., None] * ab + w[..., None] * ac
        d = ((p - q) ** 2).sum(-1)
        out_f[s:s + chunk] = d.argmin(1)
        out_d[s:s + chunk] = d.min(1)
    return out_d, out_f


def point_to_surface(points, vertices, faces):
    """flow2surf/evaluation.py:31-34: mean squared point-to-mesh distance."""
    return float(closest_point_sq_distances(points, vertices, faces)[0].mean())
