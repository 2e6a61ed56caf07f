"""Seeded synthetic inputs and random-init weights for the denoising workloads.

There are no ShapeNet meshes or trained checkpoints here, so every workload is
generated from a seed:
  - clouds: area-uniform samples of a unit sphere or of a mesh built from
    random ellipsoids and boxes, normalised to the unit sphere, plus Gaussian
    or rotation-invariant Laplace noise. The sampling, normalisation and noise
    recipes restate the reference's dataset.py:169-196 (sample_surface),
    :199-215 (normalize_points) and :229-260 (add_noise);
  - weights: every parameter of the configured Flow2SurfNet drawn from one
    seeded stream (the reference's own init zeroes the decoder output and the
    AdaLN modulation, so a freshly built model predicts v = 0).
"""

from __future__ import annotations

import math

import numpy as np

from .params import parameter_specs

DEFAULT_CONFIG = {
    "patch_size": 1024,
    "feat_dim": 192,
    "encoder_dims": [64, 128],
    "k_neighbors": 32,
    "num_blocks": 3,
    "alpha_dim": 16,
    "ffn_ratio": 8,
    "decoder_dims": [128, 64],
    "num_steps": 3,
    "alpha_clean_power": 1,
    "alpha_noisy_power": 6,
    "seed_k": 24,
    "patch_agg_beta": 5,
    "inference_chunks": 8,
    "inference_seed": 42,
}
"""The architecture and inference keys of the reference's configs/default.yaml."""


def random_parameters(cfg: dict, seed: int, velocity_scale: float = 0.1) -> dict:
    """All parameters, float32, keyed by the reference's state-dict names.

    Weights U(+-1/sqrt(fan_in)), biases U(+-0.05), norm gains 1 + U(+-0.1),
    norm shifts U(+-0.05); the decoder's output weight is scaled by
    `velocity_scale` so velocities have the magnitude of point noise.
    """
    rng = np.random.default_rng(seed)
    params = {}
    specs = parameter_specs(cfg)
    for name, shape, kind in specs:
        if kind == "weight":
            fan_in = int(np.prod(shape[1:]))
            bound = 1.0 / math.sqrt(fan_in)
            value = rng.uniform(-bound, bound, shape)
        elif kind == "bias":
            value = rng.uniform(-0.05, 0.05, shape)
        elif kind == "norm_weight":
            value = 1.0 + rng.uniform(-0.1, 0.1, shape)
        else:
            value = rng.uniform(-0.05, 0.05, shape)
        params[name] = value.astype(np.float32)
    params[specs[-1][0]] *= np.float32(velocity_scale)
    return params


# ---------------------------------------------------------------------------
# Surfaces
# ---------------------------------------------------------------------------

def _random_rotation(rng) -> np.ndarray:
    q, r = np.linalg.qr(rng.normal(size=(3, 3)))
    q = q * np.sign(np.diag(r))
    if np.linalg.det(q) < 0:
        q[:, 0] = -q[:, 0]
    return q


def ellipsoid_mesh(axes, rotation, center, n_lat=32, n_lon=64):
    """Triangulated ellipsoid (UV sphere scaled by `axes`, rotated, moved)."""
    theta = np.linspace(0.0, np.pi, n_lat + 1)
    phi = np.linspace(0.0, 2.0 * np.pi, n_lon, endpoint=False)
    t, p = np.meshgrid(theta[1:-1], phi, indexing="ij")
    ring = np.stack([np.sin(t) * np.cos(p), np.sin(t) * np.sin(p), np.cos(t)], -1).reshape(-1, 3)
    verts = np.concatenate([[[0.0, 0.0, 1.0]], ring, [[0.0, 0.0, -1.0]]], axis=0)
    faces = []
    top, bottom = 0, len(verts) - 1
    rings = n_lat - 1
    for j in range(n_lon):
        faces.append([top, 1 + j, 1 + (j + 1) % n_lon])
    for i in range(rings - 1):
        a0, b0 = 1 + i * n_lon, 1 + (i + 1) * n_lon
        for j in range(n_lon):
            j1 = (j + 1) % n_lon
            faces.append([a0 + j, b0 + j, b0 + j1])
            faces.append([a0 + j, b0 + j1, a0 + j1])
    last = 1 + (rings - 1) * n_lon
    for j in range(n_lon):
        faces.append([last + j, bottom, last + (j + 1) % n_lon])
    verts = (verts * np.asarray(axes)) @ np.asarray(rotation).T + np.asarray(center)
    return verts, np.asarray(faces, dtype=np.int64)


def box_mesh(extent, rotation, center):
    """Triangulated box with half-extents `extent`."""
    corners = np.array([[x, y, z] for x in (-1, 1) for y in (-1, 1) for z in (-1, 1)], float)
    faces = np.array([
        [0, 1, 3], [0, 3, 2], [4, 6, 7], [4, 7, 5], [0, 4, 5], [0, 5, 1],
        [2, 3, 7], [2, 7, 6], [0, 2, 6], [0, 6, 4], [1, 5, 7], [1, 7, 3]], dtype=np.int64)
    verts = (corners * np.asarray(extent)) @ np.asarray(rotation).T + np.asarray(center)
    return verts, faces


def union_mesh(seed: int, ellipsoids: int = 4, boxes: int = 2):
    """Union (concatenation) of random ellipsoids and boxes."""
    rng = np.random.default_rng(seed)
    verts, faces, offset = [], [], 0
    for _ in range(ellipsoids):
        v, f = ellipsoid_mesh(rng.uniform(0.2, 0.6, 3), _random_rotation(rng),
                              rng.uniform(-0.5, 0.5, 3))
        verts.append(v)
        faces.append(f + offset)
        offset += len(v)
    for _ in range(boxes):
        v, f = box_mesh(rng.uniform(0.1, 0.4, 3), _random_rotation(rng), rng.uniform(-0.5, 0.5, 3))
        verts.append(v)
        faces.append(f + offset)
        offset += len(v)
    return np.concatenate(verts), np.concatenate(faces)


def sample_surface(vertices, faces, num_points, rng) -> np.ndarray:
    """Area-uniform surface samples (restates dataset.py:169-196)."""
    tri = np.asarray(vertices, dtype=np.float64)[faces]
    area = 0.5 * np.linalg.norm(np.cross(tri[:, 1] - tri[:, 0], tri[:, 2] - tri[:, 0]), axis=1)
    cumulative = np.cumsum(area)
    face_idx = np.searchsorted(cumulative, rng.random(num_points) * cumulative[-1])
    origins = tri[:, 0][face_idx]
    vectors = (tri[:, 1:] - tri[:, 0][:, None, :])[face_idx]
    w = rng.random((num_points, 2, 1))
    reflected = w.sum(axis=1).reshape(-1) > 1.0
    w[reflected] = 1.0 - w[reflected]
    return ((vectors * w).sum(axis=1) + origins).astype(np.float32)


def normalize_points(points) -> np.ndarray:
    """(points - bbox centre) / max radius (restates dataset.py:199-215)."""
    points = np.asarray(points, dtype=np.float32)
    lo, hi = points.min(0), points.max(0)
    centered = points - (lo + hi) / 2
    radius = float(np.linalg.norm(centered, axis=1).max())
    return centered / radius


def bbox_diagonal(points) -> float:
    points = np.asarray(points)
    return float(np.linalg.norm(points.max(0) - points.min(0)))


def add_noise(points, noise_std, noise_type, rng) -> np.ndarray:
    """Gaussian or rotation-invariant Laplace noise (restates dataset.py:229-260):
    Laplace = Gamma(3, std/2) radius times a uniform direction."""
    points = np.asarray(points, dtype=np.float32)
    if noise_type == "gaussian":
        noise = rng.normal(0, noise_std, points.shape).astype(np.float32)
    elif noise_type == "laplace":
        d = rng.normal(size=(len(points), 3))
        d /= np.linalg.norm(d, axis=1, keepdims=True)
        radius = rng.gamma(3.0, noise_std / 2.0, size=(len(points), 1))
        noise = (radius * d).astype(np.float32)
    else:
        raise ValueError(f"Unknown noise_type: {noise_type}")
    return points + noise


# ---------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------

def sphere_cloud(num_points: int = 10_000, seed: int = 0, sigma_fraction: float = 0.02):
    """Noisy unit-sphere cloud: area-uniform points (normalised Gaussians) plus
    isotropic Gaussian noise of std sigma_fraction * bbox diagonal.
    Returns (noisy, clean) float32 (N, 3)."""
    rng = np.random.default_rng(seed)
    d = rng.normal(size=(num_points, 3))
    clean = (d / np.linalg.norm(d, axis=1, keepdims=True)).astype(np.float32)
    sigma = sigma_fraction * bbox_diagonal(clean)
    return add_noise(clean, sigma, "gaussian", rng), clean


def mesh_cloud(num_points: int = 50_000, seed: int = 4, sigma_fraction: float = 0.015,
               noise_type: str = "laplace", clean_points: int = 0):
    """Noisy cloud sampled from the random ellipsoid/box union mesh of `seed`.

    Returns (noisy, clean[, clean_reference]) float32; `clean_reference` is an
    independent clean sample of `clean_points` points when that is > 0."""
    verts, faces = union_mesh(seed)
    rng = np.random.default_rng(seed + 1_000_003)
    clean = normalize_points(sample_surface(verts, faces, num_points, rng))
    sigma = sigma_fraction * bbox_diagonal(clean)
    noisy = add_noise(clean, sigma, noise_type, rng)
    if clean_points:
        reference = normalize_points(sample_surface(verts, faces, clean_points, rng))
        return noisy, clean, reference
    return noisy, clean


def knn_patches(batch: int = 256, points: int = 1024, channels: int = 64, seed: int = 2):
    """KNN / edge micro-benchmark input: half the patches uniform in the unit
    cube, half on random ellipsoid surfaces (axes U[0.3, 1], random rotation)
    plus N(0, 0.01^2). Returns xyz (B, 3, N) and features (B, C, N) float32."""
    rng = np.random.default_rng(seed)
    xyz = np.empty((batch, points, 3), dtype=np.float32)
    half = batch // 2
    xyz[:half] = rng.uniform(0.0, 1.0, (half, points, 3))
    for b in range(half, batch):
        d = rng.normal(size=(points, 3))
        d /= np.linalg.norm(d, axis=1, keepdims=True)
        surf = (d * rng.uniform(0.3, 1.0, 3)) @ _random_rotation(rng).T
        xyz[b] = surf + rng.normal(0.0, 0.01, surf.shape)
    features = rng.normal(size=(batch, channels, points)).astype(np.float32)
    return np.ascontiguousarray(xyz.transpose(0, 2, 1)), features


def trunk_activations(batch: int = 512, points: int = 1024, channels: int = 192, seed: int = 1):
    """Trunk micro-benchmark input: x ~ N(0, 1) (B, N, C), alpha ~ U[0, 1]."""
    rng = np.random.default_rng(seed)
    x = rng.normal(size=(batch, points, channels)).astype(np.float32)
    alpha = rng.uniform(0.0, 1.0, batch).astype(np.float32)
    return x, alpha
