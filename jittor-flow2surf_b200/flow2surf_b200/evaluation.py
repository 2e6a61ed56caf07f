"""Full-cloud metrics on the GPU (flow2surf/evaluation.py:24-34)."""

from __future__ import annotations

import numpy as np
import torch

from .ops import chamfer_distances, point_to_mesh_distances


def _dev(a, dtype=torch.float32):
    if isinstance(a, torch.Tensor):
        return a.to(device="cuda", dtype=dtype)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device="cuda", dtype=dtype)


def chamfer_distance(pred, target) -> float:
    """Bidirectional squared Chamfer distance between two (N, 3) clouds (host
    arrays or CUDA tensors): mean nearest squared distance both ways."""
    return float(chamfer_distances(_dev(pred)[None], _dev(target)[None])[0].item())


def point_to_surface(points, vertices, faces) -> float:
    """Mean squared point-to-triangle-mesh distance (flow2surf/evaluation.py:31-34):
    points (M, 3), vertices (V, 3), faces (F, 3), host arrays or CUDA tensors.
    The per-point squared distances come from the GPU in float32; their mean
    is taken in float64."""
    sq, _ = point_to_mesh_distances(_dev(points), _dev(vertices), _dev(faces, torch.int32))
    return float(sq.double().mean().item())
