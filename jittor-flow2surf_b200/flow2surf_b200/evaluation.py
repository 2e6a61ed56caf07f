"""Full-cloud metric on the GPU (flow2surf/evaluation.py:24-28)."""

from __future__ import annotations

import numpy as np
import torch

from .ops import chamfer_distances


def chamfer_distance(pred, target) -> float:
    """Bidirectional squared Chamfer distance between two (N, 3) clouds (host
    arrays or CUDA tensors): mean nearest squared distance both ways."""
    def dev(a):
        if isinstance(a, torch.Tensor):
            return a.to(device="cuda", dtype=torch.float32)
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()

    return float(chamfer_distances(dev(pred)[None], dev(target)[None])[0].item())
