"""Custom operators with the reference's Python surface, backed by sm_100a kernels.

Mirrors flow2surf/models/ops/__init__.py:3-11 and
flow2surf/training/distances.py:70-98: same names, argument meaning, shape
checks and ValueError messages. Tensors are torch CUDA tensors; there is no
CPU path -- a CPU tensor or a missing library raises.
"""

from __future__ import annotations

import torch

from . import _lib


def _require_cuda(*tensors):
    for t in tensors:
        if not t.is_cuda:
            raise ValueError("flow2surf_b200 operators take CUDA tensors (no CPU path)")


def _f32(t):
    if t.dtype != torch.float32:
        raise ValueError(f"expected float32, got {t.dtype}")
    return t.contiguous()


def knn_indices(features: torch.Tensor, k: int) -> torch.Tensor:
    """Find k nearest non-self neighbors in feature space.

    features : (B, C, N) float32
    output   : (B, N, k) int32

    flow2surf/models/ops/knn.py:55-86: k < 1 raises; N <= 1 gives zeros; when
    k > N-1 the last real neighbour is repeated. Ties are broken by the lower
    index and distances are the reference kernel's fp32 expression bit for bit.
    """
    if features.dim() != 3:
        raise ValueError(f"features must be (B, C, N), got {tuple(features.shape)}")
    batch, channels, points = features.shape
    if k < 1:
        raise ValueError(f"k must be >= 1, got {k}")
    _require_cuda(features)
    out = torch.empty((batch, points, k), dtype=torch.int32, device=features.device)
    if out.numel() == 0:
        return out
    features = _f32(features)
    _lib.call("f2s_knn", _lib.ptr(features), batch, channels, points, k, _lib.ptr(out),
              _lib.stream_handle())
    return out
