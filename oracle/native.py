"""ORACLE (test infrastructure): ctypes bindings of oracle/oracle.c.

Bit-exact CPU restatements of the reference's index-producing kernels.
"""

from __future__ import annotations

import ctypes

import numpy as np

from .build import build

_LIB = None

# Contraction of `dx*dx + dy*dy + dz*dz` in the reference's nearest-distance
# kernel (flow2surf/training/cuda/nearest_distance_forward.cu:29) under nvcc's
# default -fmad=true: fmaf(dz, dz, fmaf(dx, dx, dy*dy)).
NEAREST_CONTRACTION = 0


def lib():
    global _LIB
    if _LIB is None:
        _LIB = ctypes.CDLL(str(build()))
        i64, p = ctypes.c_int64, ctypes.c_void_p
        _LIB.oracle_knn.argtypes = [p, i64, i64, i64, i64, p]
        _LIB.oracle_nearest_one_way.argtypes = [p, p, i64, i64, i64, ctypes.c_int, p, p]
        _LIB.oracle_fps.argtypes = [p, i64, i64, i64, p]
    return _LIB


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def knn(features: np.ndarray, k: int) -> np.ndarray:
    """knn_indices restated (flow2surf/models/ops/knn.py:35-66 + knn_global.cu).

    features (B, C, N) float32 -> (B, N, k) int32.
    """
    f = np.ascontiguousarray(features, dtype=np.float32)
    B, C, N = f.shape
    if k < 1:
        raise ValueError(f"k must be >= 1, got {k}")
    out = np.empty((B, N, k), dtype=np.int32)
    lib().oracle_knn(_ptr(f), B, C, N, k, _ptr(out))
    return out


def nearest_one_way(query: np.ndarray, points: np.ndarray, mode: int = NEAREST_CONTRACTION):
    """One direction of nearest_first/nearest_second (nearest_distance_forward.cu)."""
    q = np.ascontiguousarray(query, dtype=np.float32)
    p = np.ascontiguousarray(points, dtype=np.float32)
    B, M, _ = q.shape
    N = p.shape[1]
    dist = np.empty((B, M), dtype=np.float32)
    index = np.empty((B, M), dtype=np.int32)
    lib().oracle_nearest_one_way(_ptr(q), _ptr(p), B, M, N, mode, _ptr(dist), _ptr(index))
    return dist, index


def nearest_squared_distances(first: np.ndarray, second: np.ndarray,
                              mode: int = NEAREST_CONTRACTION):
    """flow2surf/training/distances.py:70-87 CUDA semantics.

    Returns (first_distance (B, M), second_index (B, M), second_distance (B, N),
    first_index (B, N)).
    """
    d1, i2 = nearest_one_way(first, second, mode)
    d2, i1 = nearest_one_way(second, first, mode)
    return d1, i2, d2, i1


def farthest_point_indices(points: np.ndarray, count: int, first: int) -> np.ndarray:
    """_farthest_point_indices (flow2surf/inference.py:19-41) with the first
    index already drawn (`rng.integers(N)`, :23)."""
    p = np.ascontiguousarray(points, dtype=np.float32)
    out = np.empty(count, dtype=np.int64)
    lib().oracle_fps(_ptr(p), p.shape[0], count, int(first), _ptr(out))
    return out
