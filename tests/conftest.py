import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
for path in (ROOT, ROOT / "jittor-flow2surf_b200"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on a B200)")
    config.addinivalue_line("markers", "slow: CPU test that takes more than a few seconds")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return dict(np.load(GOLDEN / f"{name}.npz", allow_pickle=False))
    return load


@pytest.fixture(scope="session")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda:0")


def near_tie_rows(features: np.ndarray, k: int, rel: float = 1e-5) -> np.ndarray:
    """(B, N) mask of queries whose neighbour ranks k-1/k (0-based) are closer
    than `rel` in squared distance, where two correct float32 evaluations of the
    distance may order the boundary differently."""
    f = features.astype(np.float64)
    d = ((f[:, :, :, None] - f[:, :, None, :]) ** 2).sum(1)
    B, N, _ = d.shape
    d[:, np.arange(N), np.arange(N)] = np.inf
    s = np.sort(d, axis=-1)
    ties = np.zeros((B, N), dtype=bool)
    # Adjacent ranks r, r+1 with r+1 <= k among the N-1 finite candidates.
    for r in range(max(0, min(k, N - 2))):
        gap = s[..., r + 1] - s[..., r]
        ties |= gap <= rel * np.maximum(s[..., r + 1], 1e-30)
    return ties
