"""f2s_chamfer_static: the Chamfer entry point that allocates nothing.

Some callers cannot call cudaMalloc (an out-of-memory handler, a host that
forbids device allocation once running, work that must not synchronise the
device), so this variant keeps its scratch in a built-in device array instead
of a caller workspace. It must give what f2s_chamfer gives, bit for bit (both
take the lexicographic minimum of (distance, index): this entry by the plain
scan, f2s_chamfer by the grid search once both sets hold 4096 points or
more), and once a device has been set up by a
first call it must not change the device memory in use. This file sorts
last so that, if it fails, a run that stops at the first failure has already
run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from flow2surf_b200 import _lib
from flow2surf_b200.synthetic import mesh_cloud

STATIC_MAX_POINTS = 1 << 21


def with_workspace(pred, target):
    B, M, _ = pred.shape
    N = target.shape[1]
    size = ctypes.c_size_t()
    _lib.check(_lib.lib().f2s_nearest_workspace_bytes(B, M, N, ctypes.byref(size)))
    ws = torch.empty(size.value, dtype=torch.uint8, device="cuda")
    out = torch.empty(B, dtype=torch.float64, device="cuda")
    _lib.call("f2s_chamfer", pred.data_ptr(), target.data_ptr(), B, M, N, out.data_ptr(),
              ws.data_ptr(), ws.numel(), _lib.stream_handle())
    return out.cpu().numpy()


def without_allocation(pred, target, out):
    B, M, _ = pred.shape
    N = target.shape[1]
    _lib.call("f2s_chamfer_static", pred.data_ptr(), target.data_ptr(), B, M, N,
              out.data_ptr(), _lib.stream_handle())
    return out.cpu().numpy()


def set_up_device(out):
    """The B = 0 call: only the per-device set-up (module load, scratch address)."""
    one = torch.zeros((1, 1, 3), device="cuda")
    _lib.call("f2s_chamfer_static", one.data_ptr(), one.data_ptr(), 0, 1, 1, out.data_ptr(),
              _lib.stream_handle())


@pytest.mark.gpu
def test_chamfer_static_matches_workspace_entry_twice(cuda):
    out = torch.empty(4, dtype=torch.float64, device="cuda")
    set_up_device(out)
    rng = np.random.default_rng(0)
    # first call: four 30k/25k pairs; second call: two larger, differently
    # shaped pairs, so stale keys of the first call would show up if not reset
    first_pred = torch.from_numpy(rng.normal(size=(4, 30_000, 3)).astype(np.float32)).cuda()
    first_target = torch.from_numpy(rng.normal(size=(4, 25_000, 3)).astype(np.float32)).cuda()
    clouds = [mesh_cloud(100_000, seed=s, sigma_fraction=0.01, clean_points=90_000)
              for s in (100, 101)]
    second_pred = torch.from_numpy(np.stack([c[0] for c in clouds])).cuda()
    second_target = torch.from_numpy(np.stack([c[2] for c in clouds])).cuda()
    for pred, target in ((first_pred, first_target), (second_pred, second_target)):
        got = without_allocation(pred, target, out[:pred.shape[0]])
        want = with_workspace(pred, target)
        np.testing.assert_array_equal(got, want)
        assert np.all(want > 0)


@pytest.mark.gpu
def test_chamfer_static_allocates_nothing_after_set_up(cuda):
    rng = np.random.default_rng(1)
    pred = torch.from_numpy(rng.normal(size=(2, 20_000, 3)).astype(np.float32)).cuda()
    target = torch.from_numpy(rng.normal(size=(2, 15_000, 3)).astype(np.float32)).cuda()
    out = torch.empty(2, dtype=torch.float64, device="cuda")
    set_up_device(out)
    B, M, N = 2, 20_000, 15_000
    call = lambda: _lib.call("f2s_chamfer_static", pred.data_ptr(), target.data_ptr(), B, M, N,
                             out.data_ptr(), _lib.stream_handle())
    call()
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    allocated_before = torch.cuda.memory_allocated()
    call()
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_allocated() == allocated_before
    assert free_after == free_before
    np.testing.assert_array_equal(out.cpu().numpy(), with_workspace(pred, target))


@pytest.mark.gpu
def test_chamfer_static_rejects_sizes_beyond_its_scratch(cuda):
    points = torch.zeros((1, STATIC_MAX_POINTS, 3), device="cuda")
    out = torch.empty(1, dtype=torch.float64, device="cuda")
    status = _lib.lib().f2s_chamfer_static(points.data_ptr(), points.data_ptr(), 1,
                                           STATIC_MAX_POINTS, 1, out.data_ptr(),
                                           _lib.stream_handle())
    assert status == _lib.F2S_ERR_UNSUPPORTED
    assert b"exceed the built-in scratch" in _lib.lib().f2s_last_error()
