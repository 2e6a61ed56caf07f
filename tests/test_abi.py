"""The C-ABI library loads and exports every entry point the header declares.

No compute calls: these run without a GPU.
"""

import re
from pathlib import Path

import pytest

from flow2surf_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "flow2surf_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(f2s_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "f2s_knn" in names and "f2s_last_error" in names


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"


def test_python_signatures_cover_header():
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_version_and_error_without_gpu():
    lib = _lib.lib()
    assert lib.f2s_version() >= 100
    assert isinstance(lib.f2s_last_error(), bytes)


def test_invalid_arguments_fail_before_any_device_work():
    """Argument validation happens on the host and needs no GPU."""
    lib = _lib.lib()
    assert lib.f2s_knn(None, 1, 3, 8, 0, None, None) == _lib.F2S_ERR_INVALID_ARGUMENT
    assert b"k must be >= 1" in lib.f2s_last_error()
    assert lib.f2s_knn(None, 1, 3, 8, 33, None, None) == _lib.F2S_ERR_UNSUPPORTED
    assert lib.f2s_knn(None, 1, 3, 4096, 8, None, None) == _lib.F2S_ERR_UNSUPPORTED
    assert lib.f2s_knn(None, 1, 3, 8, 4, None, None) == _lib.F2S_ERR_INVALID_ARGUMENT
    assert lib.f2s_knn(None, 0, 3, 8, 4, None, None) == _lib.F2S_OK


def test_operator_rejects_cpu_tensors():
    torch = pytest.importorskip("torch")
    from flow2surf_b200 import knn_indices

    with pytest.raises(ValueError):
        knn_indices(torch.zeros(1, 3, 8), 4)
    with pytest.raises(ValueError, match="k must be >= 1"):
        knn_indices(torch.zeros(1, 3, 8), 0)


def test_training_entries_validate_on_the_host():
    """The backward and loss entries check sizes, pointers, limits and
    workspace sizes before any device work, and a zero batch is a no-op."""
    import ctypes

    lib = _lib.lib()
    bad = _lib.F2S_ERR_INVALID_ARGUMENT
    assert lib.f2s_nearest_backward(None, None, 1, 0, 4, None, None, None, None, None, None,
                                    None) == bad
    assert lib.f2s_nearest_backward(None, None, 0, 4, 4, None, None, None, None, None, None,
                                    None) == _lib.F2S_OK
    assert lib.f2s_nearest_backward(None, None, 1, 4, 4, None, None, None, None, None, None,
                                    None) == bad
    assert b"null pointer" in lib.f2s_last_error()
    f = ctypes.c_float(1.0)
    assert lib.f2s_dcd_loss(None, None, 1, 4, 0, f, None, None, None, None, None, 0, None) == bad
    assert lib.f2s_velocity_loss(None, None, 1, 0, None, None, None, None, None) == bad
    assert lib.f2s_hpe_activation_backward(None, ctypes.c_int64(8), 300, None, None, None, None,
                                           None, None, None, 0, None) == _lib.F2S_ERR_UNSUPPORTED
    assert b"at most 256" in lib.f2s_last_error()
    assert lib.f2s_neighbor_messages_backward(None, None, None, 1, 8, 4, 320, None, None, None,
                                              None, None, None, None, None, 0,
                                              None) == _lib.F2S_ERR_UNSUPPORTED
    size = ctypes.c_size_t()
    assert lib.f2s_offset_attention_backward_workspace_bytes(2, 64, 16, 32,
                                                             ctypes.byref(size)) == _lib.F2S_OK
    assert size.value >= 2 * 2 * 64 * 64 * 4
    assert lib.f2s_neighbor_reduce_backward_workspace_bytes(1, 16, 8, 6, 64, 64,
                                                            ctypes.byref(size)) == _lib.F2S_OK
    assert size.value > 0


def test_nearest_workspace_covers_the_grid_search():
    """Below 4096 points in either set the nearest / Chamfer workspace is the
    64-bit keys alone; from 4096 points in both sets it also holds both grids
    (cell counts and starts, sorted points, the far-search list), growing
    with the sets."""
    import ctypes

    lib = _lib.lib()
    size = ctypes.c_size_t()

    def ws(B, M, N):
        assert lib.f2s_nearest_workspace_bytes(B, M, N, ctypes.byref(size)) == _lib.F2S_OK
        return size.value

    assert ws(2, 4095, 100_000) == 2 * (4095 + 100_000) * 8
    assert ws(1, 300, 257) == (300 + 257) * 8
    small, large = ws(1, 4096, 4096), ws(1, 50_000, 100_000)
    assert small > (4096 + 4096) * 8
    assert large > small and large > (50_000 + 100_000) * 8
    assert ws(4, 50_000, 100_000) > large
    assert lib.f2s_nearest_workspace_bytes(-1, 1, 1, ctypes.byref(size)) == \
        _lib.F2S_ERR_INVALID_ARGUMENT
