"""ctypes binding of libflow2surf_sm100.so (the C-ABI in include/flow2surf_b200.h).

There is no fallback: if the library is missing or CUDA is unavailable the
operators raise. Loading the library needs no GPU; calling a compute entry
point does.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIBRARY_NAME = "libflow2surf_sm100.so"
LIBRARY_PATH = Path(__file__).resolve().parent / LIBRARY_NAME

F2S_OK = 0
F2S_ERR_INVALID_ARGUMENT = 1
F2S_ERR_UNSUPPORTED = 2
F2S_ERR_CUDA = 3
F2S_ERR_WORKSPACE = 4

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float
_d = ctypes.c_double
_sz = ctypes.c_size_t

# name -> argtypes; every name here is declared in include/flow2surf_b200.h.
SIGNATURES: dict[str, list] = {
    "f2s_last_error": [],
    "f2s_version": [],
    "f2s_trace_enable": [_i],
    "f2s_trace_tag_count": [],
    "f2s_trace_tag_name": [_i],
    "f2s_trace_collect": [_p, _p],
    "f2s_knn": [_p, _i, _i, _i, _i, _p, _p],
    "f2s_offset_attention_workspace_bytes": [_i, _i, _i, _p],
    "f2s_offset_attention": [_p, _p, _p, _i, _i, _i, _i, _p, _p, _sz, _p],
    "f2s_offset_attention_tc_workspace_bytes": [_i, _i, _i, _i, _p],
    "f2s_offset_attention_tc": [_p, _p, _p, _i, _i, _i, _i, _p, _p, _sz, _p],
    "f2s_neighbor_reduce_workspace_bytes": [_i, _i, _i, _p],
    "f2s_neighbor_reduce": [_p] * 11 + [_i] * 6 + [_p, _p, _sz, _p],
    "f2s_neighbor_reduce_tc": [_p] * 11 + [_i] * 6 + [_p, _p, _sz, _p],
    "f2s_model_param_segments": [_p, _p, _p, _i, _p],
    "f2s_model_workspace_bytes": [_p, _i, _i, _p],
    "f2s_model_forward": [_p, _p, _p, _p, _i, _i, _p, _p, _sz, _p],
    "f2s_trunk_forward": [_p, _p, _p, _p, _i, _i, _p, _sz, _p],
    "f2s_fps_workspace_bytes": [_i64, _p],
    "f2s_fps": [_p, _i64, _i64, _i64, _p, _p, _sz, _p],
    "f2s_patch_index": [_p, _i64, _p, _i, _i, _d, _p, _p, _p, _p],
    "f2s_fusion_workspace_bytes": [_i64, _p],
    "f2s_fusion_build": [_p, _p, _i, _i, _i64, _p, _p, _p, _p, _sz, _p],
    "f2s_gather_patches": [_p, _p, _p, _i, _i, _p, _p],
    "f2s_fuse_euler": [_p, _p, _p, _p, _p, _p, _i64, _f, _p, _p, _p],
    "f2s_fuse_partial": [_p, _p, _p, _p, _i64, _i, _i, _i, _p, _p],
    "f2s_euler_from_sum": [_p, _p, _p, _p, _i64, _f, _p, _p, _p],
    "f2s_nearest_workspace_bytes": [_i, _i, _i, _p],
    "f2s_nearest": [_p, _p, _i, _i, _i, _p, _p, _p, _p, _p, _sz, _p],
    "f2s_chamfer": [_p, _p, _i, _i, _i, _p, _p, _sz, _p],
    "f2s_chamfer_static": [_p, _p, _i, _i, _i, _p, _p],
    "f2s_point_to_mesh_workspace_bytes": [_i, _i, _p],
    "f2s_point_to_mesh": [_p, _i, _p, _i, _p, _i, _p, _p, _p, _sz, _p],
    "f2s_linear": [_p, _i, _p, _p, _p, _i, _i, _i, _i, _i, _p],
    "f2s_device_error": [_p, _i, _p],
    "f2s_selftest_wait_timeout": [_i, _p],
    "f2s_nearest_backward": [_p, _p, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p],
    "f2s_dcd_loss_workspace_bytes": [_i, _i, _i, _p],
    "f2s_dcd_loss": [_p, _p, _i, _i, _i, _f, _p, _p, _p, _p, _p, _sz, _p],
    "f2s_velocity_loss": [_p, _p, _i, _i, _p, _p, _p, _p, _p],
    "f2s_hpe_activation_backward_workspace_bytes": [_i64, _i, _p],
    "f2s_hpe_activation_backward": [_p, _i64, _i, _p, _p, _p, _p, _p, _p, _p, _sz, _p],
    "f2s_neighbor_messages_backward_workspace_bytes": [_i, _i, _i, _p],
    "f2s_neighbor_messages_backward": [_p, _p, _p, _i, _i, _i, _i] + [_p] * 7 + [_p, _sz, _p],
    "f2s_neighbor_reduce_backward_workspace_bytes": [_i] * 6 + [_p],
    "f2s_neighbor_reduce_backward": [_p] * 11 + [_i] * 6 + [_p] * 11 + [_p, _sz, _p],
    "f2s_offset_attention_backward_workspace_bytes": [_i, _i, _i, _i, _p],
    "f2s_offset_attention_backward": [_p, _p, _p, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p, _sz,
                                      _p],
}

_RESTYPES = {"f2s_last_error": ctypes.c_char_p, "f2s_trace_tag_name": ctypes.c_char_p}

_LIB = None


class Flow2SurfError(RuntimeError):
    """A C-ABI call returned a status other than F2S_OK."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[status {status}] {message}")
        self.status = status


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIBRARY_PATH.exists():
            raise RuntimeError(
                f"{LIBRARY_NAME} is not built; run `python jittor-flow2surf_b200/build.py` "
                "(or __graft_entry__.build())")
        handle = ctypes.CDLL(str(LIBRARY_PATH))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        _LIB = handle
    return _LIB


def check(status: int) -> None:
    if status != F2S_OK:
        message = lib().f2s_last_error().decode("utf-8", "replace")
        if status in (F2S_ERR_INVALID_ARGUMENT, F2S_ERR_UNSUPPORTED):
            raise ValueError(message)
        raise Flow2SurfError(status, message)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))


DEVICE_ERRORS = {
    1: "a tensor-core kernel gave up on a bounded wait",
    2: "an fp16 intermediate of the tf32 trunk (the FFN hidden rows) was out of the fp16 range",
}


F2S_FP16_RANGE = 2  # device error word: an fp16 FFN row of the tf32 trunk overflowed


def read_device_error(stream=None, reset: bool = True) -> int:
    """The library's device error word (0, 1 or 2); synchronises `stream`."""
    value = ctypes.c_int(0)
    check(lib().f2s_device_error(ctypes.byref(value), 1 if reset else 0, stream_handle(stream)))
    return value.value


def check_device_error(stream=None) -> None:
    """Raise when the library's device error word is set (it is then
    cleared); synchronises `stream`."""
    value = ctypes.c_int(0)
    check(lib().f2s_device_error(ctypes.byref(value), 1, stream_handle(stream)))
    if value.value:
        raise Flow2SurfError(F2S_ERR_CUDA, "device error %d: %s" % (
            value.value, DEVICE_ERRORS.get(value.value, "unknown")))


def ptr(tensor) -> int | None:
    """Raw device pointer of a torch tensor (None for an empty one)."""
    return tensor.data_ptr() if tensor is not None and tensor.numel() > 0 else None


def stream_handle(stream=None) -> int | None:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream
