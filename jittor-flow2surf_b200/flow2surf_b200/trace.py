"""Per-kernel device timing through the library's launch trace.

    with trace.recording() as rec:
        ...                      # any calls into the library
    rec.kernels                  # {"gemm_swiglu": (ms, launches), ...}
"""

from __future__ import annotations

import contextlib
import ctypes

from . import _lib


def enable(on: bool = True) -> None:
    _lib.check(_lib.lib().f2s_trace_enable(1 if on else 0))


def collect() -> dict[str, tuple[float, int]]:
    """Per kernel class: (total device ms, launches) since enable(); clears."""
    lib = _lib.lib()
    n = lib.f2s_trace_tag_count()
    ms = (ctypes.c_double * n)()
    count = (ctypes.c_int64 * n)()
    _lib.check(lib.f2s_trace_collect(ms, count))
    out = {}
    for t in range(n):
        if count[t]:
            out[lib.f2s_trace_tag_name(t).decode()] = (ms[t], int(count[t]))
    return out


class _Recording:
    kernels: dict[str, tuple[float, int]]

    def __init__(self):
        self.kernels = {}

    @property
    def launches(self) -> int:
        return sum(c for _, c in self.kernels.values())

    @property
    def total_ms(self) -> float:
        return sum(ms for ms, _ in self.kernels.values())


@contextlib.contextmanager
def recording():
    rec = _Recording()
    enable(True)
    try:
        yield rec
    finally:
        rec.kernels = collect()
        enable(False)
