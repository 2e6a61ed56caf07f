"""The tcgen05 tensor-core contraction (f2s_linear) against float64 products.

bf16: inputs are bf16, so the only error is fp32 accumulation order (tested
at 1e-5 relative to the row scale). tf32: fp32 inputs read with a 10-bit
mantissa (tested at 2e-3 relative). fp32: the CUDA-core kernel (1e-6).
"""

import numpy as np
import pytest
import torch

from flow2surf_b200 import _lib

pytestmark = pytest.mark.gpu

PRECISION = {"fp32": 0, "tf32": 1, "bf16": 2, "bf16x3": 3}


def linear(x, w, b, precision):
    rows, K = x.shape
    cols = w.shape[0] // 2 if precision == "bf16x3" else w.shape[0]  # bf16x3: hi then lo
    y = torch.empty((rows, cols), dtype=torch.float32, device="cuda")
    _lib.call("f2s_linear", x.data_ptr(), x.stride(0), w.data_ptr(),
              b.data_ptr() if b is not None else None, y.data_ptr(), y.stride(0), rows, cols, K,
              PRECISION[precision], _lib.stream_handle())
    return y


def device_error():
    import ctypes
    v = ctypes.c_int(0)
    _lib.check(_lib.lib().f2s_device_error(ctypes.byref(v), 1, _lib.stream_handle()))
    return v.value


@pytest.mark.parametrize("precision", ["bf16", "tf32", "fp32", "bf16x3"])
@pytest.mark.parametrize("rows,cols,K", [(1000, 288, 192), (300, 192, 1536), (129, 3, 64),
                                         (5000, 128, 64), (1024, 1536, 192), (257, 384, 128),
                                         (77, 100, 40), (20000, 288, 192), (20000, 1536, 192)])
def test_linear_matches_float64(cuda, precision, rows, cols, K):
    """The last two shapes give every CTA several row blocks, so the weight
    tiles stay resident in shared memory (tf32 and bf16 for 288 columns,
    bf16 for 1536)."""
    g = torch.Generator(device="cpu").manual_seed(rows + cols + K)
    x = torch.randn(rows, K, generator=g)
    w = torch.randn(cols, K, generator=g) / K ** 0.5
    b = torch.randn(cols, generator=g) * 0.1
    if precision == "bf16":
        if K % 8:
            pytest.skip("bf16 rows need a 16-byte pitch")
        xd, wd = x.to(torch.bfloat16), w.to(torch.bfloat16)
        ref = xd.double() @ wd.double().T + b.double()
        tol = 1e-5
    elif precision == "bf16x3":
        if K % 8:
            pytest.skip("bf16 weight rows need a 16-byte pitch")
        # fp32 x (split in the kernel); W as its bf16 high parts, then low parts
        w_hi = w.to(torch.bfloat16)
        w_lo = (w - w_hi.float()).to(torch.bfloat16)
        xd, wd = x, torch.cat([w_hi, w_lo])
        ref = x.double() @ w.double().T + b.double()
        tol = 2e-5
    else:
        if precision == "tf32" and K % 4:
            pytest.skip("tf32 rows need a 16-byte pitch")
        xd, wd = x, w
        ref = x.double() @ w.double().T + b.double()
        tol = 2e-3 if precision == "tf32" else 1e-6
    y = linear(xd.cuda().contiguous(), wd.cuda().contiguous(), b.cuda(), precision)
    torch.cuda.synchronize()
    scale = (xd.double().abs() @ wd.double().abs().T).max().item()
    err = (y.cpu().double() - ref).abs().max().item()
    assert err <= tol * scale, f"{precision} {rows}x{cols}x{K}: err {err} scale {scale}"
    assert device_error() == 0


def test_linear_no_bias_and_strided_rows(cuda):
    x = torch.randn(600, 256, device="cuda")
    w = torch.randn(192, 128, device="cuda") / 128 ** 0.5
    xs = x[:, :128]                       # row pitch 256, K 128
    y = linear(xs.to(torch.bfloat16).contiguous(), w.to(torch.bfloat16), None, "bf16")
    y2 = linear(xs, w, None, "tf32")      # strided fp32 rows through the tensor map
    ref = xs.double() @ w.double().T
    assert (y.double() - ref).abs().max().item() < 0.05
    assert (y2.double() - ref).abs().max().item() < 0.01
    assert device_error() == 0
