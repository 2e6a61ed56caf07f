"""A minimal stand-in for the `jittor` package, backed by torch on the CPU.

Test infrastructure only: it lets the reference's own Python (its models,
operators' CPU fallbacks and patch_denoise) run in this container, where
Jittor is not installed, so that golden vectors come from the reference's
code itself. It implements just the API surface that code touches, with
Jittor's semantics where they differ from torch's:
  - Var.mean/sum(dim=, keepdims=), Var.max(dim=) returning values only;
  - nn.LayerNorm normalising with max(E[x^2] - E[x]^2, 0) and eps 1e-5;
  - nn.GELU / nn.gelu as the erf form; nn.LeakyReLU(scale=...);
  - jt.argmin returning (index, value); Var.transpose(*perm) permuting.
`jt.flags.use_cuda` is 0, so every operator takes its Jittor CPU fallback.
`DTYPE` selects the float type the shim computes in (float32 like Jittor, or
float64 to compare algorithms without rounding noise).
"""

from __future__ import annotations

import contextlib
import math
import sys
import types

import numpy as np
import torch

DTYPE = torch.float32


def _t(x):
    if isinstance(x, Var):
        return x.t
    return x


def _w(x):
    return Var(x) if isinstance(x, torch.Tensor) else x


_DTYPE_NAMES = {torch.float32: "float32", torch.float64: "float64", torch.int32: "int32",
                torch.int64: "int64", torch.bool: "bool"}


class Var:
    """Jittor Var over a torch tensor."""

    __array_priority__ = 1000

    def __init__(self, t):
        self.t = t if isinstance(t, torch.Tensor) else torch.as_tensor(t)

    # -- metadata --
    @property
    def shape(self):
        return tuple(self.t.shape)

    @property
    def ndim(self):
        return self.t.ndim

    @property
    def dtype(self):
        name = _DTYPE_NAMES.get(self.t.dtype, str(self.t.dtype))
        return "float32" if name == "float64" and DTYPE == torch.float64 else name

    def numpy(self):
        return self.t.detach().cpu().numpy()

    def stop_grad(self):
        return self

    def float32(self):
        return Var(self.t.to(DTYPE))

    def assign(self, other):
        self.t = _t(other).clone().to(self.t.dtype)
        return self

    # -- shape ops --
    def reshape(self, *shape):
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        return Var(self.t.reshape(*shape))

    def permute(self, *dims):
        return Var(self.t.permute(*dims))

    def transpose(self, *dims):
        if len(dims) == 2:
            return Var(self.t.transpose(*dims))
        return Var(self.t.permute(*dims))

    def unsqueeze(self, dim):
        return Var(self.t.unsqueeze(dim))

    def squeeze(self, dim):
        return Var(self.t.squeeze(dim))

    def expand(self, *shape):
        return Var(self.t.expand(*shape))

    # -- reductions --
    def mean(self, dim=None, keepdims=False):
        return Var(self.t.mean() if dim is None else self.t.mean(dim=dim, keepdim=keepdims))

    def sum(self, dim=None, keepdims=False):
        return Var(self.t.sum() if dim is None else self.t.sum(dim=dim, keepdim=keepdims))

    def max(self, dim=None, keepdims=False):
        if dim is None:
            return Var(self.t.max())
        return Var(self.t.max(dim=dim, keepdim=keepdims).values)

    def topk(self, k, dim=-1):
        values, indices = torch.topk(self.t, k=k, dim=dim)
        return Var(values), Var(indices.to(torch.int32))

    # -- indexing / arithmetic --
    def __getitem__(self, item):
        if isinstance(item, Var):
            item = item.t.long()
        elif isinstance(item, tuple):
            item = tuple(i.t.long() if isinstance(i, Var) else i for i in item)
        return Var(self.t[item])

    def _bin(self, other, op):
        return Var(op(self.t, _t(other)))

    def __add__(self, o): return self._bin(o, torch.add)
    def __radd__(self, o): return Var(_t(o) + self.t)
    def __sub__(self, o): return self._bin(o, torch.sub)
    def __rsub__(self, o): return Var(_t(o) - self.t)
    def __mul__(self, o): return self._bin(o, torch.mul)
    def __rmul__(self, o): return Var(_t(o) * self.t)
    def __truediv__(self, o): return self._bin(o, torch.div)
    def __rtruediv__(self, o): return Var(_t(o) / self.t)
    def __pow__(self, o): return Var(self.t ** _t(o))
    def __neg__(self): return Var(-self.t)
    def __eq__(self, o): return Var(self.t == _t(o))
    def __gt__(self, o): return Var(self.t > _t(o))
    def __lt__(self, o): return Var(self.t < _t(o))
    __hash__ = object.__hash__


def _cast(x):
    t = torch.as_tensor(np.asarray(x) if not isinstance(x, torch.Tensor) else x)
    if t.is_floating_point():
        t = t.to(DTYPE)
    return t


def array(x):
    return Var(_cast(x))


def _dt(dtype):
    return {"int32": torch.int32, "int64": torch.int64, "float32": DTYPE, None: DTYPE}[dtype]


def zeros(shape, dtype=None):
    return Var(torch.zeros(shape, dtype=_dt(dtype)))


def ones(shape, dtype=None):
    return Var(torch.ones(shape, dtype=_dt(dtype)))


def full(shape, value, dtype=None):
    return Var(torch.full(shape, float(value), dtype=_dt(dtype)))


def arange(n):
    return Var(torch.arange(n, dtype=torch.int32))


def concat(values, dim=0):
    return Var(torch.cat([_t(v) for v in values], dim=dim))


def matmul(a, b):
    return Var(torch.matmul(_t(a), _t(b)))


def sqrt(x): return Var(torch.sqrt(_t(x)))
def rsqrt(x): return Var(torch.rsqrt(_t(x)))
def exp(x): return Var(torch.exp(_t(x)))
def erf(x): return Var(torch.erf(_t(x)))


def maximum(a, b):
    ta, tb = _t(a), _t(b)
    if not isinstance(tb, torch.Tensor):
        tb = torch.tensor(tb, dtype=ta.dtype)
    return Var(torch.maximum(ta, tb))


def argmin(x, dim):
    values, index = torch.min(_t(x), dim=dim)
    return Var(index.to(torch.int32)), Var(values)


def code(*args, **kwargs):
    raise RuntimeError("jt.code kernels need CUDA; the shim runs the CPU fallbacks")


class _Flags:
    use_cuda = 0
    no_grad = False


flags = _Flags()


@contextlib.contextmanager
def no_grad():
    old = flags.no_grad
    flags.no_grad = True
    try:
        with torch.no_grad():
            yield
    finally:
        flags.no_grad = old


class Function:
    def __call__(self, *args):
        return self.execute(*args)


# ---------------------------------------------------------------------------
# nn
# ---------------------------------------------------------------------------

class Module:
    def __call__(self, *args, **kwargs):
        return self.execute(*args, **kwargs)

    def eval(self):
        return self

    def _children(self):
        for name, value in vars(self).items():
            if isinstance(value, (Var, Module)):
                yield name, value

    def named_parameters(self, prefix=""):
        for name, value in self._children():
            full_name = f"{prefix}{name}"
            if isinstance(value, Var):
                yield full_name, value
            else:
                yield from value.named_parameters(full_name + ".")

    def load_parameters(self, params: dict):
        own = dict(self.named_parameters())
        missing = set(own) - set(params)
        unexpected = set(params) - set(own)
        if missing or unexpected:
            raise KeyError(f"missing={sorted(missing)} unexpected={sorted(unexpected)}")
        for name, var in own.items():
            value = torch.as_tensor(np.asarray(params[name])).to(DTYPE)
            if tuple(value.shape) != var.shape:
                raise ValueError(f"{name}: {tuple(value.shape)} != {var.shape}")
            var.t = value.clone()


class Sequential(Module):
    def __init__(self, *layers):
        for i, layer in enumerate(layers):
            setattr(self, str(i), layer)
        self._n = len(layers)

    def __getitem__(self, i):
        return getattr(self, str(i))

    def execute(self, x):
        for i in range(self._n):
            x = self[i](x)
        return x


class ModuleList(Module):
    def __init__(self, modules):
        modules = list(modules)
        for i, m in enumerate(modules):
            setattr(self, str(i), m)
        self._n = len(modules)

    def __getitem__(self, i):
        return getattr(self, str(i))

    def __iter__(self):
        return (self[i] for i in range(self._n))

    def __len__(self):
        return self._n


def _uniform(shape, bound):
    return Var((torch.rand(shape, dtype=DTYPE) * 2 - 1) * bound)


def linear(x, weight, bias=None):
    y = torch.matmul(_t(x), _t(weight).transpose(0, 1))
    return Var(y if bias is None else y + _t(bias))


class Linear(Module):
    def __init__(self, in_features, out_features, bias=True):
        bound = 1.0 / math.sqrt(in_features)
        self.weight = _uniform((out_features, in_features), bound)
        if bias:
            self.bias = _uniform((out_features,), bound)
        else:
            self.bias = None

    def execute(self, x):
        return linear(x, self.weight, self.bias)


class Conv1d(Module):
    def __init__(self, in_channels, out_channels, kernel_size, bias=True):
        bound = 1.0 / math.sqrt(in_channels * kernel_size)
        self.weight = _uniform((out_channels, in_channels, kernel_size), bound)
        self.bias = _uniform((out_channels,), bound) if bias else None

    def execute(self, x):
        y = torch.einsum("oi,bin->bon", _t(self.weight)[:, :, 0], _t(x))
        if self.bias is not None:
            y = y + _t(self.bias)[None, :, None]
        return Var(y)


class Conv2d(Module):
    def __init__(self, in_channels, out_channels, kernel_size, bias=True):
        bound = 1.0 / math.sqrt(in_channels * kernel_size * kernel_size)
        self.weight = _uniform((out_channels, in_channels, kernel_size, kernel_size), bound)
        self.bias = _uniform((out_channels,), bound) if bias else None

    def execute(self, x):
        return conv2d(x, self.weight, self.bias)


def conv2d(x, weight, bias=None):
    w = _t(weight)[:, :, 0, 0]
    y = torch.einsum("oi,bihw->bohw", w, _t(x))
    if bias is not None:
        y = y + _t(bias)[None, :, None, None]
    return Var(y)


class LayerNorm(Module):
    """Jittor LayerNorm: var = max(E[x^2] - E[x]^2, 0), eps 1e-5, affine."""

    def __init__(self, normalized_shape, eps=1e-5, elementwise_affine=True, bias=True):
        self.eps = eps
        self.weight = Var(torch.ones(normalized_shape, dtype=DTYPE))
        self.bias = Var(torch.zeros(normalized_shape, dtype=DTYPE))

    def execute(self, x):
        t = _t(x)
        mean = t.mean(dim=-1, keepdim=True)
        second = (t * t).mean(dim=-1, keepdim=True)
        var = torch.clamp(second - mean * mean, min=0.0)
        w = _t(self.weight) / torch.sqrt(var + self.eps)
        b = _t(self.bias) - mean * w
        return Var(t * w + b)


def gelu(x):
    t = _t(x)
    return Var(t * 0.5 * (1.0 + torch.erf(t / math.sqrt(2.0))))


class GELU(Module):
    def execute(self, x):
        return gelu(x)


class SiLU(Module):
    def execute(self, x):
        t = _t(x)
        return Var(t * torch.sigmoid(t))


def leaky_relu(x, scale=0.01):
    t = _t(x)
    return Var(torch.where(t > 0, t, t * scale))


class LeakyReLU(Module):
    def __init__(self, scale=0.01):
        self.scale = scale

    def execute(self, x):
        return leaky_relu(x, self.scale)


def softmax(x, dim=None):
    return Var(torch.softmax(_t(x), dim=dim))


def bmm(a, b):
    return Var(torch.bmm(_t(a), _t(b)))


def _zero_(var):
    var.t = torch.zeros_like(var.t)
    return var


def _eye(n):
    return Var(torch.eye(n, dtype=DTYPE))


def install(dtype=torch.float32):
    """Register the shim as `jittor` (and `jittor.nn`, `jittor.init`)."""
    global DTYPE
    DTYPE = dtype
    jt = sys.modules[__name__]
    nn = types.ModuleType("jittor.nn")
    for name in ("Module", "Sequential", "ModuleList", "Linear", "Conv1d", "Conv2d",
                 "LayerNorm", "GELU", "SiLU", "LeakyReLU", "linear", "conv2d", "gelu",
                 "leaky_relu", "softmax", "bmm"):
        setattr(nn, name, getattr(jt, name))
    init = types.ModuleType("jittor.init")
    init.zero_ = _zero_
    init.eye = _eye
    module = types.ModuleType("jittor")
    for name in ("Var", "Function", "array", "zeros", "ones", "full", "arange", "concat",
                 "matmul", "sqrt", "rsqrt", "exp", "erf", "maximum", "argmin", "code",
                 "flags", "no_grad"):
        setattr(module, name, getattr(jt, name))
    dataset = types.ModuleType("jittor.dataset")

    class Dataset:  # imported by flow2surf/dataset.py; never instantiated here
        pass

    dataset.Dataset = Dataset
    module.nn = nn
    module.init = init
    module.dataset = dataset
    module.__path__ = []
    sys.modules["jittor"] = module
    sys.modules["jittor.nn"] = nn
    sys.modules["jittor.init"] = init
    sys.modules["jittor.dataset"] = dataset
    return module
