"""Flow2SurfNet with the reference's constructor, parameter names and call
signature (flow2surf/models/network.py:29-95), computed by the C-ABI forward.

Parameters live on the host as float32 NumPy arrays keyed by the reference's
state-dict names; they are composed and packed once into a device blob
(f2s_model_param_segments gives the layout) and reused until they change.
"""

from __future__ import annotations

import ctypes
import pickle

import numpy as np
import torch

from . import _lib
from .params import model_dims, parameter_specs
from .synthetic import random_parameters

MAX_STAGES, MAX_BLOCKS, MAX_DECODER = 6, 16, 4


class ModelConfig(ctypes.Structure):
    """ctypes mirror of f2s_model_config (include/flow2surf_b200.h)."""

    _fields_ = [
        ("k_neighbors", ctypes.c_int32),
        ("feat_dim", ctypes.c_int32),
        ("num_blocks", ctypes.c_int32),
        ("alpha_dim", ctypes.c_int32),
        ("ffn_ratio", ctypes.c_int32),
        ("num_stages", ctypes.c_int32),
        ("stage_dims", ctypes.c_int32 * MAX_STAGES),
        ("num_decoder", ctypes.c_int32),
        ("decoder_dims", ctypes.c_int32 * MAX_DECODER),
        ("precision", ctypes.c_int32),
        ("encoder_precision", ctypes.c_int32),
    ]


PRECISIONS = {"fp32": 0, "tf32": 1, "bf16x3": 3, "tf32_wide": 4}
"""Arithmetic of the dense contractions: fp32 CUDA-core kernels, tcgen05
tensor cores reading the fp32 operands as tf32, or (encoder only) tensor cores
on operands split into two bf16 halves (hi*hi + hi*lo + lo*hi). "tf32" keeps
the trunk's FFN rows in fp16 (tf32's mantissa, fp16's range); "tf32_wide"
(trunk only) keeps them in fp32 and is what a tf32 forward is rerun in when
those fp16 rows overflow."""


def model_config(cfg: dict, precision: str = "fp32",
                 encoder_precision: str | None = None) -> ModelConfig:
    d = model_dims(cfg)
    encoder_precision = encoder_precision or precision
    for p in (precision, encoder_precision):
        if p not in PRECISIONS:
            raise ValueError(f"precision must be one of {sorted(PRECISIONS)}, got {p!r}")
    if len(d.stage_dims) > MAX_STAGES or len(d.decoder_dims) > MAX_DECODER:
        raise ValueError("too many encoder or decoder layers for the kernels")
    c = ModelConfig()
    c.k_neighbors, c.feat_dim, c.num_blocks = d.k, d.feat_dim, d.num_blocks
    c.alpha_dim, c.ffn_ratio = d.alpha_dim, d.ffn_ratio
    c.num_stages = len(d.stage_dims)
    for i, v in enumerate(d.stage_dims):
        c.stage_dims[i] = v
    c.num_decoder = len(d.decoder_dims)
    for i, v in enumerate(d.decoder_dims):
        c.decoder_dims[i] = v
    c.precision = PRECISIONS[precision]
    c.encoder_precision = PRECISIONS[encoder_precision]
    return c


def _w2(w):
    """1x1 conv weight (out, in, 1[, 1]) -> (out, in)."""
    return np.asarray(w).reshape(w.shape[0], w.shape[1])


def round_tf32(a) -> np.ndarray:
    """Nearest tf32 value (10-bit mantissa, ties away from zero) of each
    element, as float32: tensor cores read fp32 operands by dropping the low
    13 mantissa bits, so operands rounded first carry unbiased error."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).copy()
    finite = (u & 0x7F800000) != 0x7F800000
    u[finite] = (u[finite] + 0x1000) & 0xFFFFE000
    return u.view(np.float32)


def composed_segments(cfg: dict, p: dict, trunk_tf32: bool = False,
                      encoder_tf32: bool = False) -> list[np.ndarray]:
    """Parameter segments in blob order, with the reference's exact
    factorisations (flow2surf/models/encoder.py:88-101). Weights that a tf32
    tensor-core contraction reads are rounded to the nearest tf32."""
    d = model_dims(cfg)
    f32 = lambda a: np.asarray(a, dtype=np.float32)  # noqa: E731
    enc = round_tf32 if encoder_tf32 else f32
    trk = round_tf32 if trunk_tf32 else f32
    segs = [p["alpha_emb.mlp.0.weight"], p["alpha_emb.mlp.0.bias"],
            p["alpha_emb.mlp.2.weight"], p["alpha_emb.mlp.2.bias"]]
    pre = "local_encoder.input_embed.net"
    segs += [p[f"{pre}.0.weight"], p[f"{pre}.0.bias"], p[f"{pre}.1.weight"], p[f"{pre}.1.bias"],
             p[f"{pre}.3.weight"], p[f"{pre}.3.bias"]]
    for s, cin in enumerate(d.stage_inputs):
        pre = f"local_encoder.stages.{s}"
        w = f32(p[f"{pre}.projection.weight"])[:, :, 0, 0]
        wd, wc, pos = w[:, :cin], w[:, cin:2 * cin], w[:, 2 * cin:]
        content = np.concatenate([wd, wc - wd], axis=0)
        pos64 = pos.astype(np.float64)
        contrib_w = pos64 @ np.asarray(p[f"{pre}.position_embed.net.3.weight"], np.float64)
        contrib_b = pos64 @ np.asarray(p[f"{pre}.position_embed.net.3.bias"], np.float64)
        segs += [enc(content), p[f"{pre}.position_embed.net.0.weight"],
                 p[f"{pre}.position_embed.net.0.bias"], p[f"{pre}.position_embed.net.1.weight"],
                 p[f"{pre}.position_embed.net.1.bias"], enc(contrib_w), contrib_b,
                 p[f"{pre}.norm.weight"], p[f"{pre}.norm.bias"]]
    segs += [enc(_w2(p["local_encoder.proj.0.weight"])), p["local_encoder.proj.1.weight"],
             p["local_encoder.proj.1.bias"]]
    for i in range(d.num_blocks):
        pre = f"blocks.{i}"
        segs += [p[f"{pre}.mod.1.weight"], p[f"{pre}.mod.1.bias"],
                 trk(_w2(p[f"{pre}.qkv_conv.weight"])), trk(_w2(p[f"{pre}.proj.weight"])),
                 trk(_w2(p[f"{pre}.ff_gate.weight"])), p[f"{pre}.ff_gate.bias"],
                 trk(_w2(p[f"{pre}.ff1.weight"])), p[f"{pre}.ff1.bias"],
                 trk(_w2(p[f"{pre}.ff2.weight"])), p[f"{pre}.ff2.bias"]]
    layer = 0
    for _ in d.decoder_dims:
        segs += [trk(_w2(p[f"decoder.net.{layer}.weight"])), p[f"decoder.net.{layer + 1}.weight"],
                 p[f"decoder.net.{layer + 1}.bias"]]
        layer += 3
    segs.append(trk(_w2(p[f"decoder.net.{layer}.weight"])))
    return [f32(s) for s in segs]


def pack_parameters(cfg: dict, params: dict, trunk_tf32: bool = False,
                    encoder_tf32: bool = False) -> np.ndarray:
    """Host float32 blob laid out as f2s_model_param_segments reports."""
    c = model_config(cfg)
    total = ctypes.c_int64()
    n = _lib.lib().f2s_model_param_segments(ctypes.byref(c), None, None, 0, ctypes.byref(total))
    if n <= _lib.F2S_ERR_WORKSPACE:
        _lib.check(n)
    offsets = (ctypes.c_int64 * n)()
    sizes = (ctypes.c_int64 * n)()
    _lib.lib().f2s_model_param_segments(ctypes.byref(c), offsets, sizes, n, ctypes.byref(total))
    segs = composed_segments(cfg, params, trunk_tf32, encoder_tf32)
    if len(segs) != n:
        raise RuntimeError(f"blob layout mismatch: {len(segs)} segments vs {n}")
    blob = np.zeros(total.value, dtype=np.float32)
    for seg, off, size in zip(segs, offsets, sizes):
        if seg.size != size:
            raise RuntimeError(f"blob segment size mismatch: {seg.size} vs {size}")
        blob[off:off + size] = seg.ravel()
    return blob


def reference_init(cfg: dict, seed: int = 0) -> dict:
    """Weights initialised the way the reference constructs them: random
    weights, then the zero-initialised decoder output (decoder.py:26-27) and
    AdaLN modulation (transformer.py:51-54) and identity value rows
    (transformer.py:38-40), so the fresh model predicts v = 0."""
    p = random_parameters(cfg, seed)
    d = model_dims(cfg)
    for i in range(d.num_blocks):
        p[f"blocks.{i}.mod.1.weight"][:] = 0
        p[f"blocks.{i}.mod.1.bias"][:] = 0
        qkv = p[f"blocks.{i}.qkv_conv.weight"]
        qkv[2 * d.qk_dim:, :, 0] = np.eye(d.feat_dim, dtype=np.float32)
    last = parameter_specs(cfg)[-1][0]
    p[last][:] = 0
    return p


class _ArrayUnpickler(pickle.Unpickler):
    """Unpickler for parameter files: dicts, lists and NumPy arrays only."""

    _ALLOWED = {
        ("collections", "OrderedDict"), ("builtins", "dict"), ("builtins", "list"),
        ("numpy", "ndarray"), ("numpy", "dtype"),
        ("numpy.core.multiarray", "_reconstruct"), ("numpy._core.multiarray", "_reconstruct"),
        ("numpy.core.multiarray", "scalar"), ("numpy._core.multiarray", "scalar"),
        ("numpy.core.numeric", "_frombuffer"), ("numpy._core.numeric", "_frombuffer"),
    }

    def find_class(self, module, name):
        if (module, name) in self._ALLOWED or (module == "numpy" and name.startswith("dtype")):
            return super().find_class(module, name)
        raise pickle.UnpicklingError(f"refusing to load {module}.{name} from a parameter file")


class Flow2SurfNet:
    """Predict patch velocities (flow2surf/models/network.py:29-82).

    Inputs : x_alpha (B, 3, M) float32 CUDA tensor, alpha (B,) in [0, 1]
    Output : velocity (B, M, 3) float32
    """

    def __init__(self, k: int = 32, feat_dim: int = 128, num_blocks: int = 3,
                 encoder_dims=(64, 64), alpha_dim: int = 192, ffn_ratio: int = 4,
                 decoder_dims=(128, 64), seed: int = 0, precision: str = "fp32",
                 encoder_precision: str | None = None):
        self.cfg = {"k_neighbors": k, "feat_dim": feat_dim, "num_blocks": num_blocks,
                    "encoder_dims": list(encoder_dims), "alpha_dim": alpha_dim,
                    "ffn_ratio": ffn_ratio, "decoder_dims": list(decoder_dims)}
        model_dims(self.cfg)  # validates like the reference constructor
        self.precision = precision
        self.encoder_precision = encoder_precision or precision
        self._config = model_config(self.cfg, precision, self.encoder_precision)
        self._params = reference_init(self.cfg, seed)
        self._blob = None
        self._workspace = None

    # -- parameters ---------------------------------------------------------
    def state_dict(self) -> dict:
        return {k: v.copy() for k, v in self._params.items()}

    def load_parameters(self, params: dict) -> None:
        own = {name: shape for name, shape, _ in parameter_specs(self.cfg)}
        missing, unexpected = set(own) - set(params), set(params) - set(own)
        if missing or unexpected:
            raise KeyError(f"missing={sorted(missing)} unexpected={sorted(unexpected)}")
        for name, shape in own.items():
            value = np.asarray(params[name], dtype=np.float32)
            if value.shape != tuple(shape):
                raise ValueError(f"{name}: shape {value.shape} != {tuple(shape)}")
            self._params[name] = value.copy()
        self._blob = None

    load_state_dict = load_parameters

    def save(self, path) -> None:
        """Write the parameters as the reference's Module.save does: a pickled
        {state-dict name: float32 array} dict (flow2surf/training/optimization.py:41-42,
        flow2surf/training/checkpoint.py:151-153)."""
        with open(path, "wb") as f:
            pickle.dump({k: np.ascontiguousarray(v) for k, v in self._params.items()}, f,
                        protocol=pickle.HIGHEST_PROTOCOL)

    def load(self, path) -> None:
        """Load a checkpoint the reference wrote with model.save (loaded there by
        model.load, predict.py:46): a pickled dict of parameter arrays keyed by
        state-dict name; `.npz` archives are taken too. The unpickler accepts
        only dicts, lists and NumPy arrays, so a checkpoint file cannot run code."""
        path = str(path)
        if path.endswith(".npz"):
            with np.load(path, allow_pickle=False) as z:
                params = {k: z[k] for k in z.files}
        else:
            with open(path, "rb") as f:
                params = _ArrayUnpickler(f).load()
        if not isinstance(params, dict):
            raise ValueError(f"{path}: expected a dict of parameter arrays, got {type(params)}")
        self.load_parameters({str(k): np.asarray(v) for k, v in params.items()})

    def eval(self):
        return self

    def device_blob(self, device) -> torch.Tensor:
        if self._blob is None or self._blob.device != torch.device(device):
            host = pack_parameters(self.cfg, self._params,
                                   trunk_tf32=self.precision in ("tf32", "tf32_wide"),
                                   encoder_tf32=self.encoder_precision == "tf32")
            self._blob = torch.from_numpy(host).to(device)
        return self._blob

    # -- forward ------------------------------------------------------------
    def workspace_bytes(self, batch: int, points: int) -> int:
        size = ctypes.c_size_t()
        _lib.check(_lib.lib().f2s_model_workspace_bytes(ctypes.byref(self._config), batch, points,
                                                        ctypes.byref(size)))
        return size.value

    def _workspace_for(self, batch, points, device):
        need = self.workspace_bytes(batch, points)
        ws = self._workspace
        if ws is None or ws.numel() < need or ws.device != device:
            self._workspace = torch.empty(need, dtype=torch.uint8, device=device)
        return self._workspace

    def forward_into(self, x_alpha: torch.Tensor, alpha: torch.Tensor, out: torch.Tensor,
                     workspace: torch.Tensor | None = None, config=None) -> torch.Tensor:
        batch, _, points = x_alpha.shape
        ws = workspace if workspace is not None else self._workspace_for(batch, points,
                                                                         x_alpha.device)
        blob = self.device_blob(x_alpha.device)
        _lib.call("f2s_model_forward", ctypes.byref(config or self._config), _lib.ptr(blob),
                  _lib.ptr(x_alpha), _lib.ptr(alpha), batch, points, _lib.ptr(out),
                  _lib.ptr(ws), ws.numel(), _lib.stream_handle())
        return out

    def trunk_(self, x: torch.Tensor, alpha: torch.Tensor,
               workspace: torch.Tensor | None = None) -> torch.Tensor:
        """The AdaLN-Zero blocks alone (transformer.py:75-89, with the
        AlphaEmbed conditioning of network.py:75-80), in place on a
        point-major residual stream x (B, M, feat_dim) float32 CUDA tensor
        (the reference's (B, C, M) transposed); alpha (B,)."""
        if x.dim() != 3 or x.shape[2] != self.cfg["feat_dim"]:
            raise ValueError(f"x must be (B, M, {self.cfg['feat_dim']}), got {tuple(x.shape)}")
        if alpha.dim() != 1 or alpha.shape[0] != x.shape[0]:
            raise ValueError(f"alpha must be (B,), got {tuple(alpha.shape)}")
        if not x.is_cuda or not alpha.is_cuda or x.dtype != torch.float32 or \
                not x.is_contiguous():
            raise ValueError("trunk_ takes contiguous float32 CUDA tensors (no CPU path)")
        alpha = alpha.to(torch.float32).contiguous()
        batch, points, _ = x.shape
        ws = workspace if workspace is not None else self._workspace_for(batch, points, x.device)
        blob = self.device_blob(x.device)
        _lib.call("f2s_trunk_forward", ctypes.byref(self._config), _lib.ptr(blob), _lib.ptr(x),
                  _lib.ptr(alpha), batch, points, _lib.ptr(ws), ws.numel(), _lib.stream_handle())
        return x

    def wide_ffn(self):
        """This model with the trunk's FFN rows kept in fp32 (precision
        "tf32_wide", the same packed parameters): where a "tf32" forward's
        fp16 FFN rows overflow (device error word 2), this one has no range
        limit."""
        return _WideFfn(self) if self.precision == "tf32" else self

    def __call__(self, x_alpha: torch.Tensor, alpha: torch.Tensor) -> torch.Tensor:
        if x_alpha.dim() != 3 or x_alpha.shape[1] != 3:
            raise ValueError(f"x_alpha must be (B, 3, M), got {tuple(x_alpha.shape)}")
        if alpha.dim() != 1 or alpha.shape[0] != x_alpha.shape[0]:
            raise ValueError(f"alpha must be (B,), got {tuple(alpha.shape)}")
        if not x_alpha.is_cuda or not alpha.is_cuda:
            raise ValueError("Flow2SurfNet takes CUDA tensors (no CPU path)")
        x_alpha = x_alpha.to(torch.float32).contiguous()
        alpha = alpha.to(torch.float32).contiguous()
        batch, _, points = x_alpha.shape
        out = torch.empty((batch, points, 3), dtype=torch.float32, device=x_alpha.device)
        if out.numel() == 0:
            return out
        self.forward_into(x_alpha, alpha, out)
        status = _lib.read_device_error()
        if status == _lib.F2S_FP16_RANGE and self.precision == "tf32":
            # fp16 FFN rows out of range: the same forward with fp32 rows
            self.wide_ffn().forward_into(x_alpha, alpha, out)
            status = _lib.read_device_error()
        if status:  # a bounded wait that ran out (or a range error outside tf32)
            raise _lib.Flow2SurfError(_lib.F2S_ERR_CUDA, "device error %d: %s" % (
                status, _lib.DEVICE_ERRORS.get(status, "unknown")))
        return out

    execute = __call__


class _WideFfn:
    """A "tf32" Flow2SurfNet run as "tf32_wide" (fp32 FFN rows): same
    parameters, packing and workspace layout, another model config."""

    def __init__(self, model: Flow2SurfNet):
        self.model = model
        self.config = model_config(model.cfg, "tf32_wide", model.encoder_precision)

    def workspace_bytes(self, batch: int, points: int) -> int:
        size = ctypes.c_size_t()
        _lib.check(_lib.lib().f2s_model_workspace_bytes(ctypes.byref(self.config), batch, points,
                                                        ctypes.byref(size)))
        return size.value

    def forward_into(self, x_alpha, alpha, out, workspace=None):
        return self.model.forward_into(x_alpha, alpha, out, workspace, config=self.config)


def build_model(cfg: dict, precision: str | None = None,
                encoder_precision: str | None = None) -> Flow2SurfNet:
    """flow2surf/models/network.py:85-95; `precision` (or cfg["precision"],
    default "fp32") selects the arithmetic of the trunk and decoder
    contractions, `encoder_precision` (default: the same) that of the
    neighbour stages and projection head."""
    return Flow2SurfNet(
        k=cfg["k_neighbors"],
        feat_dim=cfg["feat_dim"],
        num_blocks=cfg["num_blocks"],
        encoder_dims=cfg["encoder_dims"],
        alpha_dim=cfg["alpha_dim"],
        ffn_ratio=cfg["ffn_ratio"],
        decoder_dims=cfg["decoder_dims"],
        precision=precision or cfg.get("precision", "fp32"),
        encoder_precision=encoder_precision or cfg.get("encoder_precision"),
    )
