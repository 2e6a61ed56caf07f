"""Custom operators with the reference's Python surface, backed by sm_100a kernels.

Mirrors flow2surf/models/ops/__init__.py:3-11 and
flow2surf/training/distances.py:70-98: same names, argument meaning, shape
checks and ValueError messages. Tensors are torch CUDA tensors; there is no
CPU path -- a CPU tensor or a missing library raises.
"""

from __future__ import annotations

import ctypes

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

    flow2surf/models/ops/knn.py:35-66: k < 1 raises; N <= 1 gives zeros; when
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


def _workspace(query: str, *dims) -> torch.Tensor:
    size = ctypes.c_size_t()
    _lib.check(getattr(_lib.lib(), query)(*dims, ctypes.byref(size)))
    return torch.empty(size.value, dtype=torch.uint8, device="cuda")


def offset_attention_aggregate(query: torch.Tensor, key: torch.Tensor,
                               value: torch.Tensor, *, precision: str = "fp32") -> torch.Tensor:
    """Aggregate values using normalized offset-attention weights.

    query (B, N, d), key (B, d, N), value (B, N, C) -> (B, N, C): softmax of
    query . key over the query axis, each row divided by its sum over keys
    plus 1e-9, times value (flow2surf/models/ops/attention.py:15-19,84-106).
    `precision` "fp32" (CUDA cores, the reference's arithmetic) or "tensor"
    (tcgen05: split-bf16 scores, fp16 P V; d a multiple of 4 up to 64, C a
    multiple of 64 up to 256; ~1e-3 relative).
    """
    if precision not in ("fp32", "tensor"):
        raise ValueError(f"precision must be 'fp32' or 'tensor', got {precision!r}")
    if query.dim() != 3 or key.dim() != 3 or value.dim() != 3:
        raise ValueError("query, key, and value must be rank-3 tensors")
    if (query.shape[0] != key.shape[0] or query.shape[0] != value.shape[0]
            or query.shape[1] != key.shape[2] or query.shape[1] != value.shape[1]
            or query.shape[2] != key.shape[1]):
        raise ValueError(f"Incompatible attention shapes: {tuple(query.shape)}, "
                         f"{tuple(key.shape)}, {tuple(value.shape)}")
    _require_cuda(query, key, value)
    if _needs_grad(query, key, value):
        if precision != "fp32":
            raise ValueError("the tensor-core attention has no backward; use precision='fp32'")
        return _OffsetAttention.apply(query, key, value)
    return _attention_forward(query, key, value, precision)


def _attention_forward(query, key, value, precision="fp32"):
    batch, points, width = query.shape
    channels = value.shape[2]
    out = torch.empty((batch, points, channels), dtype=torch.float32, device=query.device)
    if out.numel() == 0:
        return out
    query, key, value = _f32(query), _f32(key), _f32(value)
    if precision == "tensor":
        ws = _workspace("f2s_offset_attention_tc_workspace_bytes", batch, points, width, channels)
        entry = "f2s_offset_attention_tc"
    else:
        ws = _workspace("f2s_offset_attention_workspace_bytes", batch, points, width)
        entry = "f2s_offset_attention"
    _lib.call(entry, _lib.ptr(query), _lib.ptr(key), _lib.ptr(value), batch, points, width,
              channels, _lib.ptr(out), _lib.ptr(ws), ws.numel(), _lib.stream_handle())
    return out


class _OffsetAttention(torch.autograd.Function):
    """Exact offset attention with its backward (_OffsetAttentionFunction,
    flow2surf/models/ops/attention.py:66-81): the forward on the fp32 kernels,
    the backward recomputing the probabilities per batch chunk."""

    @staticmethod
    def forward(ctx, query, key, value):
        query, key, value = _f32(query), _f32(key), _f32(value)
        out = _attention_forward(query, key, value)
        ctx.save_for_backward(query, key, value, out)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        query, key, value, out = ctx.saved_tensors
        batch, points, width = query.shape
        channels = value.shape[2]
        gq, gk, gv = torch.empty_like(query), torch.empty_like(key), torch.empty_like(value)
        if out.numel() == 0:
            return gq.zero_(), gk.zero_(), gv.zero_()
        grad_output = _f32(grad_output)
        ws = _workspace("f2s_offset_attention_backward_workspace_bytes", batch, points, width,
                        channels)
        _lib.call("f2s_offset_attention_backward", _lib.ptr(query), _lib.ptr(key),
                  _lib.ptr(value), batch, points, width, channels, _lib.ptr(out),
                  _lib.ptr(grad_output), _lib.ptr(gq), _lib.ptr(gk), _lib.ptr(gv), _lib.ptr(ws),
                  ws.numel(), _lib.stream_handle())
        return gq, gk, gv


def reduce_neighbor_messages(content, geometry, indices, hpe_input_weight, hpe_input_bias,
                             hpe_output_weight, hpe_output_bias, hpe_norm_weight, hpe_norm_bias,
                             message_norm_weight, message_norm_bias, *,
                             precision: str = "fp32") -> torch.Tensor:
    """Encode relative geometry and max-reduce normalized neighbor messages.

    content  : (B, 2C, N), projected neighbor and center terms
    geometry : (B, N, K, D), compact relative coordinates
    indices  : (B, N, K)
    output   : (B, C, N)

    flow2surf/models/ops/neighbor_reduce.py:244-337, with the HPE hidden
    layer, its output projection and the reduce fused in one kernel.
    `precision` "fp32" (CUDA cores) or "bf16x3" (tcgen05: the output
    projection as split-bf16 MMAs, close to fp32; D 6, H 64 or 128, C 64, 128
    or 192, K 8, 16 or 32). Differentiable in both: the backward recomputes
    the stage in fp32 (neighbor_reduce.py:155-237).
    """
    if precision not in ("fp32", "bf16x3"):
        raise ValueError(f"precision must be 'fp32' or 'bf16x3', got {precision!r}")
    channels, hidden_channels = hpe_output_weight.shape
    input_hidden_channels, input_channels = hpe_input_weight.shape
    if content.shape[1] != 2 * channels:
        raise ValueError(f"Expected {2 * channels} content channels, got {content.shape[1]}")
    if input_hidden_channels != hidden_channels:
        raise ValueError("HPE projections disagree on hidden width: "
                         f"{input_hidden_channels} != {hidden_channels}")
    if geometry.shape[-1] != input_channels:
        raise ValueError(f"Expected {input_channels} geometry channels, got {geometry.shape[-1]}")
    if tuple(geometry.shape[:3]) != tuple(indices.shape):
        raise ValueError(f"Geometry shape {tuple(geometry.shape[:3])} does not match indices "
                         f"{tuple(indices.shape)}")
    if content.shape[0] != indices.shape[0] or content.shape[2] != indices.shape[1]:
        raise ValueError(f"Content shape {tuple(content.shape)} does not match indices "
                         f"{tuple(indices.shape)}")
    tensors = (content, geometry, indices, hpe_input_weight, hpe_input_bias, hpe_output_weight,
               hpe_output_bias, hpe_norm_weight, hpe_norm_bias, message_norm_weight,
               message_norm_bias)
    _require_cuda(*tensors)
    if _needs_grad(*tensors):
        return _NeighborMessages.apply(precision, *tensors)
    return _neighbor_forward(tensors, precision)


def _neighbor_forward(tensors, precision="fp32"):
    content, geometry, indices = tensors[:3]
    channels, hidden_channels = tensors[5].shape
    input_channels = geometry.shape[-1]
    batch, points, neighbors = indices.shape
    out = torch.empty((batch, channels, points), dtype=torch.float32, device=content.device)
    if out.numel() == 0:
        return out
    if indices.dtype != torch.int32:
        raise ValueError(f"indices must be int32, got {indices.dtype}")
    floats = [_f32(t) for t in tensors[:2]] + [_f32(t) for t in tensors[3:]]
    indices = indices.contiguous()
    ws = _workspace("f2s_neighbor_reduce_workspace_bytes", batch, points, channels)
    args = [_lib.ptr(floats[0]), _lib.ptr(floats[1]), _lib.ptr(indices)]
    args += [_lib.ptr(t) for t in floats[2:]]
    entry = "f2s_neighbor_reduce_tc" if precision == "bf16x3" else "f2s_neighbor_reduce"
    _lib.call(entry, *args, batch, points, neighbors, input_channels,
              hidden_channels, channels, _lib.ptr(out), _lib.ptr(ws), ws.numel(),
              _lib.stream_handle())
    return out


class _NeighborMessages(torch.autograd.Function):
    """reduce_neighbor_messages with its backward (_NeighborMessageFunction,
    flow2surf/models/ops/neighbor_reduce.py:113-237): the fused forward (fp32,
    or the split-bf16 tensor-core kernel, about 1e-5 relative to it), and a
    backward that recomputes the HPE rows and the contribution in fp32 (the
    gradient of the fp32 function at the same inputs)."""

    @staticmethod
    def forward(ctx, precision, *tensors):
        tensors = tuple(t.contiguous() if i == 2 else _f32(t) for i, t in enumerate(tensors))
        ctx.save_for_backward(*tensors)
        return _neighbor_forward(tensors, precision)

    @staticmethod
    def backward(ctx, grad_output):
        t = ctx.saved_tensors
        content, geometry, indices = t[:3]
        channels, hidden = t[5].shape
        batch, points, neighbors = indices.shape
        dims = geometry.shape[-1]
        grads = [torch.empty_like(x) for i, x in enumerate(t) if i != 2]
        if content.numel() == 0 or indices.numel() == 0:
            return (None,) + tuple(None if i == 2 else torch.zeros_like(x) for i, x in enumerate(t))
        grad_output = _f32(grad_output)
        ws = _workspace("f2s_neighbor_reduce_backward_workspace_bytes", batch, points,
                        neighbors, dims, hidden, channels)
        _lib.call("f2s_neighbor_reduce_backward", *[_lib.ptr(x) for x in t], batch, points,
                  neighbors, dims, hidden, channels, _lib.ptr(grad_output),
                  *[_lib.ptr(g) for g in grads], _lib.ptr(ws), ws.numel(), _lib.stream_handle())
        return (None, grads[0], grads[1], None, *grads[2:])


def hpe_activation_grad(preactivation: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                        grad_hidden: torch.Tensor):
    """Gradients of the HPE activation (moment LayerNorm, eps 1e-5, then the
    exact GELU) with respect to the pre-activations (..., H), the norm weight
    and the norm bias (flow2surf/models/ops/hpe.py:82-96)."""
    if preactivation.shape != grad_hidden.shape:
        raise ValueError(f"grad_hidden {tuple(grad_hidden.shape)} does not match "
                         f"preactivation {tuple(preactivation.shape)}")
    H = preactivation.shape[-1]
    if weight.shape != (H,) or bias.shape != (H,):
        raise ValueError(f"norm weight and bias must be ({H},)")
    _require_cuda(preactivation, weight, bias, grad_hidden)
    pre, w, b, gh = (_f32(x) for x in (preactivation, weight, bias, grad_hidden))
    rows = pre.numel() // H if H else 0
    gp, gw, gb = torch.empty_like(pre), torch.empty_like(w), torch.empty_like(b)
    if rows == 0:
        return gp, gw.zero_(), gb.zero_()
    size = ctypes.c_size_t()
    _lib.check(_lib.lib().f2s_hpe_activation_backward_workspace_bytes(rows, H, ctypes.byref(size)))
    ws = torch.empty(size.value, dtype=torch.uint8, device=pre.device)
    _lib.call("f2s_hpe_activation_backward", _lib.ptr(pre), rows, H, _lib.ptr(w), _lib.ptr(b),
              _lib.ptr(gh), _lib.ptr(gp), _lib.ptr(gw), _lib.ptr(gb), _lib.ptr(ws), ws.numel(),
              _lib.stream_handle())
    return gp, gw, gb


def reduce_messages_grad(content, contribution, indices, weight, bias, output, grad_output):
    """Gradients of the normalised message max-reduction
    (_reduce_messages_grad, flow2surf/models/ops/neighbor_reduce.py:57-72):
    content (B, 2C, N), contribution (B, N, K, C), indices (B, N, K) int32,
    weight / bias (C,), the forward's output and grad_output (B, C, N) ->
    grad_content, grad_contribution, grad_weight, grad_bias. The edges that
    reach each maximum (all exact ties) are found from the recomputed
    activations, so `output` is accepted for the reference's signature only."""
    del output
    _require_cuda(content, contribution, indices, weight, bias, grad_output)
    if indices.dtype != torch.int32:
        raise ValueError(f"indices must be int32, got {indices.dtype}")
    B, N, K = indices.shape
    C = contribution.shape[-1]
    content, contribution, weight, bias, grad_output = (
        _f32(x) for x in (content, contribution, weight, bias, grad_output))
    indices = indices.contiguous()
    gc, gk = torch.empty_like(content), torch.empty_like(contribution)
    gw, gb = torch.empty_like(weight), torch.empty_like(bias)
    if B == 0:
        return gc, gk, gw.zero_(), gb.zero_()
    ws = _workspace("f2s_neighbor_messages_backward_workspace_bytes", B, N, C)
    _lib.call("f2s_neighbor_messages_backward", _lib.ptr(content), _lib.ptr(contribution),
              _lib.ptr(indices), B, N, K, C, _lib.ptr(weight), _lib.ptr(bias),
              _lib.ptr(grad_output), _lib.ptr(gc), _lib.ptr(gk), _lib.ptr(gw), _lib.ptr(gb),
              _lib.ptr(ws), ws.numel(), _lib.stream_handle())
    return gc, gk, gw, gb


def nearest_squared_distances(first: torch.Tensor, second: torch.Tensor):
    """Return distances and indices from each 3D point set to the other.

    Inputs are (B, M, 3) and (B, N, 3). Outputs are first distances and second
    indices shaped (B, M), then second distances and first indices shaped
    (B, N) (flow2surf/training/distances.py:70-87; CUDA semantics, ties to the
    lower index).
    """
    if first.dim() != 3 or first.shape[2] != 3:
        raise ValueError(f"Expected first shaped (B, M, 3), got {tuple(first.shape)}")
    if second.dim() != 3 or second.shape[2] != 3:
        raise ValueError(f"Expected second shaped (B, N, 3), got {tuple(second.shape)}")
    if first.shape[0] != second.shape[0]:
        raise ValueError(f"Batch sizes differ: {first.shape[0]} and {second.shape[0]}")
    if first.shape[1] < 1 or second.shape[1] < 1:
        raise ValueError("Point sets must be nonempty")
    if first.dtype != second.dtype:
        raise ValueError(f"Dtypes differ: {first.dtype} and {second.dtype}")
    _require_cuda(first, second)
    if _needs_grad(first, second):
        return _NearestDistance.apply(first, second)
    return _nearest_forward(first, second)


def _needs_grad(*tensors) -> bool:
    return torch.is_grad_enabled() and any(t.requires_grad for t in tensors)


def _nearest_forward(first, second):
    first, second = _f32(first), _f32(second)
    B, M, _ = first.shape
    N = second.shape[1]
    dev = first.device
    d1 = torch.empty((B, M), dtype=torch.float32, device=dev)
    i2 = torch.empty((B, M), dtype=torch.int32, device=dev)
    d2 = torch.empty((B, N), dtype=torch.float32, device=dev)
    i1 = torch.empty((B, N), dtype=torch.int32, device=dev)
    if B == 0:
        return d1, i2, d2, i1
    ws = _workspace("f2s_nearest_workspace_bytes", B, M, N)
    _lib.call("f2s_nearest", _lib.ptr(first), _lib.ptr(second), B, M, N, _lib.ptr(d1),
              _lib.ptr(i2), _lib.ptr(d2), _lib.ptr(i1), _lib.ptr(ws), ws.numel(),
              _lib.stream_handle())
    return d1, i2, d2, i1


class _NearestDistance(torch.autograd.Function):
    """Nearest squared distances with the exact coordinate gradient
    (_NearestDistanceFunction, flow2surf/training/distances.py:20-62)."""

    @staticmethod
    def forward(ctx, first, second):
        first, second = _f32(first), _f32(second)
        d1, i2, d2, i1 = _nearest_forward(first, second)
        ctx.save_for_backward(first, second, i2, i1)
        ctx.mark_non_differentiable(i2, i1)
        return d1, i2, d2, i1

    @staticmethod
    def backward(ctx, g1, _gi2, g2, _gi1):
        first, second, i2, i1 = ctx.saved_tensors
        B, M, _ = first.shape
        N = second.shape[1]
        gf = torch.empty_like(first)
        gs = torch.empty_like(second)
        g1 = None if g1 is None else _f32(g1)
        g2 = None if g2 is None else _f32(g2)
        _lib.call("f2s_nearest_backward", _lib.ptr(first), _lib.ptr(second), B, M, N,
                  _lib.ptr(i2), _lib.ptr(i1), _lib.ptr(g1) if g1 is not None else None,
                  _lib.ptr(g2) if g2 is not None else None, _lib.ptr(gf), _lib.ptr(gs),
                  _lib.stream_handle())
        return gf, gs


def chamfer_distances(pred: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """Per-item Chamfer distance (B,) float64 of (B, M, 3) and (B, N, 3) clouds:
    mean squared nearest distance both ways (flow2surf/evaluation.py:24-28)."""
    if pred.dim() != 3 or target.dim() != 3 or pred.shape[2] != 3 or target.shape[2] != 3:
        raise ValueError("pred and target must be (B, M, 3) and (B, N, 3)")
    if pred.shape[0] != target.shape[0]:
        raise ValueError(f"Batch sizes differ: {pred.shape[0]} and {target.shape[0]}")
    if pred.shape[1] < 1 or target.shape[1] < 1:
        raise ValueError("Point sets must be nonempty")
    _require_cuda(pred, target)
    pred, target = _f32(pred), _f32(target)
    B, M, _ = pred.shape
    N = target.shape[1]
    out = torch.empty(B, dtype=torch.float64, device=pred.device)
    if B == 0:
        return out
    ws = _workspace("f2s_nearest_workspace_bytes", B, M, N)
    _lib.call("f2s_chamfer", _lib.ptr(pred), _lib.ptr(target), B, M, N, _lib.ptr(out),
              _lib.ptr(ws), ws.numel(), _lib.stream_handle())
    return out


def point_to_mesh_distances(points: torch.Tensor, vertices: torch.Tensor, faces: torch.Tensor):
    """Squared distance from each point to a triangle mesh and the closest
    triangle's index: points (M, 3), vertices (V, 3), faces (F, 3) integer ->
    (sq_distance (M,) float32, face_index (M,) int32). The quantity
    point_cloud_utils' closest_points_on_mesh returns (as a distance) for
    flow2surf/evaluation.py:31-34; ties go to the smaller face index."""
    if points.dim() != 2 or points.shape[1] != 3:
        raise ValueError(f"points must be (M, 3), got {tuple(points.shape)}")
    if vertices.dim() != 2 or vertices.shape[1] != 3:
        raise ValueError(f"vertices must be (V, 3), got {tuple(vertices.shape)}")
    if faces.dim() != 2 or faces.shape[1] != 3:
        raise ValueError(f"faces must be (F, 3), got {tuple(faces.shape)}")
    _require_cuda(points, vertices, faces)
    M, V, F = points.shape[0], vertices.shape[0], faces.shape[0]
    dev = points.device
    dist = torch.empty(M, dtype=torch.float32, device=dev)
    idx = torch.empty(M, dtype=torch.int32, device=dev)
    if M == 0:
        return dist, idx
    if V == 0 or F == 0:
        raise ValueError("the mesh is empty")
    faces = faces.to(torch.int32).contiguous()
    lo, hi = int(faces.min().item()), int(faces.max().item())
    if lo < 0 or hi >= V:
        raise ValueError(f"face indices must lie in [0, {V}), got [{lo}, {hi}]")
    points, vertices = _f32(points), _f32(vertices)
    ws = _workspace("f2s_point_to_mesh_workspace_bytes", M, F)
    _lib.call("f2s_point_to_mesh", _lib.ptr(points), M, _lib.ptr(vertices), V, _lib.ptr(faces), F,
              _lib.ptr(dist), _lib.ptr(idx), _lib.ptr(ws), ws.numel(), _lib.stream_handle())
    return dist, idx
