"""Patch-level training objectives on the device (flow2surf/training/losses.py).

Same names, arguments and per-item results as the reference; both are
differentiable with respect to their point or velocity inputs, the backward
running on the same library (no CPU path).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .ops import _f32, _needs_grad, _require_cuda


def _dcd_call(pred, target, alpha, grad_loss=None, want_grads=False):
    B, M, _ = pred.shape
    N = target.shape[1]
    loss = torch.empty(B, dtype=torch.float32, device=pred.device)
    gp = torch.empty_like(pred) if want_grads else None
    gt = torch.empty_like(target) if want_grads else None
    if B == 0:
        return loss, gp, gt
    size = ctypes.c_size_t()
    _lib.check(_lib.lib().f2s_dcd_loss_workspace_bytes(B, M, N, ctypes.byref(size)))
    ws = torch.empty(size.value, dtype=torch.uint8, device=pred.device)
    _lib.call("f2s_dcd_loss", _lib.ptr(pred), _lib.ptr(target), B, M, N, float(alpha),
              _lib.ptr(loss), _lib.ptr(grad_loss), _lib.ptr(gp), _lib.ptr(gt), _lib.ptr(ws),
              ws.numel(), _lib.stream_handle())
    return loss, gp, gt


class _DcdLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred, target, alpha):
        pred, target = _f32(pred), _f32(target)
        ctx.save_for_backward(pred, target)
        ctx.alpha = alpha
        return _dcd_call(pred, target, alpha)[0]

    @staticmethod
    def backward(ctx, grad_loss):
        pred, target = ctx.saved_tensors
        _, gp, gt = _dcd_call(pred, target, ctx.alpha, _f32(grad_loss), want_grads=True)
        return gp, gt, None


def dcd_loss(pred: torch.Tensor, target: torch.Tensor, alpha: float) -> torch.Tensor:
    """Density-aware Chamfer loss per point set (B,): reciprocal
    nearest-neighbour multiplicity weights and an exponential kernel on the
    squared distances (flow2surf/training/losses.py:8-41). pred (B, M, 3),
    target (B, N, 3) float32 CUDA tensors; alpha a float."""
    if pred.dim() != 3 or pred.shape[2] != 3:
        raise ValueError(f"Expected first shaped (B, M, 3), got {tuple(pred.shape)}")
    if target.dim() != 3 or target.shape[2] != 3:
        raise ValueError(f"Expected second shaped (B, N, 3), got {tuple(target.shape)}")
    if pred.shape[0] != target.shape[0]:
        raise ValueError(f"Batch sizes differ: {pred.shape[0]} and {target.shape[0]}")
    if pred.shape[1] < 1 or target.shape[1] < 1:
        raise ValueError("Point sets must be nonempty")
    _require_cuda(pred, target)
    if _needs_grad(pred, target):
        return _DcdLoss.apply(pred, target, float(alpha))
    return _dcd_call(_f32(pred), _f32(target), float(alpha))[0]


def _velocity_call(pred, target, grad_loss=None, want_loss=True, want_grads=False):
    B, M, _ = pred.shape
    loss = torch.empty(B, dtype=torch.float32, device=pred.device) if want_loss else None
    gp = torch.empty_like(pred) if want_grads else None
    gt = torch.empty_like(target) if want_grads else None
    if B == 0 or M == 0:
        if loss is not None:
            loss.fill_(float("nan") if M == 0 else 0.0)
        return loss, (gp.zero_() if gp is not None else None), (gt.zero_() if gt is not None else None)
    _lib.call("f2s_velocity_loss", _lib.ptr(pred), _lib.ptr(target), B, M, _lib.ptr(loss),
              _lib.ptr(grad_loss), _lib.ptr(gp), _lib.ptr(gt), _lib.stream_handle())
    return loss, gp, gt


class _VelocityLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred, target):
        pred, target = _f32(pred), _f32(target)
        ctx.save_for_backward(pred, target)
        return _velocity_call(pred, target)[0]

    @staticmethod
    def backward(ctx, grad_loss):
        pred, target = ctx.saved_tensors
        _, gp, gt = _velocity_call(pred, target, _f32(grad_loss), want_loss=False,
                                   want_grads=True)
        return gp, gt


def velocity_loss(pred_velocity: torch.Tensor, target_velocity: torch.Tensor) -> torch.Tensor:
    """Mean squared L2 velocity error for each patch in the batch (B,)
    (flow2surf/training/losses.py:44-47); (B, M, 3) inputs."""
    if pred_velocity.shape != target_velocity.shape or pred_velocity.dim() != 3:
        raise ValueError(f"velocities must share a (B, M, 3) shape, got "
                         f"{tuple(pred_velocity.shape)} and {tuple(target_velocity.shape)}")
    _require_cuda(pred_velocity, target_velocity)
    if _needs_grad(pred_velocity, target_velocity):
        return _VelocityLoss.apply(pred_velocity, target_velocity)
    return _velocity_call(_f32(pred_velocity), _f32(target_velocity))[0]
