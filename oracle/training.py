"""ORACLE (test infrastructure): NumPy float64 restatements of the reference's
training losses and backward kernels, the checker of the device gradients.

Each function follows the reference file and lines it cites. Nearest indices
and distances come from the bit-exact C oracle (`native`), so the index
choices match the device exactly; everything after them runs in float64.
Only tests import this module.
"""

from __future__ import annotations

import numpy as np
from scipy.special import erf

from . import native

SQRT_HALF = 0.7071067811865476
INV_SQRT_2PI = 0.3989422804014327


# ---------------------------------------------------------------------------
# nearest distances and the losses (flow2surf/training/)
# ---------------------------------------------------------------------------

def nearest_backward(first, second, second_index, first_index, grad_first_distance,
                     grad_second_distance):
    """Coordinate gradients of the nearest squared distances
    (training/cuda/nearest_distance_backward.cu:11-40, distances.py:40-62):
    d1[b, i] = |first[b, i] - second[b, j(i)]|^2 gives first[b, i] the term
    2 g1 (first_i - second_j) and second[b, j] its negative; likewise for
    the second direction. A missing gradient counts as zero."""
    first = np.asarray(first, np.float64)
    second = np.asarray(second, np.float64)
    B, M, _ = first.shape
    N = second.shape[1]
    g1 = np.zeros((B, M)) if grad_first_distance is None else np.asarray(grad_first_distance,
                                                                          np.float64)
    g2 = np.zeros((B, N)) if grad_second_distance is None else np.asarray(grad_second_distance,
                                                                           np.float64)
    gf = np.zeros_like(first)
    gs = np.zeros_like(second)
    bi = np.arange(B)[:, None]
    t1 = 2.0 * g1[..., None] * (first - second[bi, second_index])
    gf += t1
    np.add.at(gs, (np.repeat(bi, M, 1), second_index), -t1)
    t2 = 2.0 * g2[..., None] * (second - first[bi, first_index])
    gs += t2
    np.add.at(gf, (np.repeat(bi, N, 1), first_index), -t2)
    return gf, gs


def dcd_loss(pred, target, alpha, grad_loss=None):
    """Density-aware Chamfer loss (training/losses.py:8-41) per batch item,
    and the gradients of sum_b grad_loss[b] * loss[b] with respect to pred and
    target. The reciprocal multiplicities are piecewise constant (counts of
    nearest-neighbour hits), so the gradient flows through the distances only:
    d loss / d d1[b, i] = 0.5 / M * w1 * alpha * exp(-alpha d1)."""
    pred = np.asarray(pred, np.float32)
    target = np.asarray(target, np.float32)
    B, M, _ = pred.shape
    N = target.shape[1]
    d1, i2, d2, i1 = native.nearest_squared_distances(pred, target)
    d1 = d1.astype(np.float64)
    d2 = d2.astype(np.float64)
    target_mult = np.zeros((B, N))
    pred_mult = np.zeros((B, M))
    bi = np.arange(B)[:, None]
    np.add.at(target_mult, (np.repeat(bi, M, 1), i2), 1.0)
    np.add.at(pred_mult, (np.repeat(bi, N, 1), i1), 1.0)
    w1 = 1.0 / np.maximum(target_mult[bi, i2], 1.0)
    w2 = 1.0 / np.maximum(pred_mult[bi, i1], 1.0)
    e1 = np.exp(-alpha * d1)
    e2 = np.exp(-alpha * d2)
    loss = 0.5 * ((1.0 - w1 * e1).mean(axis=1) + (1.0 - w2 * e2).mean(axis=1))
    gl = np.ones(B) if grad_loss is None else np.asarray(grad_loss, np.float64)
    g1 = gl[:, None] * 0.5 / M * w1 * alpha * e1
    g2 = gl[:, None] * 0.5 / N * w2 * alpha * e2
    gp, gt = nearest_backward(pred, target, i2, i1, g1, g2)
    return loss, gp, gt


def velocity_loss(pred_velocity, target_velocity, grad_loss=None):
    """Mean squared L2 velocity error per batch item (training/losses.py:44-47)
    and its gradients."""
    p = np.asarray(pred_velocity, np.float64)
    t = np.asarray(target_velocity, np.float64)
    err = p - t
    loss = (err * err).sum(axis=-1).mean(axis=1)
    gl = np.ones(p.shape[0]) if grad_loss is None else np.asarray(grad_loss, np.float64)
    gp = 2.0 * err / p.shape[1] * gl[:, None, None]
    return loss, gp, -gp


# ---------------------------------------------------------------------------
# HPE activation (flow2surf/models/ops/hpe.py, cuda/hpe_activation_backward.cu)
# ---------------------------------------------------------------------------

def hpe_preactivation(geometry, input_weight, input_bias):
    """project_hpe_input (hpe.py:14-18): geometry (..., D) -> (..., H)."""
    return np.asarray(geometry, np.float64) @ np.asarray(input_weight, np.float64).T + \
        np.asarray(input_bias, np.float64)


def hpe_activation(pre, weight, bias):
    """_activate_hpe (hpe.py:21-27): moment LayerNorm (eps 1e-5), exact GELU."""
    mean = pre.mean(axis=-1, keepdims=True)
    var = np.maximum((pre * pre).mean(axis=-1, keepdims=True) - mean * mean, 0.0)
    scale = weight / np.sqrt(var + 1e-5)
    x = pre * scale + (bias - mean * scale)
    return 0.5 * x * (1.0 + erf(x * SQRT_HALF))


def hpe_activation_backward(pre, weight, bias, grad_hidden):
    """hpe_activation_backward.cu:10-66 (= _hpe_activation_grad_jittor,
    hpe.py:54-84): gradients of the moment LayerNorm + exact GELU with
    respect to the pre-activations, the norm weight and the norm bias. The
    variance term is dropped where the raw variance is not positive."""
    pre = np.asarray(pre, np.float64)
    w = np.asarray(weight, np.float64)
    b = np.asarray(bias, np.float64)
    gh = np.asarray(grad_hidden, np.float64)
    H = pre.shape[-1]
    mean = pre.mean(axis=-1, keepdims=True)
    raw_var = (pre * pre).mean(axis=-1, keepdims=True) - mean * mean
    inv_std = 1.0 / np.sqrt(np.maximum(raw_var, 0.0) + 1e-5)
    normalized = (pre - mean) * inv_std
    affine = normalized * w + b
    cdf = 0.5 * (erf(affine * SQRT_HALF) + 1.0)
    gelu_grad = cdf + affine * np.exp(-0.5 * affine * affine) * INV_SQRT_2PI
    ga = gh * gelu_grad
    grad_w = (ga * normalized).reshape(-1, H).sum(axis=0)
    grad_b = ga.reshape(-1, H).sum(axis=0)
    gn = ga * w
    mean_grad = gn.mean(axis=-1, keepdims=True)
    mean_proj = (gn * normalized).mean(axis=-1, keepdims=True)
    active = (raw_var > 0.0).astype(np.float64)
    grad_pre = inv_std * (gn - mean_grad - active * normalized * mean_proj)
    return grad_pre, grad_w, grad_b


# ---------------------------------------------------------------------------
# neighbour-message reduction (flow2surf/models/ops/neighbor_reduce.py)
# ---------------------------------------------------------------------------

def _messages(content, contribution, indices):
    C = contribution.shape[-1]
    B, N, K = indices.shape
    bi = np.arange(B)[:, None, None]
    neighbor = np.transpose(content[:, :C, :], (0, 2, 1))[bi, indices]      # (B, N, K, C)
    center = np.transpose(content[:, C:, :], (0, 2, 1))[:, :, None, :]      # (B, N, 1, C)
    return neighbor + center + contribution


def messages_forward(content, contribution, indices, weight, bias):
    """_reduce_messages_jittor (neighbor_reduce.py:34-44): (B, C, N)."""
    msg = _messages(np.asarray(content, np.float64), np.asarray(contribution, np.float64),
                    indices)
    mean = msg.mean(axis=-1, keepdims=True)
    var = ((msg - mean) ** 2).mean(axis=-1, keepdims=True)
    y = (msg - mean) / np.sqrt(var + 1e-6) * weight + bias
    y = np.where(y > 0, y, 0.2 * y)
    return np.transpose(y.max(axis=2), (0, 2, 1))


def messages_backward(content, contribution, indices, weight, bias, grad_output):
    """neighbor_reduce_backward.cu:20-84: the upstream gradient of each
    (point, channel) goes to every edge whose activation equals the maximum
    over the point's K edges (all exact ties), times the LeakyReLU slope;
    then through the two-pass LayerNorm (eps 1e-6) to the message, whose
    neighbour part scatters to content[:, :C, j] and centre part sums into
    content[:, C:, n]. Returns grad_content (B, 2C, N), grad_contribution
    (B, N, K, C), grad_weight (C,), grad_bias (C,)."""
    content = np.asarray(content, np.float64)
    contribution = np.asarray(contribution, np.float64)
    w = np.asarray(weight, np.float64)
    b = np.asarray(bias, np.float64)
    go = np.transpose(np.asarray(grad_output, np.float64), (0, 2, 1))[:, :, None, :]  # (B,N,1,C)
    B, N, K = indices.shape
    C = contribution.shape[-1]
    msg = _messages(content, contribution, indices)
    mean = msg.mean(axis=-1, keepdims=True)
    centered = msg - mean
    var = (centered * centered).mean(axis=-1, keepdims=True)
    inv_std = 1.0 / np.sqrt(var + 1e-6)
    normalized = centered * inv_std
    affine = normalized * w + b
    act = np.where(affine > 0, affine, 0.2 * affine)
    slope = np.where(affine > 0, 1.0, 0.2)
    tie = act == act.max(axis=2, keepdims=True)
    upstream = np.where(tie, go * slope, 0.0)
    grad_w = (upstream * normalized).reshape(-1, C).sum(axis=0)
    grad_b = upstream.reshape(-1, C).sum(axis=0)
    weighted = upstream * w
    g = inv_std * (weighted - weighted.mean(axis=-1, keepdims=True)
                   - normalized * (weighted * normalized).mean(axis=-1, keepdims=True))
    grad_content = np.zeros_like(content)
    center = g.sum(axis=2)                                                  # (B, N, C)
    grad_content[:, C:, :] = np.transpose(center, (0, 2, 1))
    gc = np.zeros((B, N, C))
    np.add.at(gc, (np.repeat(np.arange(B)[:, None, None], N, 1).repeat(K, 2), indices), g)
    grad_content[:, :C, :] = np.transpose(gc, (0, 2, 1))
    return grad_content, g, grad_w, grad_b


def reduce_neighbor_messages(content, geometry, indices, hpe_input_weight, hpe_input_bias,
                             hpe_output_weight, hpe_output_bias, hpe_norm_weight, hpe_norm_bias,
                             message_norm_weight, message_norm_bias):
    """The op's forward (neighbor_reduce.py:84-110): (B, C, N)."""
    pre = hpe_preactivation(geometry, hpe_input_weight, hpe_input_bias)
    hidden = hpe_activation(pre, np.asarray(hpe_norm_weight, np.float64),
                            np.asarray(hpe_norm_bias, np.float64))
    contribution = hidden @ np.asarray(hpe_output_weight, np.float64).T + hpe_output_bias
    return messages_forward(content, contribution, indices, message_norm_weight,
                            message_norm_bias)


def reduce_neighbor_messages_backward(content, geometry, indices, hpe_input_weight,
                                      hpe_input_bias, hpe_output_weight, hpe_output_bias,
                                      hpe_norm_weight, hpe_norm_bias, message_norm_weight,
                                      message_norm_bias, grad_output):
    """_NeighborMessageFunction.grad (neighbor_reduce.py:155-237): the
    message-reduction backward, then through the output projection, the HPE
    activation and the input projection. Returns the gradients of content,
    geometry, the HPE input weight and bias, output weight and bias, norm
    weight and bias, and the message norm weight and bias (indices get
    none)."""
    geometry = np.asarray(geometry, np.float64)
    w_in = np.asarray(hpe_input_weight, np.float64)
    w_out = np.asarray(hpe_output_weight, np.float64)
    pre = hpe_preactivation(geometry, w_in, hpe_input_bias)
    hidden = hpe_activation(pre, np.asarray(hpe_norm_weight, np.float64),
                            np.asarray(hpe_norm_bias, np.float64))
    contribution = hidden @ w_out.T + hpe_output_bias
    g_content, g_contrib, g_mw, g_mb = messages_backward(
        content, contribution, indices, message_norm_weight, message_norm_bias, grad_output)
    C, H = w_out.shape
    flat_gc = g_contrib.reshape(-1, C)
    flat_hidden = hidden.reshape(-1, H)
    grad_hidden = flat_gc @ w_out
    g_wout = flat_gc.T @ flat_hidden
    g_bout = flat_gc.sum(axis=0)
    g_pre, g_nw, g_nb = hpe_activation_backward(pre, hpe_norm_weight, hpe_norm_bias,
                                                grad_hidden.reshape(pre.shape))
    flat_gp = g_pre.reshape(-1, H)
    flat_geo = geometry.reshape(-1, geometry.shape[-1])
    g_geo = (flat_gp @ w_in).reshape(geometry.shape)
    g_win = flat_gp.T @ flat_geo
    g_bin = flat_gp.sum(axis=0)
    return g_content, g_geo, g_win, g_bin, g_wout, g_bout, g_nw, g_nb, g_mw, g_mb


# ---------------------------------------------------------------------------
# offset attention (flow2surf/models/ops/attention.py, offset_attention.cuh)
# ---------------------------------------------------------------------------

def offset_attention(query, key, value):
    """_aggregate_jittor (attention.py:15-19): softmax of q.k over the query
    axis, rows divided by their sum over keys plus 1e-9, times value."""
    q = np.asarray(query, np.float64)
    k = np.asarray(key, np.float64)
    v = np.asarray(value, np.float64)
    s = q @ k
    p = np.exp(s - s.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    w = p / (p.sum(axis=-1, keepdims=True) + 1e-9)
    return w @ v


def offset_attention_backward(query, key, value, grad_output):
    """offset_attention_backward.cu + offset_attention.cuh:130-208: with
    G^ = G / (z + 1e-9) and r = <G^, O> per query row, dV = P^T G^,
    dP = G^ V^T - r, dS = P (dP - sum over queries of P dP) per key column,
    dQ = dS K^T, dK = Q^T dS."""
    q = np.asarray(query, np.float64)
    k = np.asarray(key, np.float64)
    v = np.asarray(value, np.float64)
    g = np.asarray(grad_output, np.float64)
    s = q @ k
    p = np.exp(s - s.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    z = p.sum(axis=-1, keepdims=True) + 1e-9
    o = (p / z) @ v
    gh = g / z
    r = (gh * o).sum(axis=-1, keepdims=True)
    dv = np.transpose(p, (0, 2, 1)) @ gh
    dp = gh @ np.transpose(v, (0, 2, 1)) - r
    ds = p * (dp - (p * dp).sum(axis=1, keepdims=True))
    dq = ds @ np.transpose(k, (0, 2, 1))
    dk = np.transpose(q, (0, 2, 1)) @ ds
    return dq, dk, dv


def near_tie_mask(content, contribution, indices, weight, bias, rel=1e-5):
    """(B, C, N) mask of the (point, channel) pairs whose two largest edge
    activations differ by less than rel x the largest magnitude without
    being equal: there a float32 recompute may pick another edge than the
    float64 restatement, so tests give those pairs no upstream gradient."""
    msg = _messages(np.asarray(content, np.float64), np.asarray(contribution, np.float64),
                    indices)
    mean = msg.mean(axis=-1, keepdims=True)
    var = ((msg - mean) ** 2).mean(axis=-1, keepdims=True)
    y = (msg - mean) / np.sqrt(var + 1e-6) * weight + bias
    y = np.where(y > 0, y, 0.2 * y)
    top = np.sort(y, axis=2)
    gap = top[:, :, -1] - top[:, :, -2]
    scale = np.abs(top[:, :, -1]) + 1e-30
    near = (gap > 0) & (gap < rel * scale)
    return np.transpose(near, (0, 2, 1))
