"""The training oracle (oracle/training.py) pinned on the CPU: each restated
backward of the reference (flow2surf/training/cuda/nearest_distance_backward.cu,
models/ops/cuda/hpe_activation_backward.cu, neighbor_reduce_backward.cu,
offset_attention_backward.cu, training/losses.py) must equal torch float64
autograd of the restated forward, and the message reduction must route the
upstream gradient to every exact tie as the reference's kernel does."""

import numpy as np
import pytest
import torch

from oracle import native
from oracle import training as ot

TOL = dict(rtol=1e-9, atol=1e-11)


def _t(a):
    return torch.tensor(np.asarray(a, np.float64), requires_grad=True)


def test_nearest_backward_matches_autograd():
    rng = np.random.default_rng(0)
    first = rng.normal(size=(2, 70, 3)).astype(np.float32)
    second = rng.normal(size=(2, 50, 3)).astype(np.float32)
    _, i2, _, i1 = native.nearest_squared_distances(first, second)
    g1, g2 = rng.normal(size=(2, 70)), rng.normal(size=(2, 50))
    f, s = _t(first), _t(second)
    bi = torch.arange(2)[:, None]
    d1 = ((f - s[bi, torch.from_numpy(i2).long()]) ** 2).sum(-1)
    d2 = ((s - f[bi, torch.from_numpy(i1).long()]) ** 2).sum(-1)
    ((d1 * torch.from_numpy(g1)).sum() + (d2 * torch.from_numpy(g2)).sum()).backward()
    gf, gs = ot.nearest_backward(first, second, i2, i1, g1, g2)
    np.testing.assert_allclose(gf, f.grad.numpy(), **TOL)
    np.testing.assert_allclose(gs, s.grad.numpy(), **TOL)
    gf0, gs0 = ot.nearest_backward(first, second, i2, i1, None, g2)
    assert np.abs(gf0).sum() > 0 and np.isfinite(gs0).all()


def test_dcd_loss_matches_autograd():
    rng = np.random.default_rng(1)
    pred = rng.normal(size=(3, 60, 3)).astype(np.float32)
    target = rng.normal(size=(3, 45, 3)).astype(np.float32)
    alpha, gl = 40.0, rng.normal(size=3)
    loss, gp, gt = ot.dcd_loss(pred, target, alpha, gl)
    _, i2, _, i1 = native.nearest_squared_distances(pred, target)
    p, t = _t(pred), _t(target)
    bi = torch.arange(3)[:, None]
    i2t, i1t = torch.from_numpy(i2).long(), torch.from_numpy(i1).long()
    d1 = ((p - t[bi, i2t]) ** 2).sum(-1)
    d2 = ((t - p[bi, i1t]) ** 2).sum(-1)
    tm = torch.zeros(3, 45, dtype=torch.float64).scatter_add(1, i2t, torch.ones(3, 60,
                                                                                 dtype=torch.float64))
    pm = torch.zeros(3, 60, dtype=torch.float64).scatter_add(1, i1t, torch.ones(3, 45,
                                                                                 dtype=torch.float64))
    w1 = 1.0 / torch.clamp(tm.gather(1, i2t), min=1.0)
    w2 = 1.0 / torch.clamp(pm.gather(1, i1t), min=1.0)
    want = 0.5 * ((1 - w1 * torch.exp(-alpha * d1)).mean(1) + (1 - w2 * torch.exp(-alpha * d2)).mean(1))
    (want * torch.from_numpy(gl)).sum().backward()
    np.testing.assert_allclose(loss, want.detach().numpy(), rtol=1e-6)  # float32 distances
    np.testing.assert_allclose(gp, p.grad.numpy(), rtol=1e-6, atol=1e-9)
    np.testing.assert_allclose(gt, t.grad.numpy(), rtol=1e-6, atol=1e-9)


def test_velocity_loss_matches_autograd():
    rng = np.random.default_rng(2)
    a, b = rng.normal(size=(2, 30, 3)), rng.normal(size=(2, 30, 3))
    loss, ga, gb = ot.velocity_loss(a, b)
    ta, tb = _t(a), _t(b)
    ((ta - tb) ** 2).sum(-1).mean(1).sum().backward()
    np.testing.assert_allclose(ga, ta.grad.numpy(), **TOL)
    np.testing.assert_allclose(gb, tb.grad.numpy(), **TOL)
    np.testing.assert_allclose(loss, ((a - b) ** 2).sum(-1).mean(1), **TOL)


def _torch_hpe(pre, w, b):
    mean = pre.mean(-1, keepdim=True)
    var = torch.clamp((pre * pre).mean(-1, keepdim=True) - mean * mean, min=0.0)
    scale = w / torch.sqrt(var + 1e-5)
    x = pre * scale + (b - mean * scale)
    return 0.5 * x * (1 + torch.erf(x * ot.SQRT_HALF))


def test_hpe_activation_backward_matches_autograd():
    rng = np.random.default_rng(3)
    pre = rng.normal(size=(2, 5, 4, 64)) * 2 + 0.3
    w, b = rng.normal(size=64), rng.normal(size=64)
    gh = rng.normal(size=pre.shape)
    tp, tw, tb = _t(pre), _t(w), _t(b)
    (_torch_hpe(tp, tw, tb) * torch.from_numpy(gh)).sum().backward()
    gp, gw, gb = ot.hpe_activation_backward(pre, w, b, gh)
    np.testing.assert_allclose(gp, tp.grad.numpy(), rtol=1e-8, atol=1e-10)
    np.testing.assert_allclose(gw, tw.grad.numpy(), rtol=1e-8, atol=1e-10)
    np.testing.assert_allclose(gb, tb.grad.numpy(), rtol=1e-8, atol=1e-10)


def _torch_messages(content, contribution, idx, w, b):
    B, N, K = idx.shape
    C = contribution.shape[-1]
    bi = torch.arange(B)[:, None, None]
    nb = content[:, :C, :].permute(0, 2, 1)[bi, idx]
    ce = content[:, C:, :].permute(0, 2, 1)[:, :, None, :]
    msg = nb + ce + contribution
    mean = msg.mean(-1, keepdim=True)
    var = ((msg - mean) ** 2).mean(-1, keepdim=True)
    y = (msg - mean) / torch.sqrt(var + 1e-6) * w + b
    y = torch.where(y > 0, y, 0.2 * y)
    return y.max(dim=2).values.permute(0, 2, 1)


def _message_case(seed, B=2, N=40, K=8, C=24):
    rng = np.random.default_rng(seed)
    content = rng.normal(size=(B, 2 * C, N))
    contribution = rng.normal(size=(B, N, K, C))
    idx = rng.integers(0, N, size=(B, N, K)).astype(np.int64)
    w, b = rng.normal(size=C), rng.normal(size=C)
    go = rng.normal(size=(B, C, N))
    return content, contribution, idx, w, b, go


def test_messages_backward_matches_autograd():
    content, contribution, idx, w, b, go = _message_case(4)
    want = ot.messages_forward(content, contribution, idx, w, b)
    tc, tk, tw, tb = _t(content), _t(contribution), _t(w), _t(b)
    out = _torch_messages(tc, tk, torch.from_numpy(idx), tw, tb)
    np.testing.assert_allclose(out.detach().numpy(), want, **TOL)
    (out * torch.from_numpy(go)).sum().backward()
    gc, gk, gw, gb = ot.messages_backward(content, contribution, idx, w, b, go)
    for got, ref in ((gc, tc), (gk, tk), (gw, tw), (gb, tb)):
        np.testing.assert_allclose(got, ref.grad.numpy(), rtol=1e-8, atol=1e-10)


def test_messages_backward_routes_to_every_tie():
    """Two identical edges (the same neighbour, no contribution difference)
    tie for the maximum wherever either wins: the reference kernel gives each
    the full upstream gradient (neighbor_reduce_backward.cu:59-62)."""
    content, contribution, idx, w, b, go = _message_case(5, K=4)
    idx[:, :, 1] = idx[:, :, 0]
    contribution[:, :, 1] = contribution[:, :, 0]
    _, gk, _, _ = ot.messages_backward(content, contribution, idx, w, b, go)
    np.testing.assert_array_equal(gk[:, :, 0], gk[:, :, 1])
    assert np.abs(gk[:, :, 0]).sum() > 0


def test_reduce_neighbor_messages_backward_matches_autograd():
    rng = np.random.default_rng(6)
    B, N, K, D, H, C = 2, 30, 8, 6, 32, 24
    content = rng.normal(size=(B, 2 * C, N))
    geometry = rng.normal(size=(B, N, K, D))
    idx = rng.integers(0, N, size=(B, N, K)).astype(np.int64)
    params = [rng.normal(size=(H, D)) * 0.5, rng.normal(size=H) * 0.1,
              rng.normal(size=(C, H)) * 0.3, rng.normal(size=C) * 0.1,
              1 + 0.1 * rng.normal(size=H), 0.1 * rng.normal(size=H),
              1 + 0.1 * rng.normal(size=C), 0.1 * rng.normal(size=C)]
    go = rng.normal(size=(B, C, N))
    tc, tg = _t(content), _t(geometry)
    tp = [_t(p) for p in params]
    pre = tg @ tp[0].T + tp[1]
    hidden = _torch_hpe(pre, tp[4], tp[5])
    contribution = hidden @ tp[2].T + tp[3]
    out = _torch_messages(tc, contribution, torch.from_numpy(idx), tp[6], tp[7])
    np.testing.assert_allclose(out.detach().numpy(),
                               ot.reduce_neighbor_messages(content, geometry, idx, *params), **TOL)
    (out * torch.from_numpy(go)).sum().backward()
    got = ot.reduce_neighbor_messages_backward(content, geometry, idx, *params, go)
    refs = [tc, tg] + tp
    for g, r in zip(got, refs):
        np.testing.assert_allclose(g, r.grad.numpy(), rtol=1e-7, atol=1e-9)


def test_offset_attention_backward_matches_autograd():
    rng = np.random.default_rng(7)
    B, N, d, C = 2, 37, 8, 12
    q, k, v = rng.normal(size=(B, N, d)), rng.normal(size=(B, d, N)), rng.normal(size=(B, N, C))
    go = rng.normal(size=(B, N, C))
    tq, tk, tv = _t(q), _t(k), _t(v)
    s = tq @ tk
    p = torch.softmax(s, dim=1)
    o = (p / (p.sum(-1, keepdim=True) + 1e-9)) @ tv
    np.testing.assert_allclose(o.detach().numpy(), ot.offset_attention(q, k, v), **TOL)
    (o * torch.from_numpy(go)).sum().backward()
    dq, dk, dv = ot.offset_attention_backward(q, k, v, go)
    for g, r in ((dq, tq), (dk, tk), (dv, tv)):
        np.testing.assert_allclose(g, r.grad.numpy(), rtol=1e-8, atol=1e-10)
