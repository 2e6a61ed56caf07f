"""Training gradients and losses on the GPU against the float64 oracle
(oracle/training.py, itself pinned to torch autograd on the CPU):
nearest_distance_backward.cu, losses.py (dcd_loss, velocity_loss),
hpe_activation_backward.cu, neighbor_reduce_backward.cu (+ the op's whole
backward, neighbor_reduce.py:155-237) and offset_attention_backward.cu.

Tolerance: the device computes in fp32 (the reference's arithmetic), so
each gradient must match the float64 oracle to 1e-4 normwise relative error
(||g - g_ref|| / ||g_ref||) and elementwise to 1e-3 relative plus 1e-4 of the
largest magnitude."""

import numpy as np
import pytest
import torch

from flow2surf_b200.losses import dcd_loss, velocity_loss
from flow2surf_b200.ops import (hpe_activation_grad, nearest_squared_distances,
                                offset_attention_aggregate, reduce_messages_grad,
                                reduce_neighbor_messages)
from oracle import native
from oracle import training as ot

pytestmark = pytest.mark.gpu


def dev(a, grad=False):
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()
    return t.requires_grad_(grad)


def close(got, want, norm=1e-4):
    got = got.detach().cpu().numpy().astype(np.float64) if torch.is_tensor(got) else got
    want = np.asarray(want, np.float64)
    scale = np.abs(want).max() + 1e-30
    err = np.linalg.norm(got - want) / (np.linalg.norm(want) + 1e-30)
    assert err < norm, f"normwise relative error {err:.3g}"
    np.testing.assert_allclose(got, want, rtol=1e-3, atol=1e-4 * scale)


@pytest.mark.parametrize("B,M,N", [(2, 300, 257), (2, 5000, 6000)])
def test_nearest_backward(cuda, B, M, N):
    rng = np.random.default_rng(M)
    first = rng.normal(size=(B, M, 3)).astype(np.float32)
    second = rng.normal(size=(B, N, 3)).astype(np.float32)
    g1, g2 = rng.normal(size=(B, M)), rng.normal(size=(B, N))
    f, s = dev(first, True), dev(second, True)
    d1, i2, d2, i1 = nearest_squared_distances(f, s)
    (d1 * dev(g1)).sum().add((d2 * dev(g2)).sum()).backward()
    _, wi2, _, wi1 = native.nearest_squared_distances(first, second)
    np.testing.assert_array_equal(i2.cpu().numpy(), wi2)
    gf, gs = ot.nearest_backward(first, second, wi2, wi1, g1, g2)
    close(f.grad, gf)
    close(s.grad, gs)


def test_nearest_backward_one_direction(cuda):
    """Only the first distances used: the second gradient is absent."""
    rng = np.random.default_rng(9)
    first = rng.normal(size=(1, 400, 3)).astype(np.float32)
    second = rng.normal(size=(1, 350, 3)).astype(np.float32)
    f, s = dev(first, True), dev(second, True)
    d1, _, _, _ = nearest_squared_distances(f, s)
    d1.sum().backward()
    _, wi2, _, wi1 = native.nearest_squared_distances(first, second)
    gf, gs = ot.nearest_backward(first, second, wi2, wi1, np.ones((1, 400)), None)
    close(f.grad, gf)
    close(s.grad, gs)


@pytest.mark.parametrize("B,M,N,alpha", [(3, 2000, 1500, 40.0), (2, 8000, 9000, 100.0)])
def test_dcd_loss(cuda, B, M, N, alpha):
    rng = np.random.default_rng(N)
    pred = (rng.normal(size=(B, M, 3)) * 0.3).astype(np.float32)
    target = (rng.normal(size=(B, N, 3)) * 0.3).astype(np.float32)
    gl = rng.normal(size=B)
    p, t = dev(pred, True), dev(target, True)
    loss = dcd_loss(p, t, alpha)
    (loss * dev(gl)).sum().backward()
    want, gp, gt = ot.dcd_loss(pred, target, alpha, gl)
    np.testing.assert_allclose(loss.detach().cpu().numpy(), want, rtol=1e-5, atol=1e-6)
    close(p.grad, gp)
    close(t.grad, gt)
    with torch.no_grad():
        np.testing.assert_allclose(dcd_loss(p, t, alpha).cpu().numpy(), want, rtol=1e-5, atol=1e-6)


def test_velocity_loss(cuda):
    rng = np.random.default_rng(3)
    a, b = rng.normal(size=(4, 1000, 3)), rng.normal(size=(4, 1000, 3))
    ta, tb = dev(a, True), dev(b, True)
    loss = velocity_loss(ta, tb)
    loss.sum().backward()
    want, ga, gb = ot.velocity_loss(a.astype(np.float32), b.astype(np.float32))
    np.testing.assert_allclose(loss.detach().cpu().numpy(), want, rtol=1e-5)
    close(ta.grad, ga)
    close(tb.grad, gb)


@pytest.mark.parametrize("H", [64, 128, 48])
def test_hpe_activation_grad(cuda, H):
    rng = np.random.default_rng(H)
    pre = rng.normal(size=(2, 64, 16, H)) * 1.5 + 0.2
    w, b = 1 + 0.2 * rng.normal(size=H), 0.1 * rng.normal(size=H)
    gh = rng.normal(size=pre.shape)
    gp, gw, gb = hpe_activation_grad(dev(pre), dev(w), dev(b), dev(gh))
    wp, ww, wb = ot.hpe_activation_backward(pre.astype(np.float32), w.astype(np.float32),
                                            b.astype(np.float32), gh.astype(np.float32))
    close(gp, wp)
    close(gw, ww)
    close(gb, wb)


def _message_case(seed, B, N, K, C):
    rng = np.random.default_rng(seed)
    content = rng.normal(size=(B, 2 * C, N)).astype(np.float32)
    contribution = rng.normal(size=(B, N, K, C)).astype(np.float32)
    idx = rng.integers(0, N, size=(B, N, K)).astype(np.int32)
    w = (1 + 0.2 * rng.normal(size=C)).astype(np.float32)
    b = (0.1 * rng.normal(size=C)).astype(np.float32)
    go = rng.normal(size=(B, C, N)).astype(np.float32)
    return content, contribution, idx, w, b, go


@pytest.mark.parametrize("C,K", [(64, 16), (192, 32), (40, 8)])
def test_reduce_messages_grad(cuda, C, K):
    content, contribution, idx, w, b, go = _message_case(C + K, 2, 200, K, C)
    go[ot.near_tie_mask(content, contribution, idx, w, b)] = 0.0
    out = ot.messages_forward(content, contribution, idx, w, b)
    got = reduce_messages_grad(dev(content), dev(contribution), torch.from_numpy(idx).cuda(),
                               dev(w), dev(b), dev(out), dev(go))
    want = ot.messages_backward(content, contribution, idx, w, b, go)
    for g, r in zip(got, want):
        close(g, r)


def test_reduce_messages_grad_ties(cuda):
    """Duplicate edges tie exactly: each gets the full upstream gradient."""
    content, contribution, idx, w, b, go = _message_case(11, 1, 150, 8, 64)
    idx[:, :, 1] = idx[:, :, 0]
    contribution[:, :, 1] = contribution[:, :, 0]
    got = reduce_messages_grad(dev(content), dev(contribution), torch.from_numpy(idx).cuda(),
                               dev(w), dev(b), None, dev(go))
    gk = got[1].cpu().numpy()
    np.testing.assert_array_equal(gk[:, :, 0], gk[:, :, 1])
    want = ot.messages_backward(content, contribution, idx, w, b, go)
    close(got[1], want[1])
    close(got[0], want[0])


@pytest.mark.parametrize("N,K,H,C,precision", [(128, 16, 64, 64, "fp32"),
                                               (96, 32, 128, 192, "fp32"),
                                               (80, 8, 36, 44, "fp32"),
                                               (40, 8, 50, 24, "fp32"),
                                               (96, 32, 128, 192, "bf16x3")])
def test_reduce_neighbor_messages_backward(cuda, N, K, H, C, precision):
    """The whole neighbour-stage backward; with the split-bf16 forward the
    backward is the same fp32 recompute, so its gradients are checked to the
    same bound."""
    rng = np.random.default_rng(N + C)
    B, D = 2, 6
    content = rng.normal(size=(B, 2 * C, N))
    geometry = rng.normal(size=(B, N, K, D))
    idx = rng.integers(0, N, size=(B, N, K)).astype(np.int32)
    params = [rng.normal(size=(H, D)) * 0.5, rng.normal(size=H) * 0.1,
              rng.normal(size=(C, H)) * (1 / np.sqrt(H)), rng.normal(size=C) * 0.1,
              1 + 0.1 * rng.normal(size=H), 0.1 * rng.normal(size=H),
              1 + 0.1 * rng.normal(size=C), 0.1 * rng.normal(size=C)]
    params = [p.astype(np.float32) for p in params]
    go = rng.normal(size=(B, C, N)).astype(np.float32)
    content, geometry = content.astype(np.float32), geometry.astype(np.float32)
    hidden = ot.hpe_activation(ot.hpe_preactivation(geometry, params[0], params[1]),
                               params[4].astype(np.float64), params[5].astype(np.float64))
    contribution = hidden @ params[2].astype(np.float64).T + params[3]
    go[ot.near_tie_mask(content, contribution, idx, params[6], params[7])] = 0.0
    inputs = [dev(content, True), dev(geometry, True), torch.from_numpy(idx).cuda()]
    inputs += [dev(p, True) for p in params]
    out = reduce_neighbor_messages(*inputs, precision=precision)
    close(out, ot.reduce_neighbor_messages(content, geometry, idx, *params),
          norm=1e-5 if precision == "fp32" else 1e-4)
    (out * dev(go)).sum().backward()
    want = ot.reduce_neighbor_messages_backward(content, geometry, idx, *params, go)
    got = [inputs[0].grad, inputs[1].grad] + [t.grad for t in inputs[3:]]
    for g, r in zip(got, want):
        close(g, r)


@pytest.mark.parametrize("B,N,d,C", [(2, 300, 48, 64), (9, 130, 16, 40)])
def test_offset_attention_backward(cuda, B, N, d, C):
    rng = np.random.default_rng(N)
    q = rng.normal(size=(B, N, d)).astype(np.float32)
    k = rng.normal(size=(B, d, N)).astype(np.float32)
    v = rng.normal(size=(B, N, C)).astype(np.float32)
    # LayerNorm'd rows as in the model (bounded scores)
    q = (q - q.mean(-1, keepdims=True)) / q.std(-1, keepdims=True)
    k = (k - k.mean(1, keepdims=True)) / k.std(1, keepdims=True)
    go = rng.normal(size=(B, N, C)).astype(np.float32)
    tq, tk, tv = dev(q, True), dev(k, True), dev(v, True)
    out = offset_attention_aggregate(tq, tk, tv)
    close(out, ot.offset_attention(q, k, v), norm=1e-5)
    (out * dev(go)).sum().backward()
    dq, dk, dv = ot.offset_attention_backward(q, k, v, go)
    close(tq.grad, dq)
    close(tk.grad, dk)
    close(tv.grad, dv)


def test_tensor_core_paths_refuse_gradients(cuda):
    q = torch.zeros(1, 64, 48, device="cuda", requires_grad=True)
    k = torch.zeros(1, 48, 64, device="cuda")
    v = torch.zeros(1, 64, 64, device="cuda")
    with pytest.raises(ValueError, match="no backward"):
        offset_attention_aggregate(q, k, v, precision="tensor")
