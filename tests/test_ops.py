"""reduce_neighbor_messages and offset_attention_aggregate on the GPU against
the oracle, with the reference's layouts and error behaviour
(flow2surf/models/ops/neighbor_reduce.py:244-337, attention.py:84-106)."""

import numpy as np
import pytest
import torch

from flow2surf_b200 import knn_indices, offset_attention_aggregate, reduce_neighbor_messages
from flow2surf_b200.synthetic import knn_patches
from oracle import native
from oracle.model import OracleNet, _channel_layer_norm, _gelu, _leaky, _moment_layer_norm


def neighbor_reduce_oracle(content, geometry, idx, wi, bi, wo, bo, gh, bh, gm, bm):
    """_reduce_messages_reference (neighbor_reduce.py:75-102) in float64."""
    content = content.astype(np.float64)
    C = wo.shape[0]
    hidden = _gelu(_moment_layer_norm(geometry @ wi.T.astype(np.float64) + bi, gh, bh))
    contrib = hidden @ wo.T.astype(np.float64) + bo
    B = content.shape[0]
    cpm = np.transpose(content, (0, 2, 1))
    neigh = cpm[np.arange(B)[:, None, None], idx, :C]
    msg = neigh + cpm[:, :, None, C:] + contrib
    msg = _channel_layer_norm(msg, 1e-6, gm, bm)
    return np.transpose(_leaky(msg).max(axis=2), (0, 2, 1))


def make_stage_inputs(B, N, K, C, H, D=6, seed=0):
    rng = np.random.default_rng(seed)
    xyz, feats = knn_patches(B, N, 2 * C, seed=seed)
    idx = native.knn(xyz, K)
    pts = np.transpose(xyz, (0, 2, 1))
    nb = pts[np.arange(B)[:, None, None], idx]
    ctr = np.broadcast_to(pts[:, :, None, :], nb.shape)
    geometry = np.concatenate([nb - ctr, ctr], -1)[..., :D].astype(np.float32)
    f = lambda *s, scale=1.0: (scale * rng.uniform(-1, 1, s)).astype(np.float32)  # noqa: E731
    weights = [f(H, D), f(H, scale=0.05), f(C, H, scale=H ** -0.5), f(C, scale=0.05),
               1 + f(H, scale=0.1), f(H, scale=0.05), 1 + f(C, scale=0.1), f(C, scale=0.05)]
    return feats, geometry, idx, weights


def run_reduce(feats, geometry, idx, w):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    wi, bi, wo, bo, gh, bh, gm, bm = w
    out = reduce_neighbor_messages(t(feats), t(geometry), t(idx), t(wi), t(bi), t(wo), t(bo),
                                   t(gh), t(bh), t(gm), t(bm))
    return out.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("K,C,H", [(16, 64, 64), (32, 64, 64), (32, 128, 64), (32, 192, 128),
                                   (7, 40, 24), (1, 16, 8)])
def test_reduce_neighbor_messages_matches_oracle(cuda, K, C, H):
    feats, geometry, idx, w = make_stage_inputs(4, 300, K, C, H, seed=K + C)
    got = run_reduce(feats, geometry, idx, w)
    want = neighbor_reduce_oracle(feats, geometry.astype(np.float64), idx, *w)
    np.testing.assert_allclose(got, want, rtol=0, atol=2e-5)


@pytest.mark.gpu
def test_reduce_neighbor_messages_microbench_shape(cuda):
    """The edge micro-benchmark stage (in, out, H) = (64, 64, 64) at K = 32."""
    feats, geometry, idx, w = make_stage_inputs(8, 1024, 32, 64, 64, seed=2)
    got = run_reduce(feats, geometry, idx, w)
    want = neighbor_reduce_oracle(feats, geometry.astype(np.float64), idx, *w)
    np.testing.assert_allclose(got, want, rtol=0, atol=2e-5)


@pytest.mark.gpu
def test_reduce_neighbor_messages_errors(cuda):
    feats, geometry, idx, w = make_stage_inputs(1, 32, 4, 16, 8, seed=1)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    wi, bi, wo, bo, gh, bh, gm, bm = [t(x) for x in w]
    with pytest.raises(ValueError, match="content channels"):
        reduce_neighbor_messages(t(feats[:, :-1]), t(geometry), t(idx), wi, bi, wo, bo, gh, bh,
                                 gm, bm)
    with pytest.raises(ValueError, match="hidden width"):
        reduce_neighbor_messages(t(feats), t(geometry), t(idx), wi[:-1], bi, wo, bo, gh, bh,
                                 gm, bm)
    with pytest.raises(ValueError, match="geometry channels"):
        reduce_neighbor_messages(t(feats), t(geometry[..., :5]), t(idx), wi, bi, wo, bo, gh,
                                 bh, gm, bm)
    with pytest.raises(ValueError, match="does not match indices"):
        reduce_neighbor_messages(t(feats), t(geometry), t(idx[:, :, :3]), wi, bi, wo, bo, gh,
                                 bh, gm, bm)


@pytest.mark.gpu
@pytest.mark.parametrize("B,N,d,C", [(2, 1024, 48, 192), (3, 100, 48, 192), (2, 257, 16, 40),
                                     (1, 1, 8, 8), (2, 65, 128, 256)])
def test_offset_attention_matches_oracle(cuda, B, N, d, C):
    rng = np.random.default_rng(N + d)
    q = rng.normal(size=(B, N, d)).astype(np.float32)
    k = rng.normal(size=(B, d, N)).astype(np.float32)
    if d == 48:  # the trunk's LN-normalised q, k: |S| up to 48
        q = _channel_layer_norm(q.astype(np.float64)).astype(np.float32)
        k = np.transpose(_channel_layer_norm(np.transpose(k, (0, 2, 1)).astype(np.float64)),
                         (0, 2, 1)).astype(np.float32)
    v = rng.normal(size=(B, N, C)).astype(np.float32)
    t = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    got = offset_attention_aggregate(t(q), t(k), t(v)).cpu().numpy()
    want = OracleNet.offset_attention(q.astype(np.float64),
                                      np.transpose(k, (0, 2, 1)).astype(np.float64),
                                      v.astype(np.float64))
    np.testing.assert_allclose(got, want, rtol=0, atol=5e-5)


@pytest.mark.gpu
def test_offset_attention_shape_errors(cuda):
    t = lambda *s: torch.zeros(*s, device="cuda")  # noqa: E731
    with pytest.raises(ValueError, match="rank-3"):
        offset_attention_aggregate(t(2, 4), t(2, 4, 4), t(2, 4, 4))
    with pytest.raises(ValueError, match="Incompatible"):
        offset_attention_aggregate(t(2, 4, 3), t(2, 3, 5), t(2, 4, 6))


def run_reduce_tc(feats, geometry, idx, w):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    wi, bi, wo, bo, gh, bh, gm, bm = w
    out = reduce_neighbor_messages(t(feats), t(geometry), t(idx), t(wi), t(bi), t(wo), t(bo),
                                   t(gh), t(bh), t(gm), t(bm), precision="bf16x3")
    return out.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("K,C,H", [(8, 64, 64), (16, 128, 64), (32, 192, 128), (32, 128, 64)])
def test_reduce_neighbor_messages_tensor_cores(cuda, K, C, H):
    """The split-bf16 tensor-core kernel behind the operator (max-abs 1e-4:
    the contraction keeps ~2^-17 relative, the rest is fp32)."""
    feats, geometry, idx, w = make_stage_inputs(4, 300, K, C, H, seed=K + C + 1)
    got = run_reduce_tc(feats, geometry, idx, w)
    want = neighbor_reduce_oracle(feats, geometry.astype(np.float64), idx, *w)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("K", [16, 32])
def test_reduce_neighbor_messages_tensor_cores_microbench(cuda, K):
    """The KNN + edge micro-benchmark batch: 256 patches x 1024 points, stage
    (in, out, H) = (64, 64, 64); every patch on the GPU, a sample of 8 patches
    (independent of the others) against the float64 oracle."""
    feats, geometry, idx, w = make_stage_inputs(256, 1024, K, 64, 64, seed=2)
    got = run_reduce_tc(feats, geometry, idx, w)
    pick = np.array([0, 37, 100, 127, 128, 170, 211, 255])
    want = neighbor_reduce_oracle(feats[pick], geometry[pick].astype(np.float64), idx[pick], *w)
    np.testing.assert_allclose(got[pick], want, rtol=0, atol=1e-4)
    assert np.isfinite(got).all()


@pytest.mark.gpu
def test_reduce_neighbor_messages_tensor_core_shape_limits(cuda):
    feats, geometry, idx, w = make_stage_inputs(1, 64, 7, 40, 24, seed=3)
    with pytest.raises(ValueError, match="outside the tensor-core kernel"):
        run_reduce_tc(feats, geometry, idx, w)


def attention_inputs(B, N, d, C, seed):
    rng = np.random.default_rng(seed)
    q = _channel_layer_norm(rng.normal(size=(B, N, d))).astype(np.float32)
    k = np.transpose(_channel_layer_norm(rng.normal(size=(B, N, d))), (0, 2, 1)).astype(np.float32)
    v = rng.normal(size=(B, N, C)).astype(np.float32)
    return q, np.ascontiguousarray(k), v


@pytest.mark.gpu
@pytest.mark.parametrize("B,N,d,C,sample", [(2, 1024, 48, 192, 2), (3, 100, 48, 192, 3),
                                            (2, 257, 16, 64, 2), (512, 1024, 48, 192, 4),
                                            (2, 900, 48, 256, 2)])
def test_offset_attention_tensor_cores(cuda, B, N, d, C, sample):
    """tcgen05 path of the operator (split-bf16 scores, fp16 P V): normwise
    relative 2e-3 and max-abs 2e-3 of the largest output; the fourth case is
    the trunk micro-benchmark's attention (512 patches x 1024 points, d 48,
    C 192), a sample of its patches against the float64 oracle. Key tiles are
    128 wide: C = 256 leaves shared memory for one K stage only, and with
    N = 900 the last tile's second 64-key V box lies wholly past N."""
    q, k, v = attention_inputs(B, N, d, C, seed=N + d)
    t = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    got = offset_attention_aggregate(t(q), t(k), t(v), precision="tensor").cpu().numpy()
    pick = np.linspace(0, B - 1, sample).astype(int)
    want = OracleNet.offset_attention(q[pick].astype(np.float64),
                                      np.transpose(k[pick], (0, 2, 1)).astype(np.float64),
                                      v[pick].astype(np.float64))
    err = got[pick] - want
    assert np.linalg.norm(err) / np.linalg.norm(want) < 2e-3
    assert np.abs(err).max() < 2e-3 * np.abs(want).max()


@pytest.mark.gpu
def test_offset_attention_tensor_core_shape_limits(cuda):
    q, k, v = attention_inputs(1, 64, 8, 40, seed=1)
    t = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    with pytest.raises(ValueError, match="outside the tensor-core kernel"):
        offset_attention_aggregate(t(q), t(k), t(v), precision="tensor")
