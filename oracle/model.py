"""ORACLE (test infrastructure): NumPy restatement of Flow2SurfNet.

Follows the reference modules line by line, in point-major layout (B, N, C)
instead of the reference's channel-major (B, C, N). Parameters are a dict keyed
by the reference's Jittor state-dict names (e.g. "blocks.0.qkv_conv.weight").
Arithmetic runs in `dtype` (float64 by default, the most accurate statement of
the reference's fp32 maths); KNN indices come from the bit-exact C oracle.
"""

from __future__ import annotations

import numpy as np
from scipy.special import erf

from . import native


def _channel_layer_norm(x, eps=1e-6, weight=None, bias=None):
    """ChannelLayerNorm (flow2surf/models/layers.py:20-27): two-pass variance."""
    mean = x.mean(axis=-1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    y = (x - mean) / np.sqrt(var + eps)
    if weight is not None:
        y = y * weight + bias
    return y


def _moment_layer_norm(x, weight, bias, eps=1e-5):
    """Jittor nn.LayerNorm and the HPE activation norm
    (flow2surf/models/ops/hpe.py:21-27, hpe_hidden_forward.cu:18-29):
    var = max(E[x^2] - E[x]^2, 0)."""
    mean = x.mean(axis=-1, keepdims=True)
    second = (x * x).mean(axis=-1, keepdims=True)
    var = np.maximum(second - mean * mean, 0.0)
    scale = weight / np.sqrt(var + eps)
    return x * scale + (bias - mean * scale)


def _gelu(x):
    """erf GELU (hpe.py:27 via nn.gelu; hpe_hidden_forward.cu:31-33)."""
    return 0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))


def _silu(x):
    return x / (1.0 + np.exp(-x))


def _leaky(x):
    return np.where(x > 0, x, 0.2 * x)


def _linear(x, w, b=None):
    y = x @ w.T
    return y if b is None else y + b


def _conv_w(w):
    """1x1 Conv1d/Conv2d weight (out, in, 1[, 1]) -> (out, in)."""
    return w.reshape(w.shape[0], w.shape[1])


class OracleNet:
    """Flow2SurfNet (flow2surf/models/network.py:29-82) restated."""

    def __init__(self, cfg: dict, params: dict, dtype=np.float64):
        self.cfg = cfg
        self.dtype = dtype
        self.p = {k: np.asarray(v, dtype=dtype) for k, v in params.items()}
        self.k = int(cfg["k_neighbors"])
        self.feat_dim = int(cfg["feat_dim"])
        self.stage_dims = list(cfg["encoder_dims"]) + [self.feat_dim]
        self.stage_inputs = [self.stage_dims[0]] + self.stage_dims[:-1]
        self.num_blocks = int(cfg["num_blocks"])
        self.decoder_dims = list(cfg["decoder_dims"])

    # -- network.py:24-26 ----------------------------------------------------
    def alpha_embed(self, alpha):
        p = self.p
        e = 2.0 * np.asarray(alpha, dtype=self.dtype)[:, None] - 1.0
        h = _silu(_linear(e, p["alpha_emb.mlp.0.weight"], p["alpha_emb.mlp.0.bias"]))
        return _linear(h, p["alpha_emb.mlp.2.weight"], p["alpha_emb.mlp.2.bias"])

    # -- encoder.py:40-71 (HPE) ---------------------------------------------
    def _hpe(self, prefix, x):
        p = self.p
        h = _linear(x, p[f"{prefix}.net.0.weight"], p[f"{prefix}.net.0.bias"])
        h = _gelu(_moment_layer_norm(h, p[f"{prefix}.net.1.weight"], p[f"{prefix}.net.1.bias"]))
        return _linear(h, p[f"{prefix}.net.3.weight"], p[f"{prefix}.net.3.bias"])

    # -- encoder.py:83-115 + neighbor_reduce.py:21-42,75-102 + hpe.py:14-50 --
    def _stage(self, s, features, xyz, idx):
        """features (B, N, Cin), xyz (B, N, 3) in dtype, idx (B, N, K)."""
        p = self.p
        pre = f"local_encoder.stages.{s}"
        cin = features.shape[-1]
        weight = p[f"{pre}.projection.weight"][:, :, 0, 0]
        delta_w = weight[:, :cin]
        center_w = weight[:, cin:2 * cin]
        position_w = weight[:, 2 * cin:]
        content_w = np.concatenate([delta_w, center_w - delta_w], axis=0)   # :88-92
        content = features @ content_w.T                                      # (B, N, 2C)
        out_w = position_w @ p[f"{pre}.position_embed.net.3.weight"]          # :95
        out_b = position_w @ p[f"{pre}.position_embed.net.3.bias"]            # :96
        cout = out_w.shape[0]

        B, N, K = idx.shape
        bidx = np.arange(B)[:, None, None]
        neighbors = xyz[bidx, idx]                                            # (B, N, K, 3)
        center = np.broadcast_to(xyz[:, :, None, :], neighbors.shape)
        geometry = np.concatenate([neighbors - center, center], axis=-1)      # :26-37
        hidden = _linear(geometry, p[f"{pre}.position_embed.net.0.weight"],
                         p[f"{pre}.position_embed.net.0.bias"])
        hidden = _gelu(_moment_layer_norm(hidden, p[f"{pre}.position_embed.net.1.weight"],
                                          p[f"{pre}.position_embed.net.1.bias"]))
        contribution = hidden @ out_w.T + out_b                              # hpe.py:46-50
        message = content[bidx, idx, :cout] + content[:, :, None, cout:] + contribution
        message = _channel_layer_norm(message, 1e-6, p[f"{pre}.norm.weight"],
                                      p[f"{pre}.norm.bias"])
        return _leaky(message).max(axis=2)                                    # (B, N, C)

    def encode(self, xyz_bcn, idx=None):
        """NeighborEncoder.execute (encoder.py:175-184). xyz (B, 3, N) f32."""
        xyz32 = np.asarray(xyz_bcn, dtype=np.float32)
        if idx is None:
            idx = native.knn(xyz32, self.k)                                    # :178
        xyz = np.transpose(xyz32, (0, 2, 1)).astype(self.dtype)
        features = self._hpe("local_encoder.input_embed", xyz)                 # :177
        outputs = []
        for s in range(len(self.stage_dims)):
            features = self._stage(s, features, xyz, idx)
            outputs.append(features)
        cat = np.concatenate(outputs, axis=-1)
        p = self.p
        y = cat @ _conv_w(p["local_encoder.proj.0.weight"]).T                 # :118-123
        y = _channel_layer_norm(y, 1e-6, p["local_encoder.proj.1.weight"],
                                p["local_encoder.proj.1.bias"])
        return _leaky(y), idx

    # -- transformer.py:57-89 + attention.py:15-19 ----------------------------
    @staticmethod
    def offset_attention(query, key_t, value):
        """_aggregate_jittor (attention.py:15-19): query (B, N, d), key_t (B, N, d)
        holding keys point-major, value (B, N, C)."""
        scores = query @ np.transpose(key_t, (0, 2, 1))                       # (B, Nq, Nk)
        scores = scores - scores.max(axis=1, keepdims=True)
        e = np.exp(scores)
        column = e / e.sum(axis=1, keepdims=True)                             # softmax over queries
        weights = column / (column.sum(axis=-1, keepdims=True) + 1e-9)
        return weights @ value

    def block(self, i, x, cond):
        p = self.p
        pre = f"blocks.{i}"
        C = x.shape[-1]
        qk = C // 4
        mod = _linear(_silu(cond), p[f"{pre}.mod.1.weight"], p[f"{pre}.mod.1.bias"])
        scale1, shift1, gate1, scale2, shift2, gate2 = [
            mod[:, None, j * C:(j + 1) * C] for j in range(6)]
        h = _channel_layer_norm(x) * (1.0 + scale1) + shift1                  # :85
        qkv = h @ _conv_w(p[f"{pre}.qkv_conv.weight"]).T
        q = _channel_layer_norm(qkv[..., :qk])                                # :61-63
        k = _channel_layer_norm(qkv[..., qk:2 * qk])
        v = qkv[..., 2 * qk:]
        offset = h - self.offset_attention(q, k, v)                           # :66-68
        x = x + gate1 * (offset @ _conv_w(p[f"{pre}.proj.weight"]).T)         # :87
        h = _channel_layer_norm(x) * (1.0 + scale2) + shift2                  # :88
        gate = _linear(h, _conv_w(p[f"{pre}.ff_gate.weight"]), p[f"{pre}.ff_gate.bias"])
        val = _linear(h, _conv_w(p[f"{pre}.ff1.weight"]), p[f"{pre}.ff1.bias"])
        ff = _linear(_silu(gate) * val, _conv_w(p[f"{pre}.ff2.weight"]), p[f"{pre}.ff2.bias"])
        return x + gate2 * ff                                                 # :89

    # -- decoder.py:8-32 ----------------------------------------------------
    def decode(self, x):
        p = self.p
        layer = 0
        for _ in self.decoder_dims:
            x = x @ _conv_w(p[f"decoder.net.{layer}.weight"]).T
            x = _channel_layer_norm(x, 1e-6, p[f"decoder.net.{layer + 1}.weight"],
                                    p[f"decoder.net.{layer + 1}.bias"])
            x = _leaky(x)
            layer += 3
        return x @ _conv_w(p[f"decoder.net.{layer}.weight"]).T                # (B, N, 3)

    def forward(self, x_alpha, alpha, idx=None, return_intermediates=False):
        """Flow2SurfNet.execute (network.py:75-82): x_alpha (B, 3, M) -> (B, M, 3)."""
        cond = self.alpha_embed(alpha)
        x, idx = self.encode(x_alpha, idx)
        inter = {"cond": cond, "knn": idx, "encoded": x}
        for i in range(self.num_blocks):
            x = self.block(i, x, cond)
            inter[f"block{i}"] = x
        v = self.decode(x)
        return (v, inter) if return_intermediates else v

    __call__ = forward
