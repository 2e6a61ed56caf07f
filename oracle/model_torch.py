"""ORACLE (test infrastructure): torch-CPU restatement of Flow2SurfNet.

The same line-by-line restatement as oracle/model.py (which cites the
reference modules), written with torch CPU tensors so that every elementwise
pass and contraction runs on all host threads. bench.py times it as the CPU
baseline; tests check it against the NumPy oracle. KNN indices come from the
bit-exact C oracle.
"""

from __future__ import annotations

import numpy as np
import torch

from . import native


def _cln(x, eps=1e-6, w=None, b=None):
    """ChannelLayerNorm, two-pass (layers.py:20-27)."""
    mean = x.mean(dim=-1, keepdim=True)
    var = ((x - mean) ** 2).mean(dim=-1, keepdim=True)
    y = (x - mean) / torch.sqrt(var + eps)
    return y if w is None else y * w + b


def _mln(x, w, b, eps=1e-5):
    """Jittor LayerNorm / HPE norm: var = max(E[x^2] - E[x]^2, 0) (hpe.py:21-27)."""
    mean = x.mean(dim=-1, keepdim=True)
    var = torch.clamp((x * x).mean(dim=-1, keepdim=True) - mean * mean, min=0.0)
    scale = w / torch.sqrt(var + eps)
    return x * scale + (b - mean * scale)


def _gelu(x):
    return 0.5 * x * (1.0 + torch.erf(x * 0.7071067811865476))


def _leaky(x):
    return torch.where(x > 0, x, 0.2 * x)


class TorchOracleNet:
    """Flow2SurfNet (flow2surf/models/network.py:29-82) on torch CPU tensors."""

    def __init__(self, cfg: dict, params: dict, dtype=torch.float32):
        self.dtype = dtype
        self.p = {k: torch.from_numpy(np.asarray(v)).to(dtype) for k, v in params.items()}
        self.k = int(cfg["k_neighbors"])
        self.stage_dims = list(cfg["encoder_dims"]) + [int(cfg["feat_dim"])]
        self.num_blocks = int(cfg["num_blocks"])
        self.decoder_dims = list(cfg["decoder_dims"])

    def _w(self, name):
        w = self.p[name]
        return w.reshape(w.shape[0], w.shape[1])

    def _hpe(self, pre, x):
        p = self.p
        h = x @ p[f"{pre}.net.0.weight"].T + p[f"{pre}.net.0.bias"]
        h = _gelu(_mln(h, p[f"{pre}.net.1.weight"], p[f"{pre}.net.1.bias"]))
        return h @ p[f"{pre}.net.3.weight"].T + p[f"{pre}.net.3.bias"]

    def _stage(self, s, f, xyz, idx):
        p = self.p
        pre = f"local_encoder.stages.{s}"
        cin = f.shape[-1]
        w = p[f"{pre}.projection.weight"][:, :, 0, 0]
        wd, wc, pos = w[:, :cin], w[:, cin:2 * cin], w[:, 2 * cin:]
        content = f @ torch.cat([wd, wc - wd], 0).T
        out_w = pos @ p[f"{pre}.position_embed.net.3.weight"]
        out_b = pos @ p[f"{pre}.position_embed.net.3.bias"]
        cout = out_w.shape[0]
        B = idx.shape[0]
        bidx = torch.arange(B)[:, None, None]
        nb = xyz[bidx, idx]
        geometry = torch.cat([nb - xyz[:, :, None, :], xyz[:, :, None, :].expand_as(nb)], -1)
        hidden = geometry @ p[f"{pre}.position_embed.net.0.weight"].T + \
            p[f"{pre}.position_embed.net.0.bias"]
        hidden = _gelu(_mln(hidden, p[f"{pre}.position_embed.net.1.weight"],
                            p[f"{pre}.position_embed.net.1.bias"]))
        msg = content[bidx, idx, :cout] + content[:, :, None, cout:] + hidden @ out_w.T + out_b
        msg = _cln(msg, 1e-6, p[f"{pre}.norm.weight"], p[f"{pre}.norm.bias"])
        return _leaky(msg).amax(dim=2)

    def _condition(self, alpha):
        """AlphaEmbed (network.py:10-26)."""
        p = self.p
        e = 2.0 * torch.from_numpy(np.asarray(alpha)).to(self.dtype)[:, None] - 1.0
        cond = torch.nn.functional.silu(e @ p["alpha_emb.mlp.0.weight"].T +
                                        p["alpha_emb.mlp.0.bias"])
        return cond @ p["alpha_emb.mlp.2.weight"].T + p["alpha_emb.mlp.2.bias"]

    def _trunk(self, x, cond):
        """AdaLN-Zero blocks (transformer.py:75-89) on point-major x (B, M, C)."""
        p = self.p
        C = x.shape[-1]
        qk = C // 4
        for i in range(self.num_blocks):
            pre = f"blocks.{i}"
            mod = torch.nn.functional.silu(cond) @ p[f"{pre}.mod.1.weight"].T + \
                p[f"{pre}.mod.1.bias"]
            s1, b1, g1, s2, b2, g2 = [mod[:, None, j * C:(j + 1) * C] for j in range(6)]
            h = _cln(x) * (1.0 + s1) + b1
            qkv = h @ self._w(f"{pre}.qkv_conv.weight").T
            q, k, v = _cln(qkv[..., :qk]), _cln(qkv[..., qk:2 * qk]), qkv[..., 2 * qk:]
            col = torch.softmax(q @ k.transpose(1, 2), dim=1)
            wts = col / (col.sum(dim=-1, keepdim=True) + 1e-9)
            x = x + g1 * ((h - wts @ v) @ self._w(f"{pre}.proj.weight").T)
            h = _cln(x) * (1.0 + s2) + b2
            gate = h @ self._w(f"{pre}.ff_gate.weight").T + p[f"{pre}.ff_gate.bias"]
            val = h @ self._w(f"{pre}.ff1.weight").T + p[f"{pre}.ff1.bias"]
            x = x + g2 * ((torch.nn.functional.silu(gate) * val) @
                          self._w(f"{pre}.ff2.weight").T + p[f"{pre}.ff2.bias"])
        return x

    def trunk(self, x: np.ndarray, alpha: np.ndarray) -> np.ndarray:
        """The trunk alone on a point-major (B, M, C) residual stream."""
        with torch.no_grad():
            xt = torch.from_numpy(np.asarray(x, dtype=np.float32)).to(self.dtype)
            return self._trunk(xt, self._condition(alpha)).to(torch.float32).numpy()

    def forward(self, x_alpha: np.ndarray, alpha: np.ndarray) -> np.ndarray:
        p = self.p
        with torch.no_grad():
            x32 = np.asarray(x_alpha, dtype=np.float32)
            idx = torch.from_numpy(native.knn(x32, self.k).astype(np.int64))
            xyz = torch.from_numpy(np.ascontiguousarray(x32.transpose(0, 2, 1))).to(self.dtype)
            cond = self._condition(alpha)
            f = self._hpe("local_encoder.input_embed", xyz)
            outs = []
            for s in range(len(self.stage_dims)):
                f = self._stage(s, f, xyz, idx)
                outs.append(f)
            x = torch.cat(outs, -1) @ self._w("local_encoder.proj.0.weight").T
            x = _leaky(_cln(x, 1e-6, p["local_encoder.proj.1.weight"],
                            p["local_encoder.proj.1.bias"]))
            x = self._trunk(x, cond)
            layer = 0
            for _ in self.decoder_dims:
                x = x @ self._w(f"decoder.net.{layer}.weight").T
                x = _leaky(_cln(x, 1e-6, p[f"decoder.net.{layer + 1}.weight"],
                                p[f"decoder.net.{layer + 1}.bias"]))
                layer += 3
            v = x @ self._w(f"decoder.net.{layer}.weight").T
            return v.to(torch.float32).numpy()

    __call__ = forward
