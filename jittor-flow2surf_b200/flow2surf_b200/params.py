"""Parameter inventory of Flow2SurfNet under the reference's state-dict names.

The names and shapes are those the reference's Jittor modules register
(flow2surf/models/network.py:40-73, encoder.py:40-173, transformer.py:30-54,
decoder.py:11-29), so a checkpoint saved by the reference maps one to one.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ModelDims:
    k: int
    feat_dim: int
    num_blocks: int
    stage_dims: tuple[int, ...]      # encoder_dims + [feat_dim]
    stage_inputs: tuple[int, ...]    # [encoder_dims[0]] + stage_dims[:-1]
    alpha_dim: int
    ffn_ratio: int
    decoder_dims: tuple[int, ...]

    @property
    def qk_dim(self) -> int:
        return self.feat_dim // 4

    @property
    def hidden(self) -> int:
        return self.feat_dim * self.ffn_ratio


def model_dims(cfg: dict) -> ModelDims:
    """Dimensions implied by a config (network.py:85-95, encoder.py:141-173)."""
    feat_dim = int(cfg["feat_dim"])
    enc = [int(d) for d in cfg["encoder_dims"]]
    stage_dims = enc + [feat_dim]
    stage_inputs = [stage_dims[0]] + stage_dims[:-1]
    dims = ModelDims(
        k=int(cfg["k_neighbors"]),
        feat_dim=feat_dim,
        num_blocks=int(cfg["num_blocks"]),
        stage_dims=tuple(stage_dims),
        stage_inputs=tuple(stage_inputs),
        alpha_dim=int(cfg["alpha_dim"]),
        ffn_ratio=int(cfg["ffn_ratio"]),
        decoder_dims=tuple(int(d) for d in cfg["decoder_dims"]),
    )
    if dims.num_blocks < 0:
        raise ValueError(f"num_blocks must be >= 0, got {dims.num_blocks}")
    if dims.ffn_ratio < 1:
        raise ValueError(f"ffn_ratio must be >= 1, got {dims.ffn_ratio}")
    if dims.alpha_dim < 1:
        raise ValueError(f"alpha_dim must be >= 1, got {dims.alpha_dim}")
    if dims.qk_dim < 1:
        raise ValueError(f"channels must be >= 4, got {feat_dim}")
    return dims


def parameter_specs(cfg: dict) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, kind) in a fixed order; kind is one of
    weight / bias / norm_weight / norm_bias."""
    d = model_dims(cfg)
    specs: list[tuple[str, tuple[int, ...], str]] = []

    def linear(prefix, out_dim, in_dim, bias=True):
        specs.append((f"{prefix}.weight", (out_dim, in_dim), "weight"))
        if bias:
            specs.append((f"{prefix}.bias", (out_dim,), "bias"))

    def conv1(prefix, out_dim, in_dim, bias=True):
        specs.append((f"{prefix}.weight", (out_dim, in_dim, 1), "weight"))
        if bias:
            specs.append((f"{prefix}.bias", (out_dim,), "bias"))

    def norm(prefix, dim):
        specs.append((f"{prefix}.weight", (dim,), "norm_weight"))
        specs.append((f"{prefix}.bias", (dim,), "norm_bias"))

    def hpe(prefix, width, in_dim):
        linear(f"{prefix}.net.0", width, in_dim)
        norm(f"{prefix}.net.1", width)
        linear(f"{prefix}.net.3", width, width)

    hidden = d.alpha_dim * 4
    linear("alpha_emb.mlp.0", hidden, 1)
    linear("alpha_emb.mlp.2", d.alpha_dim, hidden)
    hpe("local_encoder.input_embed", d.stage_dims[0], 3)
    for s, (cin, cout) in enumerate(zip(d.stage_inputs, d.stage_dims)):
        pre = f"local_encoder.stages.{s}"
        hpe(f"{pre}.position_embed", cin, 6)
        specs.append((f"{pre}.projection.weight", (cout, 3 * cin, 1, 1), "weight"))
        norm(f"{pre}.norm", cout)
    conv1("local_encoder.proj.0", d.feat_dim, sum(d.stage_dims), bias=False)
    norm("local_encoder.proj.1", d.feat_dim)
    C = d.feat_dim
    for i in range(d.num_blocks):
        pre = f"blocks.{i}"
        conv1(f"{pre}.qkv_conv", C + 2 * d.qk_dim, C, bias=False)
        conv1(f"{pre}.proj", C, C, bias=False)
        conv1(f"{pre}.ff_gate", d.hidden, C)
        conv1(f"{pre}.ff1", d.hidden, C)
        conv1(f"{pre}.ff2", C, d.hidden)
        linear(f"{pre}.mod.1", 6 * C, d.alpha_dim)
    in_dim = C
    layer = 0
    for h in d.decoder_dims:
        conv1(f"decoder.net.{layer}", h, in_dim, bias=False)
        norm(f"decoder.net.{layer + 1}", h)
        in_dim = h
        layer += 3
    conv1(f"decoder.net.{layer}", 3, in_dim, bias=False)
    return specs


def parameter_count(cfg: dict) -> int:
    total = 0
    for _, shape, _ in parameter_specs(cfg):
        n = 1
        for s in shape:
            n *= s
        total += n
    return total
