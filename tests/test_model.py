"""Flow2SurfNet forward on the GPU against the oracle (flow2surf/models/*).

Velocity tolerance: max-abs 1e-4 for the fp32 path.
"""

import numpy as np
import pytest
import torch

from flow2surf_b200 import Flow2SurfNet, build_model
from flow2surf_b200.synthetic import DEFAULT_CONFIG, random_parameters, sphere_cloud
from oracle.model import OracleNet

TINY_CONFIG = {
    "k_neighbors": 8, "feat_dim": 32, "encoder_dims": [16, 24], "num_blocks": 2,
    "alpha_dim": 8, "ffn_ratio": 2, "decoder_dims": [16, 8],
}
VELOCITY_ATOL = 1e-4


def patches_from_cloud(cloud, count, size, seed):
    rng = np.random.default_rng(seed)
    centers = cloud[rng.choice(len(cloud), count, replace=False)]
    out = []
    for c in centers:
        order = np.argsort(((cloud - c) ** 2).sum(1), kind="stable")[:size]
        out.append((cloud[order] - c).T)
    return np.ascontiguousarray(np.stack(out), dtype=np.float32)


def gpu_forward(cfg, params, x, alpha, precision="fp32", encoder_precision=None):
    model = build_model(cfg, precision=precision, encoder_precision=encoder_precision)
    model.load_parameters(params)
    v = model(torch.from_numpy(x).cuda(), torch.from_numpy(alpha).cuda())
    return v.cpu().numpy()


@pytest.mark.gpu
def test_tiny_model_matches_reference_golden(cuda, golden):
    fix = golden("model")
    params = {k[len("param/"):]: v for k, v in fix.items() if k.startswith("param/")}
    v = gpu_forward(TINY_CONFIG, params, fix["x"], fix["alpha"])
    np.testing.assert_allclose(v, fix["velocity_f64"], rtol=0, atol=VELOCITY_ATOL)
    ora = OracleNet(TINY_CONFIG, params)(fix["x"], fix["alpha"])
    np.testing.assert_allclose(v, ora, rtol=0, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("k,points", [(32, 1024), (16, 1000)])
def test_default_model_matches_oracle(cuda, k, points):
    cfg = dict(DEFAULT_CONFIG, k_neighbors=k)
    params = random_parameters(cfg, seed=0)
    cloud = sphere_cloud(20000, seed=3)[0]
    x = patches_from_cloud(cloud, 3, points, seed=k)
    alpha = np.array([0.5, 0.791531, 0.997947], dtype=np.float32)
    v = gpu_forward(cfg, params, x, alpha)
    ref, inter = OracleNet(cfg, params)(x, alpha, return_intermediates=True)
    err = np.abs(v - ref).max()
    assert err < VELOCITY_ATOL, f"max abs velocity error {err}"
    assert np.abs(ref).max() > 1e-2  # the comparison is not vacuous


@pytest.mark.gpu
@pytest.mark.parametrize("k", [32, 16])
@pytest.mark.parametrize("precision,encoder_precision,max_abs,rel_norm", [
    ("tf32", "bf16x3", VELOCITY_ATOL, 1e-3),   # tensor cores, within the fp32/tf32 bound
    ("tf32", "tf32", None, 2e-3),              # all-tf32: normwise relative bound
    ("fp32", "bf16x3", VELOCITY_ATOL, 1e-4),
])
def test_tensor_core_model_matches_oracle(cuda, k, precision, encoder_precision, max_abs,
                                          rel_norm):
    cfg = dict(DEFAULT_CONFIG, k_neighbors=k)
    params = random_parameters(cfg, seed=0)
    cloud = sphere_cloud(20000, seed=3)[0]
    x = patches_from_cloud(cloud, 4, 1024 if k == 32 else 1000, seed=k + 1)
    alpha = np.array([0.5, 0.791531, 0.997947, 1.0], dtype=np.float32)
    v = gpu_forward(cfg, params, x, alpha, precision, encoder_precision)
    ref = OracleNet(cfg, params)(x, alpha)
    rel = np.linalg.norm(v - ref) / np.linalg.norm(ref)
    assert rel < rel_norm, f"normwise relative error {rel}"
    if max_abs is not None:
        assert np.abs(v - ref).max() < max_abs, f"max abs error {np.abs(v - ref).max()}"


@pytest.mark.gpu
@pytest.mark.parametrize("points", [777, 1001])
def test_tensor_core_trunk_ragged_patches(cuda, points):
    """The bench's mode on patches whose size is not a multiple of 8: the qkv
    GEMM writes V straight into the attention's fp16 V^T, whose rows are padded
    to a multiple of 8 keys (the padding zeroed), and the last 128-key tile is
    partly past the patch."""
    cfg = dict(DEFAULT_CONFIG, k_neighbors=16)
    params = random_parameters(cfg, seed=3)
    cloud = sphere_cloud(20000, seed=6)[0]
    x = patches_from_cloud(cloud, 3, points, seed=points)
    alpha = np.array([0.4, 0.8, 1.0], dtype=np.float32)
    v = gpu_forward(cfg, params, x, alpha, "tf32", "bf16x3")
    ref = OracleNet(cfg, params)(x, alpha)
    assert np.linalg.norm(v - ref) / np.linalg.norm(ref) < 1e-3
    assert np.abs(v - ref).max() < VELOCITY_ATOL


@pytest.mark.gpu
@pytest.mark.parametrize("k,patches,points", [(8, 3, 1000), (32, 3, 999), (16, 5, 777)])
def test_split_encoder_shapes(cuda, k, patches, points):
    """The split-bf16 neighbour stage at K = 8 and on ragged batches (the
    last tile of 128 edge rows only partly filled), trunk fp32 so the encoder
    dominates the error."""
    cfg = dict(DEFAULT_CONFIG, k_neighbors=k)
    params = random_parameters(cfg, seed=2)
    cloud = sphere_cloud(20000, seed=5)[0]
    x = patches_from_cloud(cloud, patches, points, seed=k)
    alpha = np.linspace(0.3, 1.0, patches).astype(np.float32)
    v = gpu_forward(cfg, params, x, alpha, "fp32", "bf16x3")
    ref = OracleNet(cfg, params)(x, alpha)
    err = np.abs(v - ref).max()
    assert err < VELOCITY_ATOL, f"max abs velocity error {err}"
    assert np.abs(ref).max() > 1e-2


@pytest.mark.gpu
def test_default_model_reference_golden(cuda, golden):
    fix = golden("model_default")
    params = random_parameters(DEFAULT_CONFIG, seed=int(fix["params_seed"]))
    v = gpu_forward(DEFAULT_CONFIG, params, fix["x"], fix["alpha"])
    np.testing.assert_allclose(v, fix["velocity_f64"], rtol=0, atol=VELOCITY_ATOL)


@pytest.mark.gpu
def test_fresh_model_predicts_zero_velocity(cuda):
    """As constructed, the reference's model is a zero-velocity identity flow
    (decoder.py:23-27)."""
    model = build_model(DEFAULT_CONFIG)
    x = torch.randn(2, 3, 256, device="cuda") * 0.1
    v = model(x, torch.tensor([0.3, 0.7], device="cuda"))
    assert v.shape == (2, 256, 3)
    assert torch.count_nonzero(v).item() == 0


@pytest.mark.gpu
def test_batch_independence(cuda):
    """Patches are independent: a batch gives the same bits as one at a time."""
    params = random_parameters(TINY_CONFIG, seed=9)
    rng = np.random.default_rng(1)
    x = (0.2 * rng.normal(size=(5, 3, 100))).astype(np.float32)
    alpha = rng.uniform(size=5).astype(np.float32)
    full = gpu_forward(TINY_CONFIG, params, x, alpha)
    for b in range(5):
        one = gpu_forward(TINY_CONFIG, params, x[b:b + 1], alpha[b:b + 1])
        np.testing.assert_array_equal(one[0], full[b])


def test_constructor_validation_matches_reference():
    with pytest.raises(ValueError, match="num_blocks"):
        Flow2SurfNet(num_blocks=-1)
    with pytest.raises(ValueError, match="ffn_ratio"):
        Flow2SurfNet(ffn_ratio=0)
    with pytest.raises(ValueError, match="alpha_dim"):
        Flow2SurfNet(alpha_dim=0)


def test_state_dict_round_trip():
    model = build_model(DEFAULT_CONFIG)
    params = random_parameters(DEFAULT_CONFIG, seed=4)
    model.load_parameters(params)
    sd = model.state_dict()
    assert set(sd) == set(params)
    for k in params:
        np.testing.assert_array_equal(sd[k], params[k])
    bad = dict(params)
    bad.pop("blocks.0.proj.weight")
    with pytest.raises(KeyError):
        model.load_parameters(bad)


@pytest.mark.gpu
def test_fp16_ffn_overflow_falls_back_to_fp32_rows(cuda):
    """The tf32 trunk keeps the FFN input and hidden rows in fp16; a value
    outside the fp16 range sets the device error word (2) instead of passing an
    infinity on, and the forward (and the denoise) is then run again on the
    device with fp32 FFN rows ("tf32_wide"), so the result still matches the
    oracle where the reference computes one."""
    from flow2surf_b200 import _lib
    from flow2surf_b200.inference import denoise_device

    params = random_parameters(DEFAULT_CONFIG, seed=0)
    cloud = sphere_cloud(4000, seed=3)[0]
    x = patches_from_cloud(cloud, 2, 1000, seed=1)
    alpha = np.array([0.5, 0.9], dtype=np.float32)
    _lib.check_device_error()  # clear whatever an earlier test left
    big = dict(params)
    for name in ("blocks.0.ff_gate.weight", "blocks.0.ff1.weight"):
        big[name] = (params[name] * 300.0).astype(np.float32)
    model = build_model(DEFAULT_CONFIG, precision="tf32", encoder_precision="bf16x3")
    model.load_parameters(big)
    # the fp16 rows do overflow with these weights
    out = torch.empty((2, 1000, 3), device="cuda")
    model.forward_into(torch.from_numpy(x).cuda(), torch.from_numpy(alpha).cuda(), out)
    assert _lib.read_device_error() == _lib.F2S_FP16_RANGE
    # the model call reruns with fp32 rows and agrees with the oracle
    v = model(torch.from_numpy(x).cuda(), torch.from_numpy(alpha).cuda()).cpu().numpy()
    ref = OracleNet(DEFAULT_CONFIG, big)(x, alpha)
    rel = np.linalg.norm(v - ref) / np.linalg.norm(ref)
    assert rel < 2e-3, rel
    assert np.abs(ref).max() > 1e-2
    # a whole denoise completes (no exception) and leaves the word clear
    pts = torch.from_numpy(sphere_cloud(3000, seed=4)[0]).cuda()
    res = denoise_device(model, pts, 1000, 3, 2, patch_agg_beta=5.0)
    assert torch.isfinite(res).all()
    assert _lib.read_device_error() == 0


@pytest.mark.gpu
def test_bounded_wait_that_runs_out_is_reported(cuda):
    """Every tensor-core kernel bounds its mbarrier waits; a wait that runs out
    sets device error word 1 and returns instead of hanging. The self-test
    entry waits on a barrier nothing arrives on (a few thousand polls, no copy
    or MMA in flight); the word reads 1, is cleared, and the next forward runs
    clean."""
    import ctypes

    from flow2surf_b200 import _lib

    _lib.check_device_error()  # start from a clear word
    _lib.call("f2s_selftest_wait_timeout", 4096, _lib.stream_handle())
    value = ctypes.c_int(0)
    _lib.call("f2s_device_error", ctypes.byref(value), 1, _lib.stream_handle())
    assert value.value == 1
    params = random_parameters(DEFAULT_CONFIG, seed=0)
    cloud = sphere_cloud(4000, seed=3)[0]
    x = patches_from_cloud(cloud, 2, 1000, seed=1)
    alpha = np.array([0.5, 0.9], dtype=np.float32)
    v = gpu_forward(DEFAULT_CONFIG, params, x, alpha, precision="tf32", encoder_precision="bf16x3")
    _lib.check_device_error()
    assert np.isfinite(v).all()
    # a forward during which the word is set (here: set just before it) is
    # reported by the model call, not returned; the read clears the word
    model = build_model(DEFAULT_CONFIG, precision="tf32", encoder_precision="bf16x3")
    model.load_parameters(params)
    xt, at = torch.from_numpy(x).cuda(), torch.from_numpy(alpha).cuda()
    _lib.call("f2s_selftest_wait_timeout", 4096, _lib.stream_handle())
    with pytest.raises(_lib.Flow2SurfError, match="device error 1"):
        model(xt, at)
    np.testing.assert_array_equal(model(xt, at).cpu().numpy(), v)
