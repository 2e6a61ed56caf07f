"""Pin the oracle against golden vectors produced by the reference's own code.

The fixtures in tests/golden/ come from running the reference's Python
(flow2surf/flow.py, inference.py, models/*, the operators' CPU fallbacks)
through tests/golden/make_golden.py. These tests need no GPU.
"""

import numpy as np
import pytest

from conftest import near_tie_rows
from oracle import inference as oinf
from oracle import native
from oracle.model import OracleNet
from flow2surf_b200.synthetic import DEFAULT_CONFIG, random_parameters

TINY_CONFIG = {
    "k_neighbors": 8, "feat_dim": 32, "encoder_dims": [16, 24], "num_blocks": 2,
    "alpha_dim": 8, "ffn_ratio": 2, "decoder_dims": [16, 8],
}


def _params(fix):
    return {k[len("param/"):]: v for k, v in fix.items() if k.startswith("param/")}


def test_alpha_schedule_matches_reference(golden):
    fix = golden("flow")
    for i in range(5):
        n, c, p = fix[f"case{i}_args"]
        got = oinf.alpha_schedule(int(n), c, p)
        np.testing.assert_array_equal(got, fix[f"case{i}_alpha"])
    np.testing.assert_allclose(oinf.alpha_schedule(3, 1, 6), [0.791531, 0.997947, 1.0],
                               atol=1e-6)


@pytest.mark.parametrize("case", ["xyz", "pad", "feat", "single", "surface"])
def test_knn_oracle_matches_reference_cpu_path(golden, case):
    """The reference's CPU path (bmm + topk) agrees with its CUDA kernel's key
    order except where two distances are within rounding; those rows are
    excluded, all others must be identical."""
    fix = golden("knn")
    features, k = fix[f"{case}_features"], int(fix[f"{case}_k"])
    got = native.knn(features, k)
    want = fix[f"{case}_indices"]
    assert got.shape == want.shape
    if features.shape[-1] > 1:
        ok = ~near_tie_rows(features, k)
        assert ok.mean() > 0.9
        np.testing.assert_array_equal(got[ok], want[ok])
    else:
        np.testing.assert_array_equal(got, want)


def test_knn_oracle_edge_cases():
    rng = np.random.default_rng(0)
    f = rng.normal(size=(3, 3, 6)).astype(np.float32)
    out = native.knn(f, 9)                      # k > N-1: pad with the last index
    assert out.shape == (3, 6, 9)
    assert np.all(out[..., 5:] == out[..., 4:5])
    for b in range(3):
        for q in range(6):
            assert q not in out[b, q]
            assert sorted(out[b, q, :5]) == sorted(set(range(6)) - {q})
    dup = np.zeros((1, 3, 8), dtype=np.float32)   # all points coincide: ties by index
    out = native.knn(dup, 4)
    for q in range(8):
        assert list(out[0, q]) == [j for j in range(8) if j != q][:4]
    assert np.all(native.knn(rng.normal(size=(2, 3, 1)).astype(np.float32), 3) == 0)


@pytest.mark.parametrize("case", ["sphere", "dupes", "small"])
def test_fps_oracle_matches_reference(golden, case):
    fix = golden("fps")
    got = native.farthest_point_indices(fix[f"{case}_points"], int(fix[f"{case}_count"]),
                                        int(fix[f"{case}_first"]))
    np.testing.assert_array_equal(got, fix[f"{case}_indices"])


def test_model_oracle_matches_reference_float64(golden):
    """Same weights, same inputs, same KNN graph: the restatement equals the
    reference's modules to float64 rounding."""
    fix = golden("model")
    net = OracleNet(TINY_CONFIG, _params(fix))
    v = net(fix["x"], fix["alpha"], idx=fix["knn_f64"])
    np.testing.assert_allclose(v, fix["velocity_f64"], rtol=0, atol=1e-12)
    # and against the reference run in float32, as Jittor computes it
    np.testing.assert_allclose(v, fix["velocity_f32"], rtol=0, atol=2e-6)


def test_model_oracle_knn_graph_matches_reference(golden):
    fix = golden("model")
    idx = native.knn(fix["x"], TINY_CONFIG["k_neighbors"])
    ok = ~near_tie_rows(fix["x"], TINY_CONFIG["k_neighbors"])
    np.testing.assert_array_equal(idx[ok], fix["knn_f32"][ok])


def test_default_model_oracle_matches_reference(golden):
    fix = golden("model_default")
    params = random_parameters(DEFAULT_CONFIG, seed=int(fix["params_seed"]))
    import hashlib
    h = hashlib.sha256()
    for name in sorted(params):
        h.update(name.encode())
        h.update(np.ascontiguousarray(params[name], dtype=np.float32).tobytes())
    assert h.hexdigest() == str(fix["params_sha256"]), "weight generator changed"
    net = OracleNet(DEFAULT_CONFIG, params)
    v = net(fix["x"], fix["alpha"], idx=fix["knn_f64"])
    np.testing.assert_allclose(v, fix["velocity_f64"], rtol=0, atol=1e-11)


def test_patch_denoise_oracle_matches_reference(golden):
    """The reference's patch_denoise (FPS, cKDTree patches, bincount fusion,
    Euler) against the restatement, both driving the same float64 model."""
    fix = golden("denoise")
    params = random_parameters(TINY_CONFIG, seed=5)
    net = OracleNet(TINY_CONFIG, params)
    seed_idx = oinf.patch_seed_indices(fix["noisy"], 128, 4,
                                       np.random.default_rng(int(fix["rng_seed"])))
    np.testing.assert_array_equal(seed_idx, fix["seed_idx"])
    out = oinf.patch_denoise(
        net, fix["noisy"], patch_size=int(fix["arg_patch_size"]), seed_k=int(fix["arg_seed_k"]),
        num_steps=int(fix["arg_num_steps"]), num_chunks=int(fix["arg_num_chunks"]),
        rng=np.random.default_rng(int(fix["rng_seed"])),
        patch_agg_beta=float(fix["arg_patch_agg_beta"]),
        alpha_clean_power=float(fix["arg_alpha_clean_power"]),
        alpha_noisy_power=float(fix["arg_alpha_noisy_power"]))
    assert out.dtype == np.float32
    err = np.abs(out - fix["denoised_f64"])
    # identical except where a float32 KNN near-tie flips a neighbour between
    # the reference's bmm/topk CPU path and the kernel's key order
    per_point = err.max(axis=1)
    assert np.mean(per_point > 1e-6) < 0.02
    assert per_point.max() < 1e-4
    moved = np.abs(fix["denoised_f64"] - fix["noisy"]).max()
    assert moved > 1e-3


def test_nearest_oracle_matches_reference_cpu_path(golden):
    fix = golden("nearest")
    d1, i2, d2, i1 = native.nearest_squared_distances(fix["first"], fix["second"])
    # the CPU path's |a|^2 + |b|^2 - 2<a,b> cancels: its error is a few float32
    # ulps of the squared norms (<= ~10 here), not of the distance itself
    np.testing.assert_allclose(d1, fix["d1"], rtol=0, atol=1e-5)
    np.testing.assert_allclose(d2, fix["d2"], rtol=0, atol=1e-5)
    assert (i2 == fix["i2"]).mean() > 0.99
    assert (i1 == fix["i1"]).mean() > 0.99


def test_chamfer_oracle_matches_reference(golden):
    fix = golden("nearest")
    got = oinf.chamfer_distance(fix["pred"], fix["target"])
    assert abs(got - float(fix["chamfer"])) < 1e-12
    d1, _ = native.nearest_one_way(fix["pred"][None], fix["target"][None])
    d2, _ = native.nearest_one_way(fix["target"][None], fix["pred"][None])
    kernel_form = float(d1.astype(np.float64).mean() + d2.astype(np.float64).mean())
    assert abs(kernel_form - float(fix["chamfer"])) < 1e-5


def test_torch_cpu_oracle_matches_numpy_oracle(golden):
    """The torch-CPU restatement (timed as the CPU baseline) computes the same
    model as the NumPy oracle."""
    from oracle.model_torch import TorchOracleNet

    fix = golden("model")
    params = _params(fix)
    got = TorchOracleNet(TINY_CONFIG, params, dtype=__import__("torch").float64)(
        fix["x"], fix["alpha"])
    want = OracleNet(TINY_CONFIG, params)(fix["x"], fix["alpha"])
    # the torch restatement returns float32 velocities
    np.testing.assert_allclose(got, want, rtol=1e-7, atol=1e-9)
    np.testing.assert_allclose(got, fix["velocity_f64"], rtol=0, atol=1e-5)


def test_torch_float32_oracle_tracks_float64_oracle_on_default_model():
    """The float32 torch-CPU restatement is the checker of the large GPU
    parity tests (whole 50k-point denoise steps, the 64-patch trunk): on the
    default architecture it stays within 1e-6 of the float64 NumPy oracle,
    two orders below the 1e-4 velocity tolerance."""
    import torch

    from flow2surf_b200.synthetic import DEFAULT_CONFIG, random_parameters
    from oracle.model_torch import TorchOracleNet

    params = random_parameters(DEFAULT_CONFIG, seed=0)
    rng = np.random.default_rng(11)
    x = (0.1 * rng.normal(size=(2, 3, 300))).astype(np.float32)
    alpha = np.array([0.5, 0.997947], dtype=np.float32)
    ref = OracleNet(DEFAULT_CONFIG, params)
    want, inter = ref(x, alpha, return_intermediates=True)
    got = TorchOracleNet(DEFAULT_CONFIG, params)(x, alpha)
    assert np.abs(got - want).max() < 1e-6
    assert np.abs(want).max() > 1e-2
    # the trunk alone, on the encoded stream
    trunk = TorchOracleNet(DEFAULT_CONFIG, params, dtype=torch.float32).trunk(
        inter["encoded"].astype(np.float32), alpha)
    want_t = inter[f"block{DEFAULT_CONFIG['num_blocks'] - 1}"]
    assert np.abs(trunk - want_t).max() < 1e-5 * max(1.0, np.abs(want_t).max())
