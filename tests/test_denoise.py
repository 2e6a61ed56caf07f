"""Device patch_denoise against the oracle and the reference goldens
(flow2surf/inference.py:19-198)."""

import numpy as np
import pytest
import torch
from scipy.spatial import cKDTree

from flow2surf_b200 import build_model
from flow2surf_b200.inference import (DenoisePlan, _Runner, build_plan, farthest_point_indices,
                                      patch_denoise, patch_seed_count)
from flow2surf_b200.synthetic import DEFAULT_CONFIG, mesh_cloud, random_parameters, sphere_cloud
from oracle import inference as oinf
from oracle import native
from oracle.model import OracleNet

pytestmark = pytest.mark.gpu

TINY_CONFIG = {
    "k_neighbors": 8, "feat_dim": 32, "encoder_dims": [16, 24], "num_blocks": 2,
    "alpha_dim": 8, "ffn_ratio": 2, "decoder_dims": [16, 8],
}


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("case", ["sphere", "dupes", "small"])
def test_fps_reference_golden(cuda, golden, case):
    fix = golden("fps")
    got = farthest_point_indices(dev(fix[f"{case}_points"]), int(fix[f"{case}_count"]),
                                 int(fix[f"{case}_first"]))
    np.testing.assert_array_equal(got.cpu().numpy(), fix[f"{case}_indices"])


@pytest.mark.parametrize("n,count", [(50_000, 150), (100_000, 60), (130_000, 40), (257, 257),
                                     (400_000, 300), (2_400_000, 12)])
def test_fps_bit_exact(cuda, n, count):
    """Covers one CTA, 8-CTA clusters with the slice in shared memory, the
    cooperative grid (130k and 400k points) and the cluster with the running
    minima in global memory (2.4M points)."""
    pts = mesh_cloud(n, seed=4)[0] if n >= 1000 else sphere_cloud(n, seed=1)[0]
    first = 17 % n
    got = farthest_point_indices(dev(pts), count, first).cpu().numpy()
    np.testing.assert_array_equal(got, native.farthest_point_indices(pts, count, first))


def test_patch_index_matches_ckdtree(cuda):
    pts = mesh_cloud(20_000, seed=4)[0]
    seeds = native.farthest_point_indices(pts, 60, 3)
    k = 1000
    plan = build_plan(dev(pts), k, dev(seeds.astype(np.int32)), 5.0)
    nbr = plan.neighbors.cpu().numpy()
    radial = plan.radial.cpu().numpy()
    want_idx, want_r = oinf.build_patch_index(pts, seeds, k)
    assert (nbr == want_idx).mean() > 0.9999  # order may differ only on exact distance ties
    for p in range(len(seeds)):
        assert set(nbr[p]) == set(want_idx[p])
    np.testing.assert_allclose(radial, want_r, rtol=0, atol=1e-15)
    want_w = np.exp(-5.0 * want_r * want_r)
    np.testing.assert_allclose(plan.weights.cpu().numpy(), want_w, rtol=4e-16, atol=0)


def test_fusion_sums_match_bincount(cuda):
    pts = sphere_cloud(5000, seed=2)[0]
    seeds = native.farthest_point_indices(pts, 40, 0)
    plan = build_plan(dev(pts), 300, dev(seeds.astype(np.int32)), 5.0)
    nbr = plan.neighbors.cpu().numpy().reshape(-1)
    w = plan.weights.cpu().numpy().reshape(-1)
    wsum = np.bincount(nbr, weights=w, minlength=len(pts))
    np.testing.assert_array_equal(plan.weight_sum.cpu().numpy(), wsum)   # same order, same bits
    offsets = plan.offsets.cpu().numpy()
    entries = plan.entries.cpu().numpy()
    assert offsets[-1] == len(nbr)
    for n in range(0, len(pts), 97):
        seg = entries[offsets[n]:offsets[n + 1]]
        np.testing.assert_array_equal(seg, np.flatnonzero(nbr == n))


def test_fuse_euler_bit_exact(cuda):
    """aggregate_votes + Euler (inference.py:158-171,193-195), uncovered
    points included, against NumPy given the same votes."""
    pts = sphere_cloud(6000, seed=7)[0]
    seeds = native.farthest_point_indices(pts, 12, 5)
    plan = build_plan(dev(pts), 256, dev(seeds.astype(np.int32)), 5.0)
    rng = np.random.default_rng(0)
    votes = (0.05 * rng.normal(size=(12, 256, 3))).astype(np.float32)

    class Fixed:
        def __call__(self, x, alpha):
            return dev(votes)

    runner = _Runner(Fixed(), plan, 1 << 30)
    out = torch.empty_like(dev(pts))
    alphas = oinf.alpha_schedule(3, 1.0, 6.0)
    step = float(alphas[2]) - float(alphas[1])
    runner.step(dev(pts), out, float(alphas[2]), step)
    nbr = plan.neighbors.cpu().numpy()
    point_idx, w, wsum, uncovered = oinf.build_aggregation(
        nbr, plan.radial.cpu().numpy(), 5.0, len(pts))
    assert uncovered.any()
    v = oinf.aggregate_votes(votes, point_idx, w, wsum, len(pts))
    want = oinf.euler_update(pts, v, step, uncovered)
    np.testing.assert_array_equal(out.cpu().numpy(), want)


def tiny_model(params):
    model = build_model(TINY_CONFIG)
    model.load_parameters(params)
    return model


def test_patch_denoise_reference_golden(cuda, golden):
    fix = golden("denoise")
    params = random_parameters(TINY_CONFIG, seed=5)
    out = patch_denoise(
        tiny_model(params), fix["noisy"], patch_size=int(fix["arg_patch_size"]),
        seed_k=int(fix["arg_seed_k"]), num_steps=int(fix["arg_num_steps"]),
        num_chunks=int(fix["arg_num_chunks"]), rng=np.random.default_rng(int(fix["rng_seed"])),
        patch_agg_beta=float(fix["arg_patch_agg_beta"]),
        alpha_clean_power=float(fix["arg_alpha_clean_power"]),
        alpha_noisy_power=float(fix["arg_alpha_noisy_power"]))
    assert out.dtype == np.float32 and out.shape == fix["noisy"].shape
    err = np.abs(out - fix["denoised_f64"]).max(axis=1)
    # as for the oracle: equal except where a later step's KNN near-tie flips
    assert np.mean(err > 1e-4) < 0.01
    assert np.quantile(err, 0.99) < 1e-5


def test_patch_denoise_per_step_parity(cuda):
    """Each Euler step from the same input state: device step vs oracle step
    (teacher forcing removes the compounding of float32 KNN near-ties)."""
    params = random_parameters(TINY_CONFIG, seed=5)
    model = tiny_model(params)
    noisy = sphere_cloud(3000, seed=21)[0]
    trace = []
    oinf.patch_denoise(OracleNet(TINY_CONFIG, params), noisy, 128, 6, 3, 4,
                       rng=np.random.default_rng(3), patch_agg_beta=5.0,
                       alpha_clean_power=1.0, alpha_noisy_power=6.0, trace=trace)
    seeds = oinf.patch_seed_indices(noisy, 128, 6, np.random.default_rng(3))
    plan = build_plan(dev(noisy), 128, dev(seeds.astype(np.int32)), 5.0)
    runner = _Runner(model, plan, 1 << 30)
    levels = [t[0] for t in trace]               # descending: 1.0, 0.997947, 0.791531
    previous = levels[1:] + [0.0]
    for (alpha, x_in, votes, velocity, x_out), a_prev in zip(trace, previous):
        out = torch.empty_like(dev(x_in))
        runner.step(dev(x_in), out, alpha, alpha - a_prev)
        np.testing.assert_allclose(runner.votes.cpu().numpy(), votes, rtol=0, atol=1e-4)
        np.testing.assert_allclose(out.cpu().numpy(), x_out, rtol=0, atol=1e-4)


def test_single_euler_step_sphere_default_model(cuda):
    """One reverse-flow Euler step (alpha = 0.5) of a 10,000-point noisy unit
    sphere: 100 FPS patches of 1,000 points, K = 16, default architecture with
    random weights (seed 0); x' = x - 0.5 v."""
    cfg = dict(DEFAULT_CONFIG, k_neighbors=16)
    params = random_parameters(cfg, seed=0)
    model = build_model(cfg)
    model.load_parameters(params)
    noisy = sphere_cloud(10_000, seed=0)[0]
    assert patch_seed_count(10_000, 1000, 10) == 100
    seeds = oinf.patch_seed_indices(noisy, 1000, 10, np.random.default_rng(0))
    plan = build_plan(dev(noisy), 1000, dev(seeds.astype(np.int32)), 5.0)
    out = torch.empty_like(dev(noisy))
    _Runner(model, plan, 1 << 30).step(dev(noisy), out, 0.5, 0.5)
    nbr, radial = oinf.build_patch_index(noisy, seeds, 1000)
    agg = oinf.build_aggregation(nbr, radial, 5.0, len(noisy))
    votes = oinf.predict_velocity(OracleNet(cfg, params), noisy, nbr, seeds, 0.5, 10)
    v = oinf.aggregate_votes(votes, agg[0], agg[1], agg[2], len(noisy))
    want = oinf.euler_update(noisy, v, 0.5, agg[3])
    err = np.abs(out.cpu().numpy() - want).max()
    assert err < 1e-4, err
    assert np.abs(want - noisy).max() > 1e-3
