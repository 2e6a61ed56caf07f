"""The arithmetic bench.py measures (trunk tf32 with fp16 FFN rows, split-bf16
encoder) on the benchmark's own workloads, against the oracle:

* the full reverse-flow denoise of the 50,000-point Laplace-noise mesh cloud
  (150 patches of 1,000 points, K = 32, 3 Euler steps; flow2surf/inference.py
  :68-198), teacher-forced step by step;
* one Euler step (alpha = 0.5) of the 10,000-point noisy sphere with K = 16
  (100 patches of 1,000 points);
* the trunk alone (transformer.py:75-89) on 64 patches of 1,024 points with
  N(0, 1) features and alpha ~ U[0, 1] per patch, weights from seed 1.

The checker is the float32 torch-CPU restatement of the model
(oracle/model_torch.py), which stays within 1e-6 of the float64 NumPy oracle
(tests/test_oracle_golden.py); the fusion, weights and Euler update are the
NumPy restatement of the reference's (oracle/inference.py).
Tolerances: velocities (votes) and denoised points max-abs 1e-4.
"""

import functools
import os

import numpy as np
import pytest
import torch

from flow2surf_b200 import build_model
from flow2surf_b200.inference import (_Runner, build_plan, farthest_point_indices,
                                      patch_seed_count)
from flow2surf_b200.synthetic import DEFAULT_CONFIG, mesh_cloud, random_parameters, sphere_cloud
from oracle import inference as oinf
from oracle.model_torch import TorchOracleNet

pytestmark = pytest.mark.gpu

BENCH_PRECISION = dict(precision="tf32", encoder_precision="bf16x3")
VELOCITY_ATOL = 1e-4


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bench_model(cfg, params, precision="tf32", encoder_precision="bf16x3"):
    model = build_model(cfg, precision=precision, encoder_precision=encoder_precision)
    model.load_parameters(params)
    return model


def torch_oracle(cfg, params):
    torch.set_num_threads(os.cpu_count() or 1)
    return TorchOracleNet(cfg, params)


def test_denoise50k_bench_mode_teacher_forced(cuda):
    N, patch, seed_k = 50_000, 1000, 3
    cloud = mesh_cloud(N, seed=4, sigma_fraction=0.015, noise_type="laplace")[0]
    params = random_parameters(DEFAULT_CONFIG, seed=0)
    model = bench_model(DEFAULT_CONFIG, params)
    oracle = torch_oracle(DEFAULT_CONFIG, params)
    P = patch_seed_count(N, patch, seed_k)
    assert P == 150
    seeds = oinf.patch_seed_indices(cloud, patch, seed_k, np.random.default_rng(0))
    first = int(np.random.default_rng(0).integers(N))
    got_seeds = farthest_point_indices(dev(cloud), P, first).cpu().numpy()
    np.testing.assert_array_equal(got_seeds, seeds)
    plan = build_plan(dev(cloud), patch, dev(seeds.astype(np.int32)), 5.0)
    nbr = plan.neighbors.cpu().numpy().astype(np.int64)
    radial = plan.radial.cpu().numpy()
    want_idx, want_r = oinf.build_patch_index(cloud, seeds, patch)
    for p in range(P):
        assert set(nbr[p]) == set(want_idx[p])
    point_idx, w, wsum, uncovered = oinf.build_aggregation(nbr, radial, 5.0, N)
    runner = _Runner(model, plan, 1 << 34)
    alphas = oinf.alpha_schedule(3, 1.0, 6.0)
    x = cloud
    worst = 0.0
    for step in range(2, -1, -1):
        a = float(alphas[step])
        step_size = a - (float(alphas[step - 1]) if step > 0 else 0.0)
        out = torch.empty_like(dev(x))
        runner.step(dev(x), out, a, step_size)
        votes = oinf.predict_velocity(oracle, x, nbr, seeds, a, 15)
        got_votes = runner.votes.cpu().numpy()
        err = np.abs(got_votes - votes).max()
        worst = max(worst, err)
        assert err < VELOCITY_ATOL, f"step {step}: max-abs vote error {err}"
        assert np.abs(votes).max() > 1e-2
        want = oinf.euler_update(x, oinf.aggregate_votes(votes, point_idx, w, wsum, N),
                                 step_size, uncovered)
        got = out.cpu().numpy()
        assert np.abs(got - want).max() < VELOCITY_ATOL
        x = want
    print(f"denoise50k bench mode: worst vote error {worst:.3g}")


@functools.lru_cache(maxsize=1)
def _sphere_step_reference():
    cfg = dict(DEFAULT_CONFIG, k_neighbors=16)
    params = random_parameters(cfg, seed=0)
    noisy = sphere_cloud(10_000, seed=0)[0]
    seeds = oinf.patch_seed_indices(noisy, 1000, 10, np.random.default_rng(0))
    nbr, radial = oinf.build_patch_index(noisy, seeds, 1000)
    agg = oinf.build_aggregation(nbr, radial, 5.0, len(noisy))
    votes = oinf.predict_velocity(torch_oracle(cfg, params), noisy, nbr, seeds, 0.5, 10)
    v = oinf.aggregate_votes(votes, agg[0], agg[1], agg[2], len(noisy))
    return cfg, params, noisy, seeds, oinf.euler_update(noisy, v, 0.5, agg[3])


@pytest.mark.parametrize("precision,encoder_precision",
                         [("tf32", "bf16x3"), ("fp32", "bf16x3"), ("fp32", "fp32")])
def test_sphere10k_euler_step_modes(cuda, precision, encoder_precision):
    cfg, params, noisy, seeds, want = _sphere_step_reference()
    model = bench_model(cfg, params, precision, encoder_precision)
    plan = build_plan(dev(noisy), 1000, dev(seeds.astype(np.int32)), 5.0)
    out = torch.empty_like(dev(noisy))
    _Runner(model, plan, 1 << 32).step(dev(noisy), out, 0.5, 0.5)
    err = np.abs(out.cpu().numpy() - want).max()
    assert err < VELOCITY_ATOL, err
    assert np.abs(want - noisy).max() > 1e-3


@pytest.mark.parametrize("precision,max_abs,rel_norm", [
    ("tf32", None, 1e-3),
    ("fp32", 1e-4, 1e-5),
])
def test_trunk_64_patches(cuda, precision, max_abs, rel_norm):
    B, M, C = 64, 1024, DEFAULT_CONFIG["feat_dim"]
    params = random_parameters(DEFAULT_CONFIG, seed=1)
    rng = np.random.default_rng(1)
    x = rng.normal(size=(B, M, C)).astype(np.float32)
    alpha = rng.uniform(size=B).astype(np.float32)
    model = bench_model(DEFAULT_CONFIG, params, precision, "bf16x3")
    got = model.trunk_(dev(x), dev(alpha)).cpu().numpy()
    want = torch_oracle(DEFAULT_CONFIG, params).trunk(x, alpha)
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    worst = np.abs(got - want).max()
    print(f"trunk {precision}: normwise relative {rel:.3g}, max-abs {worst:.3g}")
    assert rel < rel_norm, rel
    if max_abs is not None:
        assert worst < max_abs, worst
    assert np.abs(want - x).max() > 1e-2   # the blocks changed the stream
