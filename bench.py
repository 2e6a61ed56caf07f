#!/usr/bin/env python
"""Denoised points/s of the full reverse flow on B200.

Workload (per GPU, weak scaling: each rank denoises its own cloud): a
50,000-point synthetic cloud sampled area-uniform on a random union of 4
ellipsoids and 2 boxes, normalised to the unit sphere, with rotation-invariant
Laplace noise (sigma = 0.015 x bbox diagonal); 1,000-point patches at
farthest-point seeds with ~3x overlap (seed_k = 3 -> 150 patches), the default
configuration's architecture (K = 32, feat 192, 3 trunk blocks) with random
weights (seed 0), the default schedule (3 Euler steps, alpha powers 1 / 6),
centre-weighted fusion (beta = 5). One step = one full patch_denoise of the
cloud: FPS seeds, patch index, fusion structure, 3 x (gather, model forward
over all patches, fusion + Euler).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

`value` is timed on the device with CUDA events (cloud resident in HBM, L2
flushed between steps); `e2e` is the same metric through the public
patch_denoise with a pinned host array in and a host array out. The
`reference` arm times the CPU restatement of the reference's path on the host
cores (the reference's Jittor is not installed here) on a bounded sample of
the same cloud. Two more legs ride on the line, outside the timed steps:
`chamfer` (the denoised cloud against a 100,000-point clean sample of its
surface, by the exact grid search), `one_cloud` (strong scaling: one
400,000-point cloud split by patch across the ranks, one NCCL all-reduce of
the vote sums per Euler step, with that all-reduce's own time) and `batch`
(the multi-GPU batch: 64 clouds of 100,000 points with noise sigma drawn
from U[0.005, 0.025] x the bounding-box diagonal, sharded by cloud over the
ranks, each denoised and scored by its Chamfer distance against a 100,000-point
clean sample of its surface).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "jittor-flow2surf_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "denoised points/sec (full reverse flow)"
UNIT = "points/s"
DENOISE = dict(patch_size=1000, seed_k=3, num_steps=3, patch_agg_beta=5.0,
               alpha_clean_power=1.0, alpha_noisy_power=6.0)
L2_FLUSH_BYTES = 512 << 20
TRACED_STEPS = 5


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--points", type=int, default=50_000)
    p.add_argument("--seed-k", type=int, default=DENOISE["seed_k"])
    p.add_argument("--cpu-sample-patches", type=int, default=60,
                   help="patches of the cloud in the bounded CPU-baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-one-cloud", action="store_true",
                   help="skip the strong-scaling leg (one 400k-point cloud split by patch)")
    p.add_argument("--no-batch", action="store_true",
                   help="skip the batch leg (64 clouds of 100k points sharded by cloud)")
    p.add_argument("--precision", choices=["fp32", "tf32"], default="tf32",
                   help="arithmetic of the trunk and decoder contractions")
    p.add_argument("--encoder-precision", choices=["fp32", "tf32", "bf16x3"], default="bf16x3",
                   help="arithmetic of the neighbour-stage contractions")
    p.add_argument("--one-cloud", action="store_true",
                   help="all ranks denoise one cloud of --points, its patches split across "
                        "the GPUs with one NCCL all-reduce of the vote sums per Euler step "
                        "(strong scaling) instead of one cloud per GPU")
    p.add_argument("--profile-chamfer", action="store_true",
                   help="instead of the benchmark: two Chamfer evaluations of a denoised-size "
                        "cloud against a 100,000-point clean sample and exit (ncu case)")
    p.add_argument("--profile-training", action="store_true",
                   help="instead of the benchmark: time the training losses and backward "
                        "passes at the reference's training shapes (64 patches of 1024 "
                        "points, K 32) and exit")
    p.add_argument("--profile-forward", type=int, default=0, metavar="B",
                   help="instead of the benchmark: two model forwards on B synthetic "
                        "1000-point patches and exit (a small case for ncu captures)")
    return p.parse_args()


def profile_forward(args) -> None:
    """Two forwards of the default architecture on B patches: the first warms
    up, the second is the one an ncu capture skips to (-s <launches of one
    forward>)."""
    import torch

    from flow2surf_b200 import build_model
    from flow2surf_b200.synthetic import DEFAULT_CONFIG, random_parameters

    B = args.profile_forward
    model = build_model(DEFAULT_CONFIG, precision=args.precision,
                        encoder_precision=args.encoder_precision)
    model.load_parameters(random_parameters(DEFAULT_CONFIG, seed=0))
    gen = torch.Generator().manual_seed(0)
    x = (torch.randn(B, 3, DENOISE["patch_size"], generator=gen) * 0.3).cuda()
    alpha = torch.full((B,), 0.5).cuda()
    for _ in range(2):
        v = model(x, alpha)
    torch.cuda.synchronize()
    print(json.dumps({"profile_forward": B, "checksum": float(v.abs().sum())}), flush=True)


CHAMFER_REFERENCE_POINTS = 100_000


def chamfer_leg(points, reference, repeats: int = 3) -> dict:
    """Chamfer of `points` (N, 3) against `reference` (R, 3) on the device
    (flow2surf/evaluation.py:24-28 with the nearest-distance search), timed
    with CUDA events. Sets of 4096 points or more take the exact uniform-grid
    search (the same bits as the all-pairs scan, from a few hundred candidate
    pairs per query), so the rate is given in queries (points of both sets)
    per second, not in pairs."""
    import torch

    from flow2surf_b200.ops import chamfer_distances

    a, b = points[None].contiguous(), reference[None].contiguous()
    value = chamfer_distances(a, b)  # warm-up
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(repeats):
        value = chamfer_distances(a, b)
    stop.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / repeats
    queries = a.shape[1] + b.shape[1]
    grid = min(a.shape[1], b.shape[1]) >= 4096
    return {"value": float(value.item()), "ms": ms, "points": int(a.shape[1]),
            "reference_points": int(b.shape[1]), "queries_per_s": queries / (ms * 1e-3),
            "method": "uniform grid, exact" if grid else "all pairs"}


ONE_CLOUD_POINTS = 400_000


def one_cloud_leg(model, world: int, dev, steps: int = 3, warmup: int = 1) -> dict:
    """Strong scaling: one 400,000-point cloud (the same on every rank) denoised
    with its patches split across the ranks (each rank builds the patch index
    of its own patches; one NCCL all-reduce of the float64 vote sums per Euler
    step). Device time per denoise, max over ranks; the all-reduce's own time
    from CUDA events around it."""
    import torch
    import torch.distributed as dist

    from flow2surf_b200.inference import denoise_device, patch_seed_count

    group = dist.group.WORLD if world > 1 else None
    pts = torch.from_numpy(make_cloud(ONE_CLOUD_POINTS, 0)).to(dev)
    run = lambda ev=None: denoise_device(model, pts, rng=np.random.default_rng(0),  # noqa: E731
                                         process_group=group, collective_events=ev, **DENOISE)
    for _ in range(warmup):
        run()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    events: list = []
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        run(events)
    stop.record()
    torch.cuda.synchronize(dev)
    t = torch.tensor([start.elapsed_time(stop) / steps,
                      sum(a.elapsed_time(b) for a, b in events) / steps],
                     dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ar_ms = t.tolist()
    return {"points": ONE_CLOUD_POINTS,
            "patches": patch_seed_count(ONE_CLOUD_POINTS, DENOISE["patch_size"], DENOISE["seed_k"]),
            "ranks": world, "scaling": "strong", "steps": steps, "ms_per_step": ms,
            "value": ONE_CLOUD_POINTS / (ms * 1e-3), "unit": UNIT,
            "allreduce_ms_per_step": ar_ms if world > 1 else 0.0,
            "allreduce_bytes_per_step": (DENOISE["num_steps"] * ONE_CLOUD_POINTS * 24
                                         if world > 1 else 0)}


def profile_chamfer(args) -> None:
    """Two Chamfer evaluations (denoise-size cloud vs 100k clean sample)."""
    import torch

    from flow2surf_b200.synthetic import mesh_cloud

    noisy, _, ref = mesh_cloud(args.points, seed=4, sigma_fraction=0.015, noise_type="laplace",
                               clean_points=CHAMFER_REFERENCE_POINTS)
    line = chamfer_leg(torch.from_numpy(noisy).cuda(), torch.from_numpy(ref).cuda(), repeats=1)
    print(json.dumps({"profile_chamfer": line["ms"]}), flush=True)


def _event_ms(fn, repeats: int = 3) -> float:
    import torch

    for _ in range(3):  # warm-up (the caching allocator reaches its working set too)
        fn()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(repeats):
        fn()
    stop.record()
    torch.cuda.synchronize()
    return start.elapsed_time(stop) / repeats


def profile_training(args) -> None:
    """The training losses and backward passes at the reference's training
    shapes (configs/default.yaml: 8 meshes x 8 patches of 1024 points, K 32,
    feature width 192, dcd_alpha 8000; the last neighbour stage: 6 geometry
    inputs, HPE width 128, 192 channels), forward + backward each, timed with
    CUDA events on synthetic inputs."""
    import torch

    from flow2surf_b200.losses import dcd_loss, velocity_loss
    from flow2surf_b200.ops import offset_attention_aggregate, reduce_neighbor_messages

    B, N, K, D, H, C, d = 64, 1024, 32, 6, 128, 192, 48
    g = torch.Generator(device="cuda").manual_seed(0)

    def rnd(*shape, scale=1.0, grad=True):
        return (torch.randn(*shape, generator=g, device="cuda") * scale).requires_grad_(grad)

    out = {}
    pred, target = rnd(B, N, 3, scale=0.3), rnd(B, N, 3, scale=0.3, grad=False)
    out["dcd_loss_ms"] = _event_ms(lambda: dcd_loss(pred, target, 8000.0).sum().backward())
    vp, vt = rnd(B, N, 3), rnd(B, N, 3, grad=False)
    out["velocity_loss_ms"] = _event_ms(lambda: velocity_loss(vp, vt).sum().backward())
    content = rnd(B, 2 * C, N)
    geometry = rnd(B, N, K, D)
    idx = torch.randint(0, N, (B, N, K), generator=g, device="cuda", dtype=torch.int32)
    params = [rnd(H, D, scale=0.5), rnd(H, scale=0.1), rnd(C, H, scale=H ** -0.5),
              rnd(C, scale=0.1), (1 + rnd(H, scale=0.1, grad=False)).requires_grad_(),
              rnd(H, scale=0.1), (1 + rnd(C, scale=0.1, grad=False)).requires_grad_(),
              rnd(C, scale=0.1)]
    go = torch.randn(B, C, N, generator=g, device="cuda")
    fwd = _event_ms(lambda: reduce_neighbor_messages(content, geometry, idx, *params).detach())
    both = _event_ms(lambda: (reduce_neighbor_messages(content, geometry, idx, *params) * go)
                     .sum().backward())
    out["neighbor_reduce_forward_ms"] = fwd
    out["neighbor_reduce_backward_ms"] = both - fwd
    out["neighbor_reduce_forward_bf16x3_ms"] = _event_ms(
        lambda: reduce_neighbor_messages(content, geometry, idx, *params,
                                         precision="bf16x3").detach())
    q = torch.nn.functional.layer_norm(torch.randn(B, N, d, generator=g, device="cuda"), (d,))
    k = torch.nn.functional.layer_norm(torch.randn(B, N, d, generator=g, device="cuda"),
                                       (d,)).transpose(1, 2).contiguous()
    q.requires_grad_()
    k.requires_grad_()
    v = rnd(B, N, C)
    ga = torch.randn(B, N, C, generator=g, device="cuda")
    afwd = _event_ms(lambda: offset_attention_aggregate(q, k, v).detach())
    aboth = _event_ms(lambda: (offset_attention_aggregate(q, k, v) * ga).sum().backward())
    out["offset_attention_forward_ms"] = afwd
    out["offset_attention_backward_ms"] = aboth - afwd
    flops = B * 2.0 * N * N * (3 * d + 2 * C)  # S, dV, G V^T, dQ, dK
    out["offset_attention_backward_tflops"] = flops / ((aboth - afwd) * 1e-3) / 1e12
    out["shapes"] = {"patches": B, "points": N, "k": K, "hpe": H, "channels": C, "qk": d}
    print(json.dumps({"profile_training": out}), flush=True)


def workload_config(args, world: int) -> dict:
    from flow2surf_b200.inference import patch_seed_count

    patches = patch_seed_count(args.points, DENOISE["patch_size"], args.seed_k)
    where = f"split by patch across {world} GPU(s)" if args.one_cloud else "per GPU"
    return {
        "workload": (f"full reverse-flow denoise of one {args.points:,}-point synthetic cloud "
                     f"{where} ({patches} patches x {DENOISE['patch_size']} points, "
                     f"{DENOISE['num_steps']} Euler steps)"),
        "points_per_cloud": args.points,
        "clouds": 1 if args.one_cloud else world,
        "patch_size": DENOISE["patch_size"],
        "seed_k": args.seed_k,
        "patches": patches,
        "num_steps": DENOISE["num_steps"],
        "alpha_powers": [1, 6],
        "patch_agg_beta": DENOISE["patch_agg_beta"],
        "k_neighbors": 32,
        "architecture": "configs/default.yaml (feat 192, encoder 64/128, 3 blocks, ffn x8)",
        "weights": "random init, seed 0",
        "l2": f"flushed between timed steps ({L2_FLUSH_BYTES >> 20} MiB write, untimed)",
        "parallelism": (f"one cloud sharded by patch over {world} GPU(s), NCCL all-reduce of "
                        "the float64 vote sums (24 bytes per point) per Euler step"
                        if args.one_cloud else f"shard by cloud, {world} GPU(s), no collective"),
    }


BATCH_CLOUDS = 64
BATCH_POINTS = 100_000


def batch_leg(model, world: int, rank: int, dev) -> dict:
    """The multi-GPU batch: 64 synthetic clouds of 100,000 points (the
    denoise cloud's mesh and Laplace-noise recipe, sigma drawn from
    U[0.005, 0.025] x the bounding-box diagonal per cloud), sharded by cloud
    (rank r takes clouds r, r + N, ...; no collective). Each cloud is
    denoised and its Chamfer distance to a 100,000-point clean sample of its
    surface computed on the device. Device time of a rank's whole shard, max
    over ranks; value = all 64 clouds' points / that time (total work fixed:
    strong scaling by cloud)."""
    import torch
    import torch.distributed as dist

    from flow2surf_b200.inference import denoise_device
    from flow2surf_b200.ops import chamfer_distances
    from flow2surf_b200.synthetic import mesh_cloud

    mine = list(range(rank, BATCH_CLOUDS, world))
    clouds, refs = [], []
    for i in mine:
        sigma = float(np.random.default_rng(1000 + i).uniform(0.005, 0.025))
        noisy, _, ref = mesh_cloud(BATCH_POINTS, seed=1000 + i, sigma_fraction=sigma,
                                   noise_type="laplace", clean_points=BATCH_POINTS)
        clouds.append(torch.from_numpy(noisy).to(dev))
        refs.append(torch.from_numpy(ref).to(dev)[None])
    losses = torch.zeros(len(mine), dtype=torch.float64, device=dev)

    def shard():
        for n, (pts, ref) in enumerate(zip(clouds, refs)):
            out = denoise_device(model, pts, rng=np.random.default_rng(mine[n]), **DENOISE)
            losses[n:n + 1] = chamfer_distances(out[None], ref)

    if mine:  # warm-up on the shard's first cloud
        out = denoise_device(model, clouds[0], rng=np.random.default_rng(mine[0]), **DENOISE)
        chamfer_distances(out[None], refs[0])
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    shard()
    stop.record()
    torch.cuda.synchronize(dev)
    t = torch.tensor([start.elapsed_time(stop), float(losses.sum().item())],
                     dtype=torch.float64, device=dev)
    if world > 1:
        ms_max = t[:1].clone()
        dist.all_reduce(ms_max, op=dist.ReduceOp.MAX)
        loss_sum = t[1:].clone()
        dist.all_reduce(loss_sum, op=dist.ReduceOp.SUM)
        t = torch.cat([ms_max, loss_sum])
    ms, loss_sum = t.tolist()
    return {"clouds": BATCH_CLOUDS, "points_per_cloud": BATCH_POINTS, "ranks": world,
            "sharding": "by cloud, no collective", "scaling": "strong", "ms": ms,
            "value": BATCH_CLOUDS * BATCH_POINTS / (ms * 1e-3), "unit": UNIT,
            "chamfer_mean": loss_sum / BATCH_CLOUDS,
            "noise": "Laplace, sigma U[0.005, 0.025] x bbox diagonal per cloud"}


def make_cloud(points: int, rank: int):
    from flow2surf_b200.synthetic import mesh_cloud

    return mesh_cloud(points, seed=4 + rank, sigma_fraction=0.015, noise_type="laplace")[0]


def make_model(precision: str = "fp32", encoder_precision: str | None = None):
    from flow2surf_b200 import build_model
    from flow2surf_b200.synthetic import DEFAULT_CONFIG, random_parameters

    model = build_model(DEFAULT_CONFIG, precision=precision, encoder_precision=encoder_precision)
    model.load_parameters(random_parameters(DEFAULT_CONFIG, seed=0))
    return model


# ---------------------------------------------------------------------------
# CPU arms (the oracle restatement of the reference's path)
# ---------------------------------------------------------------------------

CPU_SAMPLE_PATCHES = 15   # patches of the cloud per reference-arm step (10 steps cover all 150)


def cpu_denoise_sample(cloud: np.ndarray, net, seed_k: int, sample: int, offset: int) -> float:
    """Seconds the CPU restatement of the reference's patch_denoise
    (flow2surf/inference.py:68-198) spends on a bounded sample of the full
    denoise of `cloud`: `sample` of its P patches (a contiguous window from
    `offset`, wrapping) through everything that scales with the patches (patch
    index, aggregation weights, and for each of the 3 Euler steps the model
    forward, the vote fusion and the update), plus the cloud's farthest-point
    seeds (all P of them, a serial per-cloud cost) charged pro rata sample / P."""
    from oracle import inference as oinf

    kw = DENOISE
    N = len(cloud)
    P = oinf.patch_seed_count(N, kw["patch_size"], seed_k)
    sample = min(sample, P)
    t0 = time.perf_counter()
    seeds = oinf.patch_seed_indices(cloud, kw["patch_size"], seed_k, np.random.default_rng(0))
    t_fps = time.perf_counter() - t0
    t1 = time.perf_counter()
    sel = seeds[(offset + np.arange(sample)) % P]
    nbr, radial = oinf.build_patch_index(cloud, sel, kw["patch_size"])
    point_idx, w, wsum, uncovered = oinf.build_aggregation(nbr, radial, kw["patch_agg_beta"], N)
    alphas = oinf.alpha_schedule(kw["num_steps"], kw["alpha_clean_power"],
                                 kw["alpha_noisy_power"])
    chunk = (P + 7) // 8  # the reference's num_chunks = 8 batching
    current = cloud.copy()
    for step in range(kw["num_steps"] - 1, -1, -1):
        a = float(alphas[step])
        a_prev = float(alphas[step - 1]) if step > 0 else 0.0
        votes = oinf.predict_velocity(net, current, nbr, sel, a, chunk)
        velocity = oinf.aggregate_votes(votes, point_idx, w, wsum, N)
        current = oinf.euler_update(current, velocity, a - a_prev, uncovered)
    return t_fps * sample / P + (time.perf_counter() - t1)


def cpu_sampler(points: int, seed_k: int):
    import torch

    from flow2surf_b200.synthetic import DEFAULT_CONFIG, random_parameters
    from oracle import inference as oinf
    from oracle.model_torch import TorchOracleNet

    torch.set_num_threads(os.cpu_count())
    cloud = make_cloud(points, 0)
    net = TorchOracleNet(DEFAULT_CONFIG, random_parameters(DEFAULT_CONFIG, seed=0))
    P = oinf.patch_seed_count(points, DENOISE["patch_size"], seed_k)
    return cloud, net, P


def cpu_sample_text(sample: int, patches: int, points: int) -> str:
    return (f"CPU restatement of the reference's path (torch-CPU float32 model, NumPy/SciPy "
            f"patch index and fusion; Jittor is not installed), all {os.cpu_count()} host "
            f"threads, on the {points:,}-point cloud itself: {sample} of its {patches} patches "
            f"per step through the patch index, weights and 3 Euler steps of forward, fusion "
            f"and update, FPS charged pro rata; points/s = points x {sample}/{patches} / time")


def cpu_baseline_line(args) -> dict:
    cloud, net, P = cpu_sampler(args.points, args.seed_k)
    sample = max(1, min(args.cpu_sample_patches, P))
    seconds = cpu_denoise_sample(cloud, net, args.seed_k, sample, 0)
    value = args.points * sample / P / seconds
    return {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
            "sample": cpu_sample_text(sample, P, args.points) + f" ({seconds:.1f} s, one sample)"}


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    cloud, net, P = cpu_sampler(args.points, args.seed_k)
    sample = min(CPU_SAMPLE_PATCHES, P)
    times = []
    for i in range(args.warmup + args.steps):
        seconds = cpu_denoise_sample(cloud, net, args.seed_k, sample, (i * sample) % P)
        if i >= args.warmup:
            times.append(seconds)
    value = args.points * sample / P / statistics.mean(times)
    ms_step = 1e3 * args.points / value     # one full denoise of the cloud at this rate
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": workload_config(args, 1),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                         "sample": cpu_sample_text(sample, P, args.points)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region.

    nvidia-smi's start-up (NVML initialisation) is heavy; `__enter__` returns
    only once the first sample has arrived, so that start-up does not overlap
    the timed steps."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines: list[str] = []
        self.text = ""

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line)

    def __enter__(self):
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()
        deadline = time.time() + 15.0
        while not self.lines and time.time() < deadline and self.proc.poll() is None:
            time.sleep(0.02)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)  # one more sample after the last timed step
            self.proc.terminate()
            try:
                self.proc.wait(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
            self.reader.join(timeout=5)
        self.text = "".join(self.lines)

    def summary(self) -> dict:
        rows = []
        for line in self.text.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm_max = max(r[1] for r in rows)
        loaded = [r for r in rows if r[0] >= 0.5 * sm_max] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[2]) if v == "Active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": sm_max,
                "reasons": reasons, "samples": len(rows)}


def kernel_flops_per_point(tag: str, dims) -> float:
    """Algorithmic FLOPs per patch point of one forward, by kernel class."""
    C, Hf, qk, K = dims.feat_dim, dims.hidden, dims.qk_dim, dims.k
    M = DENOISE["patch_size"]
    nb = dims.num_blocks
    if tag == "gemm_swiglu":
        return nb * 2 * 2 * C * Hf
    if tag == "gemm_ff2":
        return nb * 2 * Hf * C
    if tag == "gemm_qkv":
        return nb * 2 * C * (C + 2 * qk)
    if tag == "gemm_proj":
        return nb * 2 * C * C
    if tag == "attn_output":
        return nb * 2 * M * (qk + C)
    if tag == "attn_colstats":
        return nb * 2 * M * qk
    if tag == "edge_stage":
        return sum(2 * K * (6 * h + h * c) for h, c in zip(dims.stage_inputs, dims.stage_dims))
    if tag == "gemm_content":
        return sum(2 * h * 2 * c for h, c in zip(dims.stage_inputs, dims.stage_dims))
    if tag == "gemm_head":
        return 2 * sum(dims.stage_dims) * C
    return 0.0


def load_traffic() -> dict:
    """DRAM bytes per launch by kernel class from the committed ncu summary."""
    path = ROOT / "profiles" / "traffic.txt"
    out = {}
    if path.exists():
        for line in path.read_text().splitlines():
            parts = line.split()
            if len(parts) >= 2 and not line.startswith("#"):
                try:
                    out[parts[0]] = float(parts[1])
                except ValueError:
                    pass
    return out


def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d["bf16_tflops_sustained"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def roofline(kernels: dict, forwards_points: float, dims) -> dict:
    """The dominant kernel's achieved rate against its bound."""
    tag, (ms, launches) = max(kernels.items(), key=lambda kv: kv[1][0])
    pk = peaks()
    flops = kernel_flops_per_point(tag, dims) * forwards_points
    traffic = load_traffic().get(tag)
    if flops > 0:
        achieved = flops / (ms * 1e-3) / 1e12
        peak = pk["bf16_tflops_sustained"]
        return {"kernel": tag, "bound": "tensor", "achieved": achieved, "peak": peak,
                "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
                "launches": launches, "avg_launch_ms": ms / launches,
                "peak_source": f"{pk['source']} bf16 dense, sustained"}
    return {"kernel": tag, "bound": "hbm", "achieved": None, "peak": pk["hbm_gbs"],
            "unit": "GB/s", "frac": None, "traffic": traffic, "launches": launches,
            "avg_launch_ms": ms / launches, "peak_source": f"{pk['source']} HBM copy"}


def run_gpu(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    from flow2surf_b200 import trace
    from flow2surf_b200.inference import (denoise_device, patch_denoise, patch_seed_count,
                                          shard_range)
    from flow2surf_b200.params import model_dims
    from flow2surf_b200.synthetic import DEFAULT_CONFIG

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    model = make_model(args.precision, args.encoder_precision)
    shard = args.one_cloud and world > 1
    group = dist.group.WORLD if shard else None
    cloud_seed = 0 if args.one_cloud else rank
    cloud = make_cloud(args.points, cloud_seed)
    points = torch.from_numpy(cloud).to(dev)
    pinned = torch.from_numpy(cloud).pin_memory()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    kw = dict(DENOISE, seed_k=args.seed_k)
    steps, warmup = args.steps, args.warmup

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def one_step():
        return denoise_device(model, points, rng=np.random.default_rng(cloud_seed),
                              process_group=group, **kw)

    for _ in range(warmup):
        one_step()
    barrier()

    # device-timed steps (value)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    gpu_id = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(gpu_id) as clocks:
        barrier()
        for i in range(steps):
            flush.fill_(i & 0xFF)
            starts[i].record()
            out = one_step()
            stops[i].record()
        barrier()
    elapsed_ms = sum(s.elapsed_time(e) for s, e in zip(starts, stops))
    total = torch.tensor([elapsed_ms], dtype=torch.float64, device=dev)

    # per-kernel breakdown: a separate pass of the same steps with a CUDA-event
    # pair around every launch (the events cost the timed steps above nothing)
    traced_steps = min(steps, TRACED_STEPS)
    with trace.recording() as rec:
        for i in range(traced_steps):
            flush.fill_(i & 0xFF)
            one_step()
        barrier()

    # end-to-end through the public API (value measured the same way, host in/out)
    e2e_s = 0.0
    for i in range(steps):
        flush.fill_(i & 0xFF)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        host_out = patch_denoise(model, pinned, num_chunks=8,
                                 rng=np.random.default_rng(cloud_seed), device=dev,
                                 process_group=group, **kw)
        e2e_s += time.perf_counter() - t0
    barrier()
    e2e = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
        dist.all_reduce(e2e, op=dist.ReduceOp.MAX)
    if not np.all(np.isfinite(host_out)) or not torch.isfinite(out).all():
        raise RuntimeError("non-finite denoised output")
    # quality leg: Chamfer of the denoised cloud against a 100k clean sample of
    # its surface (the multi-GPU configuration's loss), on the device
    from flow2surf_b200.synthetic import mesh_cloud
    reference = mesh_cloud(args.points, seed=4 + cloud_seed, sigma_fraction=0.015,
                           noise_type="laplace", clean_points=CHAMFER_REFERENCE_POINTS)[2]
    chamfer = chamfer_leg(out, torch.from_numpy(reference).to(dev))
    one_cloud = None if args.one_cloud or args.no_one_cloud else one_cloud_leg(model, world, dev)
    batch = None if args.one_cloud or args.no_batch else batch_leg(model, world, rank, dev)
    if rank != 0:
        return

    ms_step = total.item() / steps
    clouds = 1 if args.one_cloud else world
    value = clouds * args.points / (ms_step * 1e-3)
    e2e_value = clouds * args.points * steps / e2e.item()
    dims = model_dims(DEFAULT_CONFIG)
    patches = patch_seed_count(args.points, kw["patch_size"], args.seed_k)
    if shard:  # rank 0's share, which its kernel trace covers
        begin, end = shard_range(patches, rank, world)
        patches = end - begin
    forward_points = traced_steps * kw["num_steps"] * patches * kw["patch_size"]
    kernels = rec.kernels
    total_kernel_ms = sum(ms for ms, _ in kernels.values()) or 1.0
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong" if args.one_cloud else "weak",
        "vs_baseline": None, "dtype": f"trunk {args.precision}, encoder {args.encoder_precision}", "data": "synthetic (seeded mesh clouds, random-init "
        "weights; no ShapeNet or checkpoints available)",
        "config": workload_config(args, world),
        "roofline": roofline(kernels, forward_points, dims),
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(cloud.nbytes),
                "d2h_bytes_per_step": int(host_out.nbytes)},
        "chamfer": chamfer,
        "one_cloud": one_cloud,
        "batch": batch,
        "gpu_launches": rec.launches * steps // traced_steps,
        "clocks": clocks.summary(),
        "kernel_breakdown": (f"separate traced pass of {traced_steps} steps (CUDA events "
                             "around every launch on its stream); value is timed untraced"),
        "kernels": {k: {"ms_per_step": ms / traced_steps, "launches_per_step": n / traced_steps,
                        "share": ms / total_kernel_ms} for k, (ms, n) in
                    sorted(kernels.items(), key=lambda kv: -kv[1][0])},
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_line(args)
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.profile_forward > 0:
        profile_forward(args)
        return
    if args.profile_chamfer:
        profile_chamfer(args)
        return
    if args.profile_training:
        profile_training(args)
        return
    if world > 1:
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_gpu(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
