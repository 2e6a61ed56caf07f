"""Device-resident patch-wise reverse-flow inference (flow2surf/inference.py).

Same signature, validation and results as the reference's patch_denoise, with
every stage on the GPU: farthest-point seeds, the patch index, the fusion
structure, the per-step patch gather, the model forward and the fused
vote aggregation + Euler update. The host only draws the first FPS index from
`rng` (as the reference does) and copies the cloud in and out.
"""

from __future__ import annotations

import ctypes
import hashlib
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .flow import alpha_schedule

# Device memory the model's per-chunk workspace may take.
DEFAULT_WORKSPACE_BUDGET = 24 << 30
MAX_ROWS_PER_FORWARD = 1 << 20   # f2s_model_forward takes B * M below this per call


def make_rng(seed, *parts):
    """Deterministic NumPy generator from a seed and namespace parts
    (inference.py:12-16)."""
    key = "::".join([str(seed), *map(str, parts)]).encode("utf-8")
    digest = hashlib.blake2b(key, digest_size=8).digest()
    return np.random.default_rng(int.from_bytes(digest, "little") % (2**32))


def patch_seed_count(num_points, patch_size, seed_k):
    """Patch-centre count for one cloud (inference.py:44-59)."""
    num_points, patch_size, seed_k = int(num_points), int(patch_size), int(seed_k)
    if num_points < 1:
        raise ValueError(f"num_points must be >= 1, got {num_points}")
    if patch_size < 1:
        raise ValueError(f"patch_size must be >= 1, got {patch_size}")
    if seed_k < 1:
        raise ValueError(f"seed_k must be >= 1, got {seed_k}")
    effective_patch_size = min(patch_size, num_points)
    return min(num_points, max(1, int(seed_k * num_points / effective_patch_size)))


def _workspace(query: str, *dims, device) -> torch.Tensor:
    size = ctypes.c_size_t()
    _lib.check(getattr(_lib.lib(), query)(*dims, ctypes.byref(size)))
    return torch.empty(max(size.value, 1), dtype=torch.uint8, device=device)


def farthest_point_indices(points: torch.Tensor, count: int, first: int) -> torch.Tensor:
    """Device FPS, bit-exact to _farthest_point_indices (inference.py:19-41)
    given the first index (the reference's `rng.integers(N)`). Returns int32."""
    n = points.shape[0]
    out = torch.empty(count, dtype=torch.int32, device=points.device)
    ws = _workspace("f2s_fps_workspace_bytes", n, device=points.device)
    _lib.call("f2s_fps", _lib.ptr(points), n, count, int(first), _lib.ptr(out), _lib.ptr(ws),
              ws.numel(), _lib.stream_handle())
    return out


def patch_seed_indices(points, patch_size, seed_k, rng):
    """Farthest-point patch centres (inference.py:62-65); `points` is a CUDA
    tensor (N, 3) float32."""
    count = patch_seed_count(points.shape[0], patch_size, seed_k)
    first = int(rng.integers(points.shape[0]))
    return farthest_point_indices(points, count, first)


@dataclass
class DenoisePlan:
    """Per-cloud device state, fixed from the noisy input (inference.py:138-139)."""

    num_points: int
    patch_size: int
    seeds: torch.Tensor        # (P,) int32
    neighbors: torch.Tensor    # (P, k) int32, ascending distance
    radial: torch.Tensor       # (P, k) float64
    weights: torch.Tensor      # (P, k) float64
    offsets: torch.Tensor      # (N + 1,) int32
    entries: torch.Tensor      # (P * k,) int32 flat (patch, slot) in bincount order
    weight_sum: torch.Tensor   # (N,) float64

    @property
    def num_patches(self) -> int:
        return self.seeds.shape[0]


def build_plan(points: torch.Tensor, patch_size: int, seeds: torch.Tensor,
               patch_agg_beta: float) -> DenoisePlan:
    """Patch index (inference.py:110-122) and aggregation (:124-134) on device."""
    n = points.shape[0]
    P = seeds.shape[0]
    dev = points.device
    stream = _lib.stream_handle()
    neighbors = torch.empty((P, patch_size), dtype=torch.int32, device=dev)
    radial = torch.empty((P, patch_size), dtype=torch.float64, device=dev)
    weights = torch.empty((P, patch_size), dtype=torch.float64, device=dev)
    _lib.call("f2s_patch_index", _lib.ptr(points), n, _lib.ptr(seeds), P, patch_size,
              float(patch_agg_beta), _lib.ptr(neighbors), _lib.ptr(radial), _lib.ptr(weights),
              stream)
    offsets = torch.empty(n + 1, dtype=torch.int32, device=dev)
    entries = torch.empty(P * patch_size, dtype=torch.int32, device=dev)
    weight_sum = torch.empty(n, dtype=torch.float64, device=dev)
    ws = _workspace("f2s_fusion_workspace_bytes", n, device=dev)
    _lib.call("f2s_fusion_build", _lib.ptr(neighbors), _lib.ptr(weights), P, patch_size, n,
              _lib.ptr(offsets), _lib.ptr(entries), _lib.ptr(weight_sum), _lib.ptr(ws),
              ws.numel(), stream)
    return DenoisePlan(n, patch_size, seeds, neighbors, radial, weights, offsets, entries,
                       weight_sum)


def gather_patch_rows(local: torch.Tensor, num_patches: int, group) -> torch.Tensor:
    """The rows of every rank's patch range in patch order: `local` holds this
    rank's rows of `shard_range` at its top, padded to the largest range
    (ceil(P / world) rows); one all-gather, then each rank's real rows."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    chunk = local.shape[0]
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous(), group=group)
    rows = []
    for r in range(world):
        begin, end = shard_range(num_patches, r, world)
        if end - begin > chunk:
            raise ValueError("gather_patch_rows: a rank's range exceeds the padded chunk")
        rows.append(parts[r][:end - begin])
    return torch.cat(rows).contiguous()


def build_plan_sharded(points: torch.Tensor, patch_size: int, seeds: torch.Tensor,
                       patch_agg_beta: float, group) -> DenoisePlan:
    """build_plan for one cloud split across the ranks of `group`: each rank
    builds the patch index of its own patch range (`shard_range`), one
    all-gather (NCCL) per array assembles every patch's neighbours, radial
    distances and weights on every rank, and the fusion structure is built
    from them. The patch index of a seed does not depend on the other seeds,
    so the plan is the one build_plan gives, bit for bit."""
    import torch.distributed as dist

    n = points.shape[0]
    P = seeds.shape[0]
    dev = points.device
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    chunk = -(-P // world)  # the largest range
    begin, end = shard_range(P, rank, world)
    local_n = torch.zeros((chunk, patch_size), dtype=torch.int32, device=dev)
    local_r = torch.zeros((chunk, patch_size), dtype=torch.float64, device=dev)
    local_w = torch.zeros((chunk, patch_size), dtype=torch.float64, device=dev)
    if end > begin:
        _lib.call("f2s_patch_index", _lib.ptr(points), n, _lib.ptr(seeds[begin:]), end - begin,
                  patch_size, float(patch_agg_beta), _lib.ptr(local_n), _lib.ptr(local_r),
                  _lib.ptr(local_w), _lib.stream_handle())
    neighbors, radial, weights = (gather_patch_rows(x, P, group)
                                  for x in (local_n, local_r, local_w))
    offsets = torch.empty(n + 1, dtype=torch.int32, device=dev)
    entries = torch.empty(P * patch_size, dtype=torch.int32, device=dev)
    weight_sum = torch.empty(n, dtype=torch.float64, device=dev)
    ws = _workspace("f2s_fusion_workspace_bytes", n, device=dev)
    _lib.call("f2s_fusion_build", _lib.ptr(neighbors), _lib.ptr(weights), P, patch_size, n,
              _lib.ptr(offsets), _lib.ptr(entries), _lib.ptr(weight_sum), _lib.ptr(ws),
              ws.numel(), _lib.stream_handle())
    return DenoisePlan(n, patch_size, seeds, neighbors, radial, weights, offsets, entries,
                       weight_sum)


class _Runner:
    """Reusable device buffers for the integration loop of one plan."""

    def __init__(self, model, plan: DenoisePlan, workspace_budget: int):
        self.model, self.plan = model, plan
        P, k = plan.num_patches, plan.patch_size
        dev = plan.seeds.device
        self.x = torch.empty((P, 3, k), dtype=torch.float32, device=dev)
        self.votes = torch.empty((P, k, 3), dtype=torch.float32, device=dev)
        self.alpha = torch.empty(P, dtype=torch.float32, device=dev)
        self.chunk = P
        self.workspace = None
        if hasattr(model, "workspace_bytes"):
            per_patch = max(1, model.workspace_bytes(1, k))
            # also within the forward's row limit (B * M < 2^20 per call)
            row_cap = max(1, (MAX_ROWS_PER_FORWARD - 1) // k)
            self.chunk = max(1, min(P, workspace_budget // per_patch, row_cap))
            self.workspace = torch.empty(model.workspace_bytes(self.chunk, k), dtype=torch.uint8,
                                         device=dev)

    def predict(self, points: torch.Tensor, alpha_value: float, begin: int = 0,
                end: int | None = None) -> torch.Tensor:
        """Per-patch votes (P, k, 3) of patches [begin, end) (inference.py:141-153)."""
        plan = self.plan
        k = plan.patch_size
        end = plan.num_patches if end is None else end
        if end > begin:
            _lib.call("f2s_gather_patches", _lib.ptr(points), _lib.ptr(plan.neighbors[begin]),
                      _lib.ptr(plan.seeds[begin:]), end - begin, k, _lib.ptr(self.x[begin]),
                      _lib.stream_handle())
        self.alpha.fill_(alpha_value)
        for start in range(begin, end, self.chunk):
            stop = min(end, start + self.chunk)
            if self.workspace is not None:
                self.model.forward_into(self.x[start:stop], self.alpha[start:stop],
                                        self.votes[start:stop], self.workspace)
            else:
                self.votes[start:stop] = self.model(self.x[start:stop], self.alpha[start:stop])
        return self.votes

    def step(self, points: torch.Tensor, out: torch.Tensor, alpha_current: float,
             alpha_step: float) -> None:
        votes = self.predict(points, alpha_current)
        plan = self.plan
        _lib.call("f2s_fuse_euler", _lib.ptr(points), _lib.ptr(votes), _lib.ptr(plan.offsets),
                  _lib.ptr(plan.entries), _lib.ptr(plan.weights), _lib.ptr(plan.weight_sum),
                  plan.num_points, ctypes.c_float(alpha_step), _lib.ptr(out), None,
                  _lib.stream_handle())


def shard_range(num_patches: int, rank: int, world_size: int) -> tuple[int, int]:
    """Contiguous patch range [begin, end) of `rank` when one cloud's patches
    are split across `world_size` GPUs: a fixed split, so the result depends
    only on the world size."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"bad rank {rank} of world size {world_size}")
    base, extra = divmod(num_patches, world_size)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


class _ShardedRunner(_Runner):
    """One cloud across the ranks of a process group: every rank holds the
    whole cloud and plan, runs the model on its own patch range, forms the
    weighted vote sums of those patches, and one all-reduce (NCCL over NVLink)
    per Euler step adds them; the update is then identical on every rank."""

    def __init__(self, model, plan: DenoisePlan, workspace_budget: int, group):
        import torch.distributed as dist
        super().__init__(model, plan, workspace_budget)
        self.dist, self.group = dist, group
        self.begin, self.end = shard_range(plan.num_patches, dist.get_rank(group),
                                           dist.get_world_size(group))
        self.vote_sum = torch.empty((plan.num_points, 3), dtype=torch.float64,
                                    device=plan.seeds.device)
        # CUDA-event pairs around each all-reduce when timing is asked for
        self.collective_events: list | None = None

    def step(self, points: torch.Tensor, out: torch.Tensor, alpha_current: float,
             alpha_step: float) -> None:
        plan = self.plan
        votes = self.predict(points, alpha_current, self.begin, self.end)
        stream = _lib.stream_handle()
        _lib.call("f2s_fuse_partial", _lib.ptr(votes), _lib.ptr(plan.offsets),
                  _lib.ptr(plan.entries), _lib.ptr(plan.weights), plan.num_points,
                  plan.patch_size, self.begin, self.end, _lib.ptr(self.vote_sum), stream)
        if self.collective_events is not None:
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            self.dist.all_reduce(self.vote_sum, group=self.group)
            stop.record()
            self.collective_events.append((start, stop))
        else:
            self.dist.all_reduce(self.vote_sum, group=self.group)
        _lib.call("f2s_euler_from_sum", _lib.ptr(points), _lib.ptr(self.vote_sum),
                  _lib.ptr(plan.weight_sum), _lib.ptr(plan.offsets), plan.num_points,
                  ctypes.c_float(alpha_step), _lib.ptr(out), None, stream)


def denoise_device(model, points: torch.Tensor, patch_size, seed_k, num_steps, rng=None,
                   patch_seed_idx=None, patch_agg_beta=4.0, alpha_clean_power=1.0,
                   alpha_noisy_power=1.0, workspace_budget=DEFAULT_WORKSPACE_BUDGET,
                   process_group=None, collective_events=None):
    """patch_denoise on a cloud already on the GPU ((N, 3) float32 CUDA
    tensor); returns the denoised cloud as a new CUDA tensor.

    With `process_group` (an initialised torch.distributed group, one GPU per
    rank), every rank passes the same cloud and seeds and the patches are
    split across the ranks (`shard_range`); every rank returns the same
    result. The per-step sum then adds the ranks' partial float64 sums, which
    can differ from the one-GPU order in the last bit of a float64 sum. Each
    rank builds the patch index of its own patches (`build_plan_sharded`).
    `collective_events`, if a list, receives a (start, stop) CUDA-event pair
    around each per-step all-reduce."""
    if rng is None:
        rng = np.random.default_rng(0)
    num_points = points.shape[0]
    patch_size = min(int(patch_size), num_points)
    num_patches = patch_seed_count(num_points, patch_size, seed_k)
    points = points.to(torch.float32).contiguous()
    if patch_seed_idx is None:
        seeds = patch_seed_indices(points, patch_size, seed_k, rng)
    else:
        seed_idx = np.asarray(patch_seed_idx, dtype=np.int64)
        if seed_idx.shape != (num_patches,):
            raise ValueError(f"patch_seed_idx must have shape ({num_patches},), "
                             f"got {seed_idx.shape}")
        if np.any((seed_idx < 0) | (seed_idx >= num_points)):
            raise ValueError("patch_seed_idx contains an out-of-range point index")
        seeds = torch.from_numpy(seed_idx.astype(np.int32)).to(points.device)
    sharded = process_group is not None and torch.distributed.get_world_size(process_group) > 1
    plan = (build_plan_sharded(points, patch_size, seeds, patch_agg_beta, process_group)
            if sharded else build_plan(points, patch_size, seeds, patch_agg_beta))
    alphas = alpha_schedule(num_steps, alpha_clean_power, alpha_noisy_power)

    def integrate(net):
        runner = (_ShardedRunner(net, plan, workspace_budget, process_group) if sharded
                  else _Runner(net, plan, workspace_budget))
        if sharded and collective_events is not None:
            runner.collective_events = collective_events
        current = points.clone()
        spare = torch.empty_like(current)
        for step in range(num_steps - 1, -1, -1):
            alpha_current = float(alphas[step])
            alpha_previous = float(alphas[step - 1]) if step > 0 else 0.0
            runner.step(current, spare, alpha_current, alpha_current - alpha_previous)
            current, spare = spare, current
        return current

    current = integrate(model)
    status = _lib.read_device_error()
    if sharded:  # every rank takes the same path
        flag = torch.tensor([status], dtype=torch.int32, device=points.device)
        torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MAX, group=process_group)
        status = int(flag.item())
    if status == _lib.F2S_FP16_RANGE and hasattr(model, "wide_ffn"):
        # an fp16 FFN row of the tf32 trunk overflowed somewhere: the whole
        # denoise again with fp32 FFN rows (still on the device)
        current = integrate(model.wide_ffn())
        status = _lib.read_device_error()
    if status:
        raise _lib.Flow2SurfError(_lib.F2S_ERR_CUDA, "device error %d: %s" % (
            status, _lib.DEVICE_ERRORS.get(status, "unknown")))
    return current


def patch_denoise(model, pc_noisy, patch_size, seed_k, num_steps, num_chunks, rng=None,
                  patch_seed_idx=None, patch_agg_beta=4.0, alpha_clean_power=1.0,
                  alpha_noisy_power=1.0, device="cuda", process_group=None):
    """Denoise one normalized point cloud by patch-wise reverse integration.

    Drop-in for flow2surf/inference.py:68-198: `pc_noisy` is a host (N, 3)
    array and so is the result (float32). `num_chunks` is validated as the
    reference does; the GPU batches patches by a memory budget instead, which
    does not change any result because patches are independent.
    `process_group` splits the cloud's patches across the group's GPUs
    (see `denoise_device`).
    """
    if num_chunks < 1:
        raise ValueError(f"num_chunks must be >= 1, got {num_chunks}")
    if isinstance(pc_noisy, torch.Tensor):   # e.g. a pinned host tensor: asynchronous copy
        points = pc_noisy.to(device=device, dtype=torch.float32, non_blocking=True)
    else:
        host = np.ascontiguousarray(np.asarray(pc_noisy), dtype=np.float32)
        points = torch.from_numpy(host).to(device)
    out = denoise_device(model, points, patch_size, seed_k, num_steps, rng=rng,
                         patch_seed_idx=patch_seed_idx, patch_agg_beta=patch_agg_beta,
                         alpha_clean_power=alpha_clean_power,
                         alpha_noisy_power=alpha_noisy_power, process_group=process_group)
    return out.cpu().numpy()
