"""Generate golden vectors by running the reference's own Python code.

Runs in the build container only (it reads the reference checkout, which the
GPU machines do not have); its outputs are committed beside it as .npz files:

    python tests/golden/make_golden.py [--reference DIR]

The reference needs Jittor, which is absent here, so `jittor_shim` stands in
for it (torch on the CPU, `use_cuda = 0`): every operator takes the
reference's own CPU fallback, its modules, flow maths and patch_denoise run
unchanged. trimesh and point_cloud_utils are stubbed (only the mesh loader and
point-to-surface use them; neither is exercised).

Fixtures:
  flow.npz      alpha_schedule levels (flow2surf/flow.py:24-52)
  knn.npz       knn_indices CPU path (flow2surf/models/ops/knn.py:13-32)
  fps.npz       _farthest_point_indices (flow2surf/inference.py:19-41)
  model.npz     Flow2SurfNet forward, a reduced config with its weights
                embedded, in float64 and float32 (flow2surf/models/*)
  model_default.npz  default config, weights from the seeded generator
  denoise.npz   patch_denoise end to end (flow2surf/inference.py:68-198)
  nearest.npz   nearest_squared_distances CPU path and chamfer_distance
"""

from __future__ import annotations

import argparse
import hashlib
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(REPO / "jittor-flow2surf_b200"))

import jittor_shim  # noqa: E402

from flow2surf_b200.synthetic import DEFAULT_CONFIG, random_parameters, sphere_cloud  # noqa: E402

TINY_CONFIG = {
    "k_neighbors": 8, "feat_dim": 32, "encoder_dims": [16, 24], "num_blocks": 2,
    "alpha_dim": 8, "ffn_ratio": 2, "decoder_dims": [16, 8],
}


def params_digest(params: dict) -> str:
    h = hashlib.sha256()
    for name in sorted(params):
        h.update(name.encode())
        h.update(np.ascontiguousarray(params[name], dtype=np.float32).tobytes())
    return h.hexdigest()


def import_reference(reference: Path, dtype):
    for name in list(sys.modules):
        if name == "flow2surf" or name.startswith("flow2surf."):
            del sys.modules[name]
    jittor_shim.install(dtype)
    sys.modules.setdefault("trimesh", types.ModuleType("trimesh"))
    sys.modules.setdefault("point_cloud_utils", types.ModuleType("point_cloud_utils"))
    if str(reference) not in sys.path:
        sys.path.insert(0, str(reference))
    import flow2surf.evaluation as evaluation
    import flow2surf.flow as flow
    import flow2surf.inference as inference
    import flow2surf.models as models
    import flow2surf.models.encoder as encoder
    import flow2surf.models.ops.knn as knn
    import flow2surf.training.distances as distances
    return types.SimpleNamespace(flow=flow, inference=inference, models=models, encoder=encoder,
                                 knn=knn, distances=distances, evaluation=evaluation)


def build_reference_model(ref, cfg, params):
    model = ref.models.build_model(cfg)
    model.load_parameters(params)
    return model.eval()


def model_forward(ref, model, x, alpha):
    """Run the reference model, recording the KNN indices its encoder used."""
    seen = []
    original = ref.encoder.knn_indices

    def recording(features, k):
        out = original(features, k)
        seen.append(out.numpy().copy())
        return out

    ref.encoder.knn_indices = recording
    try:
        with jittor_shim.no_grad():
            v = model(jittor_shim.array(x), jittor_shim.array(alpha)).numpy()
    finally:
        ref.encoder.knn_indices = original
    return v, seen[0]


def make_flow(ref):
    cases = [(3, 1, 6), (1, 1, 1), (6, 1, 6), (10, 2.0, 3.0), (4, 0.5, 1.5)]
    out = {}
    for i, (n, c, p) in enumerate(cases):
        out[f"case{i}_args"] = np.array([n, c, p], dtype=np.float64)
        out[f"case{i}_alpha"] = ref.flow.alpha_schedule(n, c, p)
    return out


def make_knn(ref):
    rng = np.random.default_rng(11)
    cases = {
        "xyz": (rng.normal(size=(2, 3, 64)).astype(np.float32), 16),
        "pad": (rng.uniform(size=(1, 3, 5)).astype(np.float32), 8),
        "feat": (rng.normal(size=(2, 5, 40)).astype(np.float32), 7),
        "single": (rng.normal(size=(2, 3, 1)).astype(np.float32), 4),
        "surface": (sphere_cloud(200, seed=3)[0].T[None].copy(), 32),
    }
    out = {}
    for name, (features, k) in cases.items():
        out[f"{name}_features"] = features
        out[f"{name}_k"] = np.array(k)
        out[f"{name}_indices"] = ref.knn.knn_indices(jittor_shim.array(features), k).numpy()
    return out


def make_fps(ref):
    out = {}
    rng = np.random.default_rng(21)
    clouds = {
        "sphere": (sphere_cloud(3000, seed=5)[0], 30, 101),
        "dupes": (np.repeat(rng.uniform(size=(125, 3)).astype(np.float32), 4, axis=0), 40, 102),
        "small": (rng.normal(size=(7, 3)).astype(np.float32), 7, 103),
    }
    for name, (points, count, seed) in clouds.items():
        out[f"{name}_points"] = points
        out[f"{name}_count"] = np.array(count)
        out[f"{name}_seed"] = np.array(seed)
        out[f"{name}_first"] = np.array(np.random.default_rng(seed).integers(len(points)))
        out[f"{name}_indices"] = ref.inference._farthest_point_indices(
            points, count, np.random.default_rng(seed))
    return out


def make_model(reference):
    params = random_parameters(TINY_CONFIG, seed=5)
    rng = np.random.default_rng(31)
    x = (0.3 * rng.normal(size=(2, 3, 48))).astype(np.float32)
    alpha = np.array([0.25, 0.9], dtype=np.float32)
    out = {"x": x, "alpha": alpha}
    for name, value in params.items():
        out[f"param/{name}"] = value
    for tag, dtype in (("f64", torch.float64), ("f32", torch.float32)):
        ref = import_reference(reference, dtype)
        model = build_reference_model(ref, TINY_CONFIG, params)
        v, idx = model_forward(ref, model, x, alpha)
        out[f"velocity_{tag}"] = v
        out[f"knn_{tag}"] = idx
    return out


def make_model_default(reference):
    params = random_parameters(DEFAULT_CONFIG, seed=0)
    cloud = sphere_cloud(4000, seed=9)[0]
    rng = np.random.default_rng(41)
    centers = cloud[rng.choice(len(cloud), 2, replace=False)]
    x = []
    for c in centers:
        order = np.argsort(((cloud - c) ** 2).sum(1), kind="stable")[:128]
        x.append((cloud[order] - c).T)
    x = np.stack(x).astype(np.float32)
    alpha = np.array([0.5, 0.997947], dtype=np.float32)
    ref = import_reference(reference, torch.float64)
    model = build_reference_model(ref, DEFAULT_CONFIG, params)
    v, idx = model_forward(ref, model, x, alpha)
    return {"x": x, "alpha": alpha, "velocity_f64": v, "knn_f64": idx,
            "params_sha256": np.array(params_digest(params)), "params_seed": np.array(0)}


def make_denoise(reference):
    params = random_parameters(TINY_CONFIG, seed=5)
    noisy = sphere_cloud(1500, seed=13)[0]
    kwargs = dict(patch_size=128, seed_k=4, num_steps=3, num_chunks=2, patch_agg_beta=5.0,
                  alpha_clean_power=1.0, alpha_noisy_power=6.0)
    out = {"noisy": noisy, "rng_seed": np.array(7)}
    for k, v in kwargs.items():
        out[f"arg_{k}"] = np.array(v)
    for tag, dtype in (("f64", torch.float64), ("f32", torch.float32)):
        ref = import_reference(reference, dtype)
        model = build_reference_model(ref, TINY_CONFIG, params)
        out[f"denoised_{tag}"] = ref.inference.patch_denoise(
            model, noisy, rng=np.random.default_rng(7), **kwargs)
    out["seed_idx"] = ref.inference.patch_seed_indices(
        noisy, 128, 4, np.random.default_rng(7))
    return out


def make_nearest(reference):
    ref = import_reference(reference, torch.float32)
    rng = np.random.default_rng(51)
    first = rng.normal(size=(2, 300, 3)).astype(np.float32)
    second = rng.normal(size=(2, 257, 3)).astype(np.float32)
    d1, i2, d2, i1 = ref.distances.nearest_squared_distances(
        jittor_shim.array(first), jittor_shim.array(second))
    pred = sphere_cloud(2000, seed=15)[0]
    target = sphere_cloud(1700, seed=16)[1]
    return {"first": first, "second": second, "d1": d1.numpy(), "i2": i2.numpy(),
            "d2": d2.numpy(), "i1": i1.numpy(), "pred": pred, "target": target,
            "chamfer": np.array(ref.evaluation.chamfer_distance(pred, target))}


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", default="/root/reference")
    args = parser.parse_args()
    reference = Path(args.reference)
    ref32 = import_reference(reference, torch.float32)
    fixtures = {
        "flow": make_flow(ref32),
        "knn": make_knn(ref32),
        "fps": make_fps(ref32),
        "model": make_model(reference),
        "model_default": make_model_default(reference),
        "denoise": make_denoise(reference),
        "nearest": make_nearest(reference),
    }
    for name, arrays in fixtures.items():
        path = HERE / f"{name}.npz"
        np.savez_compressed(path, **arrays)
        print(f"{path.name}: {path.stat().st_size / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
