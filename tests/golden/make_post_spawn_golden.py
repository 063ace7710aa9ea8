"""Golden outputs of the reference's own post-processing and spawn search (run here, committed).

    python tests/golden/make_post_spawn_golden.py

Imports projects/environment/src/navi_environment/backends/sdfdag_backend.py from
the reference tree (with projects/contracts/src on the path; CPU torch) and
records, into post_spawn_golden.npz and spawn_golden.json:

- _postprocess_cast_outputs_tensor (:408-473) with _compute_observation_ratios_tensor
  (:366-405) on seeded distances that include NaN, +inf, -inf, negative values,
  zero, max_distance and the band / proximity / saturation bounds, for several
  fan shapes, bands and thresholds (max_distance <= 0 included);
- _observation_profile (:162-199), _spawn_candidate_score (:267-287) and
  _select_spawn_yaw_from_observation (:224-264) on seeded [Az, El] grids;
- SdfDagBackend._find_spawn_poses (:2564-2700) itself, run on the CPU with its
  attributes set as the backend sets them and its torch_sdf.cast_rays call served
  by the C restatement of the reference kernel (oracle/trace_oracle.c, pinned bit for
  bit against kernel.cu built for sm_100a), on scenes compiled by the reference's
  scene compiler (oracle/ref_scenes.py); the reference has no CPU trace of its own.

The tests compare oracle/postprocess_ref.py, oracle/spawn_ref.py and navi_b200/spawn.py
against these files without needing the reference tree.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

REF = Path(os.environ.get("NAVI_REFERENCE_ROOT", ROOT.parent / "reference"))

# (actors, az, el, max_distance, band_min, band_max, proximity)
POST_CASES = [
    (3, 12, 4, 30.0, 1.5, 13.2, 2.0),
    (2, 64, 16, 20.0, 1.5, 6.0, 2.0),
    (4, 7, 3, 30.0, 1.5, 13.2, 0.0),
    (2, 6, 5, 30.0, 9.0, 1.5, 2.0),
    (1, 1, 1, 10.0, 1.5, 6.0, 2.0),
    (2, 13, 7, 0.0, 1.5, 6.0, 2.0),
    (1, 256, 48, 30.0, 1.5, 13.2, 2.0),
]

# (az, el, max_distance, proximity, band_min, band_max)
PROFILE_CASES = [(48, 12, 30.0, 2.0, 1.5, 9.0), (8, 4, 30.0, 0.0, 1.5, 9.0), (5, 3, 20.0, 2.0, 9.0, 1.5),
                 (1, 1, 30.0, 2.0, 1.5, 9.0), (13, 7, 30.0, 2.0, 1.5, 13.2)]

# (config, scene, resolution, az, el, count, structure band max)
SPAWN_CASES = [(1, 0, 128, 64, 16, 8, 6.0), (2, 0, 128, 256, 48, 8, 13.2), (3, 0, 128, 128, 24, 5, 13.2),
               (3, 1, 64, 8, 4, 300, 13.2)]


def reference_backend():
    for sub in ("projects/environment/src", "projects/contracts/src"):
        p = str(REF / sub)
        if p not in sys.path:
            sys.path.insert(0, p)
    import navi_environment.backends.sdfdag_backend as B

    return B


def seeded_distances(rng, shape, max_distance, marks):
    """Uniform distances with NaN, +-inf, negatives, zero and exact threshold values mixed in."""
    hi = max(max_distance, 10.0) * 1.3
    d = rng.uniform(-1.0, hi, size=shape).astype(np.float32)
    pick = rng.random(shape)
    specials = [np.nan, np.inf, -np.inf, -0.5, 0.0, max_distance, np.float32(max_distance) - np.float32(1e-3),
                *marks]
    for i, v in enumerate(specials):
        lo_p = 0.02 * i
        d[(pick >= lo_p) & (pick < lo_p + 0.02)] = np.float32(v)
    flat = d.reshape(-1)
    for i, v in enumerate(specials[: flat.shape[0]]):  # every special value at least once where it fits
        flat[(7 * i) % flat.shape[0]] = np.float32(v)
    return d


def post_cases(B, out: dict) -> None:
    rng = np.random.default_rng(20260)
    for k, (a, az, el, mx, bmin, bmax, prox) in enumerate(POST_CASES):
        d = seeded_distances(rng, (a, az * el), mx, [bmin, bmax, prox])
        s = rng.integers(0, 5, size=(a, az * el)).astype(np.int32)
        res = B._postprocess_cast_outputs_tensor(
            torch.from_numpy(d), torch.from_numpy(s), az_bins=az, el_bins=el, max_distance=mx,
            structure_band_min_distance=bmin, structure_band_max_distance=bmax, proximity_distance_threshold=prox)
        names = ["depth", "semantic", "valid", "min", "starvation", "proximity", "band", "forward", "clamped"]
        out[f"post{k}_dist"] = d
        out[f"post{k}_sem"] = s
        for name, t in zip(names, res):
            arr = t.numpy()
            out[f"post{k}_{name}"] = arr.astype(np.uint8) if arr.dtype == np.bool_ else arr


def profile_cases(B, out: dict) -> None:
    rng = np.random.default_rng(40961)
    for k, (az, el, mx, prox, bmin, bmax) in enumerate(PROFILE_CASES):
        raw = seeded_distances(rng, (az, el), mx, [bmin, bmax, prox])
        valid = np.isfinite(raw)
        metric = np.clip(raw, 0.0, mx)
        kw = dict(max_distance=mx, proximity_distance_threshold=prox, structure_band_min_distance=bmin,
                  structure_band_max_distance=bmax)
        prof = B._observation_profile(metric, valid, **kw)
        score = B._spawn_candidate_score(metric, valid, **kw)
        yaw = B._select_spawn_yaw_from_observation(metric, valid, structure_band_min_distance=bmin,
                                                   structure_band_max_distance=bmax)
        out[f"prof{k}_raw"] = raw
        out[f"prof{k}_values"] = np.array([*prof, score, yaw], np.float64)


class _OracleTorchSdf:
    """Stands in for torch_sdf on the CPU: cast_rays traced by the C restatement of kernel.cu
    at its hit threshold 0.01 (kernel.cuh:7)."""

    def cast_rays(self, dag, origins, dirs, out_d, out_s, max_steps, max_distance, bbox_min, bbox_max, resolution,
                  skip_direction_validation=False):
        from oracle import oracle as O

        res = O.trace(dag.numpy().view(np.uint64), bbox_min, bbox_max, origins.numpy(), dirs.numpy(),
                      max_steps=max_steps, max_distance=max_distance, hit_epsilon=0.01)
        out_d.copy_(torch.from_numpy(res["dist"]).view(out_d.shape))
        out_s.copy_(torch.from_numpy(res["sem"]).view(out_s.shape))


def spawn_cases(B) -> list[dict]:
    from oracle import ref_scenes

    cases = []
    for config, scene, res, az, el, count, band_max in SPAWN_CASES:
        sc = ref_scenes.load_scene(config, scene, res)
        be = B.SdfDagBackend.__new__(B.SdfDagBackend)
        asset = types.SimpleNamespace(bbox_min=tuple(sc.bbox_min), bbox_max=tuple(sc.bbox_max), resolution=res)
        dag = torch.from_numpy(sc.words.view(np.int64).copy())
        be._require_asset = lambda asset=asset: asset
        be._require_dag_tensor = lambda dag=dag: dag
        be._az_bins, be._el_bins = az, el
        be._torch = torch
        be._device = torch.device("cpu")
        be._torch_sdf = _OracleTorchSdf()
        be._config = types.SimpleNamespace(sdf_max_steps=256)
        be._max_distance = 30.0
        be._bbox_min = list(sc.bbox_min)
        be._bbox_max = list(sc.bbox_max)
        be._proximity_distance_threshold = 2.0
        be._structure_band_min_distance = 1.5
        be._structure_band_max_distance = band_max
        poses = B.SdfDagBackend._find_spawn_poses(be, count)
        cases.append({"config": config, "scene": scene, "resolution": res, "azimuth_bins": az, "elevation_bins": el,
                      "count": count, "sdf_max_steps": 256, "max_distance": 30.0,
                      "proximity_distance_threshold": 2.0, "structure_band_min_distance": 1.5,
                      "structure_band_max_distance": band_max,
                      "words_sha256": hashlib.sha256(sc.words.tobytes()).hexdigest(),
                      "poses": [[float(v) for v in p] for p in poses]})
    return cases


def main() -> None:
    B = reference_backend()
    out: dict = {}
    post_cases(B, out)
    profile_cases(B, out)
    np.savez_compressed(HERE / "post_spawn_golden.npz", **out)
    spawns = spawn_cases(B)
    (HERE / "spawn_golden.json").write_text(json.dumps(spawns, indent=1) + "\n")
    print(f"{len(out)} arrays; {len(spawns)} spawn searches")


if __name__ == "__main__":
    main()
