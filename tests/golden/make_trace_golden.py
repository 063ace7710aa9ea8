"""Golden outputs of the reference's own CUDA kernel (run on a B200, committed).

    python tests/golden/make_trace_golden.py [out_dir]

Runs the reference sphere_trace_kernel (projects/torch-sdf/cpp_src/kernel.cu built
for sm_100a by oracle/build.py into oracle/_ref/) on:
  - config 1's full step (4 actors x 64 x 16 rays; rays built with eager torch ops
    on the GPU exactly as sdfdag_backend.py:1299-1312 does, plus pitch), with the
    reference's epsilon 0.01 (unmodified build) and with 1e-3 x voxel (epsilon build);
  - every known-answer case of tests/kat_cases.py.
Writes trace_golden.npz: the rays, the scene words' SHA-256, and the reference
kernel's distances and semantics.  tests/test_golden_reference_kernel.py checks the
CPU oracle against these outputs bit for bit, without a GPU.
"""

from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))


def main(out_dir: Path) -> Path:
    import torch

    from navi_b200 import scenes, tracer, workloads
    from oracle import oracle as O
    from tests.kat_cases import kat_cases

    dev = torch.device("cuda", 0)
    cfg = scenes.CONFIGS[1]
    cs = workloads.compiled_scene(1)
    pb = workloads.poses_for(1, [cs])
    fan = torch.from_numpy(workloads.fan_for(1)).to(dev)
    poses = tracer.make_poses(torch.from_numpy(pb.position).to(dev), torch.from_numpy(pb.yaw).to(dev),
                              torch.from_numpy(pb.pitch).to(dev))
    a, r = poses.shape[0], fan.shape[0]
    cy, sy, cp, sp = (poses[:, k:k + 1] for k in (3, 4, 5, 6))
    base = fan.unsqueeze(0).expand(a, -1, -1)
    by = base[..., 1] * cp - base[..., 2] * sp
    bz = base[..., 1] * sp + base[..., 2] * cp
    dirs = torch.empty((a, r, 3), dtype=torch.float32, device=dev)
    dirs[..., 0] = base[..., 0] * cy + bz * sy
    dirs[..., 1] = by
    dirs[..., 2] = -base[..., 0] * sy + bz * cy
    origins = poses[:, 0:3].unsqueeze(1).expand(-1, r, -1).contiguous()
    dag = torch.from_numpy(O.pad_words(cs.words).view(np.int64)).to(dev)
    n = a * r
    out = {
        "c1_origins": origins.cpu().numpy().reshape(n, 3),
        "c1_dirs": dirs.cpu().numpy().reshape(n, 3),
        "c1_words_sha256": np.frombuffer(hashlib.sha256(cs.words.tobytes()).digest(), np.uint8),
        "c1_bbox_min": np.array(cs.bbox_min, np.float32),
        "c1_bbox_max": np.array(cs.bbox_max, np.float32),
        "c1_eps_config": np.array([cs.hit_epsilon], np.float32),
    }
    for tag, eps_variant, eps in (("ref001", False, 0.01), ("refeps", True, cs.hit_epsilon)):
        kern = O.ReferenceKernel(eps_variant=eps_variant)
        od = torch.empty(n, dtype=torch.float32, device=dev)
        os_ = torch.empty(n, dtype=torch.int32, device=dev)
        kern.cast(dag, origins, dirs, od, os_, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                  bbox_min=cs.bbox_min, bbox_max=cs.bbox_max, resolution=cfg.resolution, hit_epsilon=eps)
        out[f"c1_{tag}_dist"] = od.cpu().numpy()
        out[f"c1_{tag}_sem"] = os_.cpu().numpy()
    kern = O.ReferenceKernel()
    for i, case in enumerate(kat_cases()):
        d = torch.from_numpy(O.pad_words(case.dag).view(np.int64)).to(dev)
        o = torch.tensor(case.origins, dtype=torch.float32, device=dev)
        v = torch.tensor(case.dirs, dtype=torch.float32, device=dev)
        od = torch.empty(o.shape[0], dtype=torch.float32, device=dev)
        os_ = torch.empty(o.shape[0], dtype=torch.int32, device=dev)
        kern.cast(d, o, v, od, os_, max_steps=case.max_steps, max_distance=case.max_distance,
                  bbox_min=case.bbox_min, bbox_max=case.bbox_max, resolution=case.resolution)
        out[f"kat_{case.name}_dist"] = od.cpu().numpy()
        out[f"kat_{case.name}_sem"] = os_.cpu().numpy()
    out_dir.mkdir(parents=True, exist_ok=True)
    path = out_dir / "trace_golden.npz"
    np.savez_compressed(path, **out)
    print(path, path.stat().st_size)
    return path


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else HERE)
