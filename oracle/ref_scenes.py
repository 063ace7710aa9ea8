"""Benchmark scenes compiled by the reference's own scene compiler — TEST INFRASTRUCTURE ONLY.

The reference arm of bench.py must not map this repository's libraries, so its
scenes come from projects/voxel-dag/src/compiler.cpp (built unmodified by
oracle/build.py into oracle/_ref/ref_voxel_dag, with the OBJ-only Assimp
stand-in) and are read back by the restatement of the reference's loader
(oracle/gmdag_ref.py, integration/voxel_dag.py:193-259).  Meshes are the seeded
synthetic scenes of navi_b200.scenes (pure numpy).  Files are cached as
``ref_c<config>_s<scene>_r<res>_<mesh hash>.gmdag`` under the scene cache; the
scenes of one configuration are compiled in parallel processes.

The reference compiler indexes voxels with 32-bit ints, which overflow above
1290^3 (compiler.cpp), so configuration 4 (2048^3) cannot come from it.
"""

from __future__ import annotations

import hashlib
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import build as OB
from . import gmdag_ref

ROOT = Path(__file__).resolve().parents[1]
MAX_RESOLUTION = 1290


@dataclass
class RefScene:
    config: int
    scene: int
    path: Path
    bbox_min: list[float]
    bbox_max: list[float]
    voxel_size: float
    resolution: int
    words: np.ndarray
    mesh: object

    @property
    def hit_epsilon(self) -> float:
        """1e-3 x voxel size in float32, the configurations' hit threshold."""
        return float(np.float32(1e-3) * np.float32(self.voxel_size))


def cache_dir() -> Path:
    return Path(os.environ.get("NAVI_SCENE_CACHE", ROOT / ".scene_cache"))


def _write_obj(path: Path, vertices: np.ndarray, triangles: np.ndarray) -> None:
    """OBJ with %.9g coordinates (strtof reads each float32 back exactly)."""
    v = np.asarray(vertices, np.float32).astype(np.float64)
    t = np.asarray(triangles, np.int64) + 1
    with path.open("w") as f:
        f.write("".join("v %.9g %.9g %.9g\n" % tuple(row) for row in v))
        f.write("".join("f %d %d %d\n" % tuple(row) for row in t))


def _digest(mesh, res: int) -> str:
    h = hashlib.sha256()
    h.update(np.asarray(mesh.vertices).tobytes())
    h.update(np.asarray(mesh.triangles).tobytes())
    h.update(str(res).encode())
    return h.hexdigest()[:16]


def compile_scene_file(config: int, scene: int, res: int) -> tuple[Path, object]:
    """Path of the reference compiler's .gmdag for (config, scene, res), compiling it if absent."""
    from navi_b200 import scenes

    if res > MAX_RESOLUTION:
        raise RuntimeError(f"the reference compiler's int voxel indexing overflows above {MAX_RESOLUTION}^3")
    exe = OB.REF_OUT / "ref_voxel_dag"
    mesh = scenes.make_scene(config, scene)
    out = cache_dir() / f"ref_c{config}_s{scene}_r{res}_{_digest(mesh, res)}.gmdag"
    if out.exists():
        return out, mesh
    if not exe.exists():
        raise RuntimeError("reference compiler not built (oracle/build.py with the reference tree)")
    out.parent.mkdir(parents=True, exist_ok=True)
    obj = out.with_suffix(f".{os.getpid()}.obj")
    tmp = out.with_suffix(f".{os.getpid()}.tmp")
    try:
        _write_obj(obj, mesh.vertices, mesh.triangles)
        r = subprocess.run([str(exe), str(obj), str(tmp), str(res)], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"reference compiler failed on c{config} s{scene}: {r.stderr.strip()}")
        os.replace(tmp, out)
    finally:
        for p in (obj, tmp):
            if p.exists():
                p.unlink()
    return out, mesh


def load_scene(config: int, scene: int, res: int) -> RefScene:
    path, mesh = compile_scene_file(config, scene, res)
    _, resolution, bmin, bmax, voxel, nodes = gmdag_ref.load_asset(path, validate_layout_flag=False)
    return RefScene(config, scene, path, list(bmin), list(bmax), voxel, resolution, nodes, mesh)


def config_scenes(config: int, workers: int = 0) -> list[RefScene]:
    """Every scene of a configuration, compiled by the reference compiler (parallel processes)."""
    from navi_b200 import scenes

    cfg = scenes.CONFIGS[config]
    n = cfg.n_scenes
    workers = workers or max(1, min(n, (os.cpu_count() or 2) // 2))
    with ThreadPoolExecutor(max_workers=workers) as pool:
        list(pool.map(lambda s: compile_scene_file(config, s, cfg.resolution), range(n)))
    return [load_scene(config, s, cfg.resolution) for s in range(n)]
