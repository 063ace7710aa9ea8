"""Benchmark-configuration workloads: compiled scenes (cached on disk), poses and fans.

Scene files are cached under ``$NAVI_SCENE_CACHE`` (default ``.scene_cache/``
at the repository root) as ``<config>_<scene>_<res>.gmdag``; a cached file is
reused only when its recorded mesh hash matches the regenerated mesh.
"""

from __future__ import annotations

import hashlib
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import gmdag, scenes
from .fan import build_spherical_ray_directions

ROOT = Path(__file__).resolve().parents[1]


def cache_dir() -> Path:
    return Path(os.environ.get("NAVI_SCENE_CACHE", ROOT / ".scene_cache"))


@dataclass
class CompiledScene:
    config: int
    scene: int
    path: Path
    asset: gmdag.GmDagAsset
    mesh: scenes.Scene

    @property
    def words(self) -> np.ndarray:
        return self.asset.nodes

    @property
    def bbox_min(self) -> list[float]:
        return list(self.asset.bbox_min)

    @property
    def bbox_max(self) -> list[float]:
        return list(self.asset.bbox_max)

    @property
    def voxel_size(self) -> float:
        return self.asset.voxel_size

    @property
    def hit_epsilon(self) -> float:
        return float(np.float32(1e-3) * np.float32(self.asset.voxel_size))


def _mesh_hash(sc: scenes.Scene, res: int) -> str:
    h = hashlib.sha256()
    h.update(sc.vertices.tobytes())
    h.update(sc.triangles.tobytes())
    h.update(str(res).encode())
    return h.hexdigest()[:16]


def _compile_device(res: int) -> int | None:
    """CUDA device for the device compiler, or None for the host compiler.

    ``$NAVI_COMPILER`` = ``host`` | ``device`` | ``auto`` (default: the device
    compiler when a GPU is visible and the resolution is a power of two).  Both
    compilers give the same words, so the cache is shared."""
    mode = os.environ.get("NAVI_COMPILER", "auto")
    if mode == "host" or res & (res - 1):
        return None
    import torch

    if not torch.cuda.is_available():
        if mode == "device":
            raise RuntimeError("NAVI_COMPILER=device but no CUDA device is visible")
        return None
    return torch.cuda.current_device()


def compiled_scene(config: int, scene: int = 0, resolution: int | None = None, threads: int = 0) -> CompiledScene:
    cfg = scenes.CONFIGS[config]
    res = resolution or cfg.resolution
    mesh = scenes.make_scene(config, scene)
    digest = _mesh_hash(mesh, res)
    d = cache_dir()
    path = d / f"c{config}_s{scene}_r{res}_{digest}.gmdag"
    if not path.exists():
        out = gmdag.compile_mesh(mesh.vertices, mesh.triangles, res, threads=threads, device=_compile_device(res))
        gmdag.write_gmdag(path, out.nodes, res, out.bbox_min, out.voxel_size)
    asset = gmdag.load_gmdag_asset(path, validate_layout=False)
    return CompiledScene(config, scene, path, asset, mesh)


@dataclass
class PoseBatch:
    position: np.ndarray  # [A, 3] f32
    yaw: np.ndarray       # [A] f32
    pitch: np.ndarray     # [A] f32
    scene: np.ndarray     # [A] i32


def poses_for(config: int, scene_list: list[CompiledScene], actors: int | None = None, seed_offset: int = 0) -> PoseBatch:
    cfg = scenes.CONFIGS[config]
    n = actors or cfg.actors
    rng = np.random.Generator(np.random.PCG64(1000 * config + 999 + seed_offset))
    scene_ids = (rng.integers(0, len(scene_list), size=n).astype(np.int32)
                 if len(scene_list) > 1 else np.zeros(n, np.int32))
    pos = np.zeros((n, 3), np.float32)
    yaw = np.zeros(n, np.float32)
    pitch = np.zeros(n, np.float32)
    for s, cs in enumerate(scene_list):
        sel = np.nonzero(scene_ids == s)[0]
        if sel.size == 0:
            continue
        p = scenes.sample_free_poses(cs.mesh, sel.size, seed=1000 * config + 500 + 17 * s + seed_offset,
                                     pitch_deg=cfg.pitch_deg)
        pos[sel] = p["position"]
        yaw[sel] = p["yaw"]
        pitch[sel] = p["pitch"]
    return PoseBatch(pos, yaw, pitch, scene_ids)


def fan_for(config: int) -> np.ndarray:
    cfg = scenes.CONFIGS[config]
    return build_spherical_ray_directions(cfg.azimuth_bins, cfg.elevation_bins)


def walk_pose_sets(config: int, scene_list: list[CompiledScene], n_sets: int, actors: int | None = None,
                   seed_offset: int = 0) -> list[PoseBatch]:
    """Successive poses of a random walk (configuration 5: 0.1 m steps, yaw jitter N(0, 5 deg),
    moves that leave free space rejected): a uniform draw, then n_sets - 1 walk steps."""
    first = poses_for(config, scene_list, actors=actors, seed_offset=seed_offset)
    sets = [first]
    meshes = [cs.mesh for cs in scene_list]
    cur = {"position": first.position, "yaw": first.yaw, "pitch": first.pitch}
    for k in range(1, n_sets):
        cur = scenes.random_walk_poses(meshes, first.scene, cur, seed=1000 * config + 777 + 31 * k + seed_offset)
        sets.append(PoseBatch(cur["position"], cur["yaw"], cur["pitch"], first.scene))
    return sets
