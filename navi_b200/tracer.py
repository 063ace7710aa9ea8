"""Python host API of the B200 sphere tracer (PyTorch only hands tensors over).

- :class:`NodePool`   device node pool re-packed from ``.gmdag`` words
- :func:`load_gmdag`  load a ``.gmdag`` file and upload it (pool + int64 DAG tensor)
- :class:`SceneSet`   pools + bounds + hit epsilons, the scene table of fan casts
- :func:`cast_rays_ex` explicit rays with hit epsilon and step-count output
- :func:`make_poses` / :func:`cast_fan`  pose-fused spherical fans

Every cast is asynchronous on the caller's current CUDA stream and never
synchronises the host.  There is no CPU path: a missing native library or a
non-CUDA tensor raises RuntimeError.
"""

from __future__ import annotations

import contextlib
import ctypes
import hashlib
import math
import os
import threading
import weakref
from dataclasses import dataclass
from pathlib import Path
from typing import Sequence

import numpy as np
import torch

from . import _native
from .gmdag import GmDagAsset, load_gmdag_asset

__all__ = [
    "NodePool",
    "SceneSet",
    "GmDagScene",
    "load_gmdag",
    "cast_rays_ex",
    "make_poses",
    "cast_fan",
    "cast_fan_observe",
    "pool_for_tensor",
    "workspace",
    "set_option",
]

DEFAULT_HIT_EPSILON = 0.01


_NVTX = os.environ.get("NAVI_NVTX", "0") not in ("", "0")


@contextlib.contextmanager
def _nvtx(name: str):
    """An NVTX range around a native call when $NAVI_NVTX is set (for nsight timelines)."""
    if not _NVTX:
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def _stream_handle(device: torch.device) -> int:
    return int(torch.cuda.current_stream(device).cuda_stream)


def workspace(device: torch.device, n_rays: int) -> torch.Tensor:
    """Scratch for one cast of n_rays rays (work counter, claim order), allocated on the current stream."""
    n = int(_native.tsdf_lib().tsdf_workspace_bytes(int(n_rays)))
    return torch.empty(n, dtype=torch.uint8, device=device)


def set_option(key: str, value: int) -> int:
    """Set a process-wide tuning knob of the native library; returns the previous value."""
    old = ctypes.c_int64()
    _native.check(_native.tsdf_lib().tsdf_set_option(key.encode(), int(value), ctypes.byref(old)), "tsdf_set_option")
    return int(old.value)


class NodePool:
    """Device node pool (32-byte octant records) built from ``.gmdag`` words."""

    def __init__(self, handle: int, device: torch.device) -> None:
        self._handle = ctypes.c_void_p(handle)
        self.device = device
        lib = _native.tsdf_lib()
        st = _native.PoolStats()
        _native.check(lib.tsdf_pool_stats_get(self._handle, ctypes.byref(st)), "tsdf_pool_stats_get")
        self.stats = {name: getattr(st, name) for name, _ in _native.PoolStats._fields_ if name != "reserved"}
        self._finalizer = weakref.finalize(self, lib.tsdf_pool_destroy, self._handle)

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._handle

    @classmethod
    def from_words(cls, words: np.ndarray, device: torch.device | str | int = "cuda") -> "NodePool":
        dev = torch.device(device) if not isinstance(device, torch.device) else device
        if dev.type != "cuda":
            raise RuntimeError("NodePool requires a CUDA device; CPU is not supported.")
        idx = dev.index if dev.index is not None else torch.cuda.current_device()
        w = np.ascontiguousarray(np.asarray(words).view(np.uint64))
        out = ctypes.c_void_p()
        lib = _native.tsdf_lib()
        _native.check(
            lib.tsdf_pool_create(w.ctypes.data_as(ctypes.c_void_p), w.shape[0], idx, 0, ctypes.byref(out)),
            "tsdf_pool_create",
        )
        return cls(out.value, torch.device("cuda", idx))

    @classmethod
    def from_tensor(cls, dag_tensor: torch.Tensor) -> "NodePool":
        """Build from the int64 CUDA DAG tensor (copies it to the host once, on the current stream)."""
        if not dag_tensor.is_cuda:
            raise RuntimeError("dag_tensor must be on CUDA. CPU tensors are not supported.")
        dev = dag_tensor.device
        out = ctypes.c_void_p()
        lib = _native.tsdf_lib()
        _native.check(
            lib.tsdf_pool_create_from_device(
                ctypes.c_void_p(dag_tensor.data_ptr()), dag_tensor.numel(), dev.index, 0,
                ctypes.c_void_p(_stream_handle(dev)), ctypes.byref(out),
            ),
            "tsdf_pool_create_from_device",
        )
        return cls(out.value, dev)

    @classmethod
    def from_file(cls, path: Path | str, device: torch.device | str | int = "cuda", *,
                  validate_layout: bool = False) -> tuple["NodePool", list[float], list[float]]:
        """Read a ``.gmdag`` file, re-pack and upload it in one native call
        (``tsdf_pool_create_from_file``); returns the pool and the float32 box the
        reference derives (bmin, bmin + voxel * resolution)."""
        dev = torch.device(device) if not isinstance(device, torch.device) else device
        if dev.type != "cuda":
            raise RuntimeError("NodePool requires a CUDA device; CPU is not supported.")
        idx = dev.index if dev.index is not None else torch.cuda.current_device()
        lib = _native.tsdf_lib()
        out = ctypes.c_void_p()
        bmin = (ctypes.c_float * 3)()
        bmax = (ctypes.c_float * 3)()
        raw = str(Path(path).expanduser().resolve()).encode()
        rc = lib.tsdf_pool_create_from_file(raw, 1 if validate_layout else 0, idx, 0, ctypes.byref(out), bmin, bmax)
        if rc == _native.TSDF_ERR_NOT_FOUND:
            raise FileNotFoundError(_native.last_error())
        _native.check(rc, "tsdf_pool_create_from_file")
        return cls(out.value, torch.device("cuda", idx)), list(bmin), list(bmax)

    def save(self, path: Path | str) -> Path:
        """Write the re-packed pool to a cache file (``tsdf_pool_save``)."""
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        _native.check(_native.tsdf_lib().tsdf_pool_save(self._handle, str(path).encode()), "tsdf_pool_save")
        return path

    @classmethod
    def load(cls, path: Path | str, device: torch.device | str | int = "cuda") -> "NodePool":
        """Upload a pool cache file written by :meth:`save` (``tsdf_pool_load``; every slot is
        checked and the record-graph height recomputed before anything reaches the device)."""
        dev = torch.device(device) if not isinstance(device, torch.device) else device
        idx = dev.index if dev.index is not None else torch.cuda.current_device()
        out = ctypes.c_void_p()
        rc = _native.tsdf_lib().tsdf_pool_load(str(path).encode(), idx, ctypes.byref(out))
        if rc == _native.TSDF_ERR_NOT_FOUND:
            raise FileNotFoundError(_native.last_error())
        _native.check(rc, "tsdf_pool_load")
        return cls(out.value, torch.device("cuda", idx))

    def close(self) -> None:
        self._finalizer()


# --- pool cache for the drop-in cast_rays(dag_tensor, ...) --------------------
# A pool is rebuilt when the tensor object, its storage pointer, its size or its
# version counter (bumped by every in-place write) changes.

_cache_lock = threading.Lock()
_pool_cache: dict[int, tuple[weakref.ref, int, int, int, NodePool]] = {}
_POOL_CACHE_LIMIT = 32


def pool_for_tensor(dag_tensor: torch.Tensor) -> NodePool:
    key = id(dag_tensor)
    version = int(dag_tensor._version)
    ptr = int(dag_tensor.data_ptr())
    numel = int(dag_tensor.numel())
    with _cache_lock:
        hit = _pool_cache.get(key)
        if hit is not None:
            ref, p, n, v, pool = hit
            if ref() is dag_tensor and p == ptr and n == numel and v == version:
                return pool
        dead = [k for k, (r, *_rest) in _pool_cache.items() if r() is None]
        for k in dead:
            _pool_cache.pop(k)
        pool = NodePool.from_tensor(dag_tensor)
        if len(_pool_cache) >= _POOL_CACHE_LIMIT:
            _pool_cache.pop(next(iter(_pool_cache)))
        _pool_cache[key] = (weakref.ref(dag_tensor), ptr, numel, version, pool)
        return pool


def register_pool(dag_tensor: torch.Tensor, pool: NodePool) -> None:
    """Record `pool` as the re-packed form of `dag_tensor` (same words), so the drop-in
    cast_rays(dag_tensor, ...) uses it until the tensor changes."""
    with _cache_lock:
        if len(_pool_cache) >= _POOL_CACHE_LIMIT:
            _pool_cache.pop(next(iter(_pool_cache)))
        _pool_cache[id(dag_tensor)] = (weakref.ref(dag_tensor), int(dag_tensor.data_ptr()), int(dag_tensor.numel()),
                                       int(dag_tensor._version), pool)


def _bbox3(values: Sequence[float], name: str) -> ctypes.Array:
    vals = [float(v) for v in values]
    if len(vals) != 3:
        raise RuntimeError(f"{name} must contain exactly 3 floats")
    return (ctypes.c_float * 3)(*vals)


def _same_device(device: torch.device, *tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and t.device != device:
            raise RuntimeError("all tensors of a cast must be on the CUDA device of the DAG")


def cast_rays_ex(
    pool: NodePool,
    origins: torch.Tensor,
    dirs: torch.Tensor,
    out_distances: torch.Tensor,
    out_semantics: torch.Tensor,
    *,
    max_steps: int,
    max_distance: float,
    bbox_min: Sequence[float],
    bbox_max: Sequence[float],
    hit_epsilon: float = DEFAULT_HIT_EPSILON,
    out_steps: torch.Tensor | None = None,
) -> None:
    """Trace rays given as [..., 3] origins/dirs into preallocated outputs [...]."""
    n = out_distances.numel()
    if origins.numel() != 3 * n or dirs.numel() != 3 * n or out_semantics.numel() != n:
        raise RuntimeError("origins/dirs must hold 3 floats per output ray")
    if out_steps is not None and (out_steps.numel() != n or out_steps.dtype != torch.int32 or not out_steps.is_contiguous()):
        raise RuntimeError("out_steps must be a contiguous int32 tensor with one entry per ray")
    _same_device(pool.device, origins, dirs, out_distances, out_semantics, out_steps)
    ws = workspace(pool.device, n)
    lib = _native.tsdf_lib()
    with _nvtx("tsdf_cast"):
        rc = lib.tsdf_cast(
            pool.handle,
            ctypes.c_void_p(origins.data_ptr()), ctypes.c_void_p(dirs.data_ptr()), n,
            ctypes.c_void_p(out_distances.data_ptr()), ctypes.c_void_p(out_semantics.data_ptr()),
            ctypes.c_void_p(out_steps.data_ptr() if out_steps is not None else None),
            int(max_steps), float(max_distance), _bbox3(bbox_min, "bbox_min"), _bbox3(bbox_max, "bbox_max"),
            float(hit_epsilon), ctypes.c_void_p(ws.data_ptr()), ctypes.c_void_p(_stream_handle(pool.device)),
        )
    _native.check(rc, "tsdf_cast")


@dataclass
class GmDagScene:
    """A loaded scene: asset metadata, its int64 DAG tensor and its node pool."""

    asset: GmDagAsset
    dag_tensor: torch.Tensor
    pool: NodePool

    @property
    def bbox_min(self) -> list[float]:
        return list(self.asset.bbox_min)

    @property
    def bbox_max(self) -> list[float]:
        return list(self.asset.bbox_max)

    @property
    def resolution(self) -> int:
        return self.asset.resolution

    @property
    def voxel_size(self) -> float:
        return self.asset.voxel_size


def _pool_cache_file(cache_dir: Path, gmdag_path: Path) -> Path:
    st = gmdag_path.stat()
    key = hashlib.sha256(f"{gmdag_path}|{st.st_size}|{st.st_mtime_ns}|{st.st_ino}".encode()).hexdigest()[:20]
    return cache_dir / f"{gmdag_path.stem}_{key}.npool"


def load_gmdag(path: Path | str, device: torch.device | str = "cuda", *, validate_layout: bool = False,
               pool_cache: Path | str | None = None) -> GmDagScene:
    """Load a ``.gmdag`` file, upload its words as an int64 tensor (as sdfdag_backend.py:1896-1900
    does) and build its node pool on the same device.

    With ``pool_cache`` (a directory) the re-packed pool is kept on disk, keyed by the
    file's path, size, mtime and inode, and later loads skip the re-pack.  The pool is
    also registered for the returned tensor, so ``torch_sdf.cast_rays(scene.dag_tensor, ...)``
    does not re-pack it either."""
    path = Path(path).expanduser().resolve()
    asset = load_gmdag_asset(path, validate_layout=validate_layout)
    dev = torch.device(device)
    dag = torch.from_numpy(asset.nodes.view(np.int64)).to(device=dev, dtype=torch.int64)
    pool = None
    cache_file = None
    if pool_cache is not None:
        cache_file = _pool_cache_file(Path(pool_cache), path)
        if cache_file.exists():
            try:
                pool = NodePool.load(cache_file, dag.device)
            except RuntimeError:
                pool = None  # unreadable cache entry: rebuild it below
            if pool is not None and pool.stats["source_words"] != asset.nodes.shape[0]:
                pool = None
    if pool is None:
        pool = NodePool.from_words(asset.nodes, dag.device)
        if cache_file is not None:
            pool.save(cache_file)
    register_pool(dag, pool)
    return GmDagScene(asset=asset, dag_tensor=dag, pool=pool)


class SceneSet:
    """Scene table for fan casts: pools with their float32 bounds and hit epsilons."""

    def __init__(
        self,
        pools: Sequence[NodePool],
        bbox_min: Sequence[Sequence[float]],
        bbox_max: Sequence[Sequence[float]],
        hit_epsilon: Sequence[float],
    ) -> None:
        if not pools:
            raise RuntimeError("a scene set needs at least one pool")
        n = len(pools)
        self.pools = list(pools)
        self.device = pools[0].device
        self.bbox_min = np.asarray(bbox_min, dtype=np.float32).reshape(n, 3)
        self.bbox_max = np.asarray(bbox_max, dtype=np.float32).reshape(n, 3)
        self.hit_epsilon = np.asarray(hit_epsilon, dtype=np.float32).reshape(n)
        handles = (ctypes.c_void_p * n)(*[p.handle.value for p in pools])
        out = ctypes.c_void_p()
        lib = _native.tsdf_lib()
        f3 = ctypes.POINTER(ctypes.c_float)
        _native.check(
            lib.tsdf_scenes_create(
                handles, n, self.bbox_min.ctypes.data_as(f3), self.bbox_max.ctypes.data_as(f3),
                self.hit_epsilon.ctypes.data_as(f3), ctypes.byref(out),
            ),
            "tsdf_scenes_create",
        )
        self._handle = out
        self._finalizer = weakref.finalize(self, lib.tsdf_scenes_destroy, out)

    def __len__(self) -> int:
        return len(self.pools)

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._handle

    def close(self) -> None:
        self._finalizer()


def make_poses(
    position: torch.Tensor,
    yaw: torch.Tensor,
    pitch: torch.Tensor | None = None,
    scene: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Pack per-actor poses into the [A, 8] float32 layout of ``tsdf_pose``.

    cos/sin come from ``torch.cos`` / ``torch.sin`` on the device, as in
    sdfdag_backend.py:1301-1302; the scene index is stored as int32 bits.
    """
    a = position.shape[0]
    dev = position.device
    poses = out if out is not None else torch.empty((a, 8), dtype=torch.float32, device=dev)
    poses[:, 0:3] = position
    poses[:, 3] = torch.cos(yaw)
    poses[:, 4] = torch.sin(yaw)
    if pitch is None:
        poses[:, 5] = 1.0
        poses[:, 6] = 0.0
    else:
        poses[:, 5] = torch.cos(pitch)
        poses[:, 6] = torch.sin(pitch)
    sc = scene if scene is not None else torch.zeros(a, dtype=torch.int32, device=dev)
    poses[:, 7] = sc.to(torch.int32).view(torch.float32)
    return poses


def cast_fan(
    scenes: SceneSet,
    poses: torch.Tensor,
    fan_dirs: torch.Tensor,
    out_distances: torch.Tensor,
    out_semantics: torch.Tensor,
    *,
    max_steps: int,
    max_distance: float,
    use_pitch: bool = False,
    out_steps: torch.Tensor | None = None,
) -> None:
    """Trace every actor's fan: out[a, r] for pose a and local direction fan_dirs[r].

    Each actor is traced in the scene its pose names (``make_poses(..., scene=)``); an
    index outside the table gives NaN distance, semantic 0 and 0 steps.  A table of one
    scene is one launch with rays claimed longest-first; a table of 2 to 64 scenes is one
    launch per scene, on library streams forked from and joined back to the current
    stream, so the outputs are ready for anything later on the current stream.  The
    workspace (``tsdf_fan_workspace_bytes``) is allocated here on the current stream.
    """
    if poses.dtype != torch.float32 or poses.dim() != 2 or poses.shape[1] != 8 or not poses.is_contiguous():
        raise RuntimeError("poses must be a contiguous float32 [actors, 8] tensor (see make_poses)")
    if fan_dirs.dtype != torch.float32 or fan_dirs.dim() != 2 or fan_dirs.shape[1] != 3 or not fan_dirs.is_contiguous():
        raise RuntimeError("fan_dirs must be a contiguous float32 [rays, 3] tensor")
    a, r = poses.shape[0], fan_dirs.shape[0]
    for name, t, dt in (("out_distances", out_distances, torch.float32), ("out_semantics", out_semantics, torch.int32)):
        if t.numel() != a * r or t.dtype != dt or not t.is_contiguous():
            raise RuntimeError(f"{name} must be a contiguous {dt} tensor of actors x rays entries")
    if out_steps is not None and (out_steps.numel() != a * r or out_steps.dtype != torch.int32 or not out_steps.is_contiguous()):
        raise RuntimeError("out_steps must be a contiguous int32 tensor of actors x rays entries")
    _same_device(scenes.device, poses, fan_dirs, out_distances, out_semantics, out_steps)
    lib = _native.tsdf_lib()
    ws = torch.empty(int(lib.tsdf_fan_workspace_bytes(scenes.handle, a, r)), dtype=torch.uint8, device=scenes.device)
    with _nvtx("tsdf_cast_fan"):
        rc = lib.tsdf_cast_fan(
            scenes.handle, ctypes.c_void_p(poses.data_ptr()), a, ctypes.c_void_p(fan_dirs.data_ptr()), r,
            1 if use_pitch else 0, ctypes.c_void_p(out_distances.data_ptr()), ctypes.c_void_p(out_semantics.data_ptr()),
            ctypes.c_void_p(out_steps.data_ptr() if out_steps is not None else None), int(max_steps),
            float(max_distance), ctypes.c_void_p(ws.data_ptr()), ctypes.c_void_p(_stream_handle(scenes.device)),
        )
    _native.check(rc, "tsdf_cast_fan")


def cast_fan_observe(
    scenes: SceneSet,
    poses: torch.Tensor,
    fan_dirs: torch.Tensor,
    azimuth_bins: int,
    elevation_bins: int,
    out_distances: torch.Tensor,
    out_semantics: torch.Tensor,
    observation: torch.Tensor,
    actor_stats: torch.Tensor,
    *,
    max_steps: int,
    max_distance: float,
    structure_band_min: float = 1.5,
    structure_band_max: float = 30.0,
    proximity_threshold: float = 2.0,
    use_pitch: bool = False,
    out_steps: torch.Tensor | None = None,
) -> None:
    """cast_fan plus the reference's post-processing (one pass over the outputs, same stream).

    observation: [actors, 3, azimuth_bins, elevation_bins] f32 (depth, semantic, valid),
    as sdfdag_backend.py:1518-1525 stacks it; actor_stats: [actors, 5] f32 (min clamped
    distance, starvation, proximity, structure band, forward structure band ratios), as
    _postprocess_cast_outputs_tensor (sdfdag_backend.py:408-473) returns them.
    """
    a, r = poses.shape[0], fan_dirs.shape[0]
    if azimuth_bins * elevation_bins != r:
        raise RuntimeError("azimuth_bins * elevation_bins must equal the fan size")
    if observation.dtype != torch.float32 or observation.numel() != 3 * a * r or not observation.is_contiguous():
        raise RuntimeError("observation must be a contiguous float32 [actors, 3, az, el] tensor")
    if actor_stats.dtype != torch.float32 or actor_stats.numel() != 5 * a or not actor_stats.is_contiguous():
        raise RuntimeError("actor_stats must be a contiguous float32 [actors, 5] tensor")
    for name, t, dt in (("out_distances", out_distances, torch.float32), ("out_semantics", out_semantics, torch.int32)):
        if t.numel() != a * r or t.dtype != dt or not t.is_contiguous():
            raise RuntimeError(f"{name} must be a contiguous {dt} tensor of actors x rays entries")
    if out_steps is not None and (out_steps.numel() != a * r or out_steps.dtype != torch.int32 or not out_steps.is_contiguous()):
        raise RuntimeError("out_steps must be a contiguous int32 tensor of actors x rays entries")
    _same_device(scenes.device, poses, fan_dirs, out_distances, out_semantics, observation, actor_stats, out_steps)
    lib = _native.tsdf_lib()
    ws = torch.empty(int(lib.tsdf_observe_workspace_bytes(scenes.handle, a, r)), dtype=torch.uint8, device=scenes.device)
    ob = _native.Observe(int(azimuth_bins), int(elevation_bins), float(structure_band_min), float(structure_band_max),
                         float(proximity_threshold), observation.data_ptr(), actor_stats.data_ptr())
    with _nvtx("tsdf_cast_fan_observe"):
        rc = lib.tsdf_cast_fan_observe(
            scenes.handle, ctypes.c_void_p(poses.data_ptr()), a, ctypes.c_void_p(fan_dirs.data_ptr()), r,
            1 if use_pitch else 0, ctypes.c_void_p(out_distances.data_ptr()), ctypes.c_void_p(out_semantics.data_ptr()),
            ctypes.c_void_p(out_steps.data_ptr() if out_steps is not None else None), int(max_steps), float(max_distance),
            ctypes.byref(ob), ctypes.c_void_p(ws.data_ptr()), ctypes.c_void_p(_stream_handle(scenes.device)),
        )
    _native.check(rc, "tsdf_cast_fan_observe")


def hit_epsilon_for(voxel_size: float) -> float:
    """The benchmark configurations' hit threshold, 1e-3 x voxel size, as float32."""
    return float(np.float32(1e-3) * np.float32(voxel_size))


def _is_finite(x: float) -> bool:
    return math.isfinite(x)
