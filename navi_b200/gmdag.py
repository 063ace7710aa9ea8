"""``.gmdag`` files: load, validate, write, and compile from a triangle mesh.

File format (projects/voxel-dag/src/compiler.hpp:22-32, docs/GMDAG.md): a
32-byte little-endian header ``<4sIIffffI`` = magic ``b"GDAG"``, version 1,
resolution, bbox_min xyz, voxel size, node count; then ``node_count`` u64 words.
A word with bit 63 set is a leaf (bits 0-15 half-float distance, bits 16-31
semantic); otherwise bits 55-62 are the child mask and bits 0-31 the index of
the child pointer table, whose entries' low 32 bits index child nodes.

:func:`load_gmdag_asset` mirrors the reference loader
(projects/environment/src/navi_environment/integration/voxel_dag.py:193-259)
with the same checks and error texts; the layout validator mirrors
``_validate_gmdag_dag_layout`` (voxel_dag.py:29-78) but walks the DAG with an
explicit stack instead of recursion.  Both run in C++ (libnavi_gmdag.so,
``gmdag_file_read`` / ``gmdag_validate_layout`` of include/gmdag.h).
"""

from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import _native

__all__ = [
    "GmDagAsset",
    "load_gmdag_asset",
    "validate_gmdag_layout",
    "write_gmdag",
    "compile_mesh",
    "half_from_float_ref",
]

_HEADER_STRUCT = struct.Struct("<4sIIffffI")


@dataclass(frozen=True, slots=True)
class GmDagAsset:
    """Loaded ``.gmdag`` asset metadata and node payload (voxel_dag.py:81-91)."""

    path: Path
    version: int
    resolution: int
    bbox_min: tuple[float, float, float]
    bbox_max: tuple[float, float, float]
    voxel_size: float
    nodes: np.ndarray


def validate_gmdag_layout(nodes: np.ndarray) -> None:
    """Reject cycles, empty internal masks and out-of-range references reachable from word 0.

    The walk runs in libnavi_gmdag.so (gmdag_validate_layout): the reference's
    depth-first order and texts (voxel_dag.py:29-78) without its recursion."""
    w = np.ascontiguousarray(np.asarray(nodes).view(np.uint64) if np.asarray(nodes).dtype.itemsize == 8
                             else np.asarray(nodes, dtype=np.uint64))
    lib = _native.gmdag_lib()
    err = _native.GmdagLayoutError()
    rc = lib.gmdag_validate_layout(w.ctypes.data_as(ctypes.c_void_p), w.shape[0], ctypes.byref(err))
    if rc != 0:
        raise RuntimeError(lib.gmdag_last_error().decode())


def load_gmdag_asset(path: Path | str, *, validate_layout: bool = True) -> GmDagAsset:
    """Load a ``.gmdag`` binary into metadata plus a contiguous node array.

    Reading and checks run in libnavi_gmdag.so (gmdag_file_read), in the order and
    with the texts of voxel_dag.py:193-259."""
    path = Path(path).expanduser().resolve()
    lib = _native.gmdag_lib()
    info = _native.GmdagFileInfo()
    layout = _native.GmdagLayoutError()
    raw = str(path).encode()
    st = lib.gmdag_file_read(raw, None, 0, 0, ctypes.byref(info), ctypes.byref(layout))
    nodes = None
    if st == _native.GMDAG_FILE_OK:
        nodes = np.empty(int(info.node_count), dtype=np.uint64)
        st = lib.gmdag_file_read(raw, nodes.ctypes.data_as(ctypes.c_void_p), nodes.shape[0],
                                 1 if validate_layout else 0, ctypes.byref(info), ctypes.byref(layout))
    if st == _native.GMDAG_FILE_NOT_FOUND:
        raise FileNotFoundError(lib.gmdag_last_error().decode())
    if st != _native.GMDAG_FILE_OK:
        raise RuntimeError(lib.gmdag_last_error().decode())
    bmin_x, bmin_y, bmin_z = (float(v) for v in info.bbox_min)
    voxel_size = float(info.voxel_size)
    resolution = int(info.resolution)
    bbox_min = (bmin_x, bmin_y, bmin_z)
    extent = voxel_size * resolution  # Python double, voxel_dag.py:244-250
    bbox_max = (bbox_min[0] + extent, bbox_min[1] + extent, bbox_min[2] + extent)
    return GmDagAsset(
        path=path,
        version=int(info.version),
        resolution=resolution,
        bbox_min=bbox_min,
        bbox_max=bbox_max,
        voxel_size=voxel_size,
        nodes=nodes,
    )


def write_gmdag(
    path: Path | str,
    nodes: np.ndarray,
    resolution: int,
    bbox_min: tuple[float, float, float] | np.ndarray,
    voxel_size: float,
) -> Path:
    """Write header + payload exactly as compiler.cpp:680-697 does."""
    path = Path(path)
    nodes = np.ascontiguousarray(np.asarray(nodes, dtype=np.uint64))
    header = _HEADER_STRUCT.pack(
        b"GDAG", 1, int(resolution), float(bbox_min[0]), float(bbox_min[1]), float(bbox_min[2]),
        float(voxel_size), int(nodes.shape[0]),
    )
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    with tmp.open("wb") as fh:
        fh.write(header)
        fh.write(nodes.tobytes())
    tmp.replace(path)
    return path


@dataclass(frozen=True)
class CompiledMesh:
    nodes: np.ndarray  # uint64 words
    resolution: int
    bbox_min: tuple[float, float, float]  # float32 values as compiled
    bbox_max: tuple[float, float, float]
    voxel_size: float
    timing: dict | None = None  # device compiler: stage times (ms) and block counts


def _mesh_arrays(vertices: np.ndarray, triangles: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    v = np.ascontiguousarray(vertices, dtype=np.float32).reshape(-1, 3)
    t = np.ascontiguousarray(triangles, dtype=np.uint32).reshape(-1, 3)
    return v, t


def _read_result(lib: ctypes.CDLL, prefix: str, handle: ctypes.c_void_p, resolution: int) -> CompiledMesh:
    try:
        n = int(getattr(lib, f"{prefix}_result_num_words")(handle))
        words = np.empty(n, dtype=np.uint64)
        getattr(lib, f"{prefix}_result_copy_words")(handle, words.ctypes.data_as(ctypes.c_void_p))
        bmin = (ctypes.c_float * 3)()
        bmax = (ctypes.c_float * 3)()
        vox = ctypes.c_float()
        getattr(lib, f"{prefix}_result_header")(handle, bmin, bmax, ctypes.byref(vox))
        timing = None
        if prefix == "gmdag_gpu":
            timing = _native.GpuCompileTiming()
            lib.gmdag_gpu_result_timing(handle, ctypes.byref(timing))
    finally:
        getattr(lib, f"{prefix}_result_free")(handle)
    return CompiledMesh(
        nodes=words,
        resolution=int(resolution),
        bbox_min=(bmin[0], bmin[1], bmin[2]),
        bbox_max=(bmax[0], bmax[1], bmax[2]),
        voxel_size=float(vox.value),
        timing=None if timing is None else {name: getattr(timing, name) for name, _ in timing._fields_},
    )


def compile_mesh(vertices: np.ndarray, triangles: np.ndarray, resolution: int, *, threads: int = 0,
                 device: int | None = None) -> CompiledMesh:
    """Compile a triangle mesh to DAG words.

    device=None runs the host compiler (OpenMP, `threads` threads); device=k runs the
    device compiler on CUDA device k (power-of-two resolutions).  Both give the same
    words."""
    v, t = _mesh_arrays(vertices, triangles)
    handle = ctypes.c_void_p()
    if device is None:
        lib, prefix = _native.gmdag_lib(), "gmdag"
        rc = lib.gmdag_compile_mesh(
            v.ctypes.data_as(ctypes.c_void_p), ctypes.c_uint64(v.shape[0]),
            t.ctypes.data_as(ctypes.c_void_p), ctypes.c_uint64(t.shape[0]),
            ctypes.c_uint32(resolution), ctypes.c_int(threads), ctypes.byref(handle),
        )
    else:
        lib, prefix = _native.gmdag_gpu_lib(), "gmdag_gpu"
        rc = lib.gmdag_gpu_compile_mesh(
            v.ctypes.data_as(ctypes.c_void_p), ctypes.c_uint64(v.shape[0]),
            t.ctypes.data_as(ctypes.c_void_p), ctypes.c_uint64(t.shape[0]),
            ctypes.c_uint32(resolution), ctypes.c_int(int(device)), ctypes.byref(handle),
        )
    if rc != 0:
        raise RuntimeError(f"gmdag compile failed: {getattr(lib, prefix + '_last_error')().decode()}")
    return _read_result(lib, prefix, handle, resolution)


def compute_sdf(vertices: np.ndarray, triangles: np.ndarray, resolution: int, *, threads: int = 0,
                device: int | None = None):
    """Stage 2 of the compiler alone: (dense grid [z, y, x] f32, bbox_min, bbox_max, voxel)."""
    v, t = _mesh_arrays(vertices, triangles)
    grid = np.empty((resolution, resolution, resolution), np.float32)
    bmin = (ctypes.c_float * 3)()
    bmax = (ctypes.c_float * 3)()
    vox = ctypes.c_float()
    if device is None:
        lib, fn, err = _native.gmdag_lib(), "gmdag_compute_sdf", "gmdag_last_error"
        arg = threads
    else:
        lib, fn, err = _native.gmdag_gpu_lib(), "gmdag_gpu_compute_sdf", "gmdag_gpu_last_error"
        arg = int(device)
    rc = getattr(lib, fn)(v.ctypes.data_as(ctypes.c_void_p), v.shape[0], t.ctypes.data_as(ctypes.c_void_p),
                          t.shape[0], resolution, arg, grid.ctypes.data_as(ctypes.c_void_p), bmin, bmax,
                          ctypes.byref(vox))
    if rc != 0:
        raise RuntimeError(f"gmdag compute_sdf failed: {getattr(lib, err)().decode()}")
    return grid, tuple(bmin), tuple(bmax), float(vox.value)


def compile_grid(grid: np.ndarray, voxel_size: float, *, threads: int = 0, device: int | None = None) -> np.ndarray:
    """Stage 3 of the compiler alone: DAG words of a dense grid [z, y, x]."""
    g = np.ascontiguousarray(grid, dtype=np.float32)
    n = g.shape[0]
    if g.shape != (n, n, n):
        raise RuntimeError("grid must be cubic [res, res, res]")
    handle = ctypes.c_void_p()
    if device is None:
        lib, prefix = _native.gmdag_lib(), "gmdag"
        rc = lib.gmdag_compile_grid(g.ctypes.data_as(ctypes.c_void_p), n, ctypes.c_float(voxel_size), threads,
                                    ctypes.byref(handle))
    else:
        lib, prefix = _native.gmdag_gpu_lib(), "gmdag_gpu"
        rc = lib.gmdag_gpu_compile_grid(g.ctypes.data_as(ctypes.c_void_p), n, ctypes.c_float(voxel_size),
                                        int(device), ctypes.byref(handle))
    if rc != 0:
        raise RuntimeError(f"gmdag compile_grid failed: {getattr(lib, prefix + '_last_error')().decode()}")
    return _read_result(lib, prefix, handle, n).nodes


def half_from_float_ref(x: float) -> int:
    """The scene compiler's float->half conversion (truncating; tiny values become +inf)."""
    return int(_native.gmdag_lib().gmdag_half_from_float(ctypes.c_float(x)))
