"""ctypes bindings of the in-tree native libraries.

The product path has no fallback: when libnavi_tsdf.so is missing or cannot be
loaded, every call that needs it raises RuntimeError.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "_lib"
# $NAVI_TSDF_DEBUG=1 selects the bounds-checked build (kernel indices checked, a device
# error word reported by every call; slower)
TSDF_PATH = LIB_DIR / ("libnavi_tsdf_debug.so" if os.environ.get("NAVI_TSDF_DEBUG", "0") not in ("", "0")
                       else "libnavi_tsdf.so")
GMDAG_PATH = LIB_DIR / "libnavi_gmdag.so"
GMDAG_GPU_PATH = LIB_DIR / "libnavi_gmdag_gpu.so"

_lock = threading.Lock()
_tsdf: ctypes.CDLL | None = None
_gmdag: ctypes.CDLL | None = None
_gmdag_gpu: ctypes.CDLL | None = None

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_int64 = ctypes.c_int64
c_uint64 = ctypes.c_uint64
c_uint32 = ctypes.c_uint32
c_float = ctypes.c_float
c_char_p = ctypes.c_char_p


class PoolStats(ctypes.Structure):
    _fields_ = [
        ("source_words", c_uint64),
        ("records", c_uint64),
        ("ext_leaves", c_uint64),
        ("device_bytes", c_uint64),
        ("root_slot", c_uint32),
        ("bfs_levels", c_uint32),
        ("device", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class Observe(ctypes.Structure):
    _fields_ = [
        ("azimuth_bins", ctypes.c_int32),
        ("elevation_bins", ctypes.c_int32),
        ("structure_band_min", c_float),
        ("structure_band_max", c_float),
        ("proximity_threshold", c_float),
        ("observation", c_void_p),
        ("actor_stats", c_void_p),
    ]


# name -> (restype, argtypes); mirrors include/tsdf.h
TSDF_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "tsdf_version": (c_int, []),
    "tsdf_last_error": (c_char_p, []),
    "tsdf_pool_create": (c_int, [c_void_p, c_uint64, c_int, c_uint32, ctypes.POINTER(c_void_p)]),
    "tsdf_pool_create_from_device": (c_int, [c_void_p, c_uint64, c_int, c_uint32, c_void_p, ctypes.POINTER(c_void_p)]),
    "tsdf_pool_create_from_file": (c_int, [c_char_p, c_int, c_int, c_uint32, ctypes.POINTER(c_void_p),
                                           ctypes.POINTER(c_float), ctypes.POINTER(c_float)]),
    "tsdf_pool_save": (c_int, [c_void_p, c_char_p]),
    "tsdf_pool_load": (c_int, [c_char_p, c_int, ctypes.POINTER(c_void_p)]),
    "tsdf_pool_destroy": (c_int, [c_void_p]),
    "tsdf_pool_stats_get": (c_int, [c_void_p, ctypes.POINTER(PoolStats)]),
    "tsdf_fan_workspace_bytes": (c_uint64, [c_void_p, c_int64, c_int64]),
    "tsdf_workspace_bytes": (c_uint64, [c_int64]),
    "tsdf_cast": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int,
                          c_float, ctypes.POINTER(c_float), ctypes.POINTER(c_float), c_float, c_void_p, c_void_p]),
    "tsdf_scenes_create": (c_int, [ctypes.POINTER(c_void_p), c_int, ctypes.POINTER(c_float), ctypes.POINTER(c_float),
                                   ctypes.POINTER(c_float), ctypes.POINTER(c_void_p)]),
    "tsdf_scenes_destroy": (c_int, [c_void_p]),
    "tsdf_cast_fan": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p,
                              c_int, c_float, c_void_p, c_void_p]),
    "tsdf_set_option": (c_int, [c_char_p, c_int64, ctypes.POINTER(c_int64)]),
    "tsdf_observe_workspace_bytes": (c_uint64, [c_void_p, c_int64, c_int64]),
    "tsdf_cast_fan_observe": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_int, c_void_p, c_void_p,
                                      c_void_p, c_int, c_float, ctypes.POINTER(Observe), c_void_p, c_void_p]),
    "tsdf_cast_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int,
                                  c_float, ctypes.POINTER(c_float), ctypes.POINTER(c_float), c_float, c_void_p]),
}

class GmdagFileInfo(ctypes.Structure):
    """gmdag_file_info of include/gmdag.h."""

    _fields_ = [
        ("magic", ctypes.c_char * 4),
        ("version", c_uint32),
        ("resolution", c_uint32),
        ("bbox_min", c_float * 3),
        ("voxel_size", c_float),
        ("node_count", c_uint32),
        ("nodes_found", c_uint64),
        ("trailing_bytes", c_uint64),
    ]


class GmdagLayoutError(ctypes.Structure):
    """gmdag_layout_error of include/gmdag.h."""

    _fields_ = [("kind", ctypes.c_int32), ("reserved", c_uint32), ("node", c_uint64), ("value", c_uint64)]


TSDF_ERR_NOT_FOUND = -6  # tsdf_status of include/tsdf.h
TSDF_ERR_FILE = -7

GMDAG_FILE_OK = 0
GMDAG_FILE_NOT_FOUND = 1

GMDAG_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "gmdag_last_error": (c_char_p, []),
    "gmdag_compile_mesh": (c_int, [c_void_p, c_uint64, c_void_p, c_uint64, c_uint32, c_int, ctypes.POINTER(c_void_p)]),
    "gmdag_result_num_words": (c_uint64, [c_void_p]),
    "gmdag_result_header": (None, [c_void_p, ctypes.POINTER(c_float), ctypes.POINTER(c_float), ctypes.POINTER(c_float)]),
    "gmdag_result_copy_words": (None, [c_void_p, c_void_p]),
    "gmdag_result_free": (None, [c_void_p]),
    "gmdag_half_from_float": (ctypes.c_uint16, [c_float]),
    "gmdag_compute_sdf": (c_int, [c_void_p, c_uint64, c_void_p, c_uint64, c_uint32, c_int, c_void_p,
                                  ctypes.POINTER(c_float), ctypes.POINTER(c_float), ctypes.POINTER(c_float)]),
    "gmdag_compile_grid": (c_int, [c_void_p, c_uint32, c_float, c_int, ctypes.POINTER(c_void_p)]),
    "gmdag_file_read": (c_int, [c_char_p, c_void_p, c_uint64, c_int, ctypes.POINTER(GmdagFileInfo),
                                ctypes.POINTER(GmdagLayoutError)]),
    "gmdag_validate_layout": (c_int, [c_void_p, c_uint64, ctypes.POINTER(GmdagLayoutError)]),
}


class GpuCompileTiming(ctypes.Structure):
    """gmdag_gpu_timing of include/gmdag.h."""

    _fields_ = [
        ("upload_ms", ctypes.c_double),
        ("seed_ms", ctypes.c_double),
        ("sweep_ms", ctypes.c_double),
        ("pyramid_ms", ctypes.c_double),
        ("levels_ms", ctypes.c_double),
        ("emit_ms", ctypes.c_double),
        ("visited_blocks", c_uint64),
        ("unique_internal", c_uint64),
    ]


GMDAG_GPU_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "gmdag_gpu_last_error": (c_char_p, []),
    "gmdag_gpu_compile_mesh": (c_int, [c_void_p, c_uint64, c_void_p, c_uint64, c_uint32, c_int,
                                       ctypes.POINTER(c_void_p)]),
    "gmdag_gpu_compute_sdf": (c_int, [c_void_p, c_uint64, c_void_p, c_uint64, c_uint32, c_int, c_void_p,
                                      ctypes.POINTER(c_float), ctypes.POINTER(c_float), ctypes.POINTER(c_float)]),
    "gmdag_gpu_compile_grid": (c_int, [c_void_p, c_uint32, c_float, c_int, ctypes.POINTER(c_void_p)]),
    "gmdag_gpu_result_num_words": (c_uint64, [c_void_p]),
    "gmdag_gpu_result_header": (None, [c_void_p, ctypes.POINTER(c_float), ctypes.POINTER(c_float),
                                       ctypes.POINTER(c_float)]),
    "gmdag_gpu_result_copy_words": (None, [c_void_p, c_void_p]),
    "gmdag_gpu_result_timing": (None, [c_void_p, ctypes.POINTER(GpuCompileTiming)]),
    "gmdag_gpu_result_free": (None, [c_void_p]),
}


def _bind(lib: ctypes.CDLL, sigs: dict[str, tuple[object, list[object]]]) -> None:
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def tsdf_lib() -> ctypes.CDLL:
    """The trace library; raises RuntimeError when it is not built or cannot load."""
    global _tsdf
    if _tsdf is None:
        with _lock:
            if _tsdf is None:
                if not TSDF_PATH.exists():
                    raise RuntimeError(
                        f"navi_b200 CUDA library not found at {TSDF_PATH}; run `python -m navi_b200.build`"
                    )
                lib = ctypes.CDLL(str(TSDF_PATH))
                _bind(lib, TSDF_SIGNATURES)
                _tsdf = lib
    return _tsdf


def gmdag_lib() -> ctypes.CDLL:
    global _gmdag
    if _gmdag is None:
        with _lock:
            if _gmdag is None:
                if not GMDAG_PATH.exists():
                    raise RuntimeError(
                        f"navi_b200 scene compiler not found at {GMDAG_PATH}; run `python -m navi_b200.build`"
                    )
                lib = ctypes.CDLL(str(GMDAG_PATH))
                _bind(lib, GMDAG_SIGNATURES)
                _gmdag = lib
    return _gmdag


def gmdag_gpu_lib() -> ctypes.CDLL:
    """The device scene compiler; raises RuntimeError when it is not built or cannot load."""
    global _gmdag_gpu
    if _gmdag_gpu is None:
        with _lock:
            if _gmdag_gpu is None:
                if not GMDAG_GPU_PATH.exists():
                    raise RuntimeError(
                        f"navi_b200 device scene compiler not found at {GMDAG_GPU_PATH}; "
                        "run `python -m navi_b200.build`"
                    )
                lib = ctypes.CDLL(str(GMDAG_GPU_PATH))
                _bind(lib, GMDAG_GPU_SIGNATURES)
                _gmdag_gpu = lib
    return _gmdag_gpu


def last_error() -> str:
    msg = tsdf_lib().tsdf_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed ({rc}): {last_error()}")
