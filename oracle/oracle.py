"""ctypes front end of the parity checkers — TEST INFRASTRUCTURE ONLY.

- :func:`trace`      the C restatement of the reference trace (trace_oracle.c),
                     OpenMP over rays; returns distances, semantics, steps and
                     per-ray DAG word-load counts (W_ref).
- :func:`point_query` one query_dag_stackless call with fresh caches.
- :func:`rotate_fan` the reference's yaw rotation of the local fan
                     (sdfdag_backend.py:1303-1310), numpy float32, every
                     product and sum rounded on its own like torch eager ops,
                     with the pitch rotation used by the benchmark configs.
- :class:`ReferenceKernel` the reference's own CUDA kernel built for sm_100a
                     (oracle/_ref/libref_trace*.so, GPU only).
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "liboracle.so"
REF_SO = HERE / "_ref" / "libref_trace.so"
REF_EPS_SO = HERE / "_ref" / "libref_trace_eps.so"

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            from . import build as _build  # noqa: F401  (oracle/build.py)

            _build.build_oracle()
        L = ctypes.CDLL(str(ORACLE_SO))
        vp = ctypes.c_void_p
        L.oracle_trace.restype = ctypes.c_int64
        L.oracle_trace.argtypes = [vp, ctypes.c_uint64, vp, vp, vp, vp, ctypes.c_int64, ctypes.c_int,
                                   ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_int, vp, vp, vp, vp]
        L.oracle_point_query.restype = ctypes.c_int
        L.oracle_point_query.argtypes = [vp, ctypes.c_uint64, vp, vp, ctypes.c_float, ctypes.c_float,
                                         ctypes.c_float, ctypes.POINTER(ctypes.c_float),
                                         ctypes.POINTER(ctypes.c_int32)]
        L.oracle_half_to_float.restype = ctypes.c_float
        L.oracle_half_to_float.argtypes = [ctypes.c_uint16]
        L.oracle_num_threads.restype = ctypes.c_int
        L.oracle_trace_mix.restype = ctypes.c_int64
        L.oracle_trace_mix.argtypes = [vp, ctypes.c_uint64, vp, vp, vp, vp, ctypes.c_int64, ctypes.c_int,
                                       ctypes.c_float, ctypes.c_float, ctypes.c_int, vp]
        _lib = L
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    return a.ctypes.data_as(ctypes.c_void_p)


def trace(
    words: np.ndarray,
    bbox_min,
    bbox_max,
    origins: np.ndarray,
    dirs: np.ndarray,
    *,
    max_steps: int,
    max_distance: float,
    hit_epsilon: float = 0.01,
    fma: bool = True,
    threads: int = 0,
) -> dict[str, np.ndarray]:
    w = np.ascontiguousarray(np.asarray(words).view(np.uint64))
    o = _f32(origins).reshape(-1, 3)
    d = _f32(dirs).reshape(-1, 3)
    n = o.shape[0]
    bmin = _f32(bbox_min).reshape(3)
    bmax = _f32(bbox_max).reshape(3)
    dist = np.empty(n, np.float32)
    sem = np.empty(n, np.int32)
    steps = np.empty(n, np.int32)
    loads = np.empty(n, np.int64)
    rc = lib().oracle_trace(
        _ptr(w), w.shape[0], _ptr(bmin), _ptr(bmax), _ptr(o), _ptr(d), n, int(max_steps),
        float(max_distance), float(hit_epsilon), 1 if fma else 0, int(threads),
        _ptr(dist), _ptr(sem), _ptr(steps), _ptr(loads),
    )
    if rc != 0:
        raise RuntimeError(f"oracle: DAG index outside the payload on ray {-rc - 1}")
    return {"dist": dist, "sem": sem, "steps": steps, "loads": loads}


MIX_NAMES = ("steps", "void_cache", "outside", "leaf_cache", "descents", "descent_leaf", "descent_void", "levels")


def step_mix(words: np.ndarray, bbox_min, bbox_max, origins: np.ndarray, dirs: np.ndarray, *, max_steps: int,
             max_distance: float, hit_epsilon: float = 0.01, threads: int = 0) -> dict[str, int]:
    """What the reference algorithm's march steps did, summed over the rays (fused position update):
    steps, void-cache hits, steps outside the box, leaf-cache hits, descents, descents ending in a
    leaf / an empty octant, and descent levels."""
    w = np.ascontiguousarray(np.asarray(words).view(np.uint64))
    o = _f32(origins).reshape(-1, 3)
    d = _f32(dirs).reshape(-1, 3)
    bmin = _f32(bbox_min).reshape(3)
    bmax = _f32(bbox_max).reshape(3)
    mix = np.zeros(len(MIX_NAMES), np.int64)
    rc = lib().oracle_trace_mix(_ptr(w), w.shape[0], _ptr(bmin), _ptr(bmax), _ptr(o), _ptr(d), o.shape[0],
                                int(max_steps), float(max_distance), float(hit_epsilon), int(threads), _ptr(mix))
    if rc != 0:
        raise RuntimeError(f"oracle: DAG index outside the payload on ray {-rc - 1}")
    return {k: int(v) for k, v in zip(MIX_NAMES, mix)}


def point_query(words: np.ndarray, bbox_min, bbox_max, p) -> tuple[float, int]:
    w = np.ascontiguousarray(np.asarray(words).view(np.uint64))
    bmin = _f32(bbox_min).reshape(3)
    bmax = _f32(bbox_max).reshape(3)
    d = ctypes.c_float()
    s = ctypes.c_int32()
    rc = lib().oracle_point_query(_ptr(w), w.shape[0], _ptr(bmin), _ptr(bmax), float(p[0]), float(p[1]),
                                  float(p[2]), ctypes.byref(d), ctypes.byref(s))
    if rc != 0:
        raise RuntimeError("oracle: DAG index outside the payload")
    return float(d.value), int(s.value)


def half_to_float(bits: int) -> float:
    return float(lib().oracle_half_to_float(bits))


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def rotate_fan(local: np.ndarray, cos_yaw, sin_yaw, cos_pitch=None, sin_pitch=None) -> np.ndarray:
    """World directions [A, R, 3] from the local fan [R, 3] and per-actor cos/sin [A].

    Each product and each sum is rounded to float32 separately, as the
    reference's eager torch ops do (sdfdag_backend.py:1303-1310).  With pitch,
    the local direction is first rotated about the local x axis:
    y' = y cos(p) - z sin(p), z' = y sin(p) + z cos(p).
    """
    b = _f32(local)[None, :, :]
    cy = _f32(cos_yaw).reshape(-1, 1)
    sy = _f32(sin_yaw).reshape(-1, 1)
    bx, by, bz = b[..., 0], b[..., 1], b[..., 2]
    if cos_pitch is not None:
        cp = _f32(cos_pitch).reshape(-1, 1)
        sp = _f32(sin_pitch).reshape(-1, 1)
        by, bz = (by * cp) - (bz * sp), (by * sp) + (bz * cp)
    else:
        by = np.broadcast_to(by, (cy.shape[0], by.shape[1]))
    x = (bx * cy) + (bz * sy)
    z = ((-bx) * sy) + (bz * cy)
    return np.ascontiguousarray(np.stack([x, np.broadcast_to(by, x.shape), z], axis=-1).astype(np.float32))


class ReferenceKernel:
    """The reference's own sphere_trace_kernel built for sm_100a (GPU only).

    ``eps_variant=True`` loads the build whose hit epsilon is settable.
    The DAG buffer handed to it must hold at least 1024 words: the reference
    stages words 0..1023 into shared memory without a bound (kernel.cu:214-220).
    """

    def __init__(self, eps_variant: bool = False) -> None:
        path = REF_EPS_SO if eps_variant else REF_SO
        if not path.exists():
            raise RuntimeError(f"reference kernel not built: {path} (run python oracle/build.py with the reference tree)")
        L = ctypes.CDLL(str(path))
        vp = ctypes.c_void_p
        L.ref_cast_rays.restype = ctypes.c_int
        L.ref_cast_rays.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                    vp, vp, ctypes.c_int]
        L.ref_synchronize.restype = ctypes.c_int
        L.ref_synchronize.argtypes = [ctypes.c_int]
        L.ref_set_hit_epsilon.restype = ctypes.c_int
        L.ref_set_hit_epsilon.argtypes = [ctypes.c_int, ctypes.c_float]
        self._lib = L
        self.eps_variant = eps_variant

    def cast(self, dag_padded, origins, dirs, out_d, out_s, *, max_steps, max_distance, bbox_min, bbox_max,
             resolution=1, hit_epsilon=None, device=0) -> None:
        """All tensor arguments are CUDA torch tensors; the call is synchronous."""
        if dag_padded.numel() < 1024:
            raise RuntimeError("reference kernel needs a DAG buffer of at least 1024 words")
        if hit_epsilon is not None:
            if not self.eps_variant:
                if np.float32(hit_epsilon) != np.float32(0.01):
                    raise RuntimeError("the unmodified reference build has epsilon 0.01")
            else:
                rc = self._lib.ref_set_hit_epsilon(device, float(hit_epsilon))
                if rc != 0:
                    raise RuntimeError(f"ref_set_hit_epsilon failed: {rc}")
        bmin = _f32(bbox_min).reshape(3)
        bmax = _f32(bbox_max).reshape(3)
        n = out_d.numel()
        rc = self._lib.ref_cast_rays(
            device, ctypes.c_void_p(dag_padded.data_ptr()), ctypes.c_void_p(origins.data_ptr()),
            ctypes.c_void_p(dirs.data_ptr()), ctypes.c_void_p(out_d.data_ptr()), ctypes.c_void_p(out_s.data_ptr()),
            n, int(max_steps), float(max_distance), _ptr(bmin), _ptr(bmax), int(resolution),
        )
        if rc != 0:
            raise RuntimeError(f"reference launch failed: {rc}")
        rc = self._lib.ref_synchronize(device)
        if rc != 0:
            raise RuntimeError(f"reference kernel failed: {rc}")


def pad_words(words: np.ndarray, minimum: int = 1024) -> np.ndarray:
    w = np.asarray(words).view(np.uint64)
    if w.shape[0] >= minimum:
        return np.ascontiguousarray(w)
    out = np.zeros(minimum, np.uint64)
    out[: w.shape[0]] = w
    return out


def reference_available() -> bool:
    return REF_SO.exists() and REF_EPS_SO.exists()


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
