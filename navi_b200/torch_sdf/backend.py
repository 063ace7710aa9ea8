"""Drop-in replacement of ``torch_sdf.backend`` (projects/torch-sdf/torch_sdf/backend.py).

Same public function, same argument order and meaning, same validation order
and error texts as the reference:

- ``cast_rays(dag_tensor, origins, dirs, out_distances, out_semantics,
  max_steps, max_distance, bbox_min, bbox_max, resolution,
  skip_direction_validation=False)`` (backend.py:145-197), with two
  keyword-only extras: ``hit_epsilon`` (the reference hard-codes 0.01,
  kernel.cuh:7) and ``out_steps`` (int32 march-iteration counts).
- ``torch_sdf_backend`` is the native module object; its ``cast_rays`` takes
  the same 11 positional arguments as the reference pybind function
  (bindings.cpp:112-120) and applies the same TORCH_CHECK contract
  (bindings.cpp:57-89) before calling the C ABI of libnavi_tsdf.so.

Strict CUDA-only path: there is no CPU fallback.  The launch goes to the
caller's current CUDA stream (the reference uses the legacy default stream).
"""

from __future__ import annotations

import math
from typing import Any

import torch

from .. import _native, tracer

_DAG_DTYPE = torch.int64
_DISTANCE_DTYPE = torch.float32
_SEMANTIC_DTYPE = torch.int32
_HIT_EPSILON = 0.01
_DIRECTION_NORM_EPS = 1e-4


class _NativeBackend:
    """The ``torch_sdf_backend`` module of the reference, over the C ABI."""

    @staticmethod
    def _check(cond: bool, msg: str) -> None:
        if not cond:
            raise RuntimeError(msg)

    def _contract(
        self,
        dag_tensor: torch.Tensor,
        origins: torch.Tensor,
        dirs: torch.Tensor,
        out_distances: torch.Tensor,
        out_semantics: torch.Tensor,
        max_steps: int,
        max_distance: float,
        bbox_min: list[float],
        bbox_max: list[float],
        resolution: int,
        skip_direction_validation: bool,
    ) -> None:
        c = self._check
        # bindings.cpp:57-89
        c(dag_tensor.is_cuda, "dag_tensor must be a CUDA tensor")
        c(origins.is_cuda, "origins must be a CUDA tensor")
        c(dirs.is_cuda, "dirs must be a CUDA tensor")
        c(out_distances.is_cuda, "out_distances must be a CUDA tensor")
        c(out_semantics.is_cuda, "out_semantics must be a CUDA tensor")
        c(origins.is_contiguous(), "origins must be contiguous")
        c(dirs.is_contiguous(), "dirs must be contiguous")
        c(out_distances.is_contiguous(), "out_distances must be contiguous")
        c(out_semantics.is_contiguous(), "out_semantics must be contiguous")
        c(dag_tensor.dtype == torch.int64, "dag_tensor must be int64")
        c(origins.dtype == torch.float32, "origins must be float32")
        c(dirs.dtype == torch.float32, "dirs must be float32")
        c(out_distances.dtype == torch.float32, "out_distances must be float32")
        c(out_semantics.dtype == torch.int32, "out_semantics must be int32")
        c(origins.dim() == 3 and origins.size(2) == 3, "origins must be [Batch, Rays, 3]")
        c(dirs.dim() == 3 and dirs.size(2) == 3, "dirs must be [Batch, Rays, 3]")
        c(tuple(dirs.shape) == tuple(origins.shape), "dirs must match origins shape")
        c(out_distances.dim() == 2, "out_distances must be [Batch, Rays]")
        c(out_semantics.dim() == 2, "out_semantics must be [Batch, Rays]")
        c(
            out_distances.size(0) == origins.size(0) and out_distances.size(1) == origins.size(1),
            "out_distances must match the [Batch, Rays] shape of origins",
        )
        c(
            out_semantics.size(0) == origins.size(0) and out_semantics.size(1) == origins.size(1),
            "out_semantics must match the [Batch, Rays] shape of origins",
        )
        c(max_steps > 0, "max_steps must be a positive integer")
        c(math.isfinite(max_distance) and max_distance > 0.0, "max_distance must be a finite positive float")
        c(resolution > 0, "resolution must be a positive integer")
        c(len(bbox_min) == 3, "bbox_min must contain exactly 3 floats")
        c(len(bbox_max) == 3, "bbox_max must contain exactly 3 floats")
        for i in range(3):
            c(math.isfinite(float(bbox_min[i])), "bbox_min must contain only finite floats")
            c(math.isfinite(float(bbox_max[i])), "bbox_max must contain only finite floats")
            c(float(bbox_min[i]) < float(bbox_max[i]), "bbox_min entries must be strictly less than bbox_max entries")
        if not skip_direction_validation:
            norms = torch.sqrt(torch.sum(dirs * dirs, -1))
            c(bool(torch.isfinite(norms).all().item()), "dirs must contain only finite direction vectors")
            max_error = float(torch.abs(norms - 1.0).amax().item())
            c(
                max_error <= _DIRECTION_NORM_EPS,
                f"dirs must be normalized within tolerance {_DIRECTION_NORM_EPS}; max error was {max_error}",
            )

    def cast_rays(
        self,
        dag_tensor: torch.Tensor,
        origins: torch.Tensor,
        dirs: torch.Tensor,
        out_distances: torch.Tensor,
        out_semantics: torch.Tensor,
        max_steps: int,
        max_distance: float,
        bbox_min: list[float],
        bbox_max: list[float],
        resolution: int,
        skip_direction_validation: bool = False,
    ) -> None:
        self.cast_rays_ex(
            dag_tensor, origins, dirs, out_distances, out_semantics, max_steps, max_distance,
            bbox_min, bbox_max, resolution, skip_direction_validation,
        )

    def cast_rays_ex(
        self,
        dag_tensor: torch.Tensor,
        origins: torch.Tensor,
        dirs: torch.Tensor,
        out_distances: torch.Tensor,
        out_semantics: torch.Tensor,
        max_steps: int,
        max_distance: float,
        bbox_min: list[float],
        bbox_max: list[float],
        resolution: int,
        skip_direction_validation: bool = False,
        hit_epsilon: float = _HIT_EPSILON,
        out_steps: torch.Tensor | None = None,
    ) -> None:
        self._contract(
            dag_tensor, origins, dirs, out_distances, out_semantics, max_steps, max_distance,
            bbox_min, bbox_max, resolution, skip_direction_validation,
        )
        pool = tracer.pool_for_tensor(dag_tensor)
        tracer.cast_rays_ex(
            pool, origins, dirs, out_distances, out_semantics,
            max_steps=max_steps, max_distance=max_distance, bbox_min=bbox_min, bbox_max=bbox_max,
            hit_epsilon=hit_epsilon, out_steps=out_steps,
        )


torch_sdf_backend: Any | None = None
try:
    _native.tsdf_lib()
    torch_sdf_backend = _NativeBackend()
    HAS_CUDA_BACKEND = True
except (OSError, RuntimeError):
    HAS_CUDA_BACKEND = False


# --- PYTHON API (backend.py:16-197) ---


def _shape_tuple(tensor: Any) -> tuple[int, ...]:
    return tuple(int(dim) for dim in tensor.shape)


def _validate_cuda_tensor(
    tensor: Any,
    *,
    name: str,
    dtype: torch.dtype,
    shape: tuple[int, ...] | None = None,
) -> None:
    if not tensor.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor. CPU tensors are not supported.")
    if tensor.dtype != dtype:
        raise RuntimeError(f"{name} must have dtype {dtype}; got {tensor.dtype}.")
    if not tensor.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous.")
    if shape is not None and _shape_tuple(tensor) != shape:
        raise RuntimeError(f"{name} must have shape {shape}; got {_shape_tuple(tensor)}.")


def _validate_cast_rays_inputs(
    dag_tensor: Any,
    origins: Any,
    dirs: Any,
    out_distances: Any,
    out_semantics: Any,
    *,
    skip_direction_validation: bool = False,
) -> None:
    if not dag_tensor.is_cuda:
        raise RuntimeError("dag_tensor must be on CUDA. CPU tensors are not supported.")
    if dag_tensor.dtype != _DAG_DTYPE:
        raise RuntimeError(f"dag_tensor must have dtype {_DAG_DTYPE}; got {dag_tensor.dtype}.")
    if not dag_tensor.is_contiguous():
        raise RuntimeError("dag_tensor must be contiguous.")
    if origins.dim() != 3 or origins.size(2) != 3:
        raise RuntimeError(f"origins must have shape [batch, rays, 3]; got {_shape_tuple(origins)}.")
    if dirs.dim() != 3 or dirs.size(2) != 3:
        raise RuntimeError(f"dirs must have shape [batch, rays, 3]; got {_shape_tuple(dirs)}.")
    batch = int(origins.size(0))
    rays = int(origins.size(1))
    if _shape_tuple(dirs) != (batch, rays, 3):
        raise RuntimeError(f"dirs must match origins shape {(batch, rays, 3)}; got {_shape_tuple(dirs)}.")
    _validate_cuda_tensor(origins, name="origins", dtype=_DISTANCE_DTYPE)
    _validate_cuda_tensor(dirs, name="dirs", dtype=_DISTANCE_DTYPE)
    _validate_cuda_tensor(out_distances, name="out_distances", dtype=_DISTANCE_DTYPE, shape=(batch, rays))
    _validate_cuda_tensor(out_semantics, name="out_semantics", dtype=_SEMANTIC_DTYPE, shape=(batch, rays))
    if not skip_direction_validation and torch.is_tensor(dirs):
        _validate_direction_norms(dirs)


def _validate_direction_norms(dirs: torch.Tensor, *, eps: float = _DIRECTION_NORM_EPS) -> None:
    norms = torch.linalg.vector_norm(dirs, dim=-1)
    if bool((~torch.isfinite(norms)).any().item()):
        raise RuntimeError("dirs must contain only finite direction vectors.")
    max_error = float(torch.abs(norms - 1.0).amax().detach().cpu().item())
    if max_error > eps:
        raise RuntimeError(f"dirs must be normalized within tolerance {eps}; max error was {max_error:.6g}.")


def _validate_bounds(bbox_min: list[float], bbox_max: list[float]) -> None:
    if len(bbox_min) != 3 or len(bbox_max) != 3:
        raise RuntimeError("bbox_min and bbox_max must each contain exactly 3 floats.")
    for index, (lower, upper) in enumerate(zip(bbox_min, bbox_max, strict=False)):
        if not math.isfinite(lower) or not math.isfinite(upper):
            raise RuntimeError("bbox_min and bbox_max must contain only finite floats.")
        if lower >= upper:
            raise RuntimeError(
                f"bbox_min[{index}] must be strictly less than bbox_max[{index}]; got {lower} >= {upper}."
            )


def _validate_runtime_parameters(
    *,
    max_steps: int,
    max_distance: float,
    bbox_min: list[float],
    bbox_max: list[float],
    resolution: int,
) -> None:
    if max_steps <= 0:
        raise RuntimeError(f"max_steps must be a positive integer; got {max_steps}.")
    if not math.isfinite(max_distance) or max_distance <= 0.0:
        raise RuntimeError(f"max_distance must be a finite positive float; got {max_distance}.")
    if resolution <= 0:
        raise RuntimeError(f"resolution must be a positive integer; got {resolution}.")
    _validate_bounds(bbox_min, bbox_max)


def cast_rays(
    dag_tensor: Any,
    origins: Any,
    dirs: Any,
    out_distances: Any,
    out_semantics: Any,
    max_steps: int,
    max_distance: float,
    bbox_min: list[float],
    bbox_max: list[float],
    resolution: int,
    skip_direction_validation: bool = False,
    *,
    hit_epsilon: float = _HIT_EPSILON,
    out_steps: Any | None = None,
) -> None:
    """
    Top-level API for TopoNav Sphere Tracing.
    Strict CUDA-only path. CPU fallback is intentionally disabled.
    """
    if not HAS_CUDA_BACKEND:
        raise RuntimeError(
            "torch_sdf_backend is not available. Build/install the CUDA extension in torch-sdf before running TopoNav."
        )
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is not available. TopoNav requires CUDA and does not support CPU fallback.")
    _validate_cast_rays_inputs(
        dag_tensor, origins, dirs, out_distances, out_semantics,
        skip_direction_validation=skip_direction_validation,
    )
    _validate_runtime_parameters(
        max_steps=max_steps, max_distance=max_distance, bbox_min=bbox_min, bbox_max=bbox_max,
        resolution=resolution,
    )
    backend = torch_sdf_backend
    if backend is None:
        raise RuntimeError("torch_sdf_backend import unexpectedly resolved to None.")
    if hit_epsilon == _HIT_EPSILON and out_steps is None:
        backend.cast_rays(
            dag_tensor, origins, dirs, out_distances, out_semantics, max_steps, max_distance,
            bbox_min, bbox_max, resolution, skip_direction_validation,
        )
    else:
        backend.cast_rays_ex(
            dag_tensor, origins, dirs, out_distances, out_semantics, max_steps, max_distance,
            bbox_min, bbox_max, resolution, skip_direction_validation, hit_epsilon, out_steps,
        )
