"""The C-ABI library loads and exports every entry point include/tsdf.h declares (no GPU needed)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from navi_b200 import _native

ROOT = Path(__file__).resolve().parents[1]


def _declared(header: Path) -> list[str]:
    text = header.read_text()
    return re.findall(r"^TSDF_API\s+[\w\s\*]+?\b(tsdf_\w+)\s*\(", text, flags=re.M)


def test_header_declares_the_cast_entry_points():
    names = _declared(ROOT / "include" / "tsdf.h")
    for required in ("tsdf_cast", "tsdf_cast_fan", "tsdf_pool_create", "tsdf_pool_create_from_device",
                     "tsdf_pool_destroy", "tsdf_last_error", "tsdf_version"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = _native.tsdf_lib()
    names = _declared(ROOT / "include" / "tsdf.h")
    assert names
    for name in names:
        assert hasattr(lib, name), name
    assert set(_native.TSDF_SIGNATURES) == set(names)


def test_version_and_workspace_query():
    lib = _native.tsdf_lib()
    assert lib.tsdf_version() == 1
    assert lib.tsdf_workspace_bytes(0) >= 8
    # counter block + 128 bucket words + 4-byte order + 1-byte key per ray, rounded to 16
    assert lib.tsdf_workspace_bytes(1000) == 256 + 512 + 4000 + 1008
    assert lib.tsdf_fan_workspace_bytes(None, 10, 0) == 256
    # scenes = NULL: the larger of one scene's claim order and a scene table's (actor order
    # rounded to 16, 1 KB of ranges and counters, 32 KB of per-scene bucket counts, the
    # 4-byte order and 1-byte key of every ray)
    assert lib.tsdf_fan_workspace_bytes(None, 10, 100) == 256 + 48 + 1024 + 32768 + 4000 + 1008
    assert lib.tsdf_fan_workspace_bytes(None, 4096, 1) == 256 + 16384 + 1024 + 32768 + 4 * 4096 + 4096
    assert lib.tsdf_observe_workspace_bytes(None, 10, 100) == lib.tsdf_fan_workspace_bytes(None, 10, 100)


def test_option_knobs_validate_their_range():
    lib = _native.tsdf_lib()
    old = ctypes.c_int64()
    assert lib.tsdf_set_option(b"chunk", 64, ctypes.byref(old)) == 0
    assert lib.tsdf_set_option(b"chunk", old.value, None) == 0
    assert lib.tsdf_set_option(b"chunk", -1, None) != 0
    assert b"chunk" in lib.tsdf_last_error()
    assert lib.tsdf_set_option(b"chunk", 1025, None) != 0
    assert old.value == 0  # the default: chosen per launch
    assert lib.tsdf_set_option(b"order", 2, None) != 0
    assert b"order" in lib.tsdf_last_error()
    assert lib.tsdf_set_option(b"per_scene", 2, None) != 0
    assert b"per_scene" in lib.tsdf_last_error()
    assert lib.tsdf_set_option(b"no_such_knob", 1, None) != 0
    assert b"unknown option" in lib.tsdf_last_error()


def test_null_arguments_are_rejected_before_any_cuda_call():
    lib = _native.tsdf_lib()
    assert lib.tsdf_pool_create(None, 0, 0, 0, None) == -1
    assert lib.tsdf_cast(None, None, None, 0, None, None, None, 1, ctypes.c_float(1.0), None, None,
                         ctypes.c_float(0.01), None, None) == -1
    assert b"pool must not be null" in lib.tsdf_last_error()


def _declared_gmdag() -> list[str]:
    text = (ROOT / "include" / "gmdag.h").read_text()
    return re.findall(r"^GMDAG_API\s+[\w\s\*]+?\b(gmdag_\w+)\s*\(", text, flags=re.M)


def test_scene_compiler_library_loads():
    lib = _native.gmdag_lib()
    for name in _native.GMDAG_SIGNATURES:
        assert hasattr(lib, name)


def test_scene_compiler_libraries_export_every_declared_symbol():
    names = _declared_gmdag()
    host = [n for n in names if not n.startswith("gmdag_gpu_")]
    dev = [n for n in names if n.startswith("gmdag_gpu_")]
    assert host and dev
    assert set(_native.GMDAG_SIGNATURES) == set(host)
    assert set(_native.GMDAG_GPU_SIGNATURES) == set(dev)
    lib = _native.gmdag_lib()
    for name in host:
        assert hasattr(lib, name), name
    gpu = _native.gmdag_gpu_lib()  # loads without a GPU: no CUDA call at load time
    for name in dev:
        assert hasattr(gpu, name), name


def test_device_compiler_validates_before_any_cuda_call():
    import ctypes

    lib = _native.gmdag_gpu_lib()
    out = ctypes.c_void_p()
    assert lib.gmdag_gpu_compile_mesh(None, 0, None, 0, 64, 0, ctypes.byref(out)) == -1
    assert b"at least one triangle" in lib.gmdag_gpu_last_error()
    v = (ctypes.c_float * 9)(0, 0, 0, 1, 0, 0, 0, 1, 0)
    i = (ctypes.c_uint32 * 3)(0, 1, 2)
    assert lib.gmdag_gpu_compile_mesh(v, 3, i, 1, 48, 0, ctypes.byref(out)) == -1
    assert b"power of two" in lib.gmdag_gpu_last_error()


@pytest.mark.parametrize("path", [_native.TSDF_PATH])
def test_library_is_built_for_sm100a_only(path):
    # the fatbin records its targets; cuobjdump is not used on purpose (no disassembly):
    # the build command is the evidence — check the build script pins the arch.
    src = (ROOT / "navi_b200" / "build.py").read_text()
    assert "arch=compute_100a,code=sm_100a" in src
    assert path.exists()
