"""Build the parity checkers (TEST INFRASTRUCTURE ONLY).

    python oracle/build.py          # oracle/_build/liboracle.so (always)
                                    # oracle/_ref/libref_trace*.so (when the reference tree exists)

- liboracle.so: the C restatement of the reference trace (trace_oracle.c),
  gcc -O2 -fopenmp -ffp-contract=off.
- libref_trace.so: the reference's own kernel.cu, unmodified, compiled for
  sm_100a straight from the reference tree with the reference's nvcc flags
  (-O3 -lineinfo, projects/torch-sdf/setup.py:44) plus ref_shim.cu.
- ref_voxel_dag: the reference scene compiler (projects/voxel-dag/src/compiler.cpp,
  unmodified) built with g++ against oracle/assimp_standin/ (an OBJ-only
  stand-in for the three Assimp headers it includes; Assimp is not available).
- libref_trace_eps.so: the same kernel with kHitEpsilon turned into a run-time
  __constant__ (ref_shim_eps.cu says how).  The copied sources live in a
  scratch folder under oracle/_ref/ only while nvcc runs.

The reference tree is read from $NAVI_REFERENCE_ROOT (default: a directory named
`reference` beside the repository); without it the prebuilt oracle/_ref files are used
as they are.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF_OUT = HERE / "_ref"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
EPS_LINE = "constexpr float kHitEpsilon = 0.01f;"
EPS_NEW = "__constant__ float kHitEpsilon = 0.01f;"


def _reference_root() -> Path:
    return Path(os.environ.get("NAVI_REFERENCE_ROOT", HERE.parent.parent / "reference"))


def _ref_src() -> Path:
    return _reference_root() / "projects" / "torch-sdf" / "cpp_src"


def _tool(*cands: str | None) -> str:
    for c in cands:
        if c and Path(c).exists():
            return c
    raise RuntimeError(f"none of {cands} exists")


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def _stale(target: Path, deps: list[Path]) -> bool:
    return not target.exists() or any(d.stat().st_mtime > target.stat().st_mtime for d in deps)


def build_oracle(force: bool = False) -> Path:
    out = BUILD / "liboracle.so"
    src = HERE / "trace_oracle.c"
    if force or _stale(out, [src]):
        BUILD.mkdir(parents=True, exist_ok=True)
        cc = _tool("/usr/bin/gcc", os.environ.get("CC"), shutil.which("gcc"))
        _run([cc, "-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
              "-fno-fast-math", str(src), "-o", str(out), "-lm"])
    return out


def build_reference(force: bool = False) -> list[Path]:
    src = _ref_src()
    if not (src / "kernel.cu").exists():
        return []
    nvcc = _tool(os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc"))
    REF_OUT.mkdir(parents=True, exist_ok=True)
    outs = []
    plain = REF_OUT / "libref_trace.so"
    if force or _stale(plain, [src / "kernel.cu", src / "kernel.cuh", HERE / "ref_shim.cu"]):
        _run([nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
              f"-I{src}", str(src / "kernel.cu"), str(HERE / "ref_shim.cu"), "-o", str(plain)])
    outs.append(plain)
    eps = REF_OUT / "libref_trace_eps.so"
    if force or _stale(eps, [src / "kernel.cu", src / "kernel.cuh", HERE / "ref_shim_eps.cu"]):
        scratch = REF_OUT / "eps_src"
        scratch.mkdir(parents=True, exist_ok=True)
        try:
            shutil.copy(src / "kernel.cu", scratch / "kernel.cu")
            header = (src / "kernel.cuh").read_text()
            if header.count(EPS_LINE) != 1:
                raise RuntimeError("kernel.cuh no longer holds the expected kHitEpsilon line")
            (scratch / "kernel.cuh").write_text(header.replace(EPS_LINE, EPS_NEW))
            _run([nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
                  f"-I{scratch}", str(HERE / "ref_shim_eps.cu"), "-o", str(eps)])
        finally:
            shutil.rmtree(scratch, ignore_errors=True)
    outs.append(eps)
    return outs


def build_reference_compiler(force: bool = False) -> list[Path]:
    """The reference voxel-dag compiler (compiler.cpp, unmodified) + the Assimp stand-in headers."""
    src = _reference_root() / "projects" / "voxel-dag" / "src"
    if not (src / "compiler.cpp").exists():
        return []
    out = REF_OUT / "ref_voxel_dag"
    standin = HERE / "assimp_standin"
    deps = [src / "compiler.cpp", src / "compiler.hpp", HERE / "ref_compile_main.cpp",
            *sorted((standin / "assimp").glob("*"))]
    if force or _stale(out, deps):
        REF_OUT.mkdir(parents=True, exist_ok=True)
        cxx = _tool("/usr/bin/g++", os.environ.get("CXX"), shutil.which("g++"))
        # default flags of a CMake Release build of the reference (no -ffast-math, no FMA target)
        _run([cxx, "-O2", "-std=c++17", f"-I{standin}", f"-I{src}", str(src / "compiler.cpp"),
              str(HERE / "ref_compile_main.cpp"), "-o", str(out)])
    return [out]


def build_all(force: bool = False) -> list[Path]:
    return [build_oracle(force), *build_reference(force), *build_reference_compiler(force)]


if __name__ == "__main__":
    for p in build_all(force="--force" in sys.argv):
        print(p)
