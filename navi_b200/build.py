"""Build the native libraries in-tree (navi_b200/_lib/).

    python -m navi_b200.build

- libnavi_tsdf.so  : the sm_100a trace kernels and the C ABI of include/tsdf.h
                     (nvcc, -gencode arch=compute_100a,code=sm_100a, static cudart)
- libnavi_tsdf_debug.so : the same with every kernel index bounds-checked
                     (-DTSDF_BOUNDS_CHECK; selected by $NAVI_TSDF_DEBUG=1)
- libnavi_gmdag.so : the host scene compiler (g++, OpenMP, -ffp-contract=off so
                     that its float arithmetic matches the reference compiler's)
- libnavi_gmdag_gpu.so : the device scene compiler (nvcc sm_100a, -fmad=false,
                     IEEE division / sqrt; same words as libnavi_gmdag.so)
- libnavi_probe.so : the L2 read-bandwidth probe of the benchmark's roofline

Both are rebuilt only when a source is newer than the library.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "_lib"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libnavi_tsdf.so")


def host_cxx() -> str:
    """A C++ compiler with OpenMP (the system g++ ships libgomp)."""
    for cand in ("/usr/bin/g++", os.environ.get("CXX"), shutil.which("g++")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("no C++ compiler found")


def host_cc() -> str:
    for cand in ("/usr/bin/gcc", os.environ.get("CC"), shutil.which("gcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("no C compiler found")


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build command failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def build_tsdf(force: bool = False, bounds_check: bool = False) -> Path:
    """libnavi_tsdf.so, or with bounds_check libnavi_tsdf_debug.so: the same library with
    every pool, leaf-table, stack and actor-order index checked in the kernels (a device
    error word, reported by the call) — the stand-in for compute-sanitizer runs."""
    out = LIB / ("libnavi_tsdf_debug.so" if bounds_check else "libnavi_tsdf.so")
    srcs = [CSRC / "tsdf_trace.cu", CSRC / "tsdf_pool.cpp", CSRC / "gmdag_io.cpp"]
    deps = srcs + [CSRC / "tsdf_internal.h", CSRC / "exit_quotient.cuh", CSRC / "gmdag_io.h", INCLUDE / "tsdf.h", INCLUDE / "gmdag.h"]
    if force or _stale(out, deps):
        LIB.mkdir(parents=True, exist_ok=True)
        tmp = out.with_suffix(".so.tmp")
        _run([
            _nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
            "-Xcompiler", "-fvisibility=hidden", "-Xlinker", "--exclude-libs,ALL", "-diag-suppress", "186",
            *(["-DTSDF_BOUNDS_CHECK"] if bounds_check else []),
            f"-I{INCLUDE}", *map(str, srcs), "-o", str(tmp),
        ])
        tmp.replace(out)
    return out


def build_gmdag(force: bool = False) -> Path:
    out = LIB / "libnavi_gmdag.so"
    srcs = [CSRC / "gmdag_compiler.cpp", CSRC / "gmdag_io.cpp"]
    if force or _stale(out, srcs + [CSRC / "gmdag_math.h", CSRC / "gmdag_io.h", INCLUDE / "gmdag.h"]):
        LIB.mkdir(parents=True, exist_ok=True)
        tmp = out.with_suffix(".so.tmp")
        _run([
            host_cxx(), "-O2", "-std=c++17", "-fPIC", "-shared", "-fopenmp",
            "-ffp-contract=off", "-fno-fast-math", f"-I{INCLUDE}", *map(str, srcs), "-o", str(tmp),
        ])
        tmp.replace(out)
    return out


def build_gmdag_gpu(force: bool = False) -> Path:
    """The device scene compiler: IEEE float semantics on both sides (no FMA
    contraction, correctly rounded division and sqrt, denormals kept), so that its
    values equal the host compiler's."""
    out = LIB / "libnavi_gmdag_gpu.so"
    src = CSRC / "gmdag_gpu.cu"
    if force or _stale(out, [src, CSRC / "gmdag_math.h", INCLUDE / "gmdag.h"]):
        LIB.mkdir(parents=True, exist_ok=True)
        tmp = out.with_suffix(".so.tmp")
        _run([
            _nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
            "-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
            "-Xcompiler", "-ffp-contract=off", "-Xcompiler", "-fvisibility=hidden",
            "-Xlinker", "--exclude-libs,ALL", f"-I{INCLUDE}", str(src), "-o", str(tmp),
        ])
        tmp.replace(out)
    return out


def build_probe(force: bool = False) -> Path:
    """libnavi_probe.so: the L2 read-bandwidth probe bench.py reports the L2 roofline against,
    and the check of the trace kernel's exit quotient against the IEEE division."""
    out = LIB / "libnavi_probe.so"
    srcs = [CSRC / "peak_probe.cu", CSRC / "quotient_check.cu"]
    if force or _stale(out, srcs + [CSRC / "exit_quotient.cuh"]):
        LIB.mkdir(parents=True, exist_ok=True)
        tmp = out.with_suffix(".so.tmp")
        _run([_nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
              *map(str, srcs), "-o", str(tmp)])
        tmp.replace(out)
    return out


def build_all(force: bool = False) -> list[Path]:
    return [build_tsdf(force), build_tsdf(force, bounds_check=True), build_gmdag(force), build_gmdag_gpu(force),
            build_probe(force)]


if __name__ == "__main__":
    for p in build_all(force="--force" in sys.argv):
        print(p)
