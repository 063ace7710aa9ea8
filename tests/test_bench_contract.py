"""bench.py's reference arm: its JSON line, and that it maps none of this repository's libraries.

The reference arm must run the reference's own code path (the oracle restating
kernel.cu on the host cores, scenes from the reference compiler), so the
process may load libraries under oracle/ only.  Runs on the CPU (the reference
CUDA kernel leg reports null without a GPU).
"""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

_PROBE = r"""
import contextlib, io, json, sys
sys.argv = ["bench.py", "--impl", "reference", "--config", "1", "--steps", "1", "--warmup", "0"]
sys.path.insert(0, ".")
import bench
buf = io.StringIO()
with contextlib.redirect_stdout(buf):
    bench.main()
maps = open("/proc/self/maps").read().splitlines()
libs = sorted({l.split()[-1] for l in maps if ".so" in l})
print(json.dumps({"line": buf.getvalue().strip(), "libs": libs}))
"""


def test_reference_arm_line_and_libraries():
    from oracle import build as OB

    if not (OB.REF_OUT / "ref_voxel_dag").exists():
        pytest.skip("reference compiler not built here")
    r = subprocess.run([sys.executable, "-c", _PROBE], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    line = json.loads(out["line"])
    assert line["impl"] == "reference"
    assert line["config"]["workload"] == "c1_room10_128"
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "rays/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    repo_libs = [p for p in out["libs"] if p.startswith(str(ROOT))]
    assert repo_libs, "the oracle library should be mapped"
    assert all(p.startswith(str(ROOT / "oracle")) for p in repo_libs), repo_libs


def test_both_arms_print_the_same_config():
    sys.path.insert(0, str(ROOT))
    import bench
    from navi_b200 import scenes

    class A:
        pose_sets = 4

    for c in (1, 2, 3, 4, 5):
        cfg = scenes.CONFIGS[c]
        for world in (1, 2, 8):
            actors = bench._actors_per_rank(cfg, world, 0)
            d = bench._config_dict(A, cfg, world, actors)
            assert d["rays_per_step_per_rank"] == actors * cfg.azimuth_bins * cfg.elevation_bins
            if c == 5:
                assert d["actors_total"] == 32768 and actors == 32768 // world
            else:
                assert actors == cfg.actors
