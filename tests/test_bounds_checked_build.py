"""The bounds-checked build (libnavi_tsdf_debug.so, -DTSDF_BOUNDS_CHECK): every node-pool,
leaf-table, stack and actor-order index the kernels use is checked, a failed check sets a
device error word that the call reports.  It stands in for compute-sanitizer runs.

CPU: the library exports the same C ABI.  GPU: in a child process with $NAVI_TSDF_DEBUG=1
(the library is chosen when navi_b200 loads it), explicit-ray, fan and multi-scene casts
and random DAGs run with no check failing and the oracle's bits.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import sys
from pathlib import Path

import pytest

from navi_b200 import _native

ROOT = Path(__file__).resolve().parents[1]


def test_debug_library_exports_the_same_abi():
    path = _native.LIB_DIR / "libnavi_tsdf_debug.so"
    assert path.exists()
    lib = ctypes.CDLL(str(path))
    for name in _native.TSDF_SIGNATURES:
        assert hasattr(lib, name), name


CHILD = r'''
import numpy as np, torch
from navi_b200 import _native, tracer, workloads
assert _native.TSDF_PATH.name == "libnavi_tsdf_debug.so"
from oracle import oracle as O
from tests.dag_fuzz import random_dag, random_rays
from tests.gpu_util import eager_world_rays
dev = torch.device("cuda", 0)

def same(a, b):
    assert np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))

cs = workloads.compiled_scene(1)
pb = workloads.poses_for(1, [cs])
fan = torch.from_numpy(workloads.fan_for(1)).to(dev)
poses = tracer.make_poses(torch.from_numpy(pb.position).to(dev), torch.from_numpy(pb.yaw).to(dev),
                          torch.from_numpy(pb.pitch).to(dev))
o, v = eager_world_rays(fan, poses, pitch=True)
ref = O.trace(cs.words, cs.bbox_min, cs.bbox_max, o.cpu().numpy(), v.cpu().numpy(), max_steps=128,
              max_distance=20.0, hit_epsilon=cs.hit_epsilon)
for descent in (0, 1):
    tracer.set_option("descent", descent)
    pool = tracer.NodePool.from_words(cs.words, dev)
    n = o.shape[0] * o.shape[1]
    d = torch.empty(n, device=dev); s = torch.empty(n, dtype=torch.int32, device=dev)
    tracer.cast_rays_ex(pool, o, v, d, s, max_steps=128, max_distance=20.0, bbox_min=cs.bbox_min,
                        bbox_max=cs.bbox_max, hit_epsilon=cs.hit_epsilon)
    same(d.cpu().numpy(), ref["dist"])
    sset = tracer.SceneSet([pool], [cs.bbox_min], [cs.bbox_max], [cs.hit_epsilon])
    tracer.cast_fan(sset, poses, fan, d, s, max_steps=128, max_distance=20.0, use_pitch=True)
    same(d.cpu().numpy(), ref["dist"])
    multi = [workloads.compiled_scene(3, k, resolution=64) for k in range(3)]
    p3 = workloads.poses_for(3, multi, actors=12)
    poses3 = tracer.make_poses(torch.from_numpy(p3.position).to(dev), torch.from_numpy(p3.yaw).to(dev), None,
                               torch.from_numpy(p3.scene).to(dev))
    ss3 = tracer.SceneSet([tracer.NodePool.from_words(c.words, dev) for c in multi], [c.bbox_min for c in multi],
                          [c.bbox_max for c in multi], [c.hit_epsilon for c in multi])
    n3 = 12 * fan.shape[0]
    d3 = torch.empty(n3, device=dev); s3 = torch.empty(n3, dtype=torch.int32, device=dev)
    tracer.cast_fan(ss3, poses3, fan, d3, s3, max_steps=128, max_distance=30.0)
    rng = np.random.default_rng(descent)
    for depth in (3, 5, 8):
        w = random_dag(rng, depth)
        oo, dd = random_rays(rng, 2000, [-1, -1, -1], [1, 1, 1], depth)
        r = O.trace(w, [-1, -1, -1], [1, 1, 1], oo, dd, max_steps=64, max_distance=5.0, hit_epsilon=0.01)
        p = tracer.NodePool.from_words(w, dev)
        dz = torch.empty(2000, device=dev); sz = torch.empty(2000, dtype=torch.int32, device=dev)
        tracer.cast_rays_ex(p, torch.from_numpy(oo).to(dev), torch.from_numpy(dd).to(dev), dz, sz, max_steps=64,
                            max_distance=5.0, bbox_min=[-1, -1, -1], bbox_max=[1, 1, 1], hit_epsilon=0.01)
        same(dz.cpu().numpy(), r["dist"])
print("bounds-checked build ok")
'''


@pytest.mark.gpu
def test_bounds_checked_build_runs_clean():
    env = dict(os.environ, NAVI_TSDF_DEBUG="1", PYTHONPATH=str(ROOT))
    proc = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=600)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-4000:]
    assert "bounds-checked build ok" in proc.stdout
