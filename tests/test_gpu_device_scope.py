"""Every C-ABI call leaves the caller's current CUDA device as it found it.

torch keeps its current device in the CUDA runtime's per-thread state, so a
library call that switched devices and did not switch back would move the
caller's later allocations and launches to the pool's GPU.  The reference
never changes the device (bindings.cpp:43-110 launches on the tensors'
device under the caller's current one).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from navi_b200 import _native, scenes, tracer, workloads
from tests.gpu_util import eager_world_rays

pytestmark = pytest.mark.gpu


def _all_calls(device: torch.device) -> None:
    """Pool creation, explicit, fan, observed-fan and allocation-free casts, pool and table release."""
    cfg = scenes.CONFIGS[1]
    cs = workloads.compiled_scene(1)
    pb = workloads.poses_for(1, [cs])
    fan = torch.from_numpy(workloads.fan_for(1)).to(device)
    poses = tracer.make_poses(torch.from_numpy(pb.position).to(device), torch.from_numpy(pb.yaw).to(device),
                              torch.from_numpy(pb.pitch).to(device))
    o, v = eager_world_rays(fan, poses)
    a, r = poses.shape[0], fan.shape[0]
    n = a * r
    pool = tracer.NodePool.from_words(cs.words, device)
    pool_t = tracer.NodePool.from_tensor(torch.from_numpy(cs.words.view(np.int64)).to(device))
    d = torch.empty(n, dtype=torch.float32, device=device)
    s = torch.empty(n, dtype=torch.int32, device=device)
    k = torch.empty(n, dtype=torch.int32, device=device)
    tracer.cast_rays_ex(pool, o, v, d, s, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                        bbox_min=cs.bbox_min, bbox_max=cs.bbox_max, hit_epsilon=cs.hit_epsilon, out_steps=k)
    sset = tracer.SceneSet([pool, pool_t], [cs.bbox_min] * 2, [cs.bbox_max] * 2, [cs.hit_epsilon] * 2)
    tracer.cast_fan(sset, poses, fan, d, s, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                    use_pitch=True, out_steps=k)
    obs = torch.empty((a, 3, cfg.azimuth_bins, cfg.elevation_bins), dtype=torch.float32, device=device)
    st = torch.empty((a, 5), dtype=torch.float32, device=device)
    tracer.cast_fan_observe(sset, poses, fan, cfg.azimuth_bins, cfg.elevation_bins, d, s, obs, st,
                            max_steps=cfg.max_steps, max_distance=cfg.max_distance, use_pitch=True)
    lib = _native.tsdf_lib()
    bmin = (ctypes.c_float * 3)(*cs.bbox_min)
    bmax = (ctypes.c_float * 3)(*cs.bbox_max)
    stream = torch.cuda.current_stream(device).cuda_stream
    _native.check(lib.tsdf_cast_noalloc(pool.handle, ctypes.c_void_p(o.data_ptr()), ctypes.c_void_p(v.data_ptr()), n,
                                        ctypes.c_void_p(d.data_ptr()), ctypes.c_void_p(s.data_ptr()),
                                        ctypes.c_void_p(k.data_ptr()), cfg.max_steps, cfg.max_distance, bmin, bmax,
                                        cs.hit_epsilon, ctypes.c_void_p(stream)), "tsdf_cast_noalloc")
    torch.cuda.synchronize(device)
    sset.close()
    pool_t.close()
    pool.close()


def test_calls_on_the_current_device_keep_it_current():
    torch.cuda.set_device(0)
    _all_calls(torch.device("cuda", 0))
    assert torch.cuda.current_device() == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_calls_on_another_device_keep_the_callers_device_current():
    """Pools, tables and casts on GPU 1 while GPU 0 is current: GPU 0 stays current."""
    torch.cuda.set_device(0)
    _all_calls(torch.device("cuda", 1))
    assert torch.cuda.current_device() == 0
    torch.cuda.set_device(1)
    _all_calls(torch.device("cuda", 0))
    assert torch.cuda.current_device() == 1
    torch.cuda.set_device(0)
