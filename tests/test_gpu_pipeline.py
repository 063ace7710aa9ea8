"""Casts with host inputs and outputs (navi_b200.pipeline) equal the device casts bit for bit.

The pipelined forms split a cast into chunks whose uploads, launches and
downloads overlap on side streams; the traced values must not change, every
output must be written, and the caller's stream must be ordered after all of it.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import torch_sdf
from navi_b200 import pipeline, scenes, tracer, workloads
from tests.gpu_util import assert_bits_equal, assert_equal, dev, eager_world_rays

pytestmark = pytest.mark.gpu


def _setup(config: int, scene_count: int | None = None, actors: int | None = None):
    cfg = scenes.CONFIGS[config]
    n_sc = scene_count or cfg.n_scenes
    scene_list = [workloads.compiled_scene(config, s, resolution=128 if config != 1 else None) for s in range(n_sc)]
    pb = workloads.poses_for(config, scene_list, actors=actors)
    d = dev()
    fan = torch.from_numpy(workloads.fan_for(config)).to(d)
    poses = tracer.make_poses(torch.from_numpy(pb.position).to(d), torch.from_numpy(pb.yaw).to(d),
                              torch.from_numpy(pb.pitch).to(d), torch.from_numpy(pb.scene).to(d))
    pools = [tracer.NodePool.from_words(cs.words, d) for cs in scene_list]
    sset = tracer.SceneSet(pools, [c.bbox_min for c in scene_list], [c.bbox_max for c in scene_list],
                           [c.hit_epsilon for c in scene_list])
    return cfg, scene_list, pb, fan, poses, pools, sset


@pytest.mark.parametrize("chunks", [1, 3, 4, 1000])
def test_cast_rays_host_equals_device_cast(chunks):
    cfg, scene_list, pb, fan, poses, pools, _ = _setup(1)
    cs = scene_list[0]
    o, v = eager_world_rays(fan, poses)
    n = o.shape[0] * o.shape[1]
    d = dev()
    want_d = torch.empty(n, dtype=torch.float32, device=d)
    want_s = torch.empty(n, dtype=torch.int32, device=d)
    want_k = torch.empty(n, dtype=torch.int32, device=d)
    tracer.cast_rays_ex(pools[0], o, v, want_d, want_s, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                        bbox_min=cs.bbox_min, bbox_max=cs.bbox_max, hit_epsilon=cs.hit_epsilon, out_steps=want_k)
    h_o = o.cpu().pin_memory()
    h_v = v.cpu().pin_memory()
    h_d = torch.full((n,), -7.0, dtype=torch.float32).pin_memory()
    h_s = torch.full((n,), -7, dtype=torch.int32).pin_memory()
    h_k = torch.full((n,), -7, dtype=torch.int32).pin_memory()
    pipeline.cast_rays_host(pools[0], h_o, h_v, h_d, h_s, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                            bbox_min=cs.bbox_min, bbox_max=cs.bbox_max, hit_epsilon=cs.hit_epsilon, out_steps=h_k,
                            chunks=chunks)
    torch.cuda.current_stream(d).synchronize()
    assert_bits_equal(h_d.numpy(), want_d.cpu().numpy(), "dist")
    assert_equal(h_s.numpy(), want_s.cpu().numpy(), "sem")
    assert_equal(h_k.numpy(), want_k.cpu().numpy(), "steps")


@pytest.mark.parametrize("chunks", [1, 4, 7])
def test_cast_fan_host_equals_device_cast_on_a_scene_table(chunks):
    cfg, scene_list, pb, fan, poses, pools, sset = _setup(3, scene_count=3, actors=40)
    a, r = poses.shape[0], fan.shape[0]
    d = dev()
    want_d = torch.empty(a * r, dtype=torch.float32, device=d)
    want_s = torch.empty(a * r, dtype=torch.int32, device=d)
    want_k = torch.empty(a * r, dtype=torch.int32, device=d)
    tracer.cast_fan(sset, poses, fan, want_d, want_s, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                    out_steps=want_k)
    h_p = poses.cpu().pin_memory()
    h_d = torch.full((a * r,), -7.0, dtype=torch.float32).pin_memory()
    h_s = torch.full((a * r,), -7, dtype=torch.int32).pin_memory()
    h_k = torch.full((a * r,), -7, dtype=torch.int32).pin_memory()
    pipeline.cast_fan_host(sset, h_p, fan, h_d, h_s, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                           out_steps=h_k, chunks=chunks)
    torch.cuda.current_stream(d).synchronize()
    assert_bits_equal(h_d.numpy(), want_d.cpu().numpy(), "dist")
    assert_equal(h_s.numpy(), want_s.cpu().numpy(), "sem")
    assert_equal(h_k.numpy(), want_k.cpu().numpy(), "steps")


def test_run_chunks_through_the_drop_in_call_orders_the_current_stream():
    """Scene groups through torch_sdf.cast_rays, pipelined; work queued on the current stream
    afterwards (a device copy of the host results' source buffers) sees finished outputs."""
    cfg, scene_list, pb, fan, poses, pools, sset = _setup(3, scene_count=3, actors=60)
    d = dev()
    order = np.argsort(pb.scene, kind="stable")
    idx = torch.from_numpy(order).to(d)
    o, v = eager_world_rays(fan, poses.index_select(0, idx), pitch=False)
    a, r = o.shape[0], o.shape[1]
    h_o, h_v = o.cpu().pin_memory(), v.cpu().pin_memory()
    g_o, g_v = torch.empty_like(o), torch.empty_like(v)
    g_d = torch.full((a, r), -7.0, dtype=torch.float32, device=d)
    g_s = torch.full((a, r), -7, dtype=torch.int32, device=d)
    h_d = torch.empty((a, r), dtype=torch.float32).pin_memory()
    h_s = torch.empty((a, r), dtype=torch.int32).pin_memory()
    dags = [torch.from_numpy(cs.words.view(np.int64)).to(d) for cs in scene_list]
    sc_sorted = pb.scene[order]
    chunks = []
    for s, cs in enumerate(scene_list):
        rows = np.nonzero(sc_sorted == s)[0]
        lo, hi = int(rows[0]), int(rows[-1]) + 1

        def run(s=s, lo=lo, hi=hi, cs=cs):
            torch_sdf.cast_rays(dags[s], g_o[lo:hi], g_v[lo:hi], g_d[lo:hi], g_s[lo:hi], cfg.max_steps,
                                cfg.max_distance, cs.bbox_min, cs.bbox_max, 128, skip_direction_validation=True,
                                hit_epsilon=cs.hit_epsilon)
        chunks.append(pipeline.Chunk(run, [(g_o[lo:hi], h_o[lo:hi]), (g_v[lo:hi], h_v[lo:hi])],
                                     [(h_d[lo:hi], g_d[lo:hi]), (h_s[lo:hi], g_s[lo:hi])]))
    pipeline.run_chunks(chunks, d)
    after = g_d.clone()  # queued on the current stream after run_chunks
    torch.cuda.current_stream(d).synchronize()
    want_d = torch.empty(a * r, dtype=torch.float32, device=d)
    want_s = torch.empty(a * r, dtype=torch.int32, device=d)
    tracer.cast_fan(sset, poses.index_select(0, idx), fan, want_d, want_s, max_steps=cfg.max_steps,
                    max_distance=cfg.max_distance)
    torch.cuda.synchronize()
    assert_bits_equal(h_d.numpy(), want_d.cpu().numpy(), "host dist")
    assert_equal(h_s.numpy(), want_s.cpu().numpy(), "host sem")
    assert_bits_equal(after.cpu().numpy(), want_d.cpu().numpy(), "device dist seen by the current stream")
