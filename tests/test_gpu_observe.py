"""The fused observation epilogue vs the reference's post-processing run by torch on the
same device (oracle/postprocess_ref.py restates sdfdag_backend.py:366-473, :1518-1525).

Tolerance: none — observation channels and per-actor statistics are compared bit for bit
(NaN compared as NaN).  Distances/semantics/steps of the observing cast must also equal
those of the plain cast.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from navi_b200 import scenes, tracer, workloads
from oracle import postprocess_ref
from tests.gpu_util import dev
from tests.kat_cases import internal_word, leaf_word

pytestmark = pytest.mark.gpu


def _bits_equal(a: torch.Tensor, b: torch.Tensor, what: str) -> None:
    x = a.detach().cpu().numpy().astype(np.float32).reshape(-1)
    y = b.detach().cpu().numpy().astype(np.float32).reshape(-1)
    nan = np.isnan(x) & np.isnan(y)
    bad = np.nonzero((x.view(np.uint32) != y.view(np.uint32)) & ~nan)[0]
    assert bad.size == 0, f"{what}: {bad.size} of {x.size} differ; first {bad[:5]}: {x[bad[:5]]} vs {y[bad[:5]]}"


def _run(sset, poses, fan, az, el, *, max_steps, max_distance, band, prox, use_pitch):
    d = poses.device
    a, r = poses.shape[0], fan.shape[0]
    od = torch.empty(a * r, device=d)
    os_ = torch.empty(a * r, dtype=torch.int32, device=d)
    ok = torch.empty(a * r, dtype=torch.int32, device=d)
    obs = torch.full((a, 3, az, el), -5.0, device=d)
    st = torch.full((a, 5), -5.0, device=d)
    tracer.cast_fan_observe(sset, poses, fan, az, el, od, os_, obs, st, max_steps=max_steps, max_distance=max_distance,
                            structure_band_min=band[0], structure_band_max=band[1], proximity_threshold=prox,
                            use_pitch=use_pitch, out_steps=ok)
    pd = torch.empty_like(od)
    ps = torch.empty_like(os_)
    pk = torch.empty_like(ok)
    tracer.cast_fan(sset, poses, fan, pd, ps, max_steps=max_steps, max_distance=max_distance, use_pitch=use_pitch,
                    out_steps=pk)
    torch.cuda.synchronize()
    _bits_equal(od, pd, "distances of the observing cast")
    assert torch.equal(os_, ps) and torch.equal(ok, pk)
    ref_obs, ref_st = postprocess_ref.postprocess(
        od.view(a, r), os_.view(a, r), az_bins=az, el_bins=el, max_distance=max_distance,
        structure_band_min_distance=band[0], structure_band_max_distance=band[1],
        proximity_distance_threshold=prox)
    _bits_equal(obs, ref_obs, "observation")
    _bits_equal(st, ref_st, "actor statistics")
    return od, st


@pytest.mark.parametrize("band,prox", [((1.5, 13.2), 2.0), ((1.5, 1.0), 0.0), ((0.5, 30.0), 25.0)])
def test_observation_matches_reference_postprocess_config1(band, prox):
    cfg = scenes.CONFIGS[1]
    cs = workloads.compiled_scene(1)
    pb = workloads.poses_for(1, [cs])
    d = dev()
    fan = torch.from_numpy(workloads.fan_for(1)).to(d)
    poses = tracer.make_poses(torch.from_numpy(pb.position).to(d), torch.from_numpy(pb.yaw).to(d),
                              torch.from_numpy(pb.pitch).to(d))
    sset = tracer.SceneSet([tracer.NodePool.from_words(cs.words, d)], [cs.bbox_min], [cs.bbox_max], [cs.hit_epsilon])
    _run(sset, poses, fan, cfg.azimuth_bins, cfg.elevation_bins, max_steps=cfg.max_steps,
         max_distance=cfg.max_distance, band=band, prox=prox, use_pitch=True)


def test_observation_matches_reference_postprocess_config2_and_multiscene():
    cfg = scenes.CONFIGS[2]
    cs = workloads.compiled_scene(2)
    pb = workloads.poses_for(2, [cs], actors=16)
    d = dev()
    fan = torch.from_numpy(workloads.fan_for(2)).to(d)
    poses = tracer.make_poses(torch.from_numpy(pb.position).to(d), torch.from_numpy(pb.yaw).to(d),
                              torch.from_numpy(pb.pitch).to(d))
    sset = tracer.SceneSet([tracer.NodePool.from_words(cs.words, d)], [cs.bbox_min], [cs.bbox_max], [cs.hit_epsilon])
    _run(sset, poses, fan, cfg.azimuth_bins, cfg.elevation_bins, max_steps=cfg.max_steps,
         max_distance=cfg.max_distance, band=(1.5, 13.2), prox=2.0, use_pitch=True)
    c3 = scenes.CONFIGS[3]
    scene_list = [workloads.compiled_scene(3, s, resolution=128) for s in range(3)]
    pb3 = workloads.poses_for(3, scene_list, actors=24)
    fan3 = torch.from_numpy(workloads.fan_for(3)).to(d)
    poses3 = tracer.make_poses(torch.from_numpy(pb3.position).to(d), torch.from_numpy(pb3.yaw).to(d), None,
                               torch.from_numpy(pb3.scene).to(d))
    sset3 = tracer.SceneSet([tracer.NodePool.from_words(c.words, d) for c in scene_list],
                            [c.bbox_min for c in scene_list], [c.bbox_max for c in scene_list],
                            [c.hit_epsilon for c in scene_list])
    _run(sset3, poses3, fan3, c3.azimuth_bins, c3.elevation_bins, max_steps=c3.max_steps,
         max_distance=c3.max_distance, band=(1.5, 13.2), prox=2.0, use_pitch=False)


def test_observation_edge_values_nan_inf_negative():
    """Leaves of NaN, +inf and negative half distances give NaN, inf and negative ray distances."""
    words = np.array([internal_word(0xFF, 1)] + list(range(9, 17)) +
                     [leaf_word(0.5, 1), 0x8000000000017E00, 0x8000000000017C00, 0x800000000001BC00,
                      leaf_word(0.25, 2), leaf_word(0.003, 3), leaf_word(2.0, 0), leaf_word(0.75, 1)], np.uint64)
    d = dev()
    sset = tracer.SceneSet([tracer.NodePool.from_words(words, d)], [(0.0, 0.0, 0.0)], [(8.0, 8.0, 8.0)], [0.01])
    az, el = 12, 6
    az_ = np.linspace(0, 2 * np.pi, az, endpoint=False, dtype=np.float32)
    el_ = np.linspace(np.pi / 2, -np.pi / 2, el, dtype=np.float32)
    ag, eg = np.meshgrid(az_, el_, indexing="ij")
    fan = torch.from_numpy(np.stack([np.cos(eg) * np.sin(ag), np.sin(eg), -np.cos(eg) * np.cos(ag)], -1)
                           .reshape(-1, 3).astype(np.float32)).to(d)
    rng = np.random.default_rng(3)
    pos = torch.from_numpy(rng.uniform(0.5, 7.5, size=(9, 3)).astype(np.float32)).to(d)
    yaw = torch.from_numpy(rng.uniform(0, 6.28, size=9).astype(np.float32)).to(d)
    poses = tracer.make_poses(pos, yaw)
    od, st = _run(sset, poses, fan, az, el, max_steps=20, max_distance=6.0, band=(0.5, 5.0), prox=1.0,
                  use_pitch=False)
    v = od.cpu().numpy()
    assert np.isnan(v).any() and np.isinf(v).any()
    # a single leaf of distance -1: rays march backwards (those that stay inside end at t < 0)
    neg = tracer.SceneSet([tracer.NodePool.from_words(np.array([0x800000000000BC00], np.uint64), d)],
                          [(0.0, 0.0, 0.0)], [(8.0, 8.0, 8.0)], [0.01])
    od, st = _run(neg, poses, fan, az, el, max_steps=7, max_distance=6.0, band=(0.5, 5.0), prox=1.0,
                  use_pitch=False)
    assert (od.cpu().numpy() < 0).any()
