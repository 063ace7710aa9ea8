"""The oracle's step mix (oracle.step_mix) accounts for every march step and word load.

Each reference step either hits the void cache, lies outside the box, hits the leaf
cache or descends; a descent ends in a leaf or an empty octant; each descent level
loads the node word and, unless it ends there, the child-pointer word
(kernel.cu:137, :198), which the per-ray load counts (W_ref) of oracle.trace add up.
"""

from __future__ import annotations

import numpy as np

from navi_b200 import scenes, workloads
from oracle import oracle as O


def test_step_mix_accounts_for_steps_and_loads():
    cfg = scenes.CONFIGS[1]
    cs = workloads.compiled_scene(1)
    pb = workloads.poses_for(1, [cs])
    fan = workloads.fan_for(1)
    d = O.rotate_fan(fan, np.cos(pb.yaw), np.sin(pb.yaw), np.cos(pb.pitch), np.sin(pb.pitch))
    o = np.repeat(pb.position[:, None, :], fan.shape[0], axis=1)
    kw = dict(max_steps=cfg.max_steps, max_distance=cfg.max_distance, hit_epsilon=cs.hit_epsilon)
    m = O.step_mix(cs.words, cs.bbox_min, cs.bbox_max, o, d, **kw)
    r = O.trace(cs.words, cs.bbox_min, cs.bbox_max, o, d, **kw)
    assert m["steps"] == int(r["steps"].sum())
    assert m["void_cache"] + m["outside"] + m["leaf_cache"] + m["descents"] == m["steps"]
    assert m["descent_leaf"] + m["descent_void"] == m["descents"]  # no 32-level fall-out on a compiled scene
    assert m["levels"] + (m["levels"] - m["descents"]) == int(r["loads"].sum())
    assert m == O.step_mix(cs.words, cs.bbox_min, cs.bbox_max, o, d, threads=1, **kw)
