"""Spawn-pose search (navi_b200/spawn.py) against the literal restatement of the
reference's numpy code (oracle/spawn_ref.py, sdfdag_backend.py:162-287, :2564-2700).

CPU: the vectorised scoring and yaw search against the per-candidate loops on random
distances (NaN, inf, values on the band and proximity bounds, tiny fans), and the
ranking/gate paths.  GPU: the whole search, probe cast on the fan kernel, against the
oracle-traced reference on compiled scenes.
"""

from __future__ import annotations

import numpy as np
import pytest

from navi_b200 import spawn
from oracle import spawn_ref

KW = dict(max_distance=30.0, proximity_distance_threshold=2.0, structure_band_min_distance=1.5,
          structure_band_max_distance=9.0)


def _distances(rng, c, az, el):
    d = rng.uniform(-1.0, 40.0, size=(c, az, el)).astype(np.float32)
    pick = rng.random((c, az, el))
    d[pick < 0.05] = np.nan
    d[(pick >= 0.05) & (pick < 0.1)] = np.inf
    d[(pick >= 0.1) & (pick < 0.13)] = np.float32(1.5)
    d[(pick >= 0.13) & (pick < 0.16)] = np.float32(9.0)
    d[(pick >= 0.16) & (pick < 0.19)] = np.float32(2.0)
    d[(pick >= 0.19) & (pick < 0.22)] = np.float32(30.0) - np.float32(1e-3)
    # a few candidates fully in the void or fully saturated, to reach the gate's paths
    d[0] = np.float32(1000.0)
    d[1] = np.inf
    return d


@pytest.mark.parametrize("az,el", [(48, 12), (8, 4), (5, 3), (1, 1), (13, 7)])
@pytest.mark.parametrize("kw", [KW, dict(KW, proximity_distance_threshold=0.0),
                                dict(KW, structure_band_min_distance=9.0, structure_band_max_distance=1.5)])
def test_vectorised_scoring_equals_reference_loops(az, el, kw):
    rng = np.random.default_rng(az * 100 + el)
    d = _distances(rng, 24, az, el)
    score, starv, yaw = spawn.score_candidates(d, **kw)
    ref = spawn_ref.score_all(d, **kw)
    assert [float(x) for x in score] == [r[0] for r in ref]
    assert [float(x) for x in starv] == [r[1] for r in ref]
    assert [float(x) for x in yaw] == [r[2] for r in ref]


def test_yaw_ties_keep_the_first_best_shift():
    d = np.full((1, 12, 4), np.float32(5.0), np.float32)  # every shift scores the same
    _, _, yaw = spawn.score_candidates(d, **KW)
    assert float(yaw[0]) == 0.0
    assert spawn_ref.score_all(d, **KW)[0][2] == 0.0


def test_candidates_follow_the_reference_grid():
    c = spawn.spawn_candidates((-11.0, -11.0, -11.0), (11.0, 11.0, 11.0))
    assert c.shape == (5 * 7 * 5, 3) and c.dtype == np.float32
    xs = np.linspace(np.float32(-11.0) + 0.2 * np.float32(22.0), np.float32(11.0) - 0.2 * np.float32(22.0), 5,
                     dtype=np.float32)
    assert np.array_equal(np.unique(c[:, 0]), np.sort(xs))
    assert np.array_equal(c[:7 * 5, 0], np.full(35, xs[0], np.float32))  # x outermost
    assert np.array_equal(c[:5, 2], xs)  # z innermost


@pytest.mark.parametrize("starv_level,count", [(0.1, 5), (0.9, 5), (0.5, 200)])
def test_ranking_and_gate(starv_level, count):
    rng = np.random.default_rng(7)
    cand = spawn.spawn_candidates((0.0, 0.0, 0.0), (10.0, 10.0, 10.0))
    score = np.round(rng.normal(size=cand.shape[0]), 1)  # ties
    starv = np.full(cand.shape[0], starv_level)
    starv[::3] = 0.2
    yaw = rng.uniform(0, 6.28, cand.shape[0])
    got = spawn.select_spawns(cand, score, starv, yaw, count)
    scored = [(float(score[i]), float(starv[i]), (float(cand[i, 0]), float(cand[i, 1]), float(cand[i, 2]),
                                                   float(yaw[i]))) for i in range(cand.shape[0])]
    scored.sort(key=lambda it: it[0], reverse=True)
    viable = [it for it in scored if it[1] < 0.70]
    if len(viable) >= count:
        want = [it[2] for it in viable[:count]]
    elif viable:
        want = [it[2] for it in viable] + [viable[0][2]] * (count - len(viable))
    else:
        want = [it[2] for it in scored[:count]]
    assert got == want


@pytest.mark.gpu
@pytest.mark.parametrize("config,bins", [(1, (64, 16)), (2, (256, 48)), (3, (128, 24))])
def test_spawn_search_matches_reference_on_compiled_scenes(config, bins):
    import torch

    from navi_b200 import tracer, workloads

    cs = workloads.compiled_scene(config, 0, resolution=128 if config == 3 else None)
    pool = tracer.NodePool.from_words(cs.words, torch.device("cuda", 0))
    kw = dict(azimuth_bins=bins[0], elevation_bins=bins[1], sdf_max_steps=256, max_distance=30.0,
              proximity_distance_threshold=2.0, structure_band_min_distance=1.5, structure_band_max_distance=6.0)
    got = spawn.find_spawn_poses(pool, cs.bbox_min, cs.bbox_max, 8, **kw)
    want = spawn_ref.find_spawn_poses(cs.words, cs.bbox_min, cs.bbox_max, 8, **kw)
    assert got == want
    assert len(got) == 8
