"""Post-processing and spawn search against the reference's own functions.

tests/golden/post_spawn_golden.npz and spawn_golden.json hold outputs of the
reference's _postprocess_cast_outputs_tensor (sdfdag_backend.py:408-473),
_observation_profile (:162-199), _spawn_candidate_score (:267-287),
_select_spawn_yaw_from_observation (:224-264) and SdfDagBackend._find_spawn_poses
(:2564-2700), made by tests/golden/make_post_spawn_golden.py from the reference
tree.  Checked here: the torch restatement that the observation kernel is compared
with on the GPU (oracle/postprocess_ref.py), the literal restatement of the spawn
search (oracle/spawn_ref.py) and the vectorised spawn scoring of the product
(navi_b200/spawn.py).  Tolerance: none (float32 bit patterns; NaN compared as NaN).
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from navi_b200 import spawn, workloads
from oracle import postprocess_ref, spawn_ref

GOLDEN = Path(__file__).parent / "golden"
POST = np.load(GOLDEN / "post_spawn_golden.npz")
SPAWNS = json.loads((GOLDEN / "spawn_golden.json").read_text())

import importlib.util  # noqa: E402

_spec = importlib.util.spec_from_file_location("mpsg", GOLDEN / "make_post_spawn_golden.py")
_mpsg = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(_mpsg)
POST_CASES = _mpsg.POST_CASES
PROFILE_CASES = _mpsg.PROFILE_CASES


def _same(got, want, what):
    g = np.ascontiguousarray(np.asarray(got))
    w = np.ascontiguousarray(np.asarray(want))
    assert g.shape == w.shape, f"{what}: shape {g.shape} vs {w.shape}"
    if g.dtype == np.float32:
        ok = (g.view(np.uint32) == w.view(np.uint32)) | (np.isnan(g) & np.isnan(w))
    else:
        ok = g == w
    bad = np.nonzero(~ok.reshape(-1))[0]
    assert bad.size == 0, f"{what}: {bad.size} differ; first {bad[:5]} got {g.reshape(-1)[bad[:5]]} want {w.reshape(-1)[bad[:5]]}"


@pytest.mark.parametrize("k", range(len(POST_CASES)))
def test_postprocess_restatement_equals_reference(k):
    a, az, el, mx, bmin, bmax, prox = POST_CASES[k]
    d = torch.from_numpy(POST[f"post{k}_dist"])
    s = torch.from_numpy(POST[f"post{k}_sem"])
    obs, stats = postprocess_ref.postprocess(d, s, az_bins=az, el_bins=el, max_distance=mx,
                                             structure_band_min_distance=bmin, structure_band_max_distance=bmax,
                                             proximity_distance_threshold=prox)
    obs, stats = obs.numpy(), stats.numpy()
    _same(obs[:, 0], POST[f"post{k}_depth"], "depth")
    _same(obs[:, 1], POST[f"post{k}_semantic"].astype(np.float32), "semantic")
    _same(obs[:, 2], POST[f"post{k}_valid"].astype(np.float32), "valid")
    for col, name in enumerate(["min", "starvation", "proximity", "band", "forward"]):
        _same(stats[:, col], POST[f"post{k}_{name}"], name)
    # the cases cover what the backend does with non-finite and out-of-range readings
    raw = POST[f"post{k}_dist"]
    if a * az * el >= 70:
        assert np.isnan(raw).any() and np.isposinf(raw).any() and np.isneginf(raw).any() and (raw < 0).any()


@pytest.mark.parametrize("k", range(len(PROFILE_CASES)))
def test_spawn_scoring_restatements_equal_reference(k):
    az, el, mx, prox, bmin, bmax = PROFILE_CASES[k]
    raw = POST[f"prof{k}_raw"]
    want = POST[f"prof{k}_values"]
    valid = np.isfinite(raw)
    metric = np.clip(raw, 0.0, mx)
    kw = dict(max_distance=mx, proximity_distance_threshold=prox, structure_band_min_distance=bmin,
              structure_band_max_distance=bmax)
    prof = spawn_ref.observation_profile(metric, valid, **kw)
    score = spawn_ref.spawn_candidate_score(metric, valid, **kw)
    yaw = spawn_ref.select_spawn_yaw(metric, valid, structure_band_min_distance=bmin, structure_band_max_distance=bmax)
    assert [*prof, score, yaw] == list(want)
    # the product's vectorised scoring (one candidate)
    s2, st2, y2 = spawn.score_candidates(raw[None], **kw)
    assert (float(s2[0]), float(st2[0]), float(y2[0])) == (want[4], want[0], want[5])


@pytest.mark.parametrize("case", SPAWNS, ids=[f"c{c['config']}s{c['scene']}r{c['resolution']}n{c['count']}" for c in SPAWNS])
def test_spawn_search_restatement_equals_reference(case):
    """The literal restatement's whole search (oracle-traced probe) returns the reference's poses."""
    cs = workloads.compiled_scene(case["config"], case["scene"], resolution=case["resolution"])
    assert hashlib.sha256(cs.words.tobytes()).hexdigest() == case["words_sha256"]
    kw = {k: case[k] for k in ("azimuth_bins", "elevation_bins", "sdf_max_steps", "max_distance",
                               "proximity_distance_threshold", "structure_band_min_distance",
                               "structure_band_max_distance")}
    got = spawn_ref.find_spawn_poses(cs.words, cs.bbox_min, cs.bbox_max, case["count"], **kw)
    assert [list(p) for p in got] == case["poses"]


@pytest.mark.gpu
@pytest.mark.parametrize("case", SPAWNS, ids=[f"c{c['config']}s{c['scene']}r{c['resolution']}n{c['count']}" for c in SPAWNS])
def test_spawn_search_on_the_gpu_equals_reference(case):
    """navi_b200.spawn (probe cast on the fan kernel, vectorised scoring) returns the reference's poses."""
    from navi_b200 import tracer

    cs = workloads.compiled_scene(case["config"], case["scene"], resolution=case["resolution"])
    pool = tracer.NodePool.from_words(cs.words, torch.device("cuda", 0))
    kw = {k: case[k] for k in ("azimuth_bins", "elevation_bins", "sdf_max_steps", "max_distance",
                               "proximity_distance_threshold", "structure_band_min_distance",
                               "structure_band_max_distance")}
    got = spawn.find_spawn_poses(pool, cs.bbox_min, cs.bbox_max, case["count"], **kw)
    assert [list(p) for p in got] == case["poses"]


def test_live_reference_postprocess_when_the_reference_tree_is_present():
    """With the reference tree at hand, a fresh seeded case straight through the reference's function."""
    if not (_mpsg.REF / "projects" / "environment" / "src").exists():
        pytest.skip("reference tree not present")
    B = _mpsg.reference_backend()
    rng = np.random.default_rng(99)
    for a, az, el, mx, bmin, bmax, prox in POST_CASES:
        d = _mpsg.seeded_distances(rng, (a, az * el), mx, [bmin, bmax, prox])
        s = rng.integers(0, 9, size=(a, az * el)).astype(np.int32)
        want = B._postprocess_cast_outputs_tensor(
            torch.from_numpy(d), torch.from_numpy(s), az_bins=az, el_bins=el, max_distance=mx,
            structure_band_min_distance=bmin, structure_band_max_distance=bmax, proximity_distance_threshold=prox)
        obs, stats = postprocess_ref.postprocess(torch.from_numpy(d), torch.from_numpy(s), az_bins=az, el_bins=el,
                                                 max_distance=mx, structure_band_min_distance=bmin,
                                                 structure_band_max_distance=bmax, proximity_distance_threshold=prox)
        _same(obs[:, 0].numpy(), want[0].numpy(), "depth")
        _same(obs[:, 2].numpy(), want[2].numpy().astype(np.float32), "valid")
        for col, idx in enumerate([3, 4, 5, 6, 7]):
            _same(stats[:, col].numpy(), want[idx].numpy(), f"stat {col}")
