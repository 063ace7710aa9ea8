"""Spawn-pose search: the environment's probe of candidate positions, on the fan kernel.

Restates ``SdfDagBackend._find_spawn_poses``
(projects/environment/src/navi_environment/backends/sdfdag_backend.py:2564-2700):
a 5 x 7 x 5 grid of candidate positions inside the middle 60% of the scene box, one
spherical probe fan per candidate (at most 48 x 12 rays), each candidate scored from
its distances (``_spawn_candidate_score`` :267-287 over ``_observation_profile``
:162-199), a forward yaw chosen per candidate (``_select_spawn_yaw_from_observation``
:224-264), then the best ``count`` candidates whose starvation is under 70%.

The probe cast is one ``tsdf_cast_fan`` launch: each candidate is an actor at yaw 0,
whose rotated fan equals the reference's unrotated probe directions bit for bit
(cos 0 = 1, sin 0 = 0 exactly), and the reference kernel's fixed hit threshold 0.01
(kernel.cuh:7) is the scene's epsilon.  No origin/direction tensors are built.

The scoring runs on the host over the [candidates, azimuth, elevation] distances, as
in the reference, vectorised with the reference's float semantics: every ratio is a
float32 mean of a 0/1 mask (an exact count over a float32 division), every score a
double-precision sum of those floats, and the yaw search keeps the first best shift.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from . import tracer
from .fan import build_spherical_ray_directions

SPAWN_MAX_STARVATION = 0.70        # sdfdag_backend.py:62
SPAWN_CANDIDATES_PER_AXIS = 5      # :63
SPAWN_HEIGHT_SAMPLES = 7           # :64
SPAWN_PROBE_AZIMUTH_BINS = 48      # :65
SPAWN_PROBE_ELEVATION_BINS = 12    # :66
REFERENCE_HIT_EPSILON = 0.01       # kernel.cuh:7, the threshold of the reference's cast


def spawn_candidates(bbox_min, bbox_max) -> np.ndarray:
    """Candidate positions [C, 3] float32, x-major then y then z (sdfdag_backend.py:2565-2590)."""
    bmin = np.array(bbox_min, dtype=np.float32)
    bmax = np.array(bbox_max, dtype=np.float32)
    extent = bmax - bmin
    xs = np.linspace(bmin[0] + 0.2 * extent[0], bmax[0] - 0.2 * extent[0], SPAWN_CANDIDATES_PER_AXIS, dtype=np.float32)
    zs = np.linspace(bmin[2] + 0.2 * extent[2], bmax[2] - 0.2 * extent[2], SPAWN_CANDIDATES_PER_AXIS, dtype=np.float32)
    ys = np.linspace(bmin[1] + 0.2 * extent[1], bmax[1] - 0.2 * extent[1], SPAWN_HEIGHT_SAMPLES, dtype=np.float32)
    gx, gy, gz = np.meshgrid(xs, ys, zs, indexing="ij")
    return np.stack([gx.reshape(-1), gy.reshape(-1), gz.reshape(-1)], axis=1).astype(np.float32)


def probe_bins(azimuth_bins: int, elevation_bins: int) -> tuple[int, int]:
    """Probe fan size (sdfdag_backend.py:2592-2593)."""
    return (min(SPAWN_PROBE_AZIMUTH_BINS, max(8, azimuth_bins)),
            min(SPAWN_PROBE_ELEVATION_BINS, max(4, elevation_bins)))


def _mean32(count: np.ndarray, n: int) -> np.ndarray:
    """np.mean of a 0/1 float32 mask with `count` ones out of n: exact sum, float32 division."""
    return count.astype(np.float32) / np.float32(n)


def score_candidates(distances: np.ndarray, *, max_distance: float, proximity_distance_threshold: float,
                     structure_band_min_distance: float, structure_band_max_distance: float):
    """Scores, starvation ratios and yaws of candidates from their probe distances [C, Az, El].

    Returns (score float64 [C], starvation float64 [C], yaw float64 [C])."""
    metric = np.asarray(distances, dtype=np.float32)
    c, az, el = metric.shape
    valid = np.isfinite(metric)
    clamped = np.clip(metric, 0.0, max_distance)  # sdfdag_backend.py:2631
    n = az * el

    # _observation_profile (:162-199)
    saturated = clamped >= max_distance - 1e-3
    starvation = _mean32(saturated.reshape(c, -1).sum(axis=1), n).astype(np.float64)
    band = np.zeros(c, np.float64)
    forward = np.zeros(c, np.float64)
    fh = max(1, az // 6)
    structure = valid & (clamped >= structure_band_min_distance) & (clamped <= structure_band_max_distance)
    s_col = structure.sum(axis=2)  # [C, Az] structure rays per azimuth column
    if structure_band_max_distance > structure_band_min_distance:
        band = _mean32(s_col.sum(axis=1), n).astype(np.float64)
        fwd_count = s_col[:, :fh].sum(axis=1) + s_col[:, az - fh:].sum(axis=1)
        forward = _mean32(fwd_count, 2 * fh * el).astype(np.float64)
    if proximity_distance_threshold <= 0.0:
        proximity = np.zeros(c, np.float64)
    else:
        near = valid & (clamped <= proximity_distance_threshold)
        proximity = _mean32(near.reshape(c, -1).sum(axis=1), n).astype(np.float64)
    proximity = np.clip(proximity, 0.0, 1.0)
    band = np.clip(band, 0.0, 1.0)
    forward = np.clip(forward, 0.0, 1.0)
    # _spawn_candidate_score (:267-287), double-precision sum of the float ratios
    score = (3.0 * band) + (2.0 * forward) - starvation - (1.5 * proximity)

    # _select_spawn_yaw_from_observation (:224-264): the forward sector of shift k is
    # the columns k .. k+fh-1 and k-fh .. k-1 (mod Az) of the rolled masks
    v_col = valid.sum(axis=2)
    idx = (np.arange(az)[:, None] + np.concatenate([np.arange(fh), np.arange(az - fh, az)])[None, :]) % az
    s_win = s_col[:, idx].sum(axis=2)  # [C, shifts]
    v_win = v_col[:, idx].sum(axis=2)
    m = 2 * fh * el
    shift_score = 2.0 * _mean32(s_win, m).astype(np.float64) + _mean32(v_win, m).astype(np.float64)
    best = np.argmax(shift_score, axis=1)  # first of equal maxima, as the strict `>` scan keeps
    yaw = np.array([float(-(2.0 * math.pi * int(k)) / az) % (2.0 * math.pi) for k in best], np.float64)
    return score, starvation, yaw


def select_spawns(candidates: np.ndarray, score: np.ndarray, starvation: np.ndarray, yaw: np.ndarray,
                  count: int, bbox_min=None, bbox_max=None) -> list[tuple[float, float, float, float]]:
    """Rank and gate (sdfdag_backend.py:2662-2700): stable sort by score, starvation < 70%."""
    scored = [(float(score[i]), float(starvation[i]),
               (float(candidates[i, 0]), float(candidates[i, 1]), float(candidates[i, 2]), float(yaw[i])))
              for i in range(candidates.shape[0])]
    scored.sort(key=lambda item: item[0], reverse=True)
    if not scored:
        center = 0.5 * (np.array(bbox_min, np.float32) + np.array(bbox_max, np.float32))
        return [(float(center[0]), float(center[1]), float(center[2]), 0.0)]
    viable = [(sc, st, sp) for sc, st, sp in scored if st < SPAWN_MAX_STARVATION]
    if len(viable) >= count:
        return [sp for _, _, sp in viable[:count]]
    if viable:
        selected = [sp for _, _, sp in viable]
        while len(selected) < count:
            selected.append(viable[0][2])
        return selected
    return [sp for _, _, sp in scored[:max(count, 1)]]


def probe_distances(pool: tracer.NodePool, bbox_min, bbox_max, candidates: np.ndarray, azimuth_bins: int,
                    elevation_bins: int, *, max_steps: int, max_distance: float) -> torch.Tensor:
    """One fan cast from every candidate at yaw 0: distances [C, Az, El] on the pool's device."""
    dev = pool.device
    fan = torch.from_numpy(build_spherical_ray_directions(azimuth_bins, elevation_bins)).to(dev)
    sset = tracer.SceneSet([pool], [list(bbox_min)], [list(bbox_max)], [REFERENCE_HIT_EPSILON])
    pos = torch.from_numpy(np.ascontiguousarray(candidates, dtype=np.float32)).to(dev)
    poses = tracer.make_poses(pos, torch.zeros(pos.shape[0], dtype=torch.float32, device=dev))
    n = pos.shape[0] * fan.shape[0]
    out_d = torch.empty(n, dtype=torch.float32, device=dev)
    out_s = torch.empty(n, dtype=torch.int32, device=dev)
    tracer.cast_fan(sset, poses, fan, out_d, out_s, max_steps=max_steps, max_distance=max_distance,
                    use_pitch=False)
    return out_d.view(pos.shape[0], azimuth_bins, elevation_bins)


def find_spawn_poses(pool: tracer.NodePool, bbox_min, bbox_max, count: int, *, azimuth_bins: int,
                     elevation_bins: int, sdf_max_steps: int, max_distance: float,
                     proximity_distance_threshold: float, structure_band_min_distance: float,
                     structure_band_max_distance: float) -> list[tuple[float, float, float, float]]:
    """(x, y, z, yaw) of `count` spawn poses, as sdfdag_backend.py:2564-2700 selects them."""
    cand = spawn_candidates(bbox_min, bbox_max)
    paz, pel = probe_bins(azimuth_bins, elevation_bins)
    dist = probe_distances(pool, bbox_min, bbox_max, cand, paz, pel,
                           max_steps=max(32, min(sdf_max_steps, 128)), max_distance=max_distance)
    score, starvation, yaw = score_candidates(
        dist.cpu().numpy(), max_distance=max_distance, proximity_distance_threshold=proximity_distance_threshold,
        structure_band_min_distance=structure_band_min_distance,
        structure_band_max_distance=structure_band_max_distance)
    return select_spawns(cand, score, starvation, yaw, count, bbox_min, bbox_max)
