"""The reference's spawn-pose search, restated literally — TEST INFRASTRUCTURE ONLY.

Follows projects/environment/src/navi_environment/backends/sdfdag_backend.py:
  _observation_profile               :162-199
  _select_spawn_yaw_from_observation :224-264
  _spawn_candidate_score             :267-287
  SdfDagBackend._find_spawn_poses    :2564-2700 (candidate grid, probe cast, ranking, gate)
with the per-candidate Python loop, np.roll per shift and np.mean calls of the
reference, and the cast done by the oracle trace (oracle/trace_oracle.c) at the
reference kernel's hit threshold 0.01 on explicit rays built as the reference builds
them (candidate origins repeated over the unrotated probe directions).  navi_b200/spawn.py
is checked against this.
"""

from __future__ import annotations

import math

import numpy as np

from oracle import oracle as O

_SPAWN_MAX_STARVATION = 0.70
_SPAWN_CANDIDATES_PER_AXIS = 5
_SPAWN_HEIGHT_SAMPLES = 7
_SPAWN_PROBE_AZIMUTH_BINS = 48
_SPAWN_PROBE_ELEVATION_BINS = 12


def build_spherical_ray_directions(azimuth_bins, elevation_bins):
    """sdfdag_backend.py:205-221."""
    az = np.linspace(0.0, 2.0 * math.pi, azimuth_bins, endpoint=False, dtype=np.float32)
    el = np.linspace(math.pi / 2.0, -math.pi / 2.0, elevation_bins, endpoint=True, dtype=np.float32)
    az_grid, el_grid = np.meshgrid(az, el, indexing="ij")
    az_flat = az_grid.reshape(-1)
    el_flat = el_grid.reshape(-1)
    cos_el = np.cos(el_flat)
    return np.stack([cos_el * np.sin(az_flat), np.sin(el_flat), -cos_el * np.cos(az_flat)], axis=-1).astype(np.float32)


def observation_profile(metric_depth, valid_2d, *, max_distance=100.0, proximity_distance_threshold,
                        structure_band_min_distance, structure_band_max_distance):
    saturated = metric_depth >= max_distance - 1e-3
    starvation_ratio = float(np.mean(saturated.astype(np.float32)))
    structure_band_ratio = 0.0
    forward_structure_ratio = 0.0
    if structure_band_max_distance > structure_band_min_distance:
        structure_mask = np.logical_and(
            valid_2d,
            np.logical_and(metric_depth >= structure_band_min_distance, metric_depth <= structure_band_max_distance),
        )
        structure_band_ratio = float(np.mean(structure_mask, dtype=np.float32))
        forward_half_bins = max(1, metric_depth.shape[0] // 6)
        forward_sector = np.concatenate(
            (structure_mask[:forward_half_bins, :], structure_mask[-forward_half_bins:, :]), axis=0
        )
        forward_structure_ratio = float(np.mean(forward_sector, dtype=np.float32))
    if proximity_distance_threshold <= 0.0:
        return starvation_ratio, 0.0, structure_band_ratio, forward_structure_ratio
    near_mask = np.logical_and(valid_2d, metric_depth <= proximity_distance_threshold)
    proximity_ratio = float(np.mean(near_mask, dtype=np.float32))
    return (
        starvation_ratio,
        max(0.0, min(1.0, proximity_ratio)),
        max(0.0, min(1.0, structure_band_ratio)),
        max(0.0, min(1.0, forward_structure_ratio)),
    )


def select_spawn_yaw(metric_depth, valid_2d, *, structure_band_min_distance, structure_band_max_distance):
    azimuth_bins = int(metric_depth.shape[0])
    if azimuth_bins <= 0:
        return 0.0
    structure_mask = np.logical_and(
        valid_2d,
        np.logical_and(metric_depth >= structure_band_min_distance, metric_depth <= structure_band_max_distance),
    )
    forward_half_bins = max(1, azimuth_bins // 6)
    best_shift = 0
    best_score = float("-inf")
    for shift in range(azimuth_bins):
        rolled_structure = np.roll(structure_mask, -shift, axis=0)
        rolled_valid = np.roll(valid_2d, -shift, axis=0)
        forward_structure = np.concatenate(
            (rolled_structure[:forward_half_bins, :], rolled_structure[-forward_half_bins:, :]), axis=0
        )
        forward_valid = np.concatenate(
            (rolled_valid[:forward_half_bins, :], rolled_valid[-forward_half_bins:, :]), axis=0
        )
        score = 2.0 * float(np.mean(forward_structure, dtype=np.float32)) + float(
            np.mean(forward_valid, dtype=np.float32)
        )
        if score > best_score:
            best_score = score
            best_shift = shift
    return float(-(2.0 * math.pi * best_shift) / azimuth_bins) % (2.0 * math.pi)


def spawn_candidate_score(metric_depth, valid_2d, **kw):
    s, p, b, f = observation_profile(metric_depth, valid_2d, **kw)
    return float((3.0 * b) + (2.0 * f) - s - (1.5 * p))


def score_all(metric_distances, *, max_distance, proximity_distance_threshold, structure_band_min_distance,
              structure_band_max_distance):
    """Per-candidate (score, starvation, yaw) lists from distances [C, Az, El] (:2630-2660)."""
    valid = np.isfinite(metric_distances)
    clamped_metric = np.clip(metric_distances, 0.0, max_distance)
    kw = dict(max_distance=max_distance, proximity_distance_threshold=proximity_distance_threshold,
              structure_band_min_distance=structure_band_min_distance,
              structure_band_max_distance=structure_band_max_distance)
    out = []
    for idx in range(metric_distances.shape[0]):
        metric_2d = clamped_metric[idx]
        valid_2d = valid[idx]
        starvation_ratio, _, _, _ = observation_profile(metric_2d, valid_2d, **kw)
        score = spawn_candidate_score(metric_2d, valid_2d, **kw)
        yaw = select_spawn_yaw(metric_2d, valid_2d, structure_band_min_distance=structure_band_min_distance,
                               structure_band_max_distance=structure_band_max_distance)
        out.append((score, starvation_ratio, yaw))
    return out


def find_spawn_poses(words, bbox_min, bbox_max, count, *, azimuth_bins, elevation_bins, sdf_max_steps,
                     max_distance, proximity_distance_threshold, structure_band_min_distance,
                     structure_band_max_distance):
    bmin = np.array(bbox_min, dtype=np.float32)
    bmax = np.array(bbox_max, dtype=np.float32)
    extent = bmax - bmin
    x_values = np.linspace(bmin[0] + 0.2 * extent[0], bmax[0] - 0.2 * extent[0], _SPAWN_CANDIDATES_PER_AXIS,
                           dtype=np.float32)
    z_values = np.linspace(bmin[2] + 0.2 * extent[2], bmax[2] - 0.2 * extent[2], _SPAWN_CANDIDATES_PER_AXIS,
                           dtype=np.float32)
    y_values = np.linspace(bmin[1] + 0.2 * extent[1], bmax[1] - 0.2 * extent[1], _SPAWN_HEIGHT_SAMPLES,
                           dtype=np.float32)
    candidates = np.array([[x, y, z] for x in x_values for y in y_values for z in z_values], dtype=np.float32)
    paz = min(_SPAWN_PROBE_AZIMUTH_BINS, max(8, azimuth_bins))
    pel = min(_SPAWN_PROBE_ELEVATION_BINS, max(4, elevation_bins))
    probe_dirs = build_spherical_ray_directions(paz, pel)
    origins = np.repeat(candidates[:, None, :], probe_dirs.shape[0], axis=1)
    dirs = np.repeat(probe_dirs[None, :, :], candidates.shape[0], axis=0)
    res = O.trace(words, bbox_min, bbox_max, origins, dirs, max_steps=max(32, min(sdf_max_steps, 128)),
                  max_distance=max_distance, hit_epsilon=0.01)
    metric = res["dist"].reshape(candidates.shape[0], paz, pel).astype(np.float32, copy=False)
    per = score_all(metric, max_distance=max_distance, proximity_distance_threshold=proximity_distance_threshold,
                    structure_band_min_distance=structure_band_min_distance,
                    structure_band_max_distance=structure_band_max_distance)
    scored = [(sc, st, (float(c[0]), float(c[1]), float(c[2]), yaw)) for (sc, st, yaw), c in zip(per, candidates)]
    scored.sort(key=lambda item: item[0], reverse=True)
    if not scored:
        center = 0.5 * (bmin + bmax)
        return [(float(center[0]), float(center[1]), float(center[2]), 0.0)]
    viable = [(sc, starv, sp) for sc, starv, sp in scored if starv < _SPAWN_MAX_STARVATION]
    if len(viable) >= count:
        return [sp for _, _, sp in viable[:count]]
    if viable:
        selected = [sp for _, _, sp in viable]
        best_spawn = viable[0][2]
        while len(selected) < count:
            selected.append(best_spawn)
        return selected
    return [sp for _, _, sp in scored[:max(count, 1)]]
