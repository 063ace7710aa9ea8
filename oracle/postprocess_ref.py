"""The reference's post-processing of cast outputs, restated in torch — TEST INFRASTRUCTURE ONLY.

Restates, op for op, so that it runs the same torch kernels on the same device:
  projects/environment/src/navi_environment/backends/sdfdag_backend.py:366-405
      _compute_observation_ratios_tensor
  projects/environment/src/navi_environment/backends/sdfdag_backend.py:408-473
      _postprocess_cast_outputs_tensor
  projects/environment/src/navi_environment/backends/sdfdag_backend.py:1518-1525
      the observation stack (depth, semantic, valid) consumed at :1402
The fused epilogue of the trace kernel is checked against this on a B200.
"""

from __future__ import annotations

import math

import torch


def observation_ratios(clamped_metric, valid_batch, *, max_distance, structure_band_min_distance,
                       structure_band_max_distance, proximity_distance_threshold):
    saturated = clamped_metric >= max_distance - 1e-3
    starvation_ratios = saturated.to(dtype=torch.float32).mean(dim=(1, 2))
    structure_band_ratios = torch.zeros_like(starvation_ratios)
    forward_structure_ratios = torch.zeros_like(starvation_ratios)
    if structure_band_max_distance > structure_band_min_distance:
        structure_mask = (
            valid_batch
            & (clamped_metric >= structure_band_min_distance)
            & (clamped_metric <= structure_band_max_distance)
        )
        structure_band_ratios = structure_mask.to(dtype=torch.float32).mean(dim=(1, 2))
        forward_half_bins = max(1, int(clamped_metric.shape[1]) // 6)
        forward_sector = torch.cat(
            (structure_mask[:, :forward_half_bins, :], structure_mask[:, -forward_half_bins:, :]), dim=1
        )
        forward_structure_ratios = forward_sector.to(dtype=torch.float32).mean(dim=(1, 2))
    if proximity_distance_threshold <= 0.0:
        proximity_ratios = torch.zeros_like(starvation_ratios)
    else:
        proximity_mask = valid_batch & (clamped_metric <= proximity_distance_threshold)
        proximity_ratios = proximity_mask.to(dtype=torch.float32).mean(dim=(1, 2))
    return (
        starvation_ratios.clamp(min=0.0, max=1.0),
        proximity_ratios.clamp(min=0.0, max=1.0),
        structure_band_ratios.clamp(min=0.0, max=1.0),
        forward_structure_ratios.clamp(min=0.0, max=1.0),
    )


def postprocess(out_distances, out_semantics, *, az_bins, el_bins, max_distance, structure_band_min_distance,
                structure_band_max_distance, proximity_distance_threshold):
    actor_count = int(out_distances.shape[0])
    metric_distances = out_distances.reshape(actor_count, az_bins, el_bins)
    semantic_batch = out_semantics.reshape(actor_count, az_bins, el_bins).to(dtype=torch.int32)
    if max_distance > 0.0:
        valid_batch = torch.isfinite(metric_distances)
        clamped_metric = metric_distances.clamp(min=0.0, max=max_distance)
        _log_denom = math.log1p(max_distance)
        depth_batch = (torch.log1p(clamped_metric) / _log_denom).clamp(min=0.0, max=1.0)
    else:
        valid_batch = torch.isfinite(metric_distances)
        clamped_metric = torch.where(valid_batch, metric_distances, torch.zeros_like(metric_distances))
        depth_batch = torch.zeros_like(metric_distances)
    min_distances = clamped_metric.amin(dim=(1, 2))
    starvation, proximity, band, forward = observation_ratios(
        clamped_metric, valid_batch, max_distance=max_distance,
        structure_band_min_distance=structure_band_min_distance,
        structure_band_max_distance=structure_band_max_distance,
        proximity_distance_threshold=proximity_distance_threshold,
    )
    observation = torch.stack(
        (depth_batch, semantic_batch.to(dtype=torch.float32), valid_batch.to(dtype=torch.float32)), dim=1
    )
    stats = torch.stack((min_distances, starvation, proximity, band, forward), dim=1)
    return observation, stats
