"""Per-rank timing statistics across GPUs (off the hot path).

Each rank traces its own actors in its own replica of the scenes; no collective
touches the trace.  After the timed region every rank contributes one small
float64 row ``[rays, device_ms, mean_steps]`` and one ``all_gather`` (NCCL on
GPUs, gloo on CPU) gives every rank the table; the job time is the slowest
rank's device time.
"""

from __future__ import annotations

import datetime
import os

import numpy as np
import torch

__all__ = ["init_from_env", "gather_rank_stats", "job_figures"]


def init_from_env(backend: str, device: torch.device | None = None, timeout_s: float = 600.0):
    """Join the process group described by RANK / WORLD_SIZE / MASTER_* (torchrun); None for one rank."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return None
    import torch.distributed as dist

    kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device is not None and backend == "nccl":
        kwargs["device_id"] = device
    dist.init_process_group(backend, **kwargs)
    return dist


def gather_rank_stats(row: torch.Tensor, dist=None) -> np.ndarray:
    """All-gather one float64 row per rank; returns the [world, k] table (same on every rank)."""
    if dist is None:
        return row.detach().cpu().numpy()[None, :]
    world = dist.get_world_size()
    parts = [torch.zeros_like(row) for _ in range(world)]
    dist.all_gather(parts, row)
    return torch.stack(parts).cpu().numpy()


def job_figures(table: np.ndarray) -> tuple[float, float]:
    """(rays of all ranks, job milliseconds = max over ranks)."""
    return float(table[:, 0].sum()), float(table[:, 1].max())
