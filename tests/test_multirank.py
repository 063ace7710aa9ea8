"""The multi-rank harness on CPU (gloo, world size 2): statistics gather, max-over-ranks
job time, and a rank that leaves before the collective (the survivor gets an error
within the process-group timeout instead of hanging).  No GPU is touched."""

from __future__ import annotations

import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, mode: str, q) -> None:
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from navi_b200 import dist_stats

    try:
        dist = dist_stats.init_from_env("gloo", timeout_s=10.0)
        if mode == "leave" and rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # flush the message before the hard exit
            os._exit(0)  # leaves between steps, before the stats collective
        row = torch.tensor([1000.0 * (rank + 1), 2.0 + rank, 40.0 + rank], dtype=torch.float64)
        table = dist_stats.gather_rank_stats(row, dist)
        q.put((rank, table.tolist(), dist_stats.job_figures(table)))
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put((rank, "error", type(exc).__name__))


def _run(mode: str, timeout: float = 60.0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=timeout) for _ in range(2)]
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda x: x[0])


def test_gather_and_max_over_ranks():
    r0, r1 = _run("ok")
    for _rank, table, (rays, job_ms) in (r0, r1):
        assert np.allclose(table, [[1000.0, 2.0, 40.0], [2000.0, 3.0, 41.0]])
        assert rays == 3000.0 and job_ms == 3.0


def test_rank_leaving_before_the_collective_fails_fast():
    r0, r1 = _run("leave")
    assert r1[1] == "left"
    assert r0[1] == "error"


def test_single_rank_needs_no_process_group(monkeypatch):
    from navi_b200 import dist_stats

    monkeypatch.setenv("WORLD_SIZE", "1")
    assert dist_stats.init_from_env("gloo") is None
    table = dist_stats.gather_rank_stats(torch.tensor([5.0, 1.5, 3.0], dtype=torch.float64))
    assert dist_stats.job_figures(table) == (5.0, 1.5)
