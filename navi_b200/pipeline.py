"""Casts whose inputs and outputs live in host memory, with the copies overlapped.

A caller that keeps rays or poses in host memory and wants results back there
pays a host-to-device copy before the trace and a device-to-host copy after
it.  Done in one piece, both copies are serial with the trace.  Split into
chunks, the upload of chunk k+1 and the download of chunk k-1 run on their own
copy streams while chunk k traces, and consecutive chunks trace on two
alternating streams, so that one chunk's last rays share the GPU with the next
chunk's first ones.  Every cast in this package is asynchronous on the current
stream, which is what makes this possible without library support.

:func:`run_chunks` is the general form (one `Chunk` per piece: copies in, a
callable that launches on the current stream, copies out).  :func:`cast_rays_host`
and :func:`cast_fan_host` apply it to explicit rays and to pose-fused fans.
Host tensors should be pinned (``tensor.pin_memory()``) for the copies to be
asynchronous.  All work is joined back to the caller's current stream before
return, so anything queued later on it sees the host outputs written; call
``torch.cuda.current_stream().synchronize()`` before reading them on the host.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass, field
from typing import Callable, Sequence

import torch

from . import tracer

__all__ = ["Chunk", "run_chunks", "cast_rays_host", "cast_fan_host"]


@dataclass
class Chunk:
    """One piece of a pipelined cast: (device, host) copy pairs in and out, and the launch."""

    run: Callable[[], None]
    h2d: Sequence[tuple[torch.Tensor, torch.Tensor]] = field(default_factory=list)
    d2h: Sequence[tuple[torch.Tensor, torch.Tensor]] = field(default_factory=list)


_streams_lock = threading.Lock()
_streams: dict[int, tuple[torch.cuda.Stream, ...]] = {}


def _side_streams(device: torch.device) -> tuple[torch.cuda.Stream, ...]:
    """(upload, download, compute A, compute B) streams of a device, made once."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _streams_lock:
        s = _streams.get(idx)
        if s is None:
            s = tuple(torch.cuda.Stream(device=torch.device("cuda", idx)) for _ in range(4))
            _streams[idx] = s
        return s


def run_chunks(chunks: Sequence[Chunk], device: torch.device) -> None:
    """Run the chunks with uploads, launches and downloads overlapped (see the module docstring).

    Device buffers must have been allocated before the call, on the current stream; the
    call orders the current stream after every copy and launch it queued."""
    if not chunks:
        return
    cur = torch.cuda.current_stream(device)
    up, down, c0, c1 = _side_streams(device)
    start = torch.cuda.Event()
    start.record(cur)
    for s in (up, down, c0, c1):
        s.wait_event(start)
    for k, ch in enumerate(chunks):
        with torch.cuda.stream(up):
            for dst, src in ch.h2d:
                dst.copy_(src, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(up)
        comp = c0 if k % 2 == 0 else c1
        comp.wait_event(ready)
        with torch.cuda.stream(comp):
            ch.run()
            done = torch.cuda.Event()
            done.record(comp)
        down.wait_event(done)
        with torch.cuda.stream(down):
            for dst, src in ch.d2h:
                dst.copy_(src, non_blocking=True)
    for s in (up, c0, c1, down):
        cur.wait_stream(s)


def _bounds(n: int, chunks: int) -> list[tuple[int, int]]:
    chunks = max(1, min(int(chunks), n)) if n else 1
    step = -(-n // chunks) if n else 0
    return [(i, min(n, i + step)) for i in range(0, n, step)] if n else []


def cast_rays_host(
    pool: tracer.NodePool,
    origins: torch.Tensor,
    dirs: torch.Tensor,
    out_distances: torch.Tensor,
    out_semantics: torch.Tensor,
    *,
    max_steps: int,
    max_distance: float,
    bbox_min: Sequence[float],
    bbox_max: Sequence[float],
    hit_epsilon: float = tracer.DEFAULT_HIT_EPSILON,
    out_steps: torch.Tensor | None = None,
    chunks: int = 4,
) -> None:
    """tracer.cast_rays_ex with host origins/dirs [N, 3] and host outputs [N], in `chunks` pieces."""
    for name, t in (("origins", origins), ("dirs", dirs), ("out_distances", out_distances),
                    ("out_semantics", out_semantics), ("out_steps", out_steps)):
        if t is not None and (t.is_cuda or not t.is_contiguous()):
            raise RuntimeError(f"{name} must be a contiguous host tensor")
    n = out_distances.numel()
    dev = pool.device
    o = origins.reshape(n, 3)
    v = dirs.reshape(n, 3)
    g_o = torch.empty((n, 3), dtype=torch.float32, device=dev)
    g_v = torch.empty((n, 3), dtype=torch.float32, device=dev)
    g_d = torch.empty(n, dtype=torch.float32, device=dev)
    g_s = torch.empty(n, dtype=torch.int32, device=dev)
    g_k = torch.empty(n, dtype=torch.int32, device=dev) if out_steps is not None else None
    h_d, h_s = out_distances.reshape(n), out_semantics.reshape(n)
    h_k = out_steps.reshape(n) if out_steps is not None else None
    pieces = []
    for lo, hi in _bounds(n, chunks):
        def run(lo=lo, hi=hi):
            tracer.cast_rays_ex(pool, g_o[lo:hi], g_v[lo:hi], g_d[lo:hi], g_s[lo:hi], max_steps=max_steps,
                                max_distance=max_distance, bbox_min=bbox_min, bbox_max=bbox_max,
                                hit_epsilon=hit_epsilon, out_steps=None if g_k is None else g_k[lo:hi])
        outs = [(h_d[lo:hi], g_d[lo:hi]), (h_s[lo:hi], g_s[lo:hi])]
        if g_k is not None:
            outs.append((h_k[lo:hi], g_k[lo:hi]))
        pieces.append(Chunk(run, [(g_o[lo:hi], o[lo:hi]), (g_v[lo:hi], v[lo:hi])], outs))
    run_chunks(pieces, dev)


def cast_fan_host(
    scenes: tracer.SceneSet,
    poses: torch.Tensor,
    fan_dirs: torch.Tensor,
    out_distances: torch.Tensor,
    out_semantics: torch.Tensor,
    *,
    max_steps: int,
    max_distance: float,
    use_pitch: bool = False,
    out_steps: torch.Tensor | None = None,
    chunks: int = 4,
) -> None:
    """tracer.cast_fan with host poses [A, 8] (make_poses layout) and host outputs [A * R],
    in `chunks` pieces of whole actors; fan_dirs stays on the device."""
    for name, t in (("poses", poses), ("out_distances", out_distances), ("out_semantics", out_semantics),
                    ("out_steps", out_steps)):
        if t is not None and (t.is_cuda or not t.is_contiguous()):
            raise RuntimeError(f"{name} must be a contiguous host tensor")
    a, r = poses.shape[0], fan_dirs.shape[0]
    dev = scenes.device
    g_p = torch.empty((a, 8), dtype=torch.float32, device=dev)
    g_d = torch.empty((a, r), dtype=torch.float32, device=dev)
    g_s = torch.empty((a, r), dtype=torch.int32, device=dev)
    g_k = torch.empty((a, r), dtype=torch.int32, device=dev) if out_steps is not None else None
    h_d, h_s = out_distances.reshape(a, r), out_semantics.reshape(a, r)
    h_k = out_steps.reshape(a, r) if out_steps is not None else None
    pieces = []
    for lo, hi in _bounds(a, chunks):
        def run(lo=lo, hi=hi):
            tracer.cast_fan(scenes, g_p[lo:hi], fan_dirs, g_d[lo:hi], g_s[lo:hi], max_steps=max_steps,
                            max_distance=max_distance, use_pitch=use_pitch,
                            out_steps=None if g_k is None else g_k[lo:hi])
        outs = [(h_d[lo:hi], g_d[lo:hi]), (h_s[lo:hi], g_s[lo:hi])]
        if g_k is not None:
            outs.append((h_k[lo:hi], g_k[lo:hi]))
        pieces.append(Chunk(run, [(g_p[lo:hi], poses[lo:hi])], outs))
    run_chunks(pieces, dev)
