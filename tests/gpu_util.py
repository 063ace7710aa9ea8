"""Helpers of the GPU parity tests."""

from __future__ import annotations

import numpy as np
import torch

from navi_b200 import tracer


def dev() -> torch.device:
    return torch.device("cuda", 0)


def eager_world_rays(fan: torch.Tensor, poses: torch.Tensor, pitch: bool = True):
    """Origins and directions built with eager torch ops, as sdfdag_backend.py:1299-1312 does
    (plus the pitch rotation of the benchmark configurations)."""
    a, r = poses.shape[0], fan.shape[0]
    cy, sy, cp, sp = (poses[:, k:k + 1] for k in (3, 4, 5, 6))
    base = fan.unsqueeze(0).expand(a, -1, -1)
    if pitch:
        by = base[..., 1] * cp - base[..., 2] * sp
        bz = base[..., 1] * sp + base[..., 2] * cp
    else:
        by = base[..., 1]
        bz = base[..., 2]
    dirs = torch.empty((a, r, 3), dtype=torch.float32, device=fan.device)
    dirs[..., 0] = base[..., 0] * cy + bz * sy
    dirs[..., 1] = by
    dirs[..., 2] = -base[..., 0] * sy + bz * cy
    origins = poses[:, 0:3].unsqueeze(1).expand(-1, r, -1).contiguous()
    return origins, dirs


def cast_explicit(words: np.ndarray, origins, dirs, *, max_steps, max_distance, bbox_min, bbox_max,
                  hit_epsilon=0.01, pool=None):
    d = dev()
    o = torch.as_tensor(np.asarray(origins, np.float32) if not torch.is_tensor(origins) else origins).to(d).contiguous()
    v = torch.as_tensor(np.asarray(dirs, np.float32) if not torch.is_tensor(dirs) else dirs).to(d).contiguous()
    n = o.numel() // 3
    out_d = torch.full((n,), -7.0, dtype=torch.float32, device=d)
    out_s = torch.full((n,), -7, dtype=torch.int32, device=d)
    out_k = torch.full((n,), -7, dtype=torch.int32, device=d)
    p = pool or tracer.NodePool.from_words(words, d)
    tracer.cast_rays_ex(p, o, v, out_d, out_s, max_steps=max_steps, max_distance=max_distance, bbox_min=bbox_min,
                        bbox_max=bbox_max, hit_epsilon=hit_epsilon, out_steps=out_k)
    torch.cuda.synchronize()
    return out_d.cpu().numpy(), out_s.cpu().numpy(), out_k.cpu().numpy()


def assert_bits_equal(got: np.ndarray, exp: np.ndarray, what: str) -> None:
    g = np.ascontiguousarray(got, dtype=np.float32).reshape(-1).view(np.uint32)
    e = np.ascontiguousarray(exp, dtype=np.float32).reshape(-1).view(np.uint32)
    bad = np.nonzero(g != e)[0]
    assert bad.size == 0, (
        f"{what}: {bad.size} of {g.size} differ; first {bad[:5]} "
        f"got {np.asarray(got).reshape(-1)[bad[:5]]} expected {np.asarray(exp).reshape(-1)[bad[:5]]}"
    )


def assert_equal(got: np.ndarray, exp: np.ndarray, what: str) -> None:
    g = np.asarray(got).reshape(-1)
    e = np.asarray(exp).reshape(-1)
    bad = np.nonzero(g != e)[0]
    assert bad.size == 0, f"{what}: {bad.size} of {g.size} differ; first {bad[:5]} got {g[bad[:5]]} expected {e[bad[:5]]}"
