"""tsdf_cast_noalloc gives the same outputs as tsdf_cast, call after call.

tsdf_cast_noalloc is for callers that cannot allocate device memory while they
run — a fixed-rate control loop that must not stall in cudaMalloc, or a host
that hands the library only buffers registered up front.  It takes no
workspace: its scratch is a static device array inside the library.  This test
calls both entry points through the C ABI (ctypes) on the same pool and rays,
twice in a row with different rays, and requires identical bits (the tolerance
of every parity test here: none).  Outputs are prefilled with sentinels so a
ray the second call skipped (a counter left over from the first call) would
show.  It builds everything it uses, so it runs alone in a fresh process as
well as after the other tests; its file name makes pytest collect it last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from navi_b200 import _native, scenes, workloads

pytestmark = pytest.mark.gpu


def _rays(config: int, seed: int, dev: torch.device):
    cs = workloads.compiled_scene(config)
    pb = workloads.poses_for(config, [cs], seed_offset=seed)
    fan = workloads.fan_for(config)
    cy, sy = np.cos(pb.yaw).astype(np.float32), np.sin(pb.yaw).astype(np.float32)
    dirs = np.stack([fan[None, :, 0] * cy[:, None] + fan[None, :, 2] * sy[:, None],
                     np.broadcast_to(fan[None, :, 1], (cy.shape[0], fan.shape[0])),
                     -fan[None, :, 0] * sy[:, None] + fan[None, :, 2] * cy[:, None]], axis=-1).astype(np.float32)
    origins = np.repeat(pb.position[:, None, :], fan.shape[0], axis=1).astype(np.float32)
    o = torch.from_numpy(np.ascontiguousarray(origins.reshape(-1, 3))).to(dev)
    d = torch.from_numpy(np.ascontiguousarray(dirs.reshape(-1, 3))).to(dev)
    return cs, o, d


def test_noalloc_cast_matches_tsdf_cast_on_consecutive_calls():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _native.tsdf_lib()
    cfg = scenes.CONFIGS[1]
    cs, _, _ = _rays(1, 1, dev)
    words = np.ascontiguousarray(cs.words)
    pool = ctypes.c_void_p()
    assert lib.tsdf_pool_create(words.ctypes.data_as(ctypes.c_void_p), words.shape[0], 0, 0, ctypes.byref(pool)) == 0
    try:
        f3 = ctypes.c_float * 3
        bmin, bmax = f3(*cs.bbox_min), f3(*cs.bbox_max)
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        for call, seed in enumerate((11, 12)):
            _, o, d = _rays(1, seed, dev)
            n = o.shape[0]
            ws = torch.zeros(int(lib.tsdf_workspace_bytes(n)), dtype=torch.uint8, device=dev)
            outs = []
            for which in ("noalloc", "workspace"):
                od = torch.full((n,), -7.0, dtype=torch.float32, device=dev)
                os_ = torch.full((n,), -7, dtype=torch.int32, device=dev)
                ok = torch.full((n,), -7, dtype=torch.int32, device=dev)
                args = (pool, ctypes.c_void_p(o.data_ptr()), ctypes.c_void_p(d.data_ptr()), n,
                        ctypes.c_void_p(od.data_ptr()), ctypes.c_void_p(os_.data_ptr()), ctypes.c_void_p(ok.data_ptr()),
                        cfg.max_steps, cfg.max_distance, bmin, bmax, cs.hit_epsilon)
                if which == "noalloc":
                    rc = lib.tsdf_cast_noalloc(*args, stream)
                else:
                    rc = lib.tsdf_cast(*args, ctypes.c_void_p(ws.data_ptr()), stream)
                assert rc == 0, lib.tsdf_last_error()
                torch.cuda.synchronize(dev)
                outs.append((od.cpu().numpy(), os_.cpu().numpy(), ok.cpu().numpy()))
            (ad, as_, ak), (bd, bs, bk) = outs
            assert (ak > 0).all(), f"call {call}: a ray was left untraced"
            assert np.array_equal(ad.view(np.uint32), bd.view(np.uint32)), f"call {call}: distances differ"
            assert np.array_equal(as_, bs), f"call {call}: semantics differ"
            assert np.array_equal(ak, bk), f"call {call}: step counts differ"
    finally:
        lib.tsdf_pool_destroy(pool)


def test_noalloc_cast_rejects_bad_arguments_without_launching():
    lib = _native.tsdf_lib()
    f3 = ctypes.c_float * 3
    assert lib.tsdf_cast_noalloc(None, None, None, 1, None, None, None, 8, 1.0, f3(0, 0, 0), f3(1, 1, 1), 0.01, None) != 0
    assert b"pool must not be null" in lib.tsdf_last_error()
