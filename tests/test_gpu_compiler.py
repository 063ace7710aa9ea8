"""The device scene compiler (libnavi_gmdag_gpu.so) against the reference compiler and the host compiler.

- words of whole compiles against the reference compiler's golden hashes
  (tests/golden/compiler_golden.json, made by tests/golden/make_compiler_golden.py);
- the SDF stage (seeding + 8 sweeps, compiler.cpp:444-536) bit for bit against the
  host compiler, including a resolution that is not a power of two;
- the DAG stage (compiler.cpp:579-674) against the host compiler on grids built to
  stress the dedup: quantised values, uniform blocks at every level, repeated
  subtrees, all-far octants, and the 1- and 2-voxel grids.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from navi_b200 import gmdag, scenes

pytestmark = pytest.mark.gpu

GOLDEN = json.loads((Path(__file__).parent / "golden" / "compiler_golden.json").read_text())


@pytest.mark.parametrize("key", sorted(GOLDEN))
def test_device_compile_equals_reference_compiler(key):
    cfg, scene, res = (int(x[1:]) for x in key.split("_"))
    sc = scenes.make_scene(cfg, scene)
    out = gmdag.compile_mesh(sc.vertices, sc.triangles, res, device=0)
    g = GOLDEN[key]
    assert out.nodes.shape[0] == g["n_words"]
    assert hashlib.sha256(out.nodes.tobytes()).hexdigest() == g["words_sha256"]
    assert list(out.bbox_min) == g["bbox_min"]
    assert out.voxel_size == g["voxel_size"]
    assert out.timing["visited_blocks"] > 0


@pytest.mark.parametrize("cfg,scene,res", [(1, 0, 128), (3, 1, 96), (2, 0, 40)])
def test_device_sdf_equals_host_sdf(cfg, scene, res):
    sc = scenes.make_scene(cfg, scene)
    g_host, bmin_h, bmax_h, vox_h = gmdag.compute_sdf(sc.vertices, sc.triangles, res)
    g_dev, bmin_d, bmax_d, vox_d = gmdag.compute_sdf(sc.vertices, sc.triangles, res, device=0)
    assert (bmin_h, bmax_h, vox_h) == (bmin_d, bmax_d, vox_d)
    assert np.array_equal(g_host.view(np.uint32), g_dev.view(np.uint32))


def _random_mesh(rng, n_tri):
    v = rng.uniform(-3.0, 3.0, size=(3 * n_tri, 3)).astype(np.float32)
    # degenerate triangles: repeated vertices and collinear points
    v[3:6] = v[3]
    v[6:9] = np.stack([v[6], v[6] * 0.5 + v[7] * 0.5, v[7]])
    return v, np.arange(3 * n_tri, dtype=np.uint32).reshape(-1, 3)


@pytest.mark.parametrize("seed,res", [(0, 32), (1, 64), (2, 17)])
def test_device_compile_random_meshes(seed, res):
    rng = np.random.default_rng(seed)
    v, t = _random_mesh(rng, 40)
    g_host = gmdag.compute_sdf(v, t, res)[0]
    g_dev = gmdag.compute_sdf(v, t, res, device=0)[0]
    assert np.array_equal(g_host.view(np.uint32), g_dev.view(np.uint32))
    if res & (res - 1) == 0:
        host = gmdag.compile_mesh(v, t, res)
        dev = gmdag.compile_mesh(v, t, res, device=0)
        assert np.array_equal(host.nodes, dev.nodes)


def _quantised_grid(rng, n, levels=4, voxel=0.1):
    """Values on a coarse lattice so that equal leaves, uniform blocks and repeated
    subtrees occur at several levels."""
    base = rng.integers(0, levels, size=(n, n, n)).astype(np.float32) * np.float32(voxel * 0.5)
    tile = base[: n // 4, : n // 4, : n // 4] if n >= 8 else base
    g = np.tile(tile, (n // tile.shape[0],) * 3)[:n, :n, :n].copy()
    # uniform regions of several sizes, some far (pruned octants), some near
    g[: n // 2, : n // 2, : n // 2] = np.float32(voxel * 40)
    if n >= 8:
        g[n // 2: n // 2 + n // 4, : n // 4, n // 2:] = np.float32(voxel * 0.3)
    return g


@pytest.mark.parametrize("n,seed", [(1, 0), (2, 1), (4, 2), (8, 3), (16, 4), (32, 5), (64, 6)])
def test_device_dag_stage_equals_host(n, seed):
    rng = np.random.default_rng(seed)
    g = _quantised_grid(rng, n)
    host = gmdag.compile_grid(g, 0.1)
    dev = gmdag.compile_grid(g, 0.1, device=0)
    assert np.array_equal(host, dev)


def test_device_dag_stage_uniform_and_far_grids():
    for value in (0.0, 0.05, 3.0, 1e-9):
        g = np.full((16, 16, 16), np.float32(value), np.float32)
        assert np.array_equal(gmdag.compile_grid(g, 0.1), gmdag.compile_grid(g, 0.1, device=0))
    # every octant of the root far from the surface, block not uniform: far leaf
    g = np.full((8, 8, 8), np.float32(5.0), np.float32)
    g[0, 0, 0] = np.float32(6.0)
    host = gmdag.compile_grid(g, 0.1)
    assert np.array_equal(host, gmdag.compile_grid(g, 0.1, device=0))
    assert host.shape[0] == 2 and int(host[0]) >> 63 == 1


def test_device_dag_stage_smooth_field():
    n = 64
    z, y, x = np.meshgrid(*(np.arange(n, dtype=np.float32),) * 3, indexing="ij")
    g = (np.abs(np.sqrt((x - 20.5) ** 2 + (y - 31.0) ** 2 + (z - 40.0) ** 2) - 12.0) * np.float32(0.05)).astype(np.float32)
    assert np.array_equal(gmdag.compile_grid(g, 0.05), gmdag.compile_grid(g, 0.05, device=0))


def test_device_compiler_rejects_bad_arguments():
    sc = scenes.make_scene(1, 0)
    with pytest.raises(RuntimeError, match="power of two"):
        gmdag.compile_mesh(sc.vertices, sc.triangles, 96, device=0)
    bad = sc.triangles.copy()
    bad[0, 0] = sc.vertices.shape[0]
    with pytest.raises(RuntimeError, match="out of range"):
        gmdag.compile_mesh(sc.vertices, bad, 64, device=0)
