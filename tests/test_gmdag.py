"""``.gmdag`` loader, writer, validator and scene compiler (CPU).

Loader cases mirror projects/environment/tests/unit/test_voxel_dag_integration.py:28-266;
round-trip cases mirror projects/torch-sdf/tests/test_gmdag_roundtrip.py:87-184.
"""

from __future__ import annotations

import struct

import numpy as np
import pytest

from navi_b200 import gmdag, scenes, workloads
from tests.kat_cases import internal_word, leaf_word

_HEADER = struct.Struct("<4sIIffffI")


def _leaf_node(distance_bits: int = 1, semantic: int = 0) -> int:
    return (1 << 63) | ((semantic & 0xFFFF) << 16) | distance_bits


def _write(path, magic=b"GDAG", version=1, res=32, bmin=(0.0, 0.0, 0.0), voxel=1.0, nodes=None, count=None, extra=b""):
    nodes = np.asarray(nodes if nodes is not None else [], dtype=np.uint64)
    n = count if count is not None else nodes.shape[0]
    path.write_bytes(_HEADER.pack(magic, version, res, *bmin, voxel, n) + nodes.tobytes() + extra)
    return path


def test_load_reads_header_and_nodes(tmp_path):
    p = _write(tmp_path / "mini.gmdag", res=64, bmin=(-2.0, -1.0, -3.0), voxel=0.25, nodes=[_leaf_node(1, 7)])
    a = gmdag.load_gmdag_asset(p)
    assert a.path == p.resolve()
    assert a.version == 1 and a.resolution == 64
    assert a.bbox_min == (-2.0, -1.0, -3.0)
    assert a.bbox_max == (14.0, 15.0, 13.0)
    assert a.voxel_size == 0.25
    assert np.array_equal(a.nodes, np.array([_leaf_node(1, 7)], np.uint64))


@pytest.mark.parametrize(
    "kwargs,match",
    [
        ({"magic": b"NOPE", "count": 0}, "Unsupported gmdag magic"),
        ({"version": 2, "nodes": [1]}, "Unsupported gmdag version"),
        ({"res": 0, "nodes": [1]}, "Invalid gmdag resolution"),
        ({"voxel": 0.0, "nodes": [1]}, "Invalid gmdag voxel size"),
        ({"voxel": float("nan"), "nodes": [1]}, "Invalid gmdag voxel size"),
        ({"count": 0}, "Invalid gmdag node count"),
        ({"nodes": [_leaf_node()], "extra": b"\x00"}, "trailing bytes detected"),
        ({"bmin": (0.0, float("inf"), 0.0), "nodes": [1]}, "non-finite bbox_min"),
        ({"nodes": [_leaf_node()], "count": 2}, "expected 2 nodes, found 1"),
    ],
)
def test_load_rejects_bad_files(tmp_path, kwargs, match):
    p = _write(tmp_path / "bad.gmdag", **kwargs)
    with pytest.raises(RuntimeError, match=match):
        gmdag.load_gmdag_asset(p)


def test_load_rejects_short_header(tmp_path):
    p = tmp_path / "short.gmdag"
    p.write_bytes(b"GDAG\x01")
    with pytest.raises(RuntimeError, match="Invalid gmdag header"):
        gmdag.load_gmdag_asset(p)


def test_load_missing_file(tmp_path):
    with pytest.raises(FileNotFoundError, match="does not exist"):
        gmdag.load_gmdag_asset(tmp_path / "nope.gmdag")


@pytest.mark.parametrize(
    "nodes,match",
    [
        ([internal_word(0, 1), _leaf_node()], "has empty child mask"),
        ([internal_word(1, 1), 9], r"child reference out of range \(9\)"),
        ([internal_word(1, 5), _leaf_node()], "child pointer table starts beyond payload"),
        ([internal_word(0b1, 1), 0], "cycle detected at node index 0"),
        ([internal_word(0b11, 1), 2], "child pointer table exceeds payload bounds"),
    ],
)
def test_layout_validation(tmp_path, nodes, match):
    p = _write(tmp_path / "layout.gmdag", nodes=nodes)
    with pytest.raises(RuntimeError, match=match):
        gmdag.load_gmdag_asset(p)
    gmdag.load_gmdag_asset(p, validate_layout=False)  # runtime loads skip the deep check


def test_validator_accepts_shared_subtrees():
    # two octants share one leaf: a DAG, not a tree
    w = np.array([internal_word(0b11, 1), 3, 3, leaf_word(0.5, 1)], np.uint64)
    gmdag.validate_gmdag_layout(w)


def test_write_then_load_round_trip(tmp_path):
    words = np.array([internal_word(0xFF, 1)] + list(range(9, 17)) + [leaf_word(0.25, s) for s in range(8)], np.uint64)
    p = gmdag.write_gmdag(tmp_path / "rt.gmdag", words, 32, (-1.5, 0.25, 3.0), 0.125)
    a = gmdag.load_gmdag_asset(p)
    assert p.stat().st_size == 32 + 8 * words.shape[0]
    assert a.resolution == 32 and a.voxel_size == 0.125
    assert a.bbox_min == (-1.5, 0.25, 3.0)
    assert a.bbox_max == (-1.5 + 4.0, 0.25 + 4.0, 3.0 + 4.0)
    assert np.array_equal(a.nodes, words)


def test_reference_half_conversion_quirks():
    # normal values truncate toward zero
    assert gmdag.half_from_float_ref(1.0) == 0x3C00
    assert gmdag.half_from_float_ref(0.1) == int(np.float16(0.0999755859375).view(np.uint16))
    # |x| in [2^-15, 2^-14): subnormal half
    assert gmdag.half_from_float_ref(2.0 ** -15) == 0x0200
    # below 2^-15 (zero included) the unsigned exponent wraps: +inf
    assert gmdag.half_from_float_ref(0.0) == 0x7C00
    assert gmdag.half_from_float_ref(1e-6) == 0x7C00
    assert gmdag.half_from_float_ref(70000.0) == 0x7C00


def _brute_force_dag(grid: np.ndarray, voxel: float) -> np.ndarray:
    """Direct restatement of compiler.cpp:579-674 on a tiny grid (recursion, full block scans)."""
    n = grid.shape[0]
    pool = [0]
    leaves: dict[int, int] = {}
    internals: dict[tuple, int] = {}

    def half(x: float) -> int:
        return gmdag.half_from_float_ref(float(np.float32(x)))

    def leaf(w: int) -> int:
        if w not in leaves:
            leaves[w] = len(pool)
            pool.append(w)
        return leaves[w]

    two = np.float32(voxel) * np.float32(2.0)

    def build(x, y, z, size):
        if size == 1:
            d = grid[z, y, x]
            return leaf((1 << 63) | ((1 if d < two else 0) << 16) | half(d))
        blk = grid[z:z + size, y:y + size, x:x + size]
        first = blk[0, 0, 0]
        if not np.any(np.abs(blk - first) > np.float32(1e-6)):
            return leaf((1 << 63) | ((1 if first < two else 0) << 16) | half(first))
        h = size // 2
        ext = np.float32(np.float32(h) * np.float32(voxel)) * np.float32(1.7321)
        mask, kids = 0, []
        for i in range(8):
            ox, oy, oz = (h if i & 1 else 0), (h if i & 2 else 0), (h if i & 4 else 0)
            if grid[z + oz:z + oz + h, y + oy:y + oy + h, x + ox:x + ox + h].min() > ext:
                continue
            kids.append(build(x + ox, y + oy, z + oz, h))
            mask |= 1 << i
        if mask == 0:
            return leaf((1 << 63) | half(blk.min()))
        key = (mask, tuple(kids))
        if key not in internals:
            p = len(pool)
            pool.append((mask << 55) | (p + 1))
            pool.extend(kids)
            internals[key] = p
        return internals[key]

    root = build(0, 0, 0, n)
    pool[0] = pool[root]
    return np.array(pool, np.uint64)


@pytest.mark.parametrize("res", [8, 16, 32])
def test_dag_stage_matches_brute_force_restatement(res):
    """The pyramid-accelerated DAG build equals a direct block-scan build on the same dense grid:
    the compiler's own SDF of a scene mesh, and synthetic grids with uniform blocks and void octants."""
    sc = scenes.make_scene(1, 0)
    grid, _bmin, _bmax, vox = gmdag.compute_sdf(sc.vertices, sc.triangles, res)
    assert np.array_equal(gmdag.compile_grid(grid, vox), _brute_force_dag(grid, vox))
    rng = np.random.default_rng(res)
    synth = rng.uniform(0.0, 3.0, size=(res, res, res)).astype(np.float32)
    synth[: res // 2, : res // 2, : res // 2] = np.float32(0.75)           # a uniform octant
    synth[res // 2:, res // 2:, :] = np.float32(50.0)                      # far-field (void) octants
    synth[0, 0, 0] = np.float32(0.0)                                       # exact zero -> +inf half
    synth[1, 1, 1] = np.float32(2.0 ** -15)                                # subnormal half
    for v in (0.25, 1.0):
        assert np.array_equal(gmdag.compile_grid(synth, v), _brute_force_dag(synth, v))


def test_full_compile_equals_sdf_then_dag_stages():
    sc = scenes.make_scene(1, 0)
    out = gmdag.compile_mesh(sc.vertices, sc.triangles, 32)
    grid, bmin, bmax, vox = gmdag.compute_sdf(sc.vertices, sc.triangles, 32)
    assert np.array_equal(out.nodes, gmdag.compile_grid(grid, vox))
    assert out.bbox_min == bmin and out.voxel_size == vox


def test_compiler_bounds_rule_and_determinism():
    sc = scenes.make_scene(1, 0)
    a = gmdag.compile_mesh(sc.vertices, sc.triangles, 64)
    b = gmdag.compile_mesh(sc.vertices, sc.triangles, 64, threads=1)
    assert np.array_equal(a.nodes, b.nodes), "thread count must not change the words"
    v = sc.vertices
    ext = float(np.max(v.max(0) - v.min(0)))
    assert a.voxel_size == pytest.approx((ext + 2.0) / 64, rel=1e-6)
    assert a.bbox_min[0] == pytest.approx(float(v[:, 0].min() + v[:, 0].max()) / 2 - (ext + 2) / 2, abs=1e-5)
    gmdag.validate_gmdag_layout(a.nodes)


def test_compiled_scene_cache_round_trip(tmp_path, monkeypatch):
    monkeypatch.setenv("NAVI_SCENE_CACHE", str(tmp_path))
    cs = workloads.compiled_scene(1, 0, resolution=32)
    assert cs.path.exists()
    again = workloads.compiled_scene(1, 0, resolution=32)
    assert np.array_equal(cs.words, again.words)
    assert cs.hit_epsilon == pytest.approx(1e-3 * cs.voxel_size, rel=1e-6)
