"""The C++ .gmdag reader and layout validator (libnavi_gmdag.so) against the literal
restatement of the reference's Python (oracle/gmdag_ref.py, voxel_dag.py:29-78, :193-259):
same outcome, same exception type and the same first message, on fuzzed DAGs and
malformed files (odd magic bytes, float formatting of the voxel size, short payloads).
"""

from __future__ import annotations

import struct

import numpy as np
import pytest

from navi_b200 import gmdag
from oracle import gmdag_ref
from tests.dag_fuzz import random_dag

_HEADER = struct.Struct("<4sIIffffI")


def _outcome(fn, *args, **kw):
    try:
        return ("ok", fn(*args, **kw))
    except (RuntimeError, FileNotFoundError) as e:
        return (type(e).__name__, str(e))


def _corrupt(rng, words):
    w = words.copy()
    n = w.shape[0]
    kind = rng.integers(0, 6)
    i = int(rng.integers(0, n))
    internal = np.nonzero((w >> np.uint64(63)) == 0)[0]
    if kind == 0 and internal.size:  # empty mask
        j = int(rng.choice(internal))
        w[j] = w[j] & np.uint64(0x007FFFFFFFFFFFFF)
    elif kind == 1 and internal.size:  # table beyond the payload
        j = int(rng.choice(internal))
        w[j] = (w[j] & np.uint64(0xFFFFFFFF00000000)) | np.uint64(n + int(rng.integers(0, 5)))
    elif kind == 2 and internal.size:  # table running past the end
        j = int(rng.choice(internal))
        w[j] = (w[j] & np.uint64(0xFFFFFFFF00000000)) | np.uint64(n - 1)
    elif kind == 3:  # child reference out of range (including a leaf word used as a pointer)
        w[i] = np.uint64(n + int(rng.integers(0, 1000))) if rng.random() < 0.5 else np.uint64(1 << 63)
    elif kind == 4 and internal.size:  # cycle back to the root or to an ancestor
        j = int(rng.choice(internal))
        base = int(w[j] & np.uint64(0xFFFFFFFF))
        if base < n:
            w[base] = np.uint64(0 if rng.random() < 0.5 else j)
    else:
        w[i] = np.uint64(int(rng.integers(0, 2**63)))
    return w


@pytest.mark.parametrize("seed", range(40))
def test_validator_first_error_equals_reference(seed):
    rng = np.random.default_rng(seed)
    words = random_dag(rng, depth=int(rng.integers(1, 6)))
    for _ in range(5):
        w = _corrupt(rng, words) if rng.random() < 0.85 else words
        want = _outcome(gmdag_ref.validate_layout, w)
        got = _outcome(gmdag.validate_gmdag_layout, w)
        assert got[0] == want[0] and (got[0] == "ok" or got[1] == want[1]), (got, want)


def test_validator_empty_payload():
    w = np.zeros(0, np.uint64)
    assert _outcome(gmdag.validate_gmdag_layout, w) == _outcome(gmdag_ref.validate_layout, w)


def _write(path, magic=b"GDAG", version=1, res=32, bmin=(0.0, 0.0, 0.0), voxel=1.0, nodes=(1 << 63,), count=None,
           extra=b""):
    nodes = np.asarray(nodes, dtype=np.uint64)
    n = nodes.shape[0] if count is None else count
    path.write_bytes(_HEADER.pack(magic, version, res, *bmin, voxel, n) + nodes.tobytes() + extra)
    return path


CASES = [
    dict(magic=b"GDAX"), dict(magic=b"\x00\x01'\""), dict(magic=b"a'bc"), dict(magic=b'a"b\\'), dict(magic=b"\n\t\r\x7f"),
    dict(version=0), dict(version=2**32 - 1), dict(res=0),
    dict(voxel=0.0), dict(voxel=-0.0), dict(voxel=-1.5), dict(voxel=float("nan")), dict(voxel=float("inf")),
    dict(voxel=float("-inf")), dict(voxel=-1e-5), dict(voxel=-0.1), dict(voxel=-3.4e38), dict(voxel=-123456789.0),
    dict(voxel=-1e16), dict(voxel=-1e15), dict(voxel=-2.5e-7), dict(voxel=-1e-4), dict(voxel=-0.00012345),
    dict(count=0), dict(bmin=(0.0, float("nan"), 0.0)), dict(bmin=(float("-inf"), 0.0, 0.0)),
    dict(count=3), dict(extra=b"\x01"), dict(extra=b"\x00" * 12), dict(count=2, extra=b"\x00" * 4),
    dict(nodes=[0], count=1), dict(nodes=[(1 << 55) | 1, 5], count=2),
]


@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("validate", [True, False])
def test_loader_matches_reference_on_malformed_files(tmp_path, case, validate):
    p = _write(tmp_path / "scene.gmdag", **CASES[case])
    want = _outcome(gmdag_ref.load_asset, p, validate_layout_flag=validate)
    got = _outcome(gmdag.load_gmdag_asset, p, validate_layout=validate)
    assert got[0] == want[0], (got, want)
    if got[0] == "ok":
        a = got[1]
        v, r, bmin, bmax, vox, nodes = want[1]
        assert (a.version, a.resolution, a.bbox_min, a.bbox_max, a.voxel_size) == (v, r, bmin, bmax, vox)
        assert np.array_equal(a.nodes, nodes)
    else:
        assert got[1] == want[1]


def test_loader_short_header_and_missing_file(tmp_path):
    p = tmp_path / "short.gmdag"
    p.write_bytes(b"GDAG\x01\x00")
    assert _outcome(gmdag.load_gmdag_asset, p) == _outcome(gmdag_ref.load_asset, p)
    q = tmp_path / "nope" / "missing.gmdag"
    assert _outcome(gmdag.load_gmdag_asset, q) == _outcome(gmdag_ref.load_asset, q)


def test_loader_on_a_compiled_scene(tmp_path):
    from navi_b200 import scenes

    sc = scenes.make_scene(1, 0)
    out = gmdag.compile_mesh(sc.vertices, sc.triangles, 64)
    p = gmdag.write_gmdag(tmp_path / "c1.gmdag", out.nodes, 64, out.bbox_min, out.voxel_size)
    a = gmdag.load_gmdag_asset(p)
    v, r, bmin, bmax, vox, nodes = gmdag_ref.load_asset(p)
    assert (a.bbox_min, a.bbox_max, a.voxel_size) == (bmin, bmax, vox)
    assert np.array_equal(a.nodes, nodes)
