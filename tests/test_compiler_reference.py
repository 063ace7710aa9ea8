"""The in-tree scene compiler against the reference compiler (projects/voxel-dag/src/compiler.cpp).

tests/golden/compiler_golden.json holds hashes of the reference compiler's
output for the test scenes, made by tests/golden/make_compiler_golden.py
(reference built by oracle/build.py with the Assimp stand-in).  When that
build is present, one more scene is compared live.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from navi_b200 import gmdag, scenes

GOLDEN = json.loads((Path(__file__).parent / "golden" / "compiler_golden.json").read_text())


@pytest.mark.parametrize("key", sorted(GOLDEN))
def test_compiler_words_equal_reference_compiler(key):
    cfg, scene, res = (int(x[1:]) for x in key.split("_"))
    sc = scenes.make_scene(cfg, scene)
    out = gmdag.compile_mesh(sc.vertices, sc.triangles, res)
    g = GOLDEN[key]
    assert out.nodes.shape[0] == g["n_words"]
    assert hashlib.sha256(out.nodes.tobytes()).hexdigest() == g["words_sha256"]
    assert list(out.bbox_min) == g["bbox_min"]
    assert out.voxel_size == g["voxel_size"]


def test_live_reference_compiler_cross_check():
    from oracle import build as OB

    if not (OB.REF_OUT / "ref_voxel_dag").exists():
        pytest.skip("reference compiler not built here")
    import importlib.util

    spec = importlib.util.spec_from_file_location("mkg", Path(__file__).parent / "golden" / "make_compiler_golden.py")
    mkg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mkg)
    ref = mkg.reference_compile(3, 2, 64)
    sc = scenes.make_scene(3, 2)
    out = gmdag.compile_mesh(sc.vertices, sc.triangles, 64)
    assert np.array_equal(ref.nodes, out.nodes)
    assert ref.bbox_min == tuple(float(x) for x in out.bbox_min)
