"""Golden hashes of the reference scene compiler's output (run here, committed).

    python tests/golden/make_compiler_golden.py

Builds each test scene's mesh, writes it as OBJ (%.9g, which strtof reads back
exactly), compiles it with the reference compiler (projects/voxel-dag/src/
compiler.cpp built by oracle/build.py against the Assimp stand-in) and records
the SHA-256 of the header and of the node words in compiler_golden.json.
"""

from __future__ import annotations

import hashlib
import json
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from navi_b200 import gmdag, scenes  # noqa: E402
from oracle import build as OB  # noqa: E402

CASES = [(1, 0, 64), (1, 0, 128), (2, 0, 128), (3, 0, 64), (3, 1, 64), (2, 0, 512)]


def write_obj(path: Path, sc: scenes.Scene) -> None:
    with path.open("w") as f:
        for v in sc.vertices:
            f.write("v %.9g %.9g %.9g\n" % (float(v[0]), float(v[1]), float(v[2])))
        for t in sc.triangles:
            f.write("f %d %d %d\n" % (t[0] + 1, t[1] + 1, t[2] + 1))


def reference_compile(config: int, scene: int, res: int) -> gmdag.GmDagAsset:
    exe = OB.REF_OUT / "ref_voxel_dag"
    if not exe.exists():
        raise RuntimeError("reference compiler not built (python oracle/build.py with the reference tree)")
    sc = scenes.make_scene(config, scene)
    with tempfile.TemporaryDirectory() as td:
        obj = Path(td) / "m.obj"
        out = Path(td) / "m.gmdag"
        write_obj(obj, sc)
        r = subprocess.run([str(exe), str(obj), str(out), str(res)], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(r.stderr)
        return gmdag.load_gmdag_asset(out, validate_layout=False)


def digest(asset: gmdag.GmDagAsset) -> dict:
    return {
        "words_sha256": hashlib.sha256(asset.nodes.tobytes()).hexdigest(),
        "n_words": int(asset.nodes.shape[0]),
        "bbox_min": list(asset.bbox_min),
        "voxel_size": asset.voxel_size,
    }


def main() -> None:
    OB.build_reference_compiler()
    out = {f"c{c}_s{s}_r{r}": digest(reference_compile(c, s, r)) for c, s, r in CASES}
    (HERE / "compiler_golden.json").write_text(json.dumps(out, indent=1) + "\n")
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
