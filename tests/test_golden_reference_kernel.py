"""The CPU oracle against outputs of the reference's own CUDA kernel (no GPU needed).

tests/golden/trace_golden.npz was written on a B200 by
tests/golden/make_trace_golden.py, which ran the reference kernel.cu (built for
sm_100a from the reference sources) on config 1's full step and on the
known-answer cases.  Bit-exact: distances as bit patterns, semantics as integers.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest

from navi_b200 import scenes, workloads
from oracle import oracle as O
from tests.kat_cases import kat_cases

GOLDEN = Path(__file__).parent / "golden" / "trace_golden.npz"
pytestmark = pytest.mark.skipif(not GOLDEN.exists(), reason="golden file not generated yet")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("tag", ["ref001", "refeps"])
def test_oracle_equals_reference_kernel_on_config1(golden, tag):
    cfg = scenes.CONFIGS[1]
    cs = workloads.compiled_scene(1)
    assert hashlib.sha256(cs.words.tobytes()).digest() == golden["c1_words_sha256"].tobytes()
    eps = 0.01 if tag == "ref001" else float(golden["c1_eps_config"][0])
    r = O.trace(cs.words, golden["c1_bbox_min"], golden["c1_bbox_max"], golden["c1_origins"], golden["c1_dirs"],
                max_steps=cfg.max_steps, max_distance=cfg.max_distance, hit_epsilon=eps)
    assert np.array_equal(r["dist"].view(np.uint32), golden[f"c1_{tag}_dist"].view(np.uint32))
    assert np.array_equal(r["sem"], golden[f"c1_{tag}_sem"])


def test_two_rounding_position_update_does_not_match(golden):
    """The reference build evaluates o + t*d with one rounding (a fused multiply-add)."""
    cfg = scenes.CONFIGS[1]
    cs = workloads.compiled_scene(1)
    r = O.trace(cs.words, golden["c1_bbox_min"], golden["c1_bbox_max"], golden["c1_origins"], golden["c1_dirs"],
                max_steps=cfg.max_steps, max_distance=cfg.max_distance, hit_epsilon=0.01, fma=False)
    assert not np.array_equal(r["dist"].view(np.uint32), golden["c1_ref001_dist"].view(np.uint32))


@pytest.mark.parametrize("case", kat_cases(), ids=lambda c: c.name)
def test_oracle_equals_reference_kernel_on_known_answers(golden, case):
    r = O.trace(case.dag, case.bbox_min, case.bbox_max, np.array(case.origins), np.array(case.dirs),
                max_steps=case.max_steps, max_distance=case.max_distance)
    assert np.array_equal(r["dist"].view(np.uint32), golden[f"kat_{case.name}_dist"].view(np.uint32))
    assert np.array_equal(r["sem"], golden[f"kat_{case.name}_sem"])
