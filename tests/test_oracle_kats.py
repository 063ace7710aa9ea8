"""The CPU oracle against the reference's own known-answer values
(projects/torch-sdf/tests/test_sphere_tracing.py:683-949)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests.kat_cases import kat_cases, leaf_word, manual_octree_reference

CASES = kat_cases()


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
@pytest.mark.parametrize("fma", [True, False])
def test_oracle_matches_reference_known_answers(case, fma):
    r = O.trace(case.dag, case.bbox_min, case.bbox_max, np.array(case.origins), np.array(case.dirs),
                max_steps=case.max_steps, max_distance=case.max_distance, fma=fma)
    case.check(r["dist"], r["sem"])


def test_oracle_step_counts_follow_the_loop_index():
    # hit at loop index 0 -> 1 step; bounded miss with max_steps=3 -> 3 steps;
    # outside the domain: 1000 jump breaks the horizon at index 0 -> 1 step
    hit = O.trace(np.array([leaf_word(0.005, 11)], np.uint64), (0, 0, 0), (1, 1, 1), [(0.5, 0.5, 0.5)],
                  [(0, 1, 0)], max_steps=4, max_distance=10.0)
    assert hit["steps"][0] == 1
    acc = O.trace(np.array([leaf_word(0.25, 4)], np.uint64), (0, 0, 0), (1, 1, 1), [(0.5, 0.5, 0.5)],
                  [(1, 0, 0)], max_steps=3, max_distance=10.0)
    assert acc["steps"][0] == 3
    out = O.trace(np.array([leaf_word(0.005, 9)], np.uint64), (0, 0, 0), (1, 1, 1), [(2.0, 0.5, 0.5)],
                  [(1, 0, 0)], max_steps=8, max_distance=2.0)
    assert out["steps"][0] == 1 and out["dist"][0] == np.float32(1000.0)


def test_oracle_point_query_matches_manual_octree_reference():
    case = [c for c in CASES if c.name == "octant_semantics"][0]
    rng = np.random.default_rng(0)
    for p in rng.uniform(-0.1, 1.1, size=(200, 3)):
        got = O.point_query(case.dag, (0, 0, 0), (1, 1, 1), p.astype(np.float32))
        exp = manual_octree_reference(case.dag, tuple(float(v) for v in p.astype(np.float32)), (0, 0, 0), (1, 1, 1))
        assert got[1] == exp[1]
        assert np.float32(got[0]) == np.float32(exp[0])


def test_oracle_half_decode_is_exact_for_every_half():
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([O.half_to_float(int(b)) for b in bits[::97]], dtype=np.float32)
    exp = ref[::97]
    nan = np.isnan(exp)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), exp[~nan].view(np.uint32))


def test_oracle_counts_dag_word_loads():
    # octant root: word 0 (node) + word 1+oct (child pointer) + leaf word = 3 loads, then a hit
    case = [c for c in CASES if c.name == "octant_semantics"][0]
    r = O.trace(case.dag, (0, 0, 0), (1, 1, 1), np.array(case.origins), np.array(case.dirs), max_steps=4,
                max_distance=10.0)
    assert list(r["loads"]) == [3] * 8


def test_oracle_rejects_out_of_range_child_reference():
    dag = np.array([((1 << 0) << 55) | 1, 5], np.uint64)  # child index 5 >= 2 words
    with pytest.raises(RuntimeError, match="outside the payload"):
        O.trace(dag, (0, 0, 0), (1, 1, 1), [(0.1, 0.1, 0.1)], [(1, 0, 0)], max_steps=2, max_distance=5.0)
