"""Known-answer DAGs and rays of the reference's native tests.

Restates the DAG builders and cases of
projects/torch-sdf/tests/test_sphere_tracing.py:26-178 (builders, point-query
reference) and :683-949 (native known-answer tests): the same words, rays,
arguments and expected values.  Shared by the oracle tests (CPU) and the
kernel tests (GPU).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable

import numpy as np


def leaf_word(distance: float, semantic: int = 0) -> int:
    bits = int(np.asarray([distance], dtype=np.float16).view(np.uint16)[0])
    return (1 << 63) | ((semantic & 0xFFFF) << 16) | bits


def internal_word(mask: int, child_base: int) -> int:
    return ((mask & 0xFF) << 55) | (child_base & 0xFFFFFFFF)


def words(values: list[int]) -> np.ndarray:
    return np.asarray(values, dtype=np.uint64)


def point_for_octant_path(octants, bbox_min, bbox_max):
    lo, hi = list(bbox_min), list(bbox_max)
    for octant in octants:
        mid = [(lo[a] + hi[a]) * 0.5 for a in range(3)]
        for a in range(3):
            if octant & (1 << a):
                lo[a] = mid[a]
            else:
                hi[a] = mid[a]
    return tuple((lo[a] + hi[a]) * 0.5 for a in range(3))


def single_path_dag_words(octants, *, distance, semantic) -> np.ndarray:
    out: list[int] = []
    slots: list[int] = []
    for depth, octant in enumerate(octants):
        ptr = len(out) + 1
        out.append(internal_word(1 << octant, ptr))
        out.append(0)
        slots.append(ptr)
        if depth > 0:
            out[slots[depth - 1]] = ptr - 1
    leaf = len(out)
    if slots:
        out[slots[-1]] = leaf
    out.append(leaf_word(distance, semantic))
    return words(out)


def prefixed_uniform_leaf_dag_words(prefix, *, distance, semantic) -> np.ndarray:
    out: list[int] = []
    slots: list[int] = []
    for depth, octant in enumerate(prefix):
        ptr = len(out) + 1
        out.append(internal_word(1 << octant, ptr))
        out.append(0)
        slots.append(ptr)
        if depth > 0:
            out[slots[depth - 1]] = ptr - 1
    ptr = len(out) + 1
    out.append(internal_word(0xFF, ptr))
    out.extend(0 for _ in range(8))
    if slots:
        out[slots[-1]] = ptr - 1
    base = len(out)
    for k in range(8):
        out[ptr + k] = base + k
    out.extend(leaf_word(distance, semantic) for _ in range(8))
    return words(out)


def manual_octree_reference(dag, origin, bbox_min, bbox_max) -> tuple[float, int]:
    """Point query of test_sphere_tracing.py:121-178 (no caches, float64 midpoints)."""
    px, py, pz = origin
    if px < bbox_min[0] or px > bbox_max[0] or py < bbox_min[1] or py > bbox_max[1] or pz < bbox_min[2] or pz > bbox_max[2]:
        return 1000.0, 0
    idx = 0
    lo, hi = list(bbox_min), list(bbox_max)
    while True:
        node = int(dag[idx])
        if (node >> 63) == 1:
            d = float(np.array([node & 0xFFFF], dtype=np.uint16).view(np.float16)[0])
            return d, int((node >> 16) & 0xFFFF)
        mid = [(lo[a] + hi[a]) * 0.5 for a in range(3)]
        p = (px, py, pz)
        octant = sum((1 << a) for a in range(3) if p[a] >= mid[a])
        for a in range(3):
            if p[a] >= mid[a]:
                lo[a] = mid[a]
            else:
                hi[a] = mid[a]
        mask = (node >> 55) & 0xFF
        if (mask & (1 << octant)) == 0:
            return 1000.0, 0
        base = node & 0xFFFFFFFF
        idx = int(dag[base + int((mask & ((1 << octant) - 1)).bit_count())])


@dataclass
class Kat:
    name: str
    dag: np.ndarray
    origins: list
    dirs: list
    max_steps: int
    max_distance: float
    bbox_min: tuple = (0.0, 0.0, 0.0)
    bbox_max: tuple = (1.0, 1.0, 1.0)
    resolution: int = 1
    # check(dist: np.ndarray, sem: np.ndarray) -> None ; raises AssertionError
    check: Callable = field(default=lambda d, s: None)


def _approx(a, b, tol):
    assert abs(float(a) - float(b)) <= tol, (a, b, tol)


def kat_cases() -> list[Kat]:
    cases: list[Kat] = []

    def outside(d, s):  # :683-694
        assert int(s[0]) == 0 and float(d[0]) > 2.0

    cases.append(Kat("outside_domain_miss", words([leaf_word(0.005, 9)]), [(2.0, 0.5, 0.5)], [(1.0, 0.0, 0.0)],
                     8, 2.0, check=outside))

    def bounded(d, s):  # :697-710
        assert int(s[0]) == 0
        _approx(d[0], 0.5, 1e-5)

    cases.append(Kat("bounded_miss_max_steps", words([leaf_word(0.5, 7)]), [(0.5, 0.5, 0.5)], [(1.0, 0.0, 0.0)],
                     1, 10.0, check=bounded))

    def accumulate(d, s):  # :713-726
        _approx(d[0], 0.75, 1e-5)
        assert int(s[0]) == 0

    cases.append(Kat("accumulate_three_steps", words([leaf_word(0.25, 4)]), [(0.5, 0.5, 0.5)], [(1.0, 0.0, 0.0)],
                     3, 10.0, check=accumulate))

    def hit(sem):
        def f(d, s):  # :729-742, :745-765
            _approx(d[0], 0.0, 1e-6)
            assert int(s[0]) == sem
        return f

    cases.append(Kat("hit_below_epsilon", words([leaf_word(0.005, 11)]), [(0.5, 0.5, 0.5)], [(0.0, 1.0, 0.0)],
                     4, 10.0, check=hit(11)))
    cases.append(Kat("overwrite_first_call", words([leaf_word(0.005, 3)]), [(0.5, 0.5, 0.5)], [(0.0, 1.0, 0.0)],
                     4, 10.0, check=hit(3)))
    cases.append(Kat("overwrite_second_call", words([leaf_word(0.5, 9)]), [(0.5, 0.5, 0.5)], [(0.0, 1.0, 0.0)],
                     1, 10.0, check=bounded))

    # :783-823 octant semantics from a manual root
    root_dag = words([internal_word(0xFF, 1)] + list(range(9, 17)) + [leaf_word(0.005, s) for s in range(1, 9)])
    octant_origins = [(0.25, 0.25, 0.25), (0.75, 0.25, 0.25), (0.25, 0.75, 0.25), (0.75, 0.75, 0.25),
                      (0.25, 0.25, 0.75), (0.75, 0.25, 0.75), (0.25, 0.75, 0.75), (0.75, 0.75, 0.75)]

    def octants(d, s):
        expected = [manual_octree_reference(root_dag, o, (0, 0, 0), (1, 1, 1)) for o in octant_origins]
        for i in range(8):
            _approx(d[i], 0.0, 1e-6)
        assert [int(v) for v in s] == [sem for _dist, sem in expected] == list(range(1, 9))

    cases.append(Kat("octant_semantics", root_dag, octant_origins, [(1.0, 0.0, 0.0)] * 8, 4, 10.0, resolution=2,
                     check=octants))

    # :826-877 sparse child mask offsets
    mask = (1 << 1) | (1 << 3) | (1 << 6)
    sparse = words([internal_word(mask, 1), 4, 5, 6, leaf_word(0.005, 11), leaf_word(0.005, 33),
                    leaf_word(0.005, 66)])
    sparse_origins = [(0.75, 0.25, 0.25), (0.75, 0.75, 0.25), (0.25, 0.75, 0.75), (0.25, 0.25, 0.25)]

    def sparse_check(d, s):
        exp = [manual_octree_reference(sparse, o, (0, 0, 0), (1, 1, 1)) for o in sparse_origins[:3]]
        for i in range(3):
            _approx(d[i], 0.0 if exp[i][0] < 0.01 else exp[i][0], 1e-6)
            assert int(s[i]) == (exp[i][1] if exp[i][0] < 0.01 else 0)
        assert [int(v) for v in s[:3]] == [11, 33, 66]
        assert int(s[3]) == 0 and float(d[3]) > 10.0

    cases.append(Kat("sparse_mask_offsets", sparse, sparse_origins, [(0.0, 1.0, 0.0)] * 4, 4, 10.0, resolution=2,
                     check=sparse_check))

    # :880-902 deep single path across repeated steps (prefix cache)
    prefix = [0, 1, 1, 1]
    deep = prefixed_uniform_leaf_dag_words(prefix, distance=0.015, semantic=23)
    deep_origin = point_for_octant_path(prefix + [0], (0.0, 0.0, 0.0), (1.0, 1.0, 1.0))

    def deep_check(d, s):
        _approx(d[0], 0.045, 2e-5)
        assert int(s[0]) == 0

    cases.append(Kat("deep_prefix_path", deep, [deep_origin], [(1.0, 0.0, 0.0)], 3, 1.0, resolution=32,
                     check=deep_check))

    # :905-923 deep leaf payload reuse (leaf cache)
    octs = [0, 1, 1, 1, 0]
    reuse = single_path_dag_words(octs, distance=0.012, semantic=19)
    reuse_origin = point_for_octant_path(octs, (0.0, 0.0, 0.0), (1.0, 1.0, 1.0))

    def reuse_check(d, s):
        _approx(d[0], 0.024, 2e-5)
        assert int(s[0]) == 0

    cases.append(Kat("deep_leaf_reuse", reuse, [reuse_origin], [(0.0, 0.0, 1.0)], 2, 1.0, resolution=32,
                     check=reuse_check))

    # :926-949 void macro-cell advance
    void_dag = words([internal_word(1 << 7, 1), 2, leaf_word(0.005, 17)])

    def void_check(d, s):
        _approx(d[0], 0.75, 1e-4)
        assert int(s[0]) == 0

    cases.append(Kat("void_advance", void_dag, [(0.25, 0.25, 0.25)], [(1.0, 0.0, 0.0)], 2, 10.0, resolution=2,
                     check=void_check))

    # :234-254 all-zero DAG contract (no expected values; must not fault)
    cases.append(Kat("zero_dag_contract", np.zeros(100, np.uint64), [(0.0, 0.0, 0.0)] * 4,
                     [(1.0, 0.0, 0.0)] * 4, 64, 30.0, resolution=128))
    return cases
