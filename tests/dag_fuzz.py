"""Random .gmdag DAGs and rays for differential tests against the oracle."""

from __future__ import annotations

import numpy as np

from tests.kat_cases import internal_word


def _half_bits(rng: np.random.Generator) -> int:
    kind = rng.integers(0, 10)
    if kind == 0:
        return 0x0000  # +0
    if kind == 1:
        return 0x7C00  # +inf (the compiler's encoding of tiny distances)
    if kind == 2:
        return int(rng.integers(1, 0x0400))  # subnormal
    if kind == 3:
        return int(np.float16(rng.uniform(0.0, 0.02)).view(np.uint16))  # near the hit threshold
    return int(np.float16(rng.uniform(0.0, 0.4)).view(np.uint16))


def random_dag(rng: np.random.Generator, depth: int, *, p_leaf: float = 0.3, p_void: float = 0.25,
               share: float = 0.2, big_semantics: bool = True) -> np.ndarray:
    """Post-order words like the compiler's: node word followed by its child table; word 0 = root copy."""
    pool: list[int] = [0]
    made: list[int] = []  # indices of internal nodes built so far (for sharing)

    def leaf() -> int:
        sem = int(rng.integers(0, 4))
        if big_semantics and rng.random() < 0.1:
            sem = int(rng.integers(0x7FFF, 0x10000))
        w = (1 << 63) | (sem << 16) | _half_bits(rng)
        pool.append(w)
        return len(pool) - 1

    def build(level: int) -> int:
        if level >= depth or rng.random() < p_leaf * (0.5 if level < 2 else 1.0):
            return leaf()
        if made and rng.random() < share:
            return int(made[rng.integers(0, len(made))])
        mask = 0
        kids = []
        for o in range(8):
            if rng.random() < p_void:
                continue
            kids.append(build(level + 1))
            mask |= 1 << o
        if mask == 0:
            return leaf()
        p = len(pool)
        pool.append(internal_word(mask, p + 1))
        pool.extend(kids)
        made.append(p)
        return p

    root = build(0)
    pool[0] = pool[root]
    return np.array(pool, dtype=np.uint64)


def grid_lines(lo: float, hi: float, depth: int) -> np.ndarray:
    """The reference's midpoint-rule lines in float32 (kernel.cu:166-176)."""
    n = 1 << depth
    b = np.zeros(n + 1, np.float32)
    b[0] = np.float32(lo)
    b[n] = np.float32(hi)
    for lvl in range(depth):
        stride = n >> lvl
        for a in range(0, n, stride):
            b[a + stride // 2] = (b[a] + b[a + stride]) * np.float32(0.5)
    return b


def random_rays(rng: np.random.Generator, n: int, bmin, bmax, depth: int):
    bmin = np.asarray(bmin, np.float32)
    bmax = np.asarray(bmax, np.float32)
    ext = bmax - bmin
    o = (bmin + rng.uniform(-0.2, 1.2, size=(n, 3)) * ext).astype(np.float32)
    # a third of the rays start exactly on grid lines of random levels, some on the box faces
    lines = [grid_lines(float(bmin[a]), float(bmax[a]), max(depth, 1)) for a in range(3)]
    sel = rng.random(n) < 0.33
    for a in range(3):
        on = sel & (rng.random(n) < 0.7)
        idx = rng.integers(0, lines[a].shape[0], size=n)
        o[on, a] = lines[a][idx[on]]
    d = rng.normal(size=(n, 3)).astype(np.float32)
    axis = rng.random(n) < 0.3
    k = rng.integers(0, 3, size=n)
    d[axis] = 0.0
    d[axis, k[axis]] = np.where(rng.random(int(axis.sum())) < 0.5, 1.0, -1.0)
    d /= np.linalg.norm(d, axis=1, keepdims=True).astype(np.float32)
    return np.ascontiguousarray(o), np.ascontiguousarray(d.astype(np.float32))
