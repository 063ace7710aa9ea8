"""Seeded synthetic scenes and poses for the benchmark configurations.

The reference measures on downloaded scene corpora (ReplicaCAD, Habitat,
Quake3 maps) that are not available here.  These scenes stand in for them:
rooms (floor plus four walls) filled with random axis-aligned boxes, spheres
and thin rods, tessellated into triangles and compiled to ``.gmdag`` by
:mod:`navi_b200.gmdag` exactly as the voxel-dag compiler would compile the
same mesh.  Every random draw comes from ``numpy.random.Generator(PCG64(seed))``
with ``seed = 1000 * config + scene``.

The analytic primitive list is kept next to the mesh; poses are sampled where
the analytic unsigned distance to every primitive exceeds a clearance
(0.5 m), by rejection.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

__all__ = [
    "CONFIGS",
    "SceneSpec",
    "Scene",
    "TraceConfig",
    "make_scene",
    "sample_free_poses",
    "random_walk_poses",
    "analytic_distance",
]


@dataclass(frozen=True)
class SceneSpec:
    cube: float
    n_prims: tuple[int, int]  # inclusive range of box+sphere count
    n_rods: int = 0
    box_side: tuple[float, float] = (0.2, 2.0)
    sphere_radius: tuple[float, float] = (0.1, 1.0)
    rod_radius: tuple[float, float] = (0.02, 0.05)
    rod_length: tuple[float, float] = (1.0, 10.0)
    n_boxes: int | None = None  # fixed split (configs 1-2); None = random split
    walls: bool = True


@dataclass(frozen=True)
class TraceConfig:
    index: int
    name: str
    scene: SceneSpec
    n_scenes: int
    resolution: int
    actors: int
    azimuth_bins: int
    elevation_bins: int
    max_steps: int
    max_distance: float
    pitch_deg: float  # poses draw pitch from U[-pitch_deg, pitch_deg]
    random_walk: bool = False

    @property
    def rays_per_actor(self) -> int:
        return self.azimuth_bins * self.elevation_bins

    @property
    def rays(self) -> int:
        return self.actors * self.rays_per_actor


_ROOM_10 = SceneSpec(cube=10.0, n_prims=(30, 30), n_boxes=20)
_ROOM_20 = SceneSpec(cube=20.0, n_prims=(90, 90), n_boxes=60)
_ROOM_20_RODS = SceneSpec(cube=20.0, n_prims=(40, 120), n_rods=200)
_ROOM_40_RODS = SceneSpec(cube=40.0, n_prims=(500, 500), n_rods=2000)

# The five configurations of the benchmark definition.  Config 3 and 5 leave
# pitch unstated; they use pitch 0 (the reference's own fan has no pitch).
CONFIGS: dict[int, TraceConfig] = {
    1: TraceConfig(1, "c1_room10_128", _ROOM_10, 1, 128, 4, 64, 16, 128, 20.0, 15.0),
    2: TraceConfig(2, "c2_room20_512", _ROOM_20, 1, 512, 64, 256, 48, 256, 30.0, 15.0),
    3: TraceConfig(3, "c3_rods8x512", _ROOM_20_RODS, 8, 512, 4096, 128, 24, 256, 30.0, 0.0),
    4: TraceConfig(4, "c4_room40_2048", _ROOM_40_RODS, 1, 2048, 16, 1024, 256, 512, 60.0, 30.0),
    5: TraceConfig(5, "c5_rods16x512", _ROOM_20_RODS, 16, 512, 32768, 256, 48, 256, 30.0, 0.0,
                   random_walk=True),
}


@dataclass
class Scene:
    """Triangle mesh plus the analytic primitives it was tessellated from."""

    seed: int
    vertices: np.ndarray  # [V, 3] float32
    triangles: np.ndarray  # [T, 3] uint32
    boxes: np.ndarray = field(default_factory=lambda: np.zeros((0, 6), np.float64))  # min xyz, max xyz
    spheres: np.ndarray = field(default_factory=lambda: np.zeros((0, 4), np.float64))  # c xyz, r
    rods: np.ndarray = field(default_factory=lambda: np.zeros((0, 7), np.float64))  # p0, p1, r
    quads: np.ndarray = field(default_factory=lambda: np.zeros((0, 6), np.float64))  # axis-aligned rects as boxes
    cube: float = 0.0


class _Mesh:
    def __init__(self) -> None:
        self.v: list[np.ndarray] = []
        self.t: list[np.ndarray] = []
        self.n = 0

    def add(self, verts: np.ndarray, tris: np.ndarray) -> None:
        self.v.append(np.asarray(verts, dtype=np.float64))
        self.t.append(np.asarray(tris, dtype=np.int64) + self.n)
        self.n += int(verts.shape[0])

    def arrays(self) -> tuple[np.ndarray, np.ndarray]:
        v = np.concatenate(self.v).astype(np.float32)
        t = np.concatenate(self.t).astype(np.uint32)
        return np.ascontiguousarray(v), np.ascontiguousarray(t)


def _box_mesh(lo: np.ndarray, hi: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    x0, y0, z0 = lo
    x1, y1, z1 = hi
    v = np.array(
        [[x0, y0, z0], [x1, y0, z0], [x1, y1, z0], [x0, y1, z0],
         [x0, y0, z1], [x1, y0, z1], [x1, y1, z1], [x0, y1, z1]]
    )
    t = np.array(
        [[0, 2, 1], [0, 3, 2], [4, 5, 6], [4, 6, 7], [0, 1, 5], [0, 5, 4],
         [2, 3, 7], [2, 7, 6], [0, 4, 7], [0, 7, 3], [1, 2, 6], [1, 6, 5]]
    )
    return v, t


def _quad_mesh(corner: np.ndarray, u: np.ndarray, w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    v = np.array([corner, corner + u, corner + u + w, corner + w])
    return v, np.array([[0, 1, 2], [0, 2, 3]])


def _sphere_mesh(c: np.ndarray, r: float, n_lon: int = 24, n_lat: int = 12) -> tuple[np.ndarray, np.ndarray]:
    verts = [c + np.array([0.0, r, 0.0])]
    for i in range(1, n_lat):
        th = math.pi * i / n_lat
        for j in range(n_lon):
            ph = 2.0 * math.pi * j / n_lon
            verts.append(c + r * np.array([math.sin(th) * math.cos(ph), math.cos(th), math.sin(th) * math.sin(ph)]))
    verts.append(c - np.array([0.0, r, 0.0]))
    v = np.array(verts)
    tris = []
    for j in range(n_lon):
        tris.append([0, 1 + (j + 1) % n_lon, 1 + j])
    for i in range(n_lat - 2):
        a = 1 + i * n_lon
        b = a + n_lon
        for j in range(n_lon):
            j1 = (j + 1) % n_lon
            tris.append([a + j, a + j1, b + j])
            tris.append([a + j1, b + j1, b + j])
    last = len(verts) - 1
    a = 1 + (n_lat - 2) * n_lon
    for j in range(n_lon):
        tris.append([last, a + j, a + (j + 1) % n_lon])
    return v, np.array(tris)


def _rod_mesh(p0: np.ndarray, p1: np.ndarray, r: float, n_side: int = 8, seg_len: float = 0.25) -> tuple[np.ndarray, np.ndarray]:
    """Capped cylinder, split along its length so every triangle stays short."""
    axis = p1 - p0
    length = float(np.linalg.norm(axis))
    a = axis / length
    ref = np.array([1.0, 0.0, 0.0]) if abs(a[0]) < 0.9 else np.array([0.0, 1.0, 0.0])
    u = np.cross(a, ref)
    u /= np.linalg.norm(u)
    w = np.cross(a, u)
    n_seg = max(1, int(math.ceil(length / seg_len)))
    ring = [r * (math.cos(2 * math.pi * k / n_side) * u + math.sin(2 * math.pi * k / n_side) * w) for k in range(n_side)]
    verts = []
    for s in range(n_seg + 1):
        base = p0 + axis * (s / n_seg)
        verts.extend(base + off for off in ring)
    c0 = len(verts)
    verts.append(p0)
    verts.append(p1)
    tris = []
    for s in range(n_seg):
        a0 = s * n_side
        b0 = a0 + n_side
        for k in range(n_side):
            k1 = (k + 1) % n_side
            tris.append([a0 + k, a0 + k1, b0 + k])
            tris.append([a0 + k1, b0 + k1, b0 + k])
    top = n_seg * n_side
    for k in range(n_side):
        k1 = (k + 1) % n_side
        tris.append([c0, k1, k])
        tris.append([c0 + 1, top + k, top + k1])
    return np.array(verts), np.array(tris)


def make_scene(config: int | TraceConfig, scene: int = 0) -> Scene:
    """Build scene ``scene`` of configuration ``config`` (seed 1000*config + scene)."""
    cfg = CONFIGS[config] if isinstance(config, int) else config
    spec = cfg.scene
    seed = 1000 * cfg.index + scene
    rng = np.random.Generator(np.random.PCG64(seed))
    L = spec.cube
    mesh = _Mesh()
    quads = []
    if spec.walls:
        # floor (y = 0) and four walls, each L x L: the mesh's bounding box is the cube
        rects = [
            (np.array([0.0, 0.0, 0.0]), np.array([L, 0.0, 0.0]), np.array([0.0, 0.0, L])),
            (np.array([0.0, 0.0, 0.0]), np.array([0.0, L, 0.0]), np.array([0.0, 0.0, L])),
            (np.array([L, 0.0, 0.0]), np.array([0.0, L, 0.0]), np.array([0.0, 0.0, L])),
            (np.array([0.0, 0.0, 0.0]), np.array([L, 0.0, 0.0]), np.array([0.0, L, 0.0])),
            (np.array([0.0, 0.0, L]), np.array([L, 0.0, 0.0]), np.array([0.0, L, 0.0])),
        ]
        for corner, u, w in rects:
            mesh.add(*_quad_mesh(corner, u, w))
            lo = np.minimum(corner, corner + u + w)
            hi = np.maximum(corner, corner + u + w)
            quads.append(np.concatenate([lo, hi]))
    lo_n, hi_n = spec.n_prims
    n_prims = int(rng.integers(lo_n, hi_n + 1))
    n_boxes = spec.n_boxes if spec.n_boxes is not None else int(rng.integers(0, n_prims + 1))
    boxes, spheres, rods = [], [], []
    for _ in range(n_boxes):
        side = rng.uniform(spec.box_side[0], spec.box_side[1], size=3)
        centre = rng.uniform(side / 2, L - side / 2)
        lo = centre - side / 2
        hi = centre + side / 2
        mesh.add(*_box_mesh(lo, hi))
        boxes.append(np.concatenate([lo, hi]))
    for _ in range(n_prims - n_boxes):
        r = float(rng.uniform(spec.sphere_radius[0], spec.sphere_radius[1]))
        c = rng.uniform(r, L - r, size=3)
        mesh.add(*_sphere_mesh(c, r))
        spheres.append(np.array([*c, r]))
    for _ in range(spec.n_rods):
        r = float(rng.uniform(spec.rod_radius[0], spec.rod_radius[1]))
        length = float(rng.uniform(spec.rod_length[0], spec.rod_length[1]))
        d = rng.normal(size=3)
        d /= np.linalg.norm(d)
        p0 = rng.uniform(0.0, L, size=3)
        p1 = np.clip(p0 + d * length, r, L - r)
        p0 = np.clip(p0, r, L - r)
        if np.linalg.norm(p1 - p0) < 0.1:
            p1 = p0 + np.clip(d, -1, 1) * 0.1
        mesh.add(*_rod_mesh(p0, p1, r))
        rods.append(np.array([*p0, *p1, r]))
    v, t = mesh.arrays()
    return Scene(
        seed=seed,
        vertices=v,
        triangles=t,
        boxes=np.array(boxes).reshape(-1, 6),
        spheres=np.array(spheres).reshape(-1, 4),
        rods=np.array(rods).reshape(-1, 7),
        quads=np.array(quads).reshape(-1, 6),
        cube=L,
    )


def analytic_distance(scene: Scene, points: np.ndarray) -> np.ndarray:
    """Unsigned distance from points [P, 3] to the scene's primitives (float64)."""
    p = np.asarray(points, dtype=np.float64).reshape(-1, 3)
    best = np.full(p.shape[0], np.inf)

    def box_dist(lo: np.ndarray, hi: np.ndarray) -> np.ndarray:
        q = np.maximum(np.maximum(lo - p, p - hi), 0.0)
        outside = np.linalg.norm(q, axis=1)
        inside = np.minimum(np.min(p - lo, axis=1), np.min(hi - p, axis=1))
        return np.where(outside > 0.0, outside, np.maximum(inside, 0.0))

    for b in np.concatenate([scene.boxes, scene.quads]) if scene.quads.size or scene.boxes.size else []:
        best = np.minimum(best, box_dist(b[:3], b[3:]))
    for s in scene.spheres:
        best = np.minimum(best, np.abs(np.linalg.norm(p - s[:3], axis=1) - s[3]))
    for r in scene.rods:
        a, b, rad = r[:3], r[3:6], r[6]
        ab = b - a
        tt = np.clip(((p - a) @ ab) / max(float(ab @ ab), 1e-12), 0.0, 1.0)
        closest = a + tt[:, None] * ab
        best = np.minimum(best, np.abs(np.linalg.norm(p - closest, axis=1) - rad))
    return best


def sample_free_poses(
    scene: Scene,
    n: int,
    *,
    seed: int,
    clearance: float = 0.5,
    pitch_deg: float = 0.0,
) -> dict[str, np.ndarray]:
    """Uniform free-space positions (clearance from every primitive), yaw U[0, 2pi), pitch U[+-pitch_deg]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    L = scene.cube
    out = np.zeros((0, 3))
    while out.shape[0] < n:
        cand = rng.uniform(clearance, L - clearance, size=(max(4 * n, 64), 3))
        ok = analytic_distance(scene, cand) > clearance
        out = np.concatenate([out, cand[ok]])
    pos = out[:n].astype(np.float32)
    yaw = rng.uniform(0.0, 2.0 * math.pi, size=n).astype(np.float32)
    pitch = (
        rng.uniform(-math.radians(pitch_deg), math.radians(pitch_deg), size=n).astype(np.float32)
        if pitch_deg > 0
        else np.zeros(n, np.float32)
    )
    return {"position": pos, "yaw": yaw, "pitch": pitch}


def random_walk_poses(
    scenes: list[Scene],
    scene_ids: np.ndarray,
    poses: dict[str, np.ndarray],
    *,
    seed: int,
    step: float = 0.1,
    yaw_jitter_deg: float = 5.0,
    clearance: float = 0.5,
) -> dict[str, np.ndarray]:
    """One random-walk step: move 0.1 m in a random horizontal direction, jitter yaw by N(0, 5 deg);
    moves that would leave free space are rejected (the actor stays)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    pos = poses["position"].astype(np.float64)
    n = pos.shape[0]
    ang = rng.uniform(0.0, 2.0 * math.pi, size=n)
    cand = pos + step * np.stack([np.cos(ang), np.zeros(n), np.sin(ang)], axis=1)
    ok = np.zeros(n, dtype=bool)
    for s, sc in enumerate(scenes):
        sel = scene_ids == s
        if not np.any(sel):
            continue
        c = cand[sel]
        inside = np.all((c > clearance) & (c < sc.cube - clearance), axis=1)
        ok[sel] = inside & (analytic_distance(sc, c) > clearance)
    new_pos = np.where(ok[:, None], cand, pos).astype(np.float32)
    yaw = (poses["yaw"] + np.radians(rng.normal(0.0, yaw_jitter_deg, size=n))).astype(np.float32)
    yaw = np.mod(yaw, np.float32(2.0 * math.pi)).astype(np.float32)
    return {"position": new_pos, "yaw": yaw, "pitch": poses["pitch"].copy()}
