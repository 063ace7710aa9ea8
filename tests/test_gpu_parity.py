"""CUDA path vs the oracle and vs the reference's own kernel, bit for bit.

Tolerance: none.  Distances are compared as float32 bit patterns, semantics
and step counts as integers.  The CUDA path is called through the C ABI
(libnavi_tsdf.so) via navi_b200.tracer and the drop-in torch_sdf.cast_rays.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import torch_sdf
from navi_b200 import scenes, tracer, workloads
from oracle import oracle as O
from tests.gpu_util import assert_bits_equal, assert_equal, cast_explicit, dev, eager_world_rays
from tests.kat_cases import kat_cases

pytestmark = pytest.mark.gpu
CASES = kat_cases()


@pytest.fixture(params=["grid", "float"])
def descent(request):
    """Run a test under both descents of the library: integer grid (default) and float."""
    old = tracer.set_option("descent", 0 if request.param == "grid" else 1)
    yield request.param
    tracer.set_option("descent", old)


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_known_answers_through_cast_rays(case):
    d = dev()
    dag = torch.from_numpy(case.dag.view(np.int64)).to(d)
    o = torch.tensor([case.origins], dtype=torch.float32, device=d)
    v = torch.tensor([case.dirs], dtype=torch.float32, device=d)
    out_d = torch.full(o.shape[:2], -7.0, dtype=torch.float32, device=d)
    out_s = torch.full(o.shape[:2], -7, dtype=torch.int32, device=d)
    out_k = torch.full(o.shape[:2], -7, dtype=torch.int32, device=d)
    torch_sdf.cast_rays(dag, o, v, out_d, out_s, case.max_steps, case.max_distance, list(case.bbox_min),
                        list(case.bbox_max), case.resolution, out_steps=out_k)
    torch.cuda.synchronize()
    got_d = out_d.cpu().numpy()[0]
    got_s = out_s.cpu().numpy()[0]
    case.check(got_d, got_s)
    ref = O.trace(case.dag, case.bbox_min, case.bbox_max, np.array(case.origins), np.array(case.dirs),
                  max_steps=case.max_steps, max_distance=case.max_distance)
    assert_bits_equal(got_d, ref["dist"], "dist")
    assert_equal(got_s, ref["sem"], "sem")
    assert_equal(out_k.cpu().numpy()[0], ref["steps"], "steps")


@pytest.mark.skipif(not O.reference_available(), reason="reference kernel not built")
@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_known_answers_match_reference_kernel(case):
    d = dev()
    kern = O.ReferenceKernel()
    dag = torch.from_numpy(O.pad_words(case.dag).view(np.int64)).to(d)
    o = torch.tensor(case.origins, dtype=torch.float32, device=d)
    v = torch.tensor(case.dirs, dtype=torch.float32, device=d)
    rd = torch.empty(o.shape[0], dtype=torch.float32, device=d)
    rs = torch.empty(o.shape[0], dtype=torch.int32, device=d)
    kern.cast(dag, o, v, rd, rs, max_steps=case.max_steps, max_distance=case.max_distance,
              bbox_min=case.bbox_min, bbox_max=case.bbox_max, resolution=case.resolution)
    got_d, got_s, _ = cast_explicit(case.dag, case.origins, case.dirs, max_steps=case.max_steps,
                                    max_distance=case.max_distance, bbox_min=case.bbox_min, bbox_max=case.bbox_max)
    assert_bits_equal(got_d, rd.cpu().numpy(), "dist vs reference kernel")
    assert_equal(got_s, rs.cpu().numpy(), "sem vs reference kernel")


def _config_rays(config: int, scene: int = 0, actors: int | None = None, resolution: int | None = None):
    cs = workloads.compiled_scene(config, scene, resolution=resolution)
    pb = workloads.poses_for(config, [cs], actors=actors)
    fan = torch.from_numpy(workloads.fan_for(config)).to(dev())
    poses = tracer.make_poses(torch.from_numpy(pb.position).to(dev()), torch.from_numpy(pb.yaw).to(dev()),
                              torch.from_numpy(pb.pitch).to(dev()))
    o, v = eager_world_rays(fan, poses, pitch=True)
    return cs, fan, poses, o, v


@pytest.mark.parametrize("eps_rule", ["config", "reference_0.01"])
def test_config1_matches_oracle_and_reference_kernel(eps_rule, descent):
    cfg = scenes.CONFIGS[1]
    cs, fan, poses, o, v = _config_rays(1)
    eps = cs.hit_epsilon if eps_rule == "config" else 0.01
    got_d, got_s, got_k = cast_explicit(cs.words, o, v, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                                        bbox_min=cs.bbox_min, bbox_max=cs.bbox_max, hit_epsilon=eps)
    on, vn = o.cpu().numpy(), v.cpu().numpy()
    ref = O.trace(cs.words, cs.bbox_min, cs.bbox_max, on, vn, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                  hit_epsilon=eps, fma=True)
    assert_bits_equal(got_d, ref["dist"], "dist vs oracle")
    assert_equal(got_s, ref["sem"], "sem vs oracle")
    assert_equal(got_k, ref["steps"], "steps vs oracle")
    if not O.reference_available():
        pytest.skip("reference kernel not built")
    kern = O.ReferenceKernel(eps_variant=(eps_rule == "config"))
    dag = torch.from_numpy(O.pad_words(cs.words).view(np.int64)).to(dev())
    rd = torch.empty(got_d.shape[0], dtype=torch.float32, device=dev())
    rs = torch.empty(got_d.shape[0], dtype=torch.int32, device=dev())
    kern.cast(dag, o, v, rd, rs, max_steps=cfg.max_steps, max_distance=cfg.max_distance, bbox_min=cs.bbox_min,
              bbox_max=cs.bbox_max, resolution=cfg.resolution, hit_epsilon=eps)
    assert_bits_equal(got_d, rd.cpu().numpy(), "dist vs reference kernel")
    assert_equal(got_s, rs.cpu().numpy(), "sem vs reference kernel")


@pytest.mark.skipif(not O.reference_available(), reason="reference kernel not built")
def test_reference_kernel_position_update_is_fused():
    """Pins how the reference build evaluates o + t*d (kernel.cu:261-263): its outputs equal the
    oracle with a fused multiply-add and differ from the two-rounding form on this workload."""
    cfg = scenes.CONFIGS[1]
    cs, fan, poses, o, v = _config_rays(1)
    kern = O.ReferenceKernel()
    dag = torch.from_numpy(O.pad_words(cs.words).view(np.int64)).to(dev())
    n = o.shape[0] * o.shape[1]
    rd = torch.empty(n, dtype=torch.float32, device=dev())
    rs = torch.empty(n, dtype=torch.int32, device=dev())
    kern.cast(dag, o, v, rd, rs, max_steps=cfg.max_steps, max_distance=cfg.max_distance, bbox_min=cs.bbox_min,
              bbox_max=cs.bbox_max, resolution=cfg.resolution)
    on, vn = o.cpu().numpy(), v.cpu().numpy()
    fused = O.trace(cs.words, cs.bbox_min, cs.bbox_max, on, vn, max_steps=cfg.max_steps,
                    max_distance=cfg.max_distance, fma=True)
    unfused = O.trace(cs.words, cs.bbox_min, cs.bbox_max, on, vn, max_steps=cfg.max_steps,
                      max_distance=cfg.max_distance, fma=False)
    ref_d = rd.cpu().numpy()
    assert_bits_equal(ref_d, fused["dist"], "reference kernel vs fused-update oracle")
    n_diff = int(np.sum(ref_d.view(np.uint32) != unfused["dist"].view(np.uint32)))
    print(f"two-rounding oracle differs on {n_diff} of {n} rays")
    assert n_diff > 0


def test_fan_matches_explicit_rays_bitwise():
    cfg = scenes.CONFIGS[1]
    cs, fan, poses, o, v = _config_rays(1)
    got_d, got_s, got_k = cast_explicit(cs.words, o, v, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                                        bbox_min=cs.bbox_min, bbox_max=cs.bbox_max, hit_epsilon=cs.hit_epsilon)
    pool = tracer.NodePool.from_words(cs.words, dev())
    sset = tracer.SceneSet([pool], [cs.bbox_min], [cs.bbox_max], [cs.hit_epsilon])
    n = got_d.shape[0]
    fd = torch.empty(n, dtype=torch.float32, device=dev())
    fs = torch.empty(n, dtype=torch.int32, device=dev())
    fk = torch.empty(n, dtype=torch.int32, device=dev())
    tracer.cast_fan(sset, poses, fan, fd, fs, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                    use_pitch=True, out_steps=fk)
    torch.cuda.synchronize()
    assert_bits_equal(fd.cpu().numpy(), got_d, "fan dist")
    assert_equal(fs.cpu().numpy(), got_s, "fan sem")
    assert_equal(fk.cpu().numpy(), got_k, "fan steps")


def test_fan_without_pitch_equals_reference_yaw_only_rays():
    cfg = scenes.CONFIGS[1]
    cs, fan, poses, _, _ = _config_rays(1)
    o, v = eager_world_rays(fan, poses, pitch=False)
    got_d, got_s, got_k = cast_explicit(cs.words, o, v, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                                        bbox_min=cs.bbox_min, bbox_max=cs.bbox_max, hit_epsilon=cs.hit_epsilon)
    sset = tracer.SceneSet([tracer.NodePool.from_words(cs.words, dev())], [cs.bbox_min], [cs.bbox_max],
                           [cs.hit_epsilon])
    n = got_d.shape[0]
    fd = torch.empty(n, dtype=torch.float32, device=dev())
    fs = torch.empty(n, dtype=torch.int32, device=dev())
    fk = torch.empty(n, dtype=torch.int32, device=dev())
    tracer.cast_fan(sset, poses, fan, fd, fs, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                    use_pitch=False, out_steps=fk)
    torch.cuda.synchronize()
    assert_bits_equal(fd.cpu().numpy(), got_d, "yaw-only fan dist")
    assert_equal(fs.cpu().numpy(), got_s, "yaw-only fan sem")
    assert_equal(fk.cpu().numpy(), got_k, "yaw-only fan steps")


def test_config2_full_step_matches_oracle(descent):
    """Full benchmark step of config 2 (64 actors x 12,288 rays, 512^3) against the oracle."""
    cfg = scenes.CONFIGS[2]
    cs, fan, poses, o, v = _config_rays(2)
    sset = tracer.SceneSet([tracer.NodePool.from_words(cs.words, dev())], [cs.bbox_min], [cs.bbox_max],
                           [cs.hit_epsilon])
    n = o.shape[0] * o.shape[1]
    fd = torch.empty(n, dtype=torch.float32, device=dev())
    fs = torch.empty(n, dtype=torch.int32, device=dev())
    fk = torch.empty(n, dtype=torch.int32, device=dev())
    tracer.cast_fan(sset, poses, fan, fd, fs, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                    use_pitch=True, out_steps=fk)
    torch.cuda.synchronize()
    ref = O.trace(cs.words, cs.bbox_min, cs.bbox_max, o.cpu().numpy(), v.cpu().numpy(), max_steps=cfg.max_steps,
                  max_distance=cfg.max_distance, hit_epsilon=cs.hit_epsilon)
    assert_bits_equal(fd.cpu().numpy(), ref["dist"], "dist")
    assert_equal(fs.cpu().numpy(), ref["sem"], "sem")
    assert_equal(fk.cpu().numpy(), ref["steps"], "steps")


def test_config4_full_step_matches_oracle():
    """Full benchmark step of config 4 (16 actors x 262,144 rays, 2048^3 scene compiled on
    the device, 40M-word pool, pitch U[-30, 30] deg, 512 steps) against the oracle."""
    cfg = scenes.CONFIGS[4]
    cs, fan, poses, o, v = _config_rays(4)
    sset = tracer.SceneSet([tracer.NodePool.from_words(cs.words, dev())], [cs.bbox_min], [cs.bbox_max],
                           [cs.hit_epsilon])
    n = o.shape[0] * o.shape[1]
    fd = torch.empty(n, dtype=torch.float32, device=dev())
    fs = torch.empty(n, dtype=torch.int32, device=dev())
    fk = torch.empty(n, dtype=torch.int32, device=dev())
    tracer.cast_fan(sset, poses, fan, fd, fs, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                    use_pitch=True, out_steps=fk)
    torch.cuda.synchronize()
    ref = O.trace(cs.words, cs.bbox_min, cs.bbox_max, o.cpu().numpy(), v.cpu().numpy(), max_steps=cfg.max_steps,
                  max_distance=cfg.max_distance, hit_epsilon=cs.hit_epsilon)
    assert_bits_equal(fd.cpu().numpy(), ref["dist"], "dist")
    assert_equal(fs.cpu().numpy(), ref["sem"], "sem")
    assert_equal(fk.cpu().numpy(), ref["steps"], "steps")
    # eps = 1e-3 voxel = 2.05e-5 lies below the smallest finite leaf distance the compiler
    # can encode (distances under 2^-15 become +inf halves), so no ray of this config can
    # register a hit: every ray marches to the horizon or to max_steps.
    assert not np.any(ref["sem"] != 0)
    assert (ref["steps"] > 8).mean() > 0.5


def test_multiscene_fan_matches_per_scene_oracle(descent):
    """Config-3 style scenes (rods) at 128^3, three scenes resident together, actors assigned at random."""
    cfg = scenes.CONFIGS[3]
    scene_list = [workloads.compiled_scene(3, s, resolution=128) for s in range(3)]
    pb = workloads.poses_for(3, scene_list, actors=48)
    fan_np = workloads.fan_for(3)
    fan = torch.from_numpy(fan_np).to(dev())
    d = dev()
    poses = tracer.make_poses(torch.from_numpy(pb.position).to(d), torch.from_numpy(pb.yaw).to(d),
                              torch.from_numpy(pb.pitch).to(d), torch.from_numpy(pb.scene).to(d))
    pools = [tracer.NodePool.from_words(cs.words, d) for cs in scene_list]
    sset = tracer.SceneSet(pools, [cs.bbox_min for cs in scene_list], [cs.bbox_max for cs in scene_list],
                           [cs.hit_epsilon for cs in scene_list])
    a, r = poses.shape[0], fan.shape[0]
    fd = torch.empty(a * r, dtype=torch.float32, device=d)
    fs = torch.empty(a * r, dtype=torch.int32, device=d)
    fk = torch.empty(a * r, dtype=torch.int32, device=d)
    tracer.cast_fan(sset, poses, fan, fd, fs, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                    use_pitch=False, out_steps=fk)
    torch.cuda.synchronize()
    o, v = eager_world_rays(fan, poses, pitch=False)
    on, vn = o.cpu().numpy(), v.cpu().numpy()
    fd_, fs_, fk_ = (x.cpu().numpy().reshape(a, r) for x in (fd, fs, fk))
    assert len(set(pb.scene.tolist())) == 3
    for s, cs in enumerate(scene_list):
        m = pb.scene == s
        ref = O.trace(cs.words, cs.bbox_min, cs.bbox_max, on[m], vn[m], max_steps=cfg.max_steps,
                      max_distance=cfg.max_distance, hit_epsilon=cs.hit_epsilon)
        assert_bits_equal(fd_[m], ref["dist"], f"scene {s} dist")
        assert_equal(fs_[m], ref["sem"], f"scene {s} sem")
        assert_equal(fk_[m], ref["steps"], f"scene {s} steps")


def _grid_aligned_rays(cs, n: int, seed: int):
    """Rays that start exactly on cell faces and run along axes (the inclusive/strict cache bounds matter)."""
    rng = np.random.default_rng(seed)
    lo = np.asarray(cs.bbox_min, np.float64)
    vox = cs.voxel_size
    res = cs.asset.resolution
    idx = rng.integers(1, res - 1, size=(n, 3))
    origins = (lo + idx * vox).astype(np.float32)
    axes = rng.integers(0, 6, size=n)
    dirs = np.zeros((n, 3), np.float32)
    dirs[np.arange(n), axes % 3] = np.where(axes < 3, 1.0, -1.0)
    return origins, dirs


def test_edge_cases_grid_aligned_outside_and_tiny_components(descent):
    cfg = scenes.CONFIGS[1]
    cs = workloads.compiled_scene(1)
    o1, d1 = _grid_aligned_rays(cs, 3000, 1)
    rng = np.random.default_rng(2)
    # origins outside the domain, pointing in and out
    o2 = rng.uniform(-5.0, 16.0, size=(2000, 3)).astype(np.float32)
    d2 = rng.normal(size=(2000, 3)).astype(np.float32)
    d2 /= np.linalg.norm(d2, axis=1, keepdims=True)
    # direction components at and around the 1e-4 threshold of the exit distance
    d3 = rng.normal(size=(2000, 3)).astype(np.float32)
    d3[:, rng.integers(0, 3)] = rng.choice(np.array([0.0, 1e-4, -1e-4, 9.9e-5, 1.01e-4, -0.0], np.float32), 2000)
    d3 /= np.linalg.norm(d3, axis=1, keepdims=True).astype(np.float32)
    o3 = rng.uniform(0.0, 10.0, size=(2000, 3)).astype(np.float32)
    origins = np.concatenate([o1, o2, o3])
    dirs = np.concatenate([d1, d2, d3]).astype(np.float32)
    for max_steps, horizon in ((1, 20.0), (cfg.max_steps, cfg.max_distance), (5000, 2000.0)):
        got_d, got_s, got_k = cast_explicit(cs.words, origins, dirs, max_steps=max_steps, max_distance=horizon,
                                            bbox_min=cs.bbox_min, bbox_max=cs.bbox_max, hit_epsilon=0.01)
        ref = O.trace(cs.words, cs.bbox_min, cs.bbox_max, origins, dirs, max_steps=max_steps, max_distance=horizon,
                      hit_epsilon=0.01)
        assert_bits_equal(got_d, ref["dist"], f"dist (max_steps={max_steps})")
        assert_equal(got_s, ref["sem"], f"sem (max_steps={max_steps})")
        assert_equal(got_k, ref["steps"], f"steps (max_steps={max_steps})")


@pytest.mark.parametrize("n", [0, 1, 31, 33, 1000, 4097])
def test_ragged_and_empty_batches(n):
    cfg = scenes.CONFIGS[1]
    cs = workloads.compiled_scene(1)
    rng = np.random.default_rng(n)
    origins = rng.uniform(0.5, 9.5, size=(n, 3)).astype(np.float32)
    dirs = rng.normal(size=(n, 3)).astype(np.float32)
    if n:
        dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    got_d, got_s, got_k = cast_explicit(cs.words, origins.reshape(n, 3), dirs.reshape(n, 3), max_steps=cfg.max_steps,
                                        max_distance=cfg.max_distance, bbox_min=cs.bbox_min, bbox_max=cs.bbox_max,
                                        hit_epsilon=cs.hit_epsilon)
    assert got_d.shape == (n,)
    if n:
        ref = O.trace(cs.words, cs.bbox_min, cs.bbox_max, origins, dirs, max_steps=cfg.max_steps,
                      max_distance=cfg.max_distance, hit_epsilon=cs.hit_epsilon)
        assert_bits_equal(got_d, ref["dist"], "dist")
        assert_equal(got_s, ref["sem"], "sem")
        assert_equal(got_k, ref["steps"], "steps")


def test_repeated_casts_are_deterministic_and_overwrite_outputs():
    cfg = scenes.CONFIGS[1]
    cs, fan, poses, o, v = _config_rays(1)
    a = cast_explicit(cs.words, o, v, max_steps=cfg.max_steps, max_distance=cfg.max_distance, bbox_min=cs.bbox_min,
                      bbox_max=cs.bbox_max, hit_epsilon=cs.hit_epsilon)
    b = cast_explicit(cs.words, o, v, max_steps=cfg.max_steps, max_distance=cfg.max_distance, bbox_min=cs.bbox_min,
                      bbox_max=cs.bbox_max, hit_epsilon=cs.hit_epsilon)
    for x, y in zip(a, b):
        assert np.array_equal(np.asarray(x).view(np.uint32), np.asarray(y).view(np.uint32))


def test_cast_runs_on_the_callers_stream():
    cfg = scenes.CONFIGS[1]
    cs, fan, poses, o, v = _config_rays(1)
    d = dev()
    pool = tracer.NodePool.from_words(cs.words, d)
    n = o.shape[0] * o.shape[1]
    s = torch.cuda.Stream(d)
    out_d = torch.zeros(n, dtype=torch.float32, device=d)
    out_s = torch.zeros(n, dtype=torch.int32, device=d)
    s.wait_stream(torch.cuda.current_stream(d))
    with torch.cuda.stream(s):
        tracer.cast_rays_ex(pool, o, v, out_d, out_s, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                            bbox_min=cs.bbox_min, bbox_max=cs.bbox_max, hit_epsilon=cs.hit_epsilon)
        done = torch.cuda.Event()
        done.record(s)
    done.synchronize()
    ref = cast_explicit(cs.words, o, v, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                        bbox_min=cs.bbox_min, bbox_max=cs.bbox_max, hit_epsilon=cs.hit_epsilon, pool=pool)
    assert_bits_equal(out_d.cpu().numpy(), ref[0], "side-stream dist")


def test_pool_cache_tracks_in_place_dag_updates():
    d = dev()
    from tests.kat_cases import leaf_word

    dag = torch.from_numpy(np.array([leaf_word(0.005, 3)], np.uint64).view(np.int64)).to(d)
    o = torch.tensor([[[0.5, 0.5, 0.5]]], device=d)
    v = torch.tensor([[[0.0, 1.0, 0.0]]], device=d)
    out_d = torch.zeros((1, 1), device=d)
    out_s = torch.zeros((1, 1), dtype=torch.int32, device=d)
    torch_sdf.cast_rays(dag, o, v, out_d, out_s, 4, 10.0, [0, 0, 0], [1, 1, 1], 1)
    assert int(out_s.item()) == 3
    dag.copy_(torch.from_numpy(np.array([leaf_word(0.5, 9)], np.uint64).view(np.int64)).to(d))
    torch_sdf.cast_rays(dag, o, v, out_d, out_s, 1, 10.0, [0, 0, 0], [1, 1, 1], 1)
    assert int(out_s.item()) == 0
    assert abs(float(out_d.item()) - 0.5) < 1e-6


# ---------------------------------------------------------------- randomized DAGs


@pytest.mark.parametrize("seed", range(12))
def test_random_dags_match_oracle(seed):
    from tests.dag_fuzz import random_dag, random_rays

    rng = np.random.default_rng(1000 + seed)
    depth = int(rng.integers(1, 9))
    dag = random_dag(rng, depth)
    if seed % 3 == 0:
        bmin, bmax = (0.0, 0.0, 0.0), (1.0, 1.0, 1.0)
    elif seed % 3 == 1:
        bmin, bmax = (-3.25, 0.5, 7.0), (4.75, 2.0, 13.5)  # non-cubic box
    else:
        bmin, bmax = (-1.0, -1.0, -1.0), (11.0, 11.0, 11.0)
    o, d = random_rays(rng, 6000, bmin, bmax, depth)
    for eps, steps, horizon in ((0.01, 64, 30.0), (0.25, 7, 3.0)):
        got_d, got_s, got_k = cast_explicit(dag, o, d, max_steps=steps, max_distance=horizon, bbox_min=bmin,
                                            bbox_max=bmax, hit_epsilon=eps)
        ref = O.trace(dag, bmin, bmax, o, d, max_steps=steps, max_distance=horizon, hit_epsilon=eps)
        assert_bits_equal(got_d, ref["dist"], f"seed {seed} depth {depth} dist")
        assert_equal(got_s, ref["sem"], f"seed {seed} sem")
        assert_equal(got_k, ref["steps"], f"seed {seed} steps")


def test_float_descent_fallback_deep_cyclic_and_degenerate():
    """DAGs the integer grid does not cover: 14 levels deep, a cycle, and a box too thin for
    distinct grid lines; all traced by the float-descent kernel, still bit-exact."""
    from tests.dag_fuzz import random_rays
    from tests.kat_cases import leaf_word, single_path_dag_words

    rng = np.random.default_rng(7)
    deep_octs = [int(x) for x in rng.integers(0, 8, size=14)]
    deep = single_path_dag_words(deep_octs, distance=0.004, semantic=5)
    cyclic = np.array([internal_word_(0b10000001, 1), 0, 3, leaf_word(0.003, 2)], np.uint64)
    cases = [(deep, (0.0, 0.0, 0.0), (1.0, 1.0, 1.0)), (cyclic, (0.0, 0.0, 0.0), (1.0, 1.0, 1.0)),
             (single_path_dag_words([1, 2, 3, 4, 5, 6], distance=0.5, semantic=1), (1e6, 0.0, 0.0),
              (1e6 + 0.0625, 1.0, 1.0))]
    for words, bmin, bmax in cases:
        o, d = random_rays(rng, 3000, bmin, bmax, 6)
        got_d, got_s, got_k = cast_explicit(words, o, d, max_steps=40, max_distance=5.0, bbox_min=bmin,
                                            bbox_max=bmax)
        ref = O.trace(words, bmin, bmax, o, d, max_steps=40, max_distance=5.0)
        assert_bits_equal(got_d, ref["dist"], "dist")
        assert_equal(got_s, ref["sem"], "sem")
        assert_equal(got_k, ref["steps"], "steps")


def internal_word_(mask: int, base: int) -> int:
    from tests.kat_cases import internal_word

    return internal_word(mask, base)


def test_pool_from_file_and_pool_cache(tmp_path):
    """tsdf_pool_create_from_file and the on-disk pool cache give the pool of from_words
    (same records, same casts), and a damaged cache file is rejected before upload."""
    from navi_b200 import gmdag

    cs, fan, poses, o, v = _config_rays(1)
    cfg = scenes.CONFIGS[1]
    path = gmdag.write_gmdag(tmp_path / "c1.gmdag", cs.words, cfg.resolution, cs.bbox_min, cs.voxel_size)
    ref_pool = tracer.NodePool.from_words(cs.words, dev())
    pool, bmin, bmax = tracer.NodePool.from_file(path, dev(), validate_layout=True)
    asset = gmdag.load_gmdag_asset(path)
    assert bmin == [float(np.float32(x)) for x in asset.bbox_min]
    assert bmax == [float(np.float32(x)) for x in asset.bbox_max]
    assert pool.stats == ref_pool.stats

    def cast(p):
        d = torch.empty(o.shape[0] * o.shape[1], device=dev())
        s = torch.empty(o.shape[0] * o.shape[1], dtype=torch.int32, device=dev())
        tracer.cast_rays_ex(p, o, v, d, s, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                            bbox_min=cs.bbox_min, bbox_max=cs.bbox_max, hit_epsilon=cs.hit_epsilon)
        torch.cuda.synchronize()
        return d.cpu().numpy(), s.cpu().numpy()

    want = cast(ref_pool)
    for p in (pool,):
        got = cast(p)
        assert_bits_equal(got[0], want[0], "dist")
        assert_equal(got[1], want[1], "sem")
    scene = tracer.load_gmdag(path, dev(), pool_cache=tmp_path / "pools")
    cached = list((tmp_path / "pools").glob("*.npool"))
    assert len(cached) == 1
    again = tracer.load_gmdag(path, dev(), pool_cache=tmp_path / "pools")
    assert again.pool.stats == ref_pool.stats
    got = cast(again.pool)
    assert_bits_equal(got[0], want[0], "dist (cached pool)")
    assert tracer.pool_for_tensor(scene.dag_tensor) is scene.pool
    raw = bytearray(cached[0].read_bytes())
    raw[40 + 4 * 3] = 0xFE  # first record, slot 3: an internal index far out of range
    raw[40 + 4 * 3 + 3] = 0x3F
    bad = tmp_path / "bad.npool"
    bad.write_bytes(bytes(raw))
    with pytest.raises(RuntimeError, match="out of range"):
        tracer.NodePool.load(bad, dev())
    bad.write_bytes(bytes(raw[:60]))
    with pytest.raises(RuntimeError, match="truncated"):
        tracer.NodePool.load(bad, dev())
    with pytest.raises(FileNotFoundError):
        tracer.NodePool.from_file(tmp_path / "missing.gmdag", dev())


def test_multiscene_actor_with_unknown_scene_is_not_traced(descent):
    """A pose whose scene index is outside the scene table: its rays get NaN, semantic 0,
    0 steps; every other actor's rays are traced as usual."""
    scene_list = [workloads.compiled_scene(3, s, resolution=64) for s in range(2)]
    pools = [tracer.NodePool.from_words(cs.words, dev()) for cs in scene_list]
    sset = tracer.SceneSet(pools, [c.bbox_min for c in scene_list], [c.bbox_max for c in scene_list],
                           [c.hit_epsilon for c in scene_list])
    pb = workloads.poses_for(3, scene_list, actors=6)
    sc = pb.scene.copy()
    sc[2] = 7
    sc[4] = -1
    fan = torch.from_numpy(workloads.fan_for(1)).to(dev())
    poses = tracer.make_poses(torch.from_numpy(pb.position).to(dev()), torch.from_numpy(pb.yaw).to(dev()),
                              None, torch.from_numpy(sc).to(dev()))
    n = 6 * fan.shape[0]
    d = torch.empty(n, device=dev())
    s = torch.empty(n, dtype=torch.int32, device=dev())
    k = torch.empty(n, dtype=torch.int32, device=dev())
    tracer.cast_fan(sset, poses, fan, d, s, max_steps=64, max_distance=30.0, out_steps=k)
    torch.cuda.synchronize()
    d = d.cpu().numpy().reshape(6, -1)
    s = s.cpu().numpy().reshape(6, -1)
    k = k.cpu().numpy().reshape(6, -1)
    for a in (2, 4):
        assert np.all(np.isnan(d[a])) and np.all(s[a] == 0) and np.all(k[a] == 0)
    for a in (0, 1, 3, 5):
        assert not np.any(np.isnan(d[a])) and np.all(k[a] > 0)


@pytest.mark.parametrize("opts", [
    {"smem_records": 1024}, {"smem_records": 37}, {"leaf_run": 0}, {"leaf_run": 8}, {"chunk": 1},
    {"chunk": 64}, {"blocks_per_sm": 1}, {"order": 0}, {"per_scene": 0}, {"per_scene": 0, "leaf_run": 0},
    {"descent": 1},
    {"smem_records": 1024, "leaf_run": 3, "chunk": 3, "blocks_per_sm": 2, "order": 0},
])
def test_tuning_options_do_not_change_results(opts):
    """Every knob of tsdf_set_option changes scheduling only: single- and multi-scene fan
    casts give the default build's bits under each setting."""
    cfg = scenes.CONFIGS[1]
    cs, fan, poses, _, _ = _config_rays(1)
    multi = [workloads.compiled_scene(3, s, resolution=64) for s in range(3)]
    pb3 = workloads.poses_for(3, multi, actors=24)
    poses3 = tracer.make_poses(torch.from_numpy(pb3.position).to(dev()), torch.from_numpy(pb3.yaw).to(dev()),
                               None, torch.from_numpy(pb3.scene).to(dev()))
    sets = [
        (tracer.SceneSet([tracer.NodePool.from_words(cs.words, dev())], [cs.bbox_min], [cs.bbox_max],
                         [cs.hit_epsilon]), poses, True),
        (tracer.SceneSet([tracer.NodePool.from_words(c.words, dev()) for c in multi], [c.bbox_min for c in multi],
                         [c.bbox_max for c in multi], [c.hit_epsilon for c in multi]), poses3, False),
    ]

    def run():
        out = []
        for sset, p, pitch in sets:
            n = p.shape[0] * fan.shape[0]
            d = torch.empty(n, device=dev())
            s = torch.empty(n, dtype=torch.int32, device=dev())
            k = torch.empty(n, dtype=torch.int32, device=dev())
            tracer.cast_fan(sset, p, fan, d, s, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                            use_pitch=pitch, out_steps=k)
            torch.cuda.synchronize()
            out.append((d.cpu().numpy(), s.cpu().numpy(), k.cpu().numpy()))
        return out

    want = run()
    old = {k: tracer.set_option(k, v) for k, v in opts.items()}
    try:
        got = run()
    finally:
        for k, v in old.items():
            tracer.set_option(k, v)
    for (gd, gs, gk), (wd, ws, wk) in zip(got, want):
        assert_bits_equal(gd, wd, f"dist under {opts}")
        assert_equal(gs, ws, f"sem under {opts}")
        assert_equal(gk, wk, f"steps under {opts}")


@pytest.mark.parametrize("n", [1, 2047, 2048, 2049, 3 * 2048 + 5, 70001])
def test_claim_order_traces_every_ray_once(n):
    """Single-scene launches claim rays longest scene-box exit first, through a bucket
    order built on the device (per-block ranks, one reservation per bucket and block).
    Every ray must be traced exactly once whatever the bucket mix: sentinel-prefilled
    outputs under the default order equal index order bit for bit and the oracle.  The
    rays mix one crowded bucket (copies of one ray), rays that start outside the box and
    leave it, and random rays, over sizes around the 2048-ray scatter tile."""
    cfg = scenes.CONFIGS[1]
    cs = workloads.compiled_scene(1)
    rng = np.random.default_rng(n)
    origins = rng.uniform(0.5, 9.5, size=(n, 3)).astype(np.float32)
    dirs = rng.normal(size=(n, 3)).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    third = n // 3
    origins[:third] = origins[0]
    dirs[:third] = dirs[0]
    out = slice(third, third + n // 4)
    origins[out] = np.array([-3.0, 5.0, 5.0], np.float32)
    dirs[out] = np.array([-1.0, 0.0, 0.0], np.float32)
    kw = dict(max_steps=cfg.max_steps, max_distance=cfg.max_distance, bbox_min=cs.bbox_min, bbox_max=cs.bbox_max,
              hit_epsilon=cs.hit_epsilon)
    pool = tracer.NodePool.from_words(cs.words, dev())
    ordered = cast_explicit(cs.words, origins, dirs, pool=pool, **kw)
    old = tracer.set_option("order", 0)
    try:
        plain = cast_explicit(cs.words, origins, dirs, pool=pool, **kw)
    finally:
        tracer.set_option("order", old)
    assert np.all(ordered[2] >= 0), "a ray was left untraced"
    assert_bits_equal(ordered[0], plain[0], "dist")
    assert_equal(ordered[1], plain[1], "sem")
    assert_equal(ordered[2], plain[2], "steps")
    pick = np.unique(np.concatenate([np.arange(min(n, 64)), rng.integers(0, n, size=min(n, 512))]))
    ref = O.trace(cs.words, cs.bbox_min, cs.bbox_max, origins[pick], dirs[pick], max_steps=cfg.max_steps,
                  max_distance=cfg.max_distance, hit_epsilon=cs.hit_epsilon)
    assert_bits_equal(ordered[0][pick], ref["dist"], "dist vs oracle")
    assert_equal(ordered[1][pick], ref["sem"], "sem vs oracle")
    assert_equal(ordered[2][pick], ref["steps"], "steps vs oracle")


@pytest.mark.parametrize("az,el,actors", [(1, 1, 5), (17, 5, 9), (255, 47, 3), (3, 1, 700)])
def test_fan_sizes_and_actor_indexing(az, el, actors):
    """Fans of any size: ray (actor, k) = index actor * (az * el) + k, checked against the
    oracle on explicit rays (the kernel splits ray indices without a hardware division)."""
    from navi_b200.fan import build_spherical_ray_directions

    cs = workloads.compiled_scene(1)
    pb = workloads.poses_for(1, [cs], actors=actors)
    fan = torch.from_numpy(build_spherical_ray_directions(az, el)).to(dev())
    poses = tracer.make_poses(torch.from_numpy(pb.position).to(dev()), torch.from_numpy(pb.yaw).to(dev()),
                              torch.from_numpy(pb.pitch).to(dev()))
    o, v = eager_world_rays(fan, poses, pitch=True)
    sset = tracer.SceneSet([tracer.NodePool.from_words(cs.words, dev())], [cs.bbox_min], [cs.bbox_max],
                           [cs.hit_epsilon])
    n = actors * az * el
    d = torch.empty(n, device=dev())
    s = torch.empty(n, dtype=torch.int32, device=dev())
    k = torch.empty(n, dtype=torch.int32, device=dev())
    tracer.cast_fan(sset, poses, fan, d, s, max_steps=128, max_distance=20.0, use_pitch=True, out_steps=k)
    torch.cuda.synchronize()
    ref = O.trace(cs.words, cs.bbox_min, cs.bbox_max, o.cpu().numpy(), v.cpu().numpy(), max_steps=128,
                  max_distance=20.0, hit_epsilon=cs.hit_epsilon)
    assert_bits_equal(d.cpu().numpy(), ref["dist"], "dist")
    assert_equal(s.cpu().numpy(), ref["sem"], "sem")
    assert_equal(k.cpu().numpy(), ref["steps"], "steps")


def _multiscene_setup(config, actors=None):
    cfg = scenes.CONFIGS[config]
    scene_list = [workloads.compiled_scene(config, s) for s in range(cfg.n_scenes)]
    pb = workloads.poses_for(config, scene_list, actors=actors)
    fan = torch.from_numpy(workloads.fan_for(config)).to(dev())
    pools = [tracer.NodePool.from_words(cs.words, dev()) for cs in scene_list]
    sset = tracer.SceneSet(pools, [c.bbox_min for c in scene_list], [c.bbox_max for c in scene_list],
                           [c.hit_epsilon for c in scene_list])
    return cfg, scene_list, pb, fan, pools, sset


def _poses(pb, sel, scene_ids):
    return tracer.make_poses(torch.from_numpy(pb.position[sel]).to(dev()), torch.from_numpy(pb.yaw[sel]).to(dev()),
                             torch.from_numpy(pb.pitch[sel]).to(dev()), torch.from_numpy(scene_ids).to(dev()))


def _sampled_oracle_check(cfg, scene_list, pb, fan, d, s, k, n_sample, seed):
    rng = np.random.default_rng(seed)
    r = fan.shape[0]
    rays = np.sort(rng.choice(pb.position.shape[0] * r, size=n_sample, replace=False))
    actor, ki = rays // r, rays % r
    fan_np = fan.cpu().numpy()
    # the cos/sin the kernel uses: torch.cos / torch.sin on the device, as in the poses
    pose = _poses(pb, np.arange(pb.position.shape[0]), pb.scene).cpu().numpy()
    dirs = O.rotate_fan(fan_np, pose[:, 3], pose[:, 4])
    for sc in np.unique(pb.scene[actor]):
        m = pb.scene[actor] == sc
        cs = scene_list[sc]
        o = pb.position[actor[m]]
        v = dirs[actor[m], ki[m]]
        ref = O.trace(cs.words, cs.bbox_min, cs.bbox_max, o, v, max_steps=cfg.max_steps,
                      max_distance=cfg.max_distance, hit_epsilon=cs.hit_epsilon)
        assert_bits_equal(d[rays[m]], ref["dist"], f"dist scene {sc}")
        assert_equal(s[rays[m]], ref["sem"], f"sem scene {sc}")
        assert_equal(k[rays[m]], ref["steps"], f"steps scene {sc}")


def test_config3_full_step_multiscene_equals_per_scene_launches_and_oracle():
    """Config 3 at full size (8 scenes, 4096 actors x 3072 rays = 12.6 M rays): one
    multi-scene launch equals the eight single-scene launches of the same actors bit for
    bit; 200,000 sampled rays equal the oracle."""
    cfg, scene_list, pb, fan, pools, sset = _multiscene_setup(3)
    a, r = pb.position.shape[0], fan.shape[0]
    n = a * r
    d = torch.empty(n, device=dev())
    s = torch.empty(n, dtype=torch.int32, device=dev())
    k = torch.empty(n, dtype=torch.int32, device=dev())
    tracer.cast_fan(sset, _poses(pb, np.arange(a), pb.scene), fan, d, s, max_steps=cfg.max_steps,
                    max_distance=cfg.max_distance, out_steps=k)
    torch.cuda.synchronize()
    d, s, k = (x.cpu().numpy().reshape(a, r) for x in (d, s, k))
    for sc, cs in enumerate(scene_list):
        sel = np.nonzero(pb.scene == sc)[0]
        one = tracer.SceneSet([pools[sc]], [cs.bbox_min], [cs.bbox_max], [cs.hit_epsilon])
        m = sel.shape[0] * r
        ds = torch.empty(m, device=dev())
        ss = torch.empty(m, dtype=torch.int32, device=dev())
        ks = torch.empty(m, dtype=torch.int32, device=dev())
        tracer.cast_fan(one, _poses(pb, sel, np.zeros(sel.shape[0], np.int32)), fan, ds, ss, max_steps=cfg.max_steps,
                        max_distance=cfg.max_distance, out_steps=ks)
        torch.cuda.synchronize()
        assert_bits_equal(d[sel].reshape(-1), ds.cpu().numpy(), f"scene {sc} dist")
        assert_equal(s[sel].reshape(-1), ss.cpu().numpy(), f"scene {sc} sem")
        assert_equal(k[sel].reshape(-1), ks.cpu().numpy(), f"scene {sc} steps")
    _sampled_oracle_check(cfg, scene_list, pb, fan, d.reshape(-1), s.reshape(-1), k.reshape(-1), 200_000, 3)


def test_config5_step_sampled_oracle_and_determinism():
    """Config 5's scenes and fan (16 scenes, 256 x 48 rays) for 4096 actors (50 M rays, the
    per-rank share at 8 GPUs): 200,000 sampled rays equal the oracle; a second launch gives
    the same bits."""
    cfg, scene_list, pb, fan, pools, sset = _multiscene_setup(5, actors=4096)
    a, r = pb.position.shape[0], fan.shape[0]
    n = a * r
    poses = _poses(pb, np.arange(a), pb.scene)
    outs = []
    for _ in range(2):
        d = torch.empty(n, device=dev())
        s = torch.empty(n, dtype=torch.int32, device=dev())
        k = torch.empty(n, dtype=torch.int32, device=dev())
        tracer.cast_fan(sset, poses, fan, d, s, max_steps=cfg.max_steps, max_distance=cfg.max_distance, out_steps=k)
        torch.cuda.synchronize()
        outs.append((d.cpu().numpy(), s.cpu().numpy(), k.cpu().numpy()))
        del d, s, k
    assert_bits_equal(outs[0][0], outs[1][0], "repeat dist")
    assert_equal(outs[0][2], outs[1][2], "repeat steps")
    _sampled_oracle_check(cfg, scene_list, pb, fan, *outs[0], 200_000, 5)


@pytest.mark.parametrize("n_scenes", [2, 64, 65])
def test_scene_tables_per_scene_launches_and_multi_scene_kernel(n_scenes):
    """Scene tables of 2 and 64 scenes take one single-scene launch per scene (actor
    ranges from the device scene sort, launches alternating on two library streams); 65
    scenes take the multi-scene kernel.  Random DAGs of depths 1-5 in non-cubic boxes
    (one cyclic DAG, traced by the float descent, in tables of 3+ scenes), a scene with
    no actors, and actors whose scene index is outside the table: the outputs equal the
    multi-scene kernel's bit for bit and the oracle on each actor's explicit rays;
    actors of no scene get NaN distance, semantic 0 and 0 steps."""
    from navi_b200.fan import build_spherical_ray_directions
    from tests.dag_fuzz import random_dag
    from tests.kat_cases import leaf_word

    rng = np.random.default_rng(500 + n_scenes)
    dags, bmins, bmaxs, eps = [], [], [], []
    for i in range(n_scenes):
        if i == 2:
            dags.append(np.array([internal_word_(0b10000001, 1), 0, 3, leaf_word(0.003, 2)], np.uint64))
        else:
            dags.append(random_dag(rng, int(rng.integers(1, 6))))
        lo = rng.uniform(-2.0, 0.0, size=3).astype(np.float32)
        bmins.append(tuple(float(x) for x in lo))
        bmaxs.append(tuple(float(x) for x in lo + rng.uniform(0.5, 3.0, size=3).astype(np.float32)))
        eps.append(float(rng.choice([0.01, 0.05, 0.2])))
    sset = tracer.SceneSet([tracer.NodePool.from_words(w, dev()) for w in dags], bmins, bmaxs, eps)
    actors = 3 * n_scenes + 5
    scene = rng.integers(0, n_scenes, size=actors).astype(np.int32)
    scene[scene == 1] = 0                       # scene 1 has no actors
    scene[rng.choice(actors, size=4, replace=False)] = [n_scenes, n_scenes + 3, -1, 1 << 20]
    pos = np.empty((actors, 3), np.float32)
    for a in range(actors):
        s = scene[a] if 0 <= scene[a] < n_scenes else 0
        lo, hi = np.array(bmins[s], np.float32), np.array(bmaxs[s], np.float32)
        pos[a] = lo + rng.uniform(0.05, 0.95, size=3).astype(np.float32) * (hi - lo)
    yaw = rng.uniform(-np.pi, np.pi, size=actors).astype(np.float32)
    pitch = rng.uniform(-0.3, 0.3, size=actors).astype(np.float32)
    poses = tracer.make_poses(torch.from_numpy(pos).to(dev()), torch.from_numpy(yaw).to(dev()),
                              torch.from_numpy(pitch).to(dev()), torch.from_numpy(scene).to(dev()))
    fan = torch.from_numpy(build_spherical_ray_directions(9, 3)).to(dev())
    r = fan.shape[0]
    kw = dict(max_steps=48, max_distance=5.0, use_pitch=True)

    def run():
        d = torch.full((actors * r,), -7.0, device=dev())
        s = torch.full((actors * r,), -7, dtype=torch.int32, device=dev())
        k = torch.full((actors * r,), -7, dtype=torch.int32, device=dev())
        tracer.cast_fan(sset, poses, fan, d, s, out_steps=k, **kw)
        torch.cuda.synchronize()
        return d.cpu().numpy().reshape(actors, r), s.cpu().numpy().reshape(actors, r), k.cpu().numpy().reshape(actors, r)

    got = run()
    old = tracer.set_option("per_scene", 0)
    try:
        multi = run()
    finally:
        tracer.set_option("per_scene", old)
    for g, m, what in zip(got, multi, ("dist", "sem", "steps")):
        if what == "dist":
            assert_bits_equal(g, m, "dist vs multi-scene kernel")
        else:
            assert_equal(g, m, f"{what} vs multi-scene kernel")
    o, v = eager_world_rays(fan, poses, pitch=True)
    o, v = o.cpu().numpy(), v.cpu().numpy()
    for s in range(n_scenes):
        sel = np.nonzero(scene == s)[0]
        if sel.size == 0:
            continue
        ref = O.trace(dags[s], bmins[s], bmaxs[s], o[sel].reshape(-1, 3), v[sel].reshape(-1, 3),
                      max_steps=48, max_distance=5.0, hit_epsilon=eps[s])
        assert_bits_equal(got[0][sel].reshape(-1), ref["dist"], f"scene {s} dist")
        assert_equal(got[1][sel].reshape(-1), ref["sem"], f"scene {s} sem")
        assert_equal(got[2][sel].reshape(-1), ref["steps"], f"scene {s} steps")
    bad = np.nonzero((scene < 0) | (scene >= n_scenes))[0]
    assert bad.size == 4
    assert np.all(np.isnan(got[0][bad])) and np.all(got[1][bad] == 0) and np.all(got[2][bad] == 0)


def test_concurrent_callers_on_their_own_streams():
    """The reference's trainer casts from several rollout groups at once, each on its own
    torch stream (the C ABI is reentrant: ctypes drops the GIL during the call).  Four
    host threads, each on its own stream with its own poses and outputs, alternate
    single-scene casts (claim order in the call's workspace) and three-scene casts
    (per-scene launches on the library's shared streams, forked from and joined back to
    the caller's stream).  Every result equals the same cast made alone."""
    import threading

    cfg1, cfg3 = scenes.CONFIGS[1], scenes.CONFIGS[3]
    cs = workloads.compiled_scene(1)
    multi = [workloads.compiled_scene(3, s, resolution=64) for s in range(3)]
    single = tracer.SceneSet([tracer.NodePool.from_words(cs.words, dev())], [cs.bbox_min], [cs.bbox_max],
                             [cs.hit_epsilon])
    table = tracer.SceneSet([tracer.NodePool.from_words(c.words, dev()) for c in multi], [c.bbox_min for c in multi],
                            [c.bbox_max for c in multi], [c.hit_epsilon for c in multi])
    fan1 = torch.from_numpy(workloads.fan_for(1)).to(dev())
    fan3 = torch.from_numpy(workloads.fan_for(3)).to(dev())

    def job(i):
        pb1 = workloads.poses_for(1, [cs], actors=16, seed_offset=100 + i)
        pb3 = workloads.poses_for(3, multi, actors=48, seed_offset=200 + i)
        p1 = tracer.make_poses(torch.from_numpy(pb1.position).to(dev()), torch.from_numpy(pb1.yaw).to(dev()),
                               torch.from_numpy(pb1.pitch).to(dev()))
        p3 = tracer.make_poses(torch.from_numpy(pb3.position).to(dev()), torch.from_numpy(pb3.yaw).to(dev()),
                               None, torch.from_numpy(pb3.scene).to(dev()))
        return [(single, p1, fan1, cfg1, True), (table, p3, fan3, cfg3, False)]

    def cast(sset, p, fan, cfg, pitch):
        n = p.shape[0] * fan.shape[0]
        d = torch.empty(n, device=dev())
        s = torch.empty(n, dtype=torch.int32, device=dev())
        k = torch.empty(n, dtype=torch.int32, device=dev())
        tracer.cast_fan(sset, p, fan, d, s, max_steps=cfg.max_steps, max_distance=cfg.max_distance, use_pitch=pitch,
                        out_steps=k)
        return d, s, k

    jobs = [job(i) for i in range(4)]
    torch.cuda.synchronize()
    want = [[tuple(x.cpu() for x in cast(*c)) for c in js] for js in jobs]
    got = [[None, None] for _ in jobs]
    errors = []

    def worker(i):
        try:
            st = torch.cuda.Stream(dev())
            st.wait_stream(torch.cuda.current_stream(dev()))
            with torch.cuda.stream(st):
                for rep in range(6):
                    c = jobs[i][rep % 2]
                    out = cast(*c)
                    got[i][rep % 2] = out
                st.synchronize()
        except Exception as exc:  # reported below; a thread's failure must fail the test
            errors.append(repr(exc))

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    torch.cuda.synchronize()
    for i in range(4):
        for j in range(2):
            gd, gs, gk = (x.cpu() for x in got[i][j])
            wd, ws, wk = want[i][j]
            assert_bits_equal(gd.numpy(), wd.numpy(), f"thread {i} cast {j} dist")
            assert_equal(gs.numpy(), ws.numpy(), f"thread {i} cast {j} sem")
            assert_equal(gk.numpy(), wk.numpy(), f"thread {i} cast {j} steps")


def test_non_finite_and_degenerate_rays(descent):
    """Origins with NaN or +-inf coordinates, origins on the box faces and corners, and
    directions with every component at or below the 1e-4 threshold of the exit distance
    (kernel.cu:54-85 then keeps its 1000 m) or exactly zero: the grid descent's sentinel
    lines and the void exit's no-valid-axis case give the oracle's bits."""
    cfg = scenes.CONFIGS[1]
    cs = workloads.compiled_scene(1)
    lo = np.asarray(cs.bbox_min, np.float32)
    hi = np.asarray(cs.bbox_max, np.float32)
    rng = np.random.default_rng(11)
    origins, dirs = [], []
    inside = rng.uniform(0.5, 9.5, size=(64, 3)).astype(np.float32)
    for k, bad in enumerate([np.nan, np.inf, -np.inf]):
        for axis in range(3):
            o = inside.copy()
            o[:, axis] = bad
            origins.append(o)
            dirs.append(rng.normal(size=(64, 3)).astype(np.float32))
    corners = np.array([[x, y, z] for x in (lo[0], hi[0]) for y in (lo[1], hi[1]) for z in (lo[2], hi[2])], np.float32)
    origins.append(np.repeat(corners, 8, axis=0))
    dirs.append(rng.normal(size=(64, 3)).astype(np.float32))
    tiny = rng.choice(np.array([0.0, -0.0, 1e-4, -1e-4, 5e-5, -3e-5], np.float32), size=(64, 3))
    origins.append(inside)
    dirs.append(tiny)
    zero = np.zeros((64, 3), np.float32)
    zero[::2, 1] = np.float32(1e-4)
    origins.append(inside)
    dirs.append(zero)
    o = np.concatenate(origins).astype(np.float32)
    v = np.concatenate(dirs).astype(np.float32)
    norm = np.linalg.norm(v, axis=1, keepdims=True)
    big = norm[:, 0] > 1e-3
    v[big] = (v[big] / norm[big]).astype(np.float32)
    for max_steps, horizon in ((cfg.max_steps, cfg.max_distance), (3, 5000.0)):
        got_d, got_s, got_k = cast_explicit(cs.words, o, v, max_steps=max_steps, max_distance=horizon,
                                            bbox_min=cs.bbox_min, bbox_max=cs.bbox_max, hit_epsilon=0.01)
        ref = O.trace(cs.words, cs.bbox_min, cs.bbox_max, o, v, max_steps=max_steps, max_distance=horizon,
                      hit_epsilon=0.01)
        same = (got_d.view(np.uint32) == ref["dist"].view(np.uint32)) | (np.isnan(got_d) & np.isnan(ref["dist"]))
        assert same.all(), f"dist differs on {np.nonzero(~same)[0][:5]}"
        assert_equal(got_s, ref["sem"], "sem")
        assert_equal(got_k, ref["steps"], "steps")
