"""Benchmark: batched sphere tracing of spherical ray fans through .gmdag DAGs on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl navi|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)

A step is one cast of every actor's full fan of the configuration (default:
config 2, 64 actors x 256 x 48 rays = 786,432 rays, one 512^3 scene).  With N
ranks each rank traces its own actors in its own replica of the scene(s)
(weak scaling; config 5 splits a fixed actor set instead, strong scaling).

Timing: per step, CUDA events on the launching stream around the cast; L2 is
flushed (a buffer of 2x the L2 size is written) between steps, outside the
events; W warm-up steps first; the job time is the max over ranks (gathered
over NCCL).  Printed: one JSON line on rank 0.

`--impl reference` times the reference algorithm on the host cores instead
(the C restatement in oracle/, OpenMP over rays, all host threads) on a
bounded sample of the same workload; it also times the reference's own CUDA
kernel built for sm_100a (oracle/_ref) on the same rays when that build exists.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "rays/sec per B200 and whole box (1/2/4/8 GPUs); % of L2/HBM roofline"
UNIT = "rays/s"
FALLBACK_HBM_GBS = 6650.0


def _args() -> argparse.Namespace:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--impl", choices=["navi", "reference"], default="navi")
    ap.add_argument("--pose-sets", type=int, default=4, help="distinct pose sets cycled over the steps")
    ap.add_argument("--actors", type=int, default=0,
                    help="actors per rank instead of the configuration's (0 = the configuration's; for small profiles)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-actors", type=int, default=0, help="actors in the CPU-baseline sample (0 = auto)")
    ap.add_argument("--descent", choices=["grid", "float"], default="grid",
                    help="library descent: integer grid (default) or float; both give identical results")
    return ap.parse_args()


# ----------------------------------------------------------------------------- helpers


def _peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (ValueError, KeyError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc: subprocess.Popen | None = None
        self.lines: list[str] = []
        self._thread: threading.Thread | None = None

    def __enter__(self) -> "ClockSampler":
        visible = os.environ.get("CUDA_VISIBLE_DEVICES")
        ident = str(self.gpu)
        if visible:
            ids = [v.strip() for v in visible.split(",") if v.strip()]
            if self.gpu < len(ids):
                ident = ids[self.gpu]
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", ident],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
            self._thread = threading.Thread(target=self._read, daemon=True)
            self._thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self) -> None:
        assert self.proc is not None and self.proc.stdout is not None
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc) -> None:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self._thread is not None:
                self._thread.join(timeout=2)

    def summary(self) -> dict:
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = max(smax, float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- workload


def _workload(config: int, rank: int, world: int, pose_sets: int, actors_override: int = 0):
    """Scenes (compiled, cached) and this rank's pose sets."""
    from navi_b200 import scenes, workloads

    cfg = scenes.CONFIGS[config]
    scene_list = [workloads.compiled_scene(config, s) for s in range(cfg.n_scenes)]
    strong = config == 5
    actors = actors_override or (cfg.actors // world if strong else cfg.actors)
    if config == 5:  # poses re-drawn each step by a random walk (0.1 m, yaw jitter N(0, 5 deg))
        sets = workloads.walk_pose_sets(config, scene_list, pose_sets, actors=actors, seed_offset=1 + 7919 * rank)
    else:
        sets = [workloads.poses_for(config, scene_list, actors=actors, seed_offset=1 + 7919 * rank + 104729 * k)
                for k in range(pose_sets)]
    return cfg, scene_list, sets, strong


def workloads_pose_subset(pb, sel):
    """The actors `sel` of a pose batch."""
    from navi_b200 import workloads

    return workloads.PoseBatch(pb.position[sel], pb.yaw[sel], pb.pitch[sel], pb.scene[sel])


def _device_poses(torch, tracer, pb, dev):
    pos = torch.from_numpy(pb.position).to(dev)
    yaw = torch.from_numpy(pb.yaw).to(dev)
    pitch = torch.from_numpy(pb.pitch).to(dev)
    scene = torch.from_numpy(pb.scene).to(dev)
    return tracer.make_poses(pos, yaw, pitch, scene)


def _eager_dirs(torch, fan_dev, poses_dev):
    """World directions as the reference builds them (eager torch ops; sdfdag_backend.py:1299-1312)."""
    cy = poses_dev[:, 3:4]
    sy = poses_dev[:, 4:5]
    cp = poses_dev[:, 5:6]
    sp = poses_dev[:, 6:7]
    a = poses_dev.shape[0]
    base = fan_dev.unsqueeze(0).expand(a, -1, -1)
    by = base[..., 1] * cp - base[..., 2] * sp
    bz = base[..., 1] * sp + base[..., 2] * cp
    dirs = torch.empty((a, fan_dev.shape[0], 3), dtype=torch.float32, device=fan_dev.device)
    dirs[..., 0] = base[..., 0] * cy + bz * sy
    dirs[..., 1] = by
    dirs[..., 2] = -base[..., 0] * sy + bz * cy
    origins = poses_dev[:, 0:3].unsqueeze(1).expand(-1, fan_dev.shape[0], -1).contiguous()
    return origins, dirs


# ----------------------------------------------------------------------------- reference arm


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    from oracle import build as OB

    OB.build_oracle()
    cfg, scene_list, sets, _strong = _workload(args.config, 0, 1, 1, args.actors)
    from navi_b200.fan import build_spherical_ray_directions

    fan = build_spherical_ray_directions(cfg.azimuth_bins, cfg.elevation_bins)
    pb = sets[0]
    cores = O.cpu_count()
    # bounded sample: enough actors for a few seconds per step on this host
    sample = args.cpu_sample_actors or max(1, min(pb.position.shape[0], int(2 * cores)))
    sel = np.arange(sample)
    dirs = O.rotate_fan(fan, np.cos(pb.yaw[sel]), np.sin(pb.yaw[sel]), np.cos(pb.pitch[sel]), np.sin(pb.pitch[sel]))
    origins = np.repeat(pb.position[sel][:, None, :], fan.shape[0], axis=1)
    sc_ids = pb.scene[sel]
    rays = origins.shape[0] * origins.shape[1]

    def one_step():
        for s, cs in enumerate(scene_list):
            m = sc_ids == s
            if not np.any(m):
                continue
            O.trace(cs.words, cs.bbox_min, cs.bbox_max, origins[m], dirs[m], max_steps=cfg.max_steps,
                    max_distance=cfg.max_distance, hit_epsilon=cs.hit_epsilon, threads=cores)

    for _ in range(args.warmup):
        one_step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_step()
    dt = time.perf_counter() - t0
    value = rays * args.steps / dt
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1e3 * dt / args.steps,
        "higher_is_better": True,
        "scaling": "strong" if args.config == 5 else "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded scenes compiled to .gmdag; seeded free-space poses)",
        "config": {"workload": cfg.name, "config_index": cfg.index, "rays_per_step": rays,
                   "sample": f"{sample} of {pb.position.shape[0]} actors of one pose set"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{sample} actors x {fan.shape[0]} rays per step (oracle/trace_oracle.c, OpenMP)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    line["ref_cuda_kernel"] = _time_reference_kernel(cfg, scene_list, sets[0], fan, args)
    print(json.dumps(line), flush=True)


def _time_reference_kernel(cfg, scene_list, pb, fan, args) -> dict | None:
    """The reference's own CUDA kernel (sm_100a build of kernel.cu) on the full explicit-ray step.

    With several scenes, the reference casts one scene at a time (sdfdag_backend.py:864-887):
    one launch per scene over that scene's actors, the step time being the sum."""
    try:
        import torch

        if not torch.cuda.is_available():
            return None
        from oracle import oracle as O
        from navi_b200 import tracer

        kern = O.ReferenceKernel(eps_variant=True)
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": str(exc)}
    dev = torch.device("cuda", 0)
    fan_dev = torch.from_numpy(fan).to(dev)
    groups = []
    for s, cs in enumerate(scene_list):
        sel = np.nonzero(pb.scene == s)[0] if len(scene_list) > 1 else np.arange(pb.position.shape[0])
        if sel.size == 0:
            continue
        sub = workloads_pose_subset(pb, sel)
        poses_s = _device_poses(torch, tracer, sub, dev)
        o_s, d_s = _eager_dirs(torch, fan_dev, poses_s)
        n_s = o_s.shape[0] * o_s.shape[1]
        groups.append((cs, torch.from_numpy(O.pad_words(cs.words).view(np.int64)).to(dev), o_s, d_s,
                       torch.empty(n_s, dtype=torch.float32, device=dev), torch.empty(n_s, dtype=torch.int32, device=dev)))
    n = sum(g[2].shape[0] * g[2].shape[1] for g in groups)
    flush = torch.empty(2 * torch.cuda.get_device_properties(dev).L2_cache_size, dtype=torch.uint8, device=dev)
    ms = []
    legacy = torch.cuda.default_stream(dev)
    for i in range(args.warmup + max(3, min(args.steps, 20))):
        flush.zero_()
        step_ms = 0.0
        for cs, dag, o_s, d_s, od, osem in groups:
            torch.cuda.synchronize()
            s0 = torch.cuda.Event(enable_timing=True)
            e0 = torch.cuda.Event(enable_timing=True)
            s0.record(legacy)
            kern.cast(dag, o_s, d_s, od, osem, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                      bbox_min=cs.bbox_min, bbox_max=cs.bbox_max, resolution=cfg.resolution,
                      hit_epsilon=cs.hit_epsilon)
            e0.record(legacy)
            torch.cuda.synchronize()
            step_ms += s0.elapsed_time(e0)
        if i >= args.warmup:
            ms.append(step_ms)
    if len(groups) != 1:
        return {"value": n / (float(np.mean(ms)) / 1e3), "unit": UNIT, "ms_per_step": float(np.mean(ms)),
                "launches_per_step": len(groups),
                "timing": "CUDA events on the legacy default stream around each per-scene launch, summed per step "
                          "(mean), L2 flushed between steps",
                "build": "oracle/_ref/libref_trace_eps.so: reference kernel.cu for sm_100a, kHitEpsilon settable"}
    _, _, origins, _, out_d, out_s = groups[0]
    from oracle import postprocess_ref

    band = _band(scene_list)
    pp = []
    for i in range(max(3, min(args.steps, 10)) + 1):
        torch.cuda.synchronize()
        s0 = torch.cuda.Event(enable_timing=True)
        e0 = torch.cuda.Event(enable_timing=True)
        s0.record()
        postprocess_ref.postprocess(out_d.view(origins.shape[0], -1), out_s.view(origins.shape[0], -1),
                                    az_bins=cfg.azimuth_bins, el_bins=cfg.elevation_bins,
                                    max_distance=cfg.max_distance, structure_band_min_distance=band[0],
                                    structure_band_max_distance=band[1], proximity_distance_threshold=2.0)
        e0.record()
        torch.cuda.synchronize()
        if i:
            pp.append(s0.elapsed_time(e0))
    return {"value": n / (float(np.mean(ms)) / 1e3), "unit": UNIT, "ms_per_step": float(np.mean(ms)),
            "postprocess_ms": float(np.mean(pp)),
            "postprocess": "the reference's torch ops after the cast (sdfdag_backend.py:408-473, :1518-1525)",
            "timing": "CUDA events on the legacy default stream around each launch (mean), L2 flushed between",
            "build": "oracle/_ref/libref_trace_eps.so: reference kernel.cu for sm_100a, kHitEpsilon settable"}


# ----------------------------------------------------------------------------- navi arm


def run_navi(args) -> None:
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from navi_b200 import dist_stats

    dist = dist_stats.init_from_env("nccl", dev)

    from navi_b200 import tracer
    from navi_b200.fan import build_spherical_ray_directions

    tracer.set_option("descent", 0 if args.descent == "grid" else 1)
    # rank 0 compiles (and caches) the scenes first; the others then read the cache
    if dist is not None and rank != 0:
        dist.barrier()
    cfg, scene_list, sets, strong = _workload(args.config, rank, world, args.pose_sets, args.actors)
    if dist is not None and rank == 0:
        dist.barrier()

    fan_np = build_spherical_ray_directions(cfg.azimuth_bins, cfg.elevation_bins)
    fan = torch.from_numpy(fan_np).to(dev)
    pools = [tracer.NodePool.from_words(cs.words, dev) for cs in scene_list]
    sset = tracer.SceneSet(pools, [cs.bbox_min for cs in scene_list], [cs.bbox_max for cs in scene_list],
                           [cs.hit_epsilon for cs in scene_list])
    use_pitch = cfg.pitch_deg > 0
    poses = [_device_poses(torch, tracer, pb, dev) for pb in sets]
    actors = poses[0].shape[0]
    r = fan.shape[0]
    n = actors * r
    out_d = torch.empty(n, dtype=torch.float32, device=dev)
    out_s = torch.empty(n, dtype=torch.int32, device=dev)
    out_steps = torch.empty(n, dtype=torch.int32, device=dev)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    flush = torch.empty(2 * l2, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def cast(k: int) -> None:
        tracer.cast_fan(sset, poses[k % len(poses)], fan, out_d, out_s, max_steps=cfg.max_steps,
                        max_distance=cfg.max_distance, use_pitch=use_pitch, out_steps=out_steps)

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(dev.index if dev.index is not None else 0) as clocks:
        time.sleep(0.3)  # let nvidia-smi start sampling
        for k in range(args.warmup):
            flush.zero_()
            cast(k)
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)
        wall0 = time.perf_counter()
        for k in range(args.steps):
            flush.zero_()
            starts[k].record(stream)
            cast(k)
            ends[k].record(stream)
        torch.cuda.synchronize(dev)
        wall1 = time.perf_counter()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    my_ms = float(sum(step_ms))
    steps_mean = float(out_steps.float().mean().item())

    # explicit-ray kernel on the same rays (the drop-in cast_rays path), device-resident
    o_dev, d_dev = _eager_dirs(torch, fan, poses[0])
    ex_ms = []
    for k in range(max(3, min(args.steps, 10))):
        flush.zero_()
        s0 = torch.cuda.Event(enable_timing=True)
        e0 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        tracer.cast_rays_ex(pools[0], o_dev, d_dev, out_d, out_s, max_steps=cfg.max_steps,
                            max_distance=cfg.max_distance, bbox_min=scene_list[0].bbox_min,
                            bbox_max=scene_list[0].bbox_max, hit_epsilon=scene_list[0].hit_epsilon)
        e0.record(stream)
        torch.cuda.synchronize(dev)
        if k > 0 or args.steps < 2:
            ex_ms.append(s0.elapsed_time(e0))
    explicit = None
    if len(scene_list) == 1:
        explicit = {"value": n / (np.median(ex_ms) / 1e3), "unit": UNIT, "ms_per_step": float(np.median(ex_ms))}

    observe = None if args.no_e2e else _observe(torch, tracer, args, cfg, sset, poses[0], fan, use_pitch, flush, dev,
                                                 scene_list)
    e2e = None if args.no_e2e or len(scene_list) != 1 else _e2e(torch, args, cfg, scene_list[0], o_dev, d_dev, flush, dev)
    e2e_fan = None if args.no_e2e else _e2e_fan(torch, tracer, args, cfg, sset, sets[0], fan, use_pitch, flush, dev)

    # gather per-rank [rays, ms, steps_mean] over NCCL; job time = max over ranks
    stats = torch.tensor([float(n * args.steps), my_ms, steps_mean], dtype=torch.float64, device=dev)
    table = dist_stats.gather_rank_stats(stats, dist)
    total_rays, job_ms = dist_stats.job_figures(table)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = _cpu_baseline(args, cfg, scene_list, sets[0], fan_np, poses[0].cpu().numpy())

    if rank == 0:
        value = total_rays / (job_ms / 1e3)
        per_launch_ms = job_ms / args.steps
        peak, peak_kind = _peaks()
        w_ref = cpu["w_ref_mean"] if cpu else None
        roof = None
        if w_ref is not None:
            bytes_per_ray = 8.0 * w_ref + 12.0
            achieved = n * bytes_per_ray / (float(np.mean(step_ms)) / 1e3) / 1e9
            roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                    "traffic": _traffic(cfg.name), "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                    "bytes_per_ray": bytes_per_ray, "w_ref_mean": w_ref,
                    "kernel": "trace_kernel<fan>"}
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": per_launch_ms,
            "higher_is_better": True,
            "scaling": "strong" if strong else "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded scenes compiled to .gmdag by the in-tree voxel-dag compiler; seeded free-space poses)",
            "config": {
                "workload": cfg.name,
                "config_index": cfg.index,
                "scenes": len(scene_list),
                "resolution": cfg.resolution,
                "actors_per_rank": actors,
                "rays_per_actor": r,
                "rays_per_step_per_rank": n,
                "max_steps": cfg.max_steps,
                "max_distance": cfg.max_distance,
                "hit_epsilon": "1e-3 x voxel",
                "pitch_deg": cfg.pitch_deg,
                "poses": (f"random walk: {args.pose_sets} successive steps cycled" if args.config == 5
                          else f"uniform in free space: {args.pose_sets} independent sets cycled"),
                "parallelism": f"dp{world} (scene replica per GPU, no hot-path collective)",
                "l2": "flushed between steps (2 x L2 bytes written), outside the timed events",
                "pool_bytes": int(sum(p.stats["device_bytes"] for p in pools)),
                "descent": args.descent,
            },
            # per step: one scene: the claim-order key and scatter kernels and the trace kernel;
            # 2-64 scenes: the scene sort, per scene the key, scatter and trace kernels, and
            # the unknown-scene fill
            "gpu_launches": args.steps * (3 if len(scene_list) == 1 else
                                          (3 * len(scene_list) + 2 if len(scene_list) <= 64 else 2)),
            "clocks": clocks.summary(),
            "e2e": e2e,
            "e2e_fan": e2e_fan,
            "explicit_rays": explicit,
            "observe": observe,
            "roofline": roof,
            "cpu_baseline": None if cpu is None else {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "per_rank_ms": [float(x) for x in table[:, 1]],
            "mean_steps_per_ray": float(np.mean(table[:, 2])),
            "wall_s": wall1 - wall0,
        }
        print(json.dumps(line), flush=True)
    del sset, pools
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def _traffic(workload: str):
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(workload)
    except ValueError:
        return None


def _observe(torch, tracer, args, cfg, sset, poses, fan, use_pitch, flush, dev, scene_list) -> dict:
    """Cast followed by the reference's post-processing as one pass over its outputs
    (observation [A,3,Az,El] + per-actor ratios).  The reference's own post-processing
    (eager torch ops after the cast) is timed by the --impl reference arm."""
    a, r = poses.shape[0], fan.shape[0]
    az, el = cfg.azimuth_bins, cfg.elevation_bins
    band = _band(scene_list)
    od = torch.empty(a * r, device=dev)
    os_ = torch.empty(a * r, dtype=torch.int32, device=dev)
    obs = torch.empty((a, 3, az, el), device=dev)
    st = torch.empty((a, 5), device=dev)
    stream = torch.cuda.current_stream(dev)

    def fused():
        tracer.cast_fan_observe(sset, poses, fan, az, el, od, os_, obs, st, max_steps=cfg.max_steps,
                                max_distance=cfg.max_distance, structure_band_min=band[0], structure_band_max=band[1],
                                proximity_threshold=2.0, use_pitch=use_pitch)

    fused()
    ms = []
    for _ in range(max(3, min(args.steps, 10))):
        flush.zero_()
        s0 = torch.cuda.Event(enable_timing=True)
        e0 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        fused()
        e0.record(stream)
        torch.cuda.synchronize(dev)
        ms.append(s0.elapsed_time(e0))
    return {"cast_observe_ms": float(np.mean(ms)), "structure_band": list(band), "proximity": 2.0}


def _band(scene_list) -> tuple[float, float]:
    """Structure band of the reference env: [1.5, min(0.6 x extent, 50)] (sdfdag_backend.py:1920-1926)."""
    ext = float(scene_list[0].bbox_max[0] - scene_list[0].bbox_min[0])
    return 1.5, max(2.5, min(0.6 * ext, 50.0))


def _e2e(torch, args, cfg, cs, o_dev, d_dev, flush, dev) -> dict:
    """torch_sdf.cast_rays (the reference-facing call) with pinned host inputs and outputs."""
    import torch_sdf

    b, r = o_dev.shape[0], o_dev.shape[1]
    h_o = o_dev.cpu().pin_memory()
    h_d = d_dev.cpu().pin_memory()
    h_od = torch.empty((b, r), dtype=torch.float32).pin_memory()
    h_os = torch.empty((b, r), dtype=torch.int32).pin_memory()
    g_o = torch.empty_like(o_dev)
    g_d = torch.empty_like(d_dev)
    g_od = torch.empty((b, r), dtype=torch.float32, device=dev)
    g_os = torch.empty((b, r), dtype=torch.int32, device=dev)
    dag = torch.from_numpy(cs.words.view(np.int64)).to(dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        g_o.copy_(h_o, non_blocking=True)
        g_d.copy_(h_d, non_blocking=True)
        torch_sdf.cast_rays(dag, g_o, g_d, g_od, g_os, cfg.max_steps, cfg.max_distance, cs.bbox_min,
                            cs.bbox_max, cfg.resolution, skip_direction_validation=True,
                            hit_epsilon=cs.hit_epsilon)
        h_od.copy_(g_od, non_blocking=True)
        h_os.copy_(g_os, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    ms = []
    for _ in range(max(3, min(args.steps, 10))):
        flush.zero_()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        step()
        e.record(stream)
        torch.cuda.synchronize(dev)
        ms.append(s.elapsed_time(e))
    n = b * r
    return {"value": n / (float(np.mean(ms)) / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(2 * n * 12),
            "d2h_bytes_per_step": int(n * 8), "api": "torch_sdf.cast_rays (pinned host origins/dirs in, dist/sem out)"}


def _e2e_fan(torch, tracer, args, cfg, sset, pb, fan, use_pitch, flush, dev) -> dict:
    """Pose-fused cast with the per-actor poses uploaded and dist/sem/steps read back every step."""
    a = pb.position.shape[0]
    r = fan.shape[0]
    n = a * r
    h_pos = torch.from_numpy(pb.position).pin_memory()
    h_yaw = torch.from_numpy(pb.yaw).pin_memory()
    h_pitch = torch.from_numpy(pb.pitch).pin_memory()
    h_scene = torch.from_numpy(pb.scene).pin_memory()
    g_pos = torch.empty((a, 3), dtype=torch.float32, device=dev)
    g_yaw = torch.empty(a, dtype=torch.float32, device=dev)
    g_pitch = torch.empty(a, dtype=torch.float32, device=dev)
    g_scene = torch.empty(a, dtype=torch.int32, device=dev)
    poses = torch.empty((a, 8), dtype=torch.float32, device=dev)
    g_d = torch.empty(n, dtype=torch.float32, device=dev)
    g_s = torch.empty(n, dtype=torch.int32, device=dev)
    g_k = torch.empty(n, dtype=torch.int32, device=dev)
    h_d = torch.empty(n, dtype=torch.float32).pin_memory()
    h_s = torch.empty(n, dtype=torch.int32).pin_memory()
    h_k = torch.empty(n, dtype=torch.int32).pin_memory()
    stream = torch.cuda.current_stream(dev)

    def step():
        g_pos.copy_(h_pos, non_blocking=True)
        g_yaw.copy_(h_yaw, non_blocking=True)
        g_pitch.copy_(h_pitch, non_blocking=True)
        g_scene.copy_(h_scene, non_blocking=True)
        tracer.make_poses(g_pos, g_yaw, g_pitch, g_scene, out=poses)
        tracer.cast_fan(sset, poses, fan, g_d, g_s, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                        use_pitch=use_pitch, out_steps=g_k)
        h_d.copy_(g_d, non_blocking=True)
        h_s.copy_(g_s, non_blocking=True)
        h_k.copy_(g_k, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    ms = []
    for _ in range(max(3, min(args.steps, 10))):
        flush.zero_()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        step()
        e.record(stream)
        torch.cuda.synchronize(dev)
        ms.append(s.elapsed_time(e))
    return {"value": n / (float(np.mean(ms)) / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(a * 24),
            "d2h_bytes_per_step": int(n * 12), "api": "navi_b200.tracer.cast_fan (host poses in, dist/sem/steps out)"}


def _cpu_baseline(args, cfg, scene_list, pb, fan_np, poses_host) -> dict:
    """Reference algorithm on the host cores (oracle/ C restatement, OpenMP), on a bounded sample.

    Also returns the mean DAG word loads per ray (W_ref) of the sample, the
    per-ray figure of the roofline accounting."""
    from oracle import build as OB
    from oracle import oracle as O

    OB.build_oracle()
    cores = O.cpu_count()
    a = pb.position.shape[0]
    sample = args.cpu_sample_actors or max(1, min(a, 2 * cores))
    sel = np.arange(sample)
    ph = poses_host[sel]
    dirs = O.rotate_fan(fan_np, ph[:, 3], ph[:, 4], ph[:, 5], ph[:, 6])
    origins = np.repeat(pb.position[sel][:, None, :], fan_np.shape[0], axis=1)
    loads = []
    rays = 0
    t0 = time.perf_counter()
    for s, cs in enumerate(scene_list):
        m = pb.scene[sel] == s
        if not np.any(m):
            continue
        res = O.trace(cs.words, cs.bbox_min, cs.bbox_max, origins[m], dirs[m], max_steps=cfg.max_steps,
                      max_distance=cfg.max_distance, hit_epsilon=cs.hit_epsilon, threads=cores)
        loads.append(res["loads"])
        rays += res["loads"].shape[0]
    dt = time.perf_counter() - t0
    return {"value": rays / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{sample} of {a} actors x {fan_np.shape[0]} rays (oracle/trace_oracle.c, OpenMP, {cores} threads)",
            "w_ref_mean": float(np.concatenate(loads).mean())}


def main() -> None:
    args = _args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_navi(args)


if __name__ == "__main__":
    main()
