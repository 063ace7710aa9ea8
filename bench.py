"""Benchmark: batched sphere tracing of spherical ray fans through .gmdag DAGs on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl navi|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)

A step is one cast of every actor's full fan of the configuration.  The default
is configuration 5, the largest that fits one GPU: 16 resident 512^3 scenes,
32,768 actors x 256 x 48 rays = 402,653,184 rays per step, the actors split
evenly across the N ranks (strong scaling; every rank holds a replica of all
scenes).  Configurations 1-4 give every rank the full configuration (weak
scaling).  At N=1 the line also carries configurations 2, 3 and 4 measured in
the same run (`configs`; --extra-configs).

Timing: per step, CUDA events on the launching stream around the cast; L2 is
flushed (a buffer of 2x the L2 size is written) between steps, outside the
events; W warm-up steps first; the job time is the max over ranks (gathered
over NCCL after the timed region).  `e2e` is the same cast through the drop-in
torch_sdf.cast_rays with host (pinned) origins/dirs copied in and host
distances/semantics copied out inside the timed region, one call per scene
group (the reference backend casts one scene at a time) or per quarter of a
single scene's rays, the copies overlapped with the casts on side streams
(navi_b200.pipeline); at N>1 it is box-wide (rays of all ranks over the slowest
rank's time).  Printed: one JSON line on rank 0.

`--impl reference` times the reference algorithm on the host cores instead
(the C restatement in oracle/, OpenMP over rays, all host threads) on a
bounded sample of the same workload, with scenes compiled by the reference's
own compiler (oracle/_ref); it also times the reference's own CUDA kernel built
for sm_100a (oracle/_ref) on the same rays when that build exists.  That arm
maps none of this repository's libraries.
"""

from __future__ import annotations

import argparse
import ctypes
import json
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
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=5)
    ap.add_argument("--impl", choices=["navi", "reference"], default="navi")
    ap.add_argument("--pose-sets", type=int, default=4, help="distinct pose sets cycled over the steps")
    ap.add_argument("--actors", type=int, default=0,
                    help="actors per rank instead of the configuration's (0 = the configuration's; for small profiles)")
    ap.add_argument("--extra-configs", default="2,3,4",
                    help="configurations also measured at N=1 and reported under `configs` ('' for none)")
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
    """nvidia-smi clocks and throttle reasons sampled every 100 ms while running."""

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


def _actors_per_rank(cfg, world: int, override: int) -> int:
    return override or (cfg.actors // world if cfg.index == 5 else cfg.actors)


def _pose_sets(config: int, scene_list, rank: int, pose_sets: int, actors: int):
    """This rank's pose sets: config 5 a random walk (0.1 m, yaw jitter N(0, 5 deg)), the
    others independent uniform draws.  scene_list entries need only `.mesh`."""
    from navi_b200 import workloads

    if config == 5:
        return workloads.walk_pose_sets(config, scene_list, pose_sets, actors=actors, seed_offset=1 + 7919 * rank)
    return [workloads.poses_for(config, scene_list, actors=actors, seed_offset=1 + 7919 * rank + 104729 * k)
            for k in range(pose_sets)]


def _config_dict(args, cfg, world: int, actors: int) -> dict:
    """The workload description printed by both arms (identical for the same command)."""
    r = cfg.azimuth_bins * cfg.elevation_bins
    return {
        "workload": cfg.name,
        "config_index": cfg.index,
        "scenes": cfg.n_scenes,
        "resolution": cfg.resolution,
        "actors_total": actors * world if cfg.index == 5 else cfg.actors * world,
        "actors_per_rank": actors,
        "rays_per_actor": r,
        "rays_per_step_per_rank": actors * r,
        "max_steps": cfg.max_steps,
        "max_distance": cfg.max_distance,
        "hit_epsilon": "1e-3 x voxel",
        "pitch_deg": cfg.pitch_deg,
        "poses": (f"random walk: {args.pose_sets} successive steps cycled" if cfg.index == 5
                  else f"uniform in free space: {args.pose_sets} independent sets cycled"),
        "parallelism": f"dp{world} (scene replica per GPU, actors split, no hot-path collective)" if cfg.index == 5
        else f"dp{world} (scene replica per GPU, full configuration per rank, no hot-path collective)",
        "l2": "flushed between steps (2 x L2 bytes written), outside the timed events",
    }


def _eager_pose_rays(torch, fan_dev, position, yaw, pitch, use_pitch: bool):
    """World rays as the reference builds them: cos/sin by torch.cos / torch.sin on the device,
    each product and sum an eager op (sdfdag_backend.py:1299-1312), plus the configurations'
    pitch rotation of the local fan; origins = position repeated per ray."""
    a, r = position.shape[0], fan_dev.shape[0]
    cy = torch.cos(yaw).unsqueeze(1)
    sy = torch.sin(yaw).unsqueeze(1)
    base = fan_dev.unsqueeze(0).expand(a, -1, -1)
    if use_pitch:
        cp = torch.cos(pitch).unsqueeze(1)
        sp = torch.sin(pitch).unsqueeze(1)
        by = base[..., 1] * cp - base[..., 2] * sp
        bz = base[..., 1] * sp + base[..., 2] * cp
    else:
        by = base[..., 1]
        bz = base[..., 2]
    dirs = torch.empty((a, r, 3), dtype=torch.float32, device=fan_dev.device)
    dirs[..., 0] = base[..., 0] * cy + bz * sy
    dirs[..., 1] = by
    dirs[..., 2] = -base[..., 0] * sy + bz * cy
    origins = position.unsqueeze(1).expand(-1, r, -1).contiguous()
    return origins, dirs


def _band(scene_list) -> tuple[float, float]:
    """Structure band of the reference env: [1.5, min(0.6 x extent, 50)] (sdfdag_backend.py:1920-1926)."""
    ext = float(scene_list[0].bbox_max[0] - scene_list[0].bbox_min[0])
    return 1.5, max(2.5, min(0.6 * ext, 50.0))


def _traffic(workload: str):
    """DRAM bytes per step of the trace kernels, from the committed ncu summaries."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        v = json.loads(p.read_text()).get(workload)
    except ValueError:
        return None
    return v


# ----------------------------------------------------------------------------- reference arm


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from navi_b200 import scenes
    from navi_b200.fan import build_spherical_ray_directions
    from oracle import build as OB
    from oracle import oracle as O
    from oracle import ref_scenes

    OB.build_oracle()
    cfg = scenes.CONFIGS[args.config]
    scene_note = "projects/voxel-dag compiler (oracle/_ref/ref_voxel_dag), read by oracle/gmdag_ref.py"
    if cfg.resolution <= ref_scenes.MAX_RESOLUTION:
        scene_list = ref_scenes.config_scenes(args.config)
    else:  # the reference compiler's int voxel indices overflow above 1290^3
        from navi_b200 import workloads

        scene_list = [workloads.compiled_scene(args.config, s) for s in range(cfg.n_scenes)]
        scene_note = ("in-tree compiler (the reference compiler overflows its int voxel indices above 1290^3; "
                      "the in-tree compiler's words equal it bit for bit at 64^3-512^3)")
    actors = _actors_per_rank(cfg, world, args.actors)
    sets = _pose_sets(args.config, scene_list, 0, 1, actors)
    fan = build_spherical_ray_directions(cfg.azimuth_bins, cfg.elevation_bins)
    pb = sets[0]
    cores = O.cpu_count()
    # bounded sample: enough actors for a fraction of a second per step on this host
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
        "config": _config_dict(args, cfg, world, actors),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{sample} of {pb.position.shape[0]} actors x {fan.shape[0]} rays per step of rank 0's "
                                   f"share (oracle/trace_oracle.c, the reference kernel restated in C, OpenMP, "
                                   f"{cores} threads; the reference has no CPU trace path)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "scenes_from": scene_note,
    }
    line["ref_cuda_kernel"] = _time_reference_kernel(cfg, scene_list, pb, fan, args)
    print(json.dumps(line), flush=True)


def _time_reference_kernel(cfg, scene_list, pb, fan, args) -> dict | None:
    """The reference's own CUDA kernel (sm_100a build of kernel.cu) on every ray of rank 0's step.

    With several scenes, the reference casts one scene at a time (sdfdag_backend.py:864-887):
    one launch per scene over that scene's actors, the step time being the sum."""
    try:
        import torch

        if not torch.cuda.is_available():
            return None
        from oracle import oracle as O

        kern = O.ReferenceKernel(eps_variant=True)
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": str(exc)}
    dev = torch.device("cuda", 0)
    fan_dev = torch.from_numpy(fan).to(dev)
    use_pitch = cfg.pitch_deg > 0
    groups = []
    for s, cs in enumerate(scene_list):
        sel = np.nonzero(pb.scene == s)[0]
        if sel.size == 0:
            continue
        o_s, d_s = _eager_pose_rays(torch, fan_dev, torch.from_numpy(pb.position[sel]).to(dev),
                                    torch.from_numpy(pb.yaw[sel]).to(dev), torch.from_numpy(pb.pitch[sel]).to(dev),
                                    use_pitch)
        n_s = o_s.shape[0] * o_s.shape[1]
        groups.append((cs, torch.from_numpy(O.pad_words(cs.words).view(np.int64)).to(dev), o_s, d_s,
                       torch.empty(n_s, dtype=torch.float32, device=dev), torch.empty(n_s, dtype=torch.int32, device=dev)))
    n = sum(g[2].shape[0] * g[2].shape[1] for g in groups)
    flush = torch.empty(2 * torch.cuda.get_device_properties(dev).L2_cache_size, dtype=torch.uint8, device=dev)
    legacy = torch.cuda.default_stream(dev)
    n_timed = max(1, min(args.steps, 3 if n > 50_000_000 else 20))
    n_warm = 1 if n > 50_000_000 else max(1, args.warmup)
    ms = []
    for i in range(n_warm + n_timed):
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
        if i >= n_warm:
            ms.append(step_ms)
    out = {"value": n / (float(np.mean(ms)) / 1e3), "unit": UNIT, "ms_per_step": float(np.mean(ms)),
           "rays_per_step": int(n), "launches_per_step": len(groups), "steps_timed": len(ms),
           "timing": "CUDA events on the legacy default stream around each per-scene launch, summed per step "
                     "(mean), L2 flushed between steps",
           "build": "oracle/_ref/libref_trace_eps.so: reference kernel.cu for sm_100a, kHitEpsilon settable"}
    if len(groups) == 1:
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
        out["postprocess_ms"] = float(np.mean(pp))
        out["postprocess"] = "the reference's torch ops after the cast (sdfdag_backend.py:408-473, :1518-1525)"
    return out


# ----------------------------------------------------------------------------- navi arm


class FanWorkload:
    """One configuration on one rank: scenes (compiled, cached), pools, scene table, poses, buffers."""

    def __init__(self, torch, args, config: int, rank: int, world: int, dev, pose_sets: int, actors_override: int = 0,
                 dist=None):
        from navi_b200 import scenes, tracer, workloads
        from navi_b200.fan import build_spherical_ray_directions

        self.cfg = cfg = scenes.CONFIGS[config]
        # rank 0 compiles (and caches) the scenes first; the others then read the cache
        if dist is not None and rank != 0:
            dist.barrier()
        self.scene_list = [workloads.compiled_scene(config, s) for s in range(cfg.n_scenes)]
        if dist is not None and rank == 0:
            dist.barrier()
        self.actors = _actors_per_rank(cfg, world, actors_override)
        self.sets = _pose_sets(config, self.scene_list, rank, pose_sets, self.actors)
        self.fan_np = build_spherical_ray_directions(cfg.azimuth_bins, cfg.elevation_bins)
        self.fan = torch.from_numpy(self.fan_np).to(dev)
        self.pools = [tracer.NodePool.from_words(cs.words, dev) for cs in self.scene_list]
        self.sset = tracer.SceneSet(self.pools, [cs.bbox_min for cs in self.scene_list],
                                    [cs.bbox_max for cs in self.scene_list],
                                    [cs.hit_epsilon for cs in self.scene_list])
        self.use_pitch = cfg.pitch_deg > 0
        self.poses = [self._device_poses(torch, pb, dev) for pb in self.sets]
        self.r = self.fan.shape[0]
        self.n = self.actors * self.r
        self.out_d = torch.empty(self.n, dtype=torch.float32, device=dev)
        self.out_s = torch.empty(self.n, dtype=torch.int32, device=dev)
        self.out_steps = torch.empty(self.n, dtype=torch.int32, device=dev)
        self.dev = dev
        self.pool_bytes = int(sum(p.stats["device_bytes"] for p in self.pools))

    @staticmethod
    def _device_poses(torch, pb, dev):
        from navi_b200 import tracer

        return tracer.make_poses(torch.from_numpy(pb.position).to(dev), torch.from_numpy(pb.yaw).to(dev),
                                 torch.from_numpy(pb.pitch).to(dev), torch.from_numpy(pb.scene).to(dev))

    def cast(self, k: int) -> None:
        from navi_b200 import tracer

        tracer.cast_fan(self.sset, self.poses[k % len(self.poses)], self.fan, self.out_d, self.out_s,
                        max_steps=self.cfg.max_steps, max_distance=self.cfg.max_distance, use_pitch=self.use_pitch,
                        out_steps=self.out_steps)

    def launches_per_step(self) -> int:
        # one scene: the claim-order key and scatter kernels and the trace kernel; 2-64 scenes:
        # the scene sort, per scene the key, scatter and trace kernels, and the unknown-scene fill
        ns = len(self.scene_list)
        return 3 if ns == 1 else (3 * ns + 2 if ns <= 64 else 2)

    def close(self) -> None:
        self.sset.close()
        for p in self.pools:
            p.close()


def _timed_steps(torch, wl: FanWorkload, steps: int, warmup: int, flush, stream, dist=None, clocks=None):
    """W untimed casts, then `steps` casts each bracketed by CUDA events on `stream` (L2 flushed
    before each, outside the events); barrier + synchronize on both sides of the timed loop."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for k in range(warmup):
        flush.zero_()
        wl.cast(k)
    torch.cuda.synchronize(wl.dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(wl.dev)
    wall0 = time.perf_counter()
    for k in range(steps):
        flush.zero_()
        starts[k].record(stream)
        wl.cast(k)
        ends[k].record(stream)
    torch.cuda.synchronize(wl.dev)
    wall1 = time.perf_counter()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)], wall1 - wall0


def _l2_read_peak(torch, dev) -> dict | None:
    """Measured L2 read bandwidth: a 16-byte-load read loop over an L2-resident buffer
    (navi_b200/csrc/peak_probe.cu), best of 10 launches, CUDA events."""
    lib_path = ROOT / "navi_b200" / "_lib" / "libnavi_probe.so"
    if not lib_path.exists():
        return None
    lib = ctypes.CDLL(str(lib_path))
    lib.navi_probe_l2_read.restype = ctypes.c_int
    lib.navi_probe_l2_read.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                       ctypes.c_void_p]
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    blocks = sms * 4  # 4 blocks of 512 threads per SM
    per_sweep = blocks * 512 * 8 * 16  # bytes one sweep of the grid reads (8 loads in flight per thread)
    sweeps = max(1, (32 << 20) // per_sweep)
    nbytes = sweeps * per_sweep
    reps = 64
    buf = torch.randint(0, 1 << 30, (nbytes // 4,), dtype=torch.int32, device=dev)
    sink = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    ms = []
    for i in range(13):
        s0 = torch.cuda.Event(enable_timing=True)
        e0 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        rc = lib.navi_probe_l2_read(ctypes.c_void_p(buf.data_ptr()), nbytes, reps, blocks,
                                    ctypes.c_void_p(sink.data_ptr()), ctypes.c_void_p(stream.cuda_stream))
        e0.record(stream)
        if rc != 0:
            return None
        torch.cuda.synchronize(dev)
        if i >= 3:
            ms.append(s0.elapsed_time(e0))
    gbs = nbytes * reps / (min(ms) / 1e3) / 1e9
    return {"gbs": gbs, "buffer_bytes": int(nbytes), "bytes_per_launch": int(nbytes * reps),
            "how": "navi_b200/csrc/peak_probe.cu: ld.global.cg 16-byte loads over an L2-resident buffer, "
                   f"{blocks} x 512 threads, best of 10 launches (CUDA events)"}


def _w_ref(cfg, scene_list, pb, fan_np, poses_host, sample: int) -> tuple[float, float, int, int]:
    """Mean DAG word loads per ray of the reference algorithm (W_ref) on a sample of actors,
    counted by the oracle (oracle/trace_oracle.c, all host threads); also the oracle's
    rays/s on that sample."""
    from oracle import build as OB
    from oracle import oracle as O

    OB.build_oracle()
    cores = O.cpu_count()
    sel = np.arange(min(sample, pb.position.shape[0]))
    ph = poses_host[sel]
    dirs = O.rotate_fan(fan_np, ph[:, 3], ph[:, 4], ph[:, 5], ph[:, 6])
    origins = np.repeat(pb.position[sel][:, None, :], fan_np.shape[0], axis=1)
    loads = []
    t0 = time.perf_counter()
    for s, cs in enumerate(scene_list):
        m = pb.scene[sel] == s
        if not np.any(m):
            continue
        res = O.trace(cs.words, cs.bbox_min, cs.bbox_max, origins[m], dirs[m], max_steps=cfg.max_steps,
                      max_distance=cfg.max_distance, hit_epsilon=cs.hit_epsilon, threads=cores)
        loads.append(res["loads"])
    dt = time.perf_counter() - t0
    allv = np.concatenate(loads)
    return float(allv.mean()), allv.shape[0] / dt, cores, int(sel.shape[0])


def _roofline(n_rays: int, step_ms: list[float], w_ref: float, hbm: float, hbm_kind: str, l2: dict | None,
              traffic) -> dict:
    bytes_per_ray = 8.0 * w_ref + 12.0
    achieved = n_rays * bytes_per_ray / (float(np.mean(step_ms)) / 1e3) / 1e9
    roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
            "traffic": traffic, "peak_source": f"{hbm_kind} hbm_gbs (MEASURED_PEAKS.json)",
            "bytes_per_ray": bytes_per_ray, "w_ref_mean": w_ref, "kernel": "trace_grid_kernel<fan>",
            "per": "step (one cast of every actor of the rank)"}
    if l2 is not None:
        roof["l2_peak"] = l2["gbs"]
        roof["l2_frac"] = achieved / l2["gbs"]
        roof["l2_peak_source"] = "measured live: " + l2["how"]
    return roof


def _explicit(torch, wl: FanWorkload, args, flush, stream) -> dict:
    """The explicit-ray kernel (tracer.cast_rays_ex, the path under torch_sdf.cast_rays) on the
    same rays, device-resident."""
    from navi_b200 import tracer

    pb, cs = wl.sets[0], wl.scene_list[0]
    o, v = _eager_pose_rays(torch, wl.fan, torch.from_numpy(pb.position).to(wl.dev), torch.from_numpy(pb.yaw).to(wl.dev),
                            torch.from_numpy(pb.pitch).to(wl.dev), wl.use_pitch)
    ms = []
    for k in range(max(3, min(args.steps, 10))):
        flush.zero_()
        s0 = torch.cuda.Event(enable_timing=True)
        e0 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        tracer.cast_rays_ex(wl.pools[0], o, v, wl.out_d, wl.out_s, max_steps=wl.cfg.max_steps,
                            max_distance=wl.cfg.max_distance, bbox_min=cs.bbox_min, bbox_max=cs.bbox_max,
                            hit_epsilon=cs.hit_epsilon)
        e0.record(stream)
        torch.cuda.synchronize(wl.dev)
        if k > 0:
            ms.append(s0.elapsed_time(e0))
    return {"value": wl.n / (float(np.median(ms)) / 1e3), "unit": UNIT, "ms_per_step": float(np.median(ms))}


def _observe(torch, wl: FanWorkload, args, flush) -> dict:
    """Cast followed by the reference's post-processing as one pass over its outputs
    (observation [A,3,Az,El] + per-actor ratios)."""
    from navi_b200 import tracer

    cfg = wl.cfg
    a, r = wl.actors, wl.r
    band = _band(wl.scene_list)
    obs = torch.empty((a, 3, cfg.azimuth_bins, cfg.elevation_bins), device=wl.dev)
    st = torch.empty((a, 5), device=wl.dev)
    stream = torch.cuda.current_stream(wl.dev)

    def fused():
        tracer.cast_fan_observe(wl.sset, wl.poses[0], wl.fan, cfg.azimuth_bins, cfg.elevation_bins, wl.out_d,
                                wl.out_s, obs, st, max_steps=cfg.max_steps, max_distance=cfg.max_distance,
                                structure_band_min=band[0], structure_band_max=band[1], proximity_threshold=2.0,
                                use_pitch=wl.use_pitch)

    fused()
    ms = []
    for _ in range(max(2, min(args.steps, 5))):
        flush.zero_()
        s0 = torch.cuda.Event(enable_timing=True)
        e0 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        fused()
        e0.record(stream)
        torch.cuda.synchronize(wl.dev)
        ms.append(s0.elapsed_time(e0))
    return {"cast_observe_ms": float(np.mean(ms)), "structure_band": list(band), "proximity": 2.0}


def _e2e(torch, wl: FanWorkload, args, flush, dist) -> tuple[dict, float, float]:
    """torch_sdf.cast_rays (the reference-facing call) with pinned host origins/dirs in and
    host distances/semantics out, every copy inside the timed region.  One call per scene
    group (the reference backend casts one scene at a time, sdfdag_backend.py:864-887), or per
    quarter of a single scene's rays; uploads, casts and downloads overlap on side streams
    (navi_b200.pipeline).  Returns (line entry, rays per step, mean ms per step)."""
    import torch_sdf
    from navi_b200 import pipeline, tracer

    cfg, dev = wl.cfg, wl.dev
    pb, r = wl.sets[0], wl.r
    order = np.argsort(pb.scene, kind="stable")
    groups = []  # (scene, actor lo, actor hi) in the sorted order
    if len(wl.scene_list) == 1:
        q = -(-pb.position.shape[0] // 4)
        groups = [(0, lo, min(lo + q, pb.position.shape[0])) for lo in range(0, pb.position.shape[0], q)]
    else:
        sc_sorted = pb.scene[order]
        for s in range(len(wl.scene_list)):
            idx = np.nonzero(sc_sorted == s)[0]
            if idx.size:
                groups.append((s, int(idx[0]), int(idx[-1]) + 1))
    a = pb.position.shape[0]
    n = a * r
    h_o = torch.empty((a, r, 3), dtype=torch.float32, pin_memory=True)
    h_v = torch.empty((a, r, 3), dtype=torch.float32, pin_memory=True)
    pos = torch.from_numpy(pb.position[order]).to(dev)
    yaw = torch.from_numpy(pb.yaw[order]).to(dev)
    pitch = torch.from_numpy(pb.pitch[order]).to(dev)
    step = 1024
    for lo in range(0, a, step):  # world rays built on the device as the reference does, staged to the host
        o, v = _eager_pose_rays(torch, wl.fan, pos[lo:lo + step], yaw[lo:lo + step], pitch[lo:lo + step],
                                wl.use_pitch)
        h_o[lo:lo + step].copy_(o)
        h_v[lo:lo + step].copy_(v)
    del o, v
    h_d = torch.empty((a, r), dtype=torch.float32, pin_memory=True)
    h_s = torch.empty((a, r), dtype=torch.int32, pin_memory=True)
    g_o = torch.empty((a, r, 3), dtype=torch.float32, device=dev)
    g_v = torch.empty((a, r, 3), dtype=torch.float32, device=dev)
    g_d = torch.empty((a, r), dtype=torch.float32, device=dev)
    g_s = torch.empty((a, r), dtype=torch.int32, device=dev)
    dags = [torch.from_numpy(cs.words.view(np.int64)).to(dev) for cs in wl.scene_list]
    for dag, pool in zip(dags, wl.pools):
        tracer.register_pool(dag, pool)  # same words: the drop-in call reuses the resident pool
    chunks = []
    for s, lo, hi in groups:
        cs = wl.scene_list[s]

        def run(s=s, lo=lo, hi=hi, cs=cs):
            torch_sdf.cast_rays(dags[s], g_o[lo:hi], g_v[lo:hi], g_d[lo:hi], g_s[lo:hi], cfg.max_steps,
                                cfg.max_distance, cs.bbox_min, cs.bbox_max, cfg.resolution,
                                skip_direction_validation=True, hit_epsilon=cs.hit_epsilon)
        chunks.append(pipeline.Chunk(run, [(g_o[lo:hi], h_o[lo:hi]), (g_v[lo:hi], h_v[lo:hi])],
                                     [(h_d[lo:hi], g_d[lo:hi]), (h_s[lo:hi], g_s[lo:hi])]))
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(1, min(args.warmup, 2))):
        pipeline.run_chunks(chunks, dev)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    ms = []
    for _ in range(max(2, min(args.steps, 5))):
        flush.zero_()
        s0 = torch.cuda.Event(enable_timing=True)
        e0 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        pipeline.run_chunks(chunks, dev)
        e0.record(stream)
        torch.cuda.synchronize(dev)
        ms.append(s0.elapsed_time(e0))
    mean_ms = float(np.mean(ms))
    entry = {"value": n / (mean_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(n * 24),
             "d2h_bytes_per_step": int(n * 8),
             "api": f"torch_sdf.cast_rays, {len(groups)} calls per step (pinned host origins/dirs in, dist/sem out; "
                    "copies overlapped on side streams by navi_b200.pipeline)"}
    return entry, float(n), mean_ms


def _e2e_fan(torch, wl: FanWorkload, args, flush) -> dict:
    """Pose-fused cast with host poses in and host dist/sem/steps out (navi_b200.pipeline.cast_fan_host)."""
    from navi_b200 import pipeline

    cfg = wl.cfg
    a, r = wl.actors, wl.r
    n = a * r
    h_p = wl.poses[0].cpu().pin_memory()
    h_d = torch.empty(n, dtype=torch.float32, pin_memory=True)
    h_s = torch.empty(n, dtype=torch.int32, pin_memory=True)
    h_k = torch.empty(n, dtype=torch.int32, pin_memory=True)
    stream = torch.cuda.current_stream(wl.dev)

    def step():
        pipeline.cast_fan_host(wl.sset, h_p, wl.fan, h_d, h_s, max_steps=cfg.max_steps,
                               max_distance=cfg.max_distance, use_pitch=wl.use_pitch, out_steps=h_k, chunks=4)

    step()
    torch.cuda.synchronize(wl.dev)
    ms = []
    for _ in range(max(2, min(args.steps, 5))):
        flush.zero_()
        s0 = torch.cuda.Event(enable_timing=True)
        e0 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        step()
        e0.record(stream)
        torch.cuda.synchronize(wl.dev)
        ms.append(s0.elapsed_time(e0))
    return {"value": n / (float(np.mean(ms)) / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(a * 32),
            "d2h_bytes_per_step": int(n * 12), "ms_per_step": float(np.mean(ms)), "rays_per_step": n,
            "api": "navi_b200.pipeline.cast_fan_host (host poses in, dist/sem/steps out, 4 chunks overlapped)"}


def _extra_config(torch, args, config: int, dev, flush, stream, hbm, hbm_kind, l2) -> dict:
    """Another configuration on this GPU in the same run: value, step time and roofline."""
    wl = FanWorkload(torch, args, config, 0, 1, dev, 2)
    steps = max(3, min(args.steps, 10))
    step_ms, _ = _timed_steps(torch, wl, steps, 2, flush, stream)
    entry = {"value": wl.n / (float(np.mean(step_ms)) / 1e3), "unit": UNIT, "ms_per_step": float(np.mean(step_ms)),
             "rays_per_step": wl.n, "steps": steps, "scenes": len(wl.scene_list), "pool_bytes": wl.pool_bytes}
    if not args.no_cpu_baseline:
        cores = os.cpu_count() or 8
        sample = max(1, min(wl.actors, 2 if wl.r > 100_000 else min(2 * cores, 64)))
        w_ref, cpu_rays_s, threads, used = _w_ref(wl.cfg, wl.scene_list, wl.sets[0], wl.fan_np,
                                                  wl.poses[0].cpu().numpy(), sample)
        entry["roofline"] = _roofline(wl.n, step_ms, w_ref, hbm, hbm_kind, l2, _traffic(wl.cfg.name))
        entry["cpu_baseline"] = {"value": cpu_rays_s, "unit": UNIT, "cores": threads, "kind": "port",
                                 "sample": f"{used} of {wl.actors} actors x {wl.r} rays (oracle/trace_oracle.c, OpenMP)"}
    wl.close()
    del wl
    torch.cuda.empty_cache()
    return entry


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
    from navi_b200 import dist_stats, tracer

    dist = dist_stats.init_from_env("nccl", dev)
    tracer.set_option("descent", 0 if args.descent == "grid" else 1)
    wl = FanWorkload(torch, args, args.config, rank, world, dev, args.pose_sets, args.actors, dist)
    cfg = wl.cfg
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    flush = torch.empty(2 * l2, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    with ClockSampler(dev.index if dev.index is not None else 0) as clocks:
        time.sleep(0.3)  # let nvidia-smi start sampling
        step_ms, wall_s = _timed_steps(torch, wl, args.steps, args.warmup, flush, stream, dist)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    my_ms = float(sum(step_ms))
    steps_mean = float(wl.out_steps.float().mean().item())

    # explicit-ray kernel on the same rays (the drop-in cast_rays path), device-resident; one scene only
    explicit = None if len(wl.scene_list) != 1 else _explicit(torch, wl, args, flush, stream)
    observe = None if args.no_e2e else _observe(torch, wl, args, flush)
    e2e, e2e_rays, e2e_ms = (None, 0.0, 0.0) if args.no_e2e else _e2e(torch, wl, args, flush, dist)
    e2e_fan = None if args.no_e2e else _e2e_fan(torch, wl, args, flush)

    # gather per-rank [rays, ms, steps, e2e rays, e2e ms, fan e2e rays, fan e2e ms] over NCCL;
    # every job time is the max over ranks
    fan_rays = float(e2e_fan["rays_per_step"]) if e2e_fan else 0.0
    fan_ms = float(e2e_fan["ms_per_step"]) if e2e_fan else 0.0
    stats = torch.tensor([float(wl.n * args.steps), my_ms, steps_mean, e2e_rays, e2e_ms, fan_rays, fan_ms],
                         dtype=torch.float64, device=dev)
    table = dist_stats.gather_rank_stats(stats, dist)
    total_rays, job_ms = dist_stats.job_figures(table)

    line = None
    if rank == 0:
        hbm, hbm_kind = _peaks()
        l2peak = _l2_read_peak(torch, dev)
        roof, cpu = None, None
        if not args.no_cpu_baseline:
            cores = os.cpu_count() or 8
            sample = args.cpu_sample_actors or max(1, min(wl.actors, 2 * cores))
            w_ref, cpu_rays_s, threads, used = _w_ref(cfg, wl.scene_list, wl.sets[0], wl.fan_np,
                                                      wl.poses[0].cpu().numpy(), sample)
            if world == 1:  # the CPU baseline is reported at N=1 only
                cpu = {"value": cpu_rays_s, "unit": UNIT, "cores": threads, "kind": "port",
                       "sample": f"{used} of {wl.actors} actors x {wl.r} rays (oracle/trace_oracle.c, the reference "
                                 f"kernel restated in C, OpenMP, {threads} threads)"}
            # per GPU: this rank's rays over the slowest rank's step time
            roof = _roofline(wl.n, [job_ms / args.steps], w_ref, hbm, hbm_kind, l2peak,
                             _traffic(cfg.name) if world == 1 else None)
            if world > 1:
                roof["scope"] = f"per GPU: one rank's rays over the slowest of {world} ranks' mean step time"
        value = total_rays / (job_ms / 1e3)
        if e2e is not None:
            e2e = dict(e2e)
            e2e["value"] = float(table[:, 3].sum()) / (float(table[:, 4].max()) / 1e3)
            if world > 1:
                e2e["scope"] = f"box: rays of all {world} ranks over the slowest rank's mean step time"
        if e2e_fan is not None:
            e2e_fan = dict(e2e_fan)
            e2e_fan["value"] = float(table[:, 5].sum()) / (float(table[:, 6].max()) / 1e3)
            if world > 1:
                e2e_fan["scope"] = f"box: rays of all {world} ranks over the slowest rank's mean step time"
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": job_ms / args.steps,
            "higher_is_better": True,
            "scaling": "strong" if cfg.index == 5 else "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded scenes compiled to .gmdag by the in-tree voxel-dag compiler; seeded free-space poses)",
            "config": _config_dict(args, cfg, world, wl.actors),
            "gpu_launches": args.steps * wl.launches_per_step(),
            "clocks": clocks.summary(),
            "e2e": e2e,
            "e2e_fan": e2e_fan,
            "explicit_rays": explicit,
            "observe": observe,
            "roofline": roof,
            "cpu_baseline": cpu,
            "l2_read_peak": l2peak,
            "pool_bytes": wl.pool_bytes,
            "descent": args.descent,
            "per_rank_ms": [float(x) for x in table[:, 1]],
            "mean_steps_per_ray": float(np.mean(table[:, 2])),
            "wall_s": wall_s,
        }
    wl.close()
    del wl
    torch.cuda.empty_cache()
    if rank == 0 and world == 1 and args.extra_configs:
        hbm, hbm_kind = _peaks()
        extras = {}
        for c in (int(x) for x in args.extra_configs.split(",") if x.strip()):
            if c == args.config:
                continue
            from navi_b200 import scenes

            extras[scenes.CONFIGS[c].name] = _extra_config(torch, args, c, dev, flush, stream, hbm, hbm_kind,
                                                           line["l2_read_peak"])
        line["configs"] = extras
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    args = _args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_navi(args)


if __name__ == "__main__":
    main()
