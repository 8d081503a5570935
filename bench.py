#!/usr/bin/env python
# SPDX-License-Identifier: Apache-2.0
"""Exact radius + 3NN query throughput on B200; prints one JSON line.

Workload (the 64-scene configuration, scenes sharded across GPUs, no
data-path collective): 64 FPS-ordered synthetic room scenes of 24,000 points
(seeds 0..63); scene i runs on GPU i mod N, so each of N GPUs answers 64 / N
scenes (strong scaling).  Per scene: prefixes 24000/6000/1500/375/94, radius
r = 0.1/0.2/0.4/0.8 with K = 32 (31,875 computed rows), the down-sampling
rows served by the reuse cache after its value checks (7,969 rows) and 3NN
on every decoder stage (31,875 rows).  Unit: answered query rows per second,
all GPUs together.

* ``value``: one step = rebuild the prefix forest of the rank's scenes and
  run every stage (``gsa_b200.hierarchy.Batch``), inputs resident in HBM;
  the step runs as one captured CUDA graph or as direct launches, whichever
  a short calibration before timing finds faster (``step_mode``); device
  time from CUDA events per step, L2 flushed (256 MiB write) between steps
  outside the timed events; max over ranks.  ``weak`` (N > 1): the same with
  64 scenes on every GPU.
* ``e2e``: the same rows through the drop-in ``QuerySession`` API, one scene
  at a time, points copied from pinned host memory and every output row
  copied back to pinned host memory inside the timed region (a scene's rows
  on a copy stream while the next scene runs).  ``e2e_fixed_graph``: the
  same through ``fixed_graph_forward`` with the measured "frozen" policy
  (``prefix``, ``verify=False``).  ``e2e_concurrent_sessions``: the session
  API from two host threads, each on its own stream.  ``e2e_batched``: the
  same with the batched engine.
* ``roofline``: the query kernel with the largest share of step time,
  algorithmic bytes (radius 12 + 4K B per query, 3NN 36 B per query) over its
  measured time, against the measured HBM copy bandwidth.
* ``cpu_baseline``: the NumPy oracle (a port of the reference's test oracle)
  on one scene, one core, rank 0 at N=1.

``--impl reference`` runs the reference instead, on rank 0 only: its CPU
algorithm (the oracle port) on all host cores for ``value``, and, in
``ref_cuda``, the reference's own GPU path (its unmodified ``QuerySession``
with its CUDA kernels built from source for sm_100a) on the same scenes,
timed per call with CUDA events.
"""

import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "exact radius+3NN queries/sec at 1/2/4/8 B200; % of HBM roofline"
UNIT = "queries/s"
SCENES = 64
SIZES = (24000, 6000, 1500, 375, 94)
RADII = (0.1, 0.2, 0.4, 0.8)
K = 32
FALLBACK_HBM_GBS = 6650.0
TRAFFIC_PROFILE = ROOT / "profiles" / "dram_traffic_room64.json"


def rows_per_scene():
    return sum(SIZES[:4]), sum(SIZES[1:5]), sum(SIZES[:4])


def config(total, world):
    ball, hit, nn = rows_per_scene()
    return {
        "workload": f"room hierarchy, {total} FPS-ordered scenes x {SIZES[0]} points, scene i on GPU i mod {world}",
        "scenes_total": total,
        "scenes_per_gpu": -(-total // world),
        "scene_seeds": "0..scenes_total-1",
        "points_per_scene": SIZES[0],
        "prefixes": list(SIZES),
        "radii": list(RADII),
        "k": K,
        "rows_per_scene": {"radius_computed": ball, "reuse_hits": hit, "nn3": nn},
        "parallelism": "scene-sharded, one process per GPU",
        "l2": "flushed between timed steps (256 MiB write, outside the step events)",
    }


def parse():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--scenes", type=int, default=SCENES, help="scenes of the whole job")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-configs", action="store_true",
                   help="skip the 1M-point room and the clustered stress scene (N=1 runs)")
    p.add_argument("--write-traffic-profile", metavar="NCU_CSV",
                   help="write the DRAM traffic profile from an ncu --csv capture of the frontier "
                        "kernels' first hierarchy run (see TRAFFIC_SOURCES) and exit")
    return p.parse_args()


# --------------------------------------------------------------------------
# reference arm: the oracle port on all host cores, and the reference's own
# GPU path


def _ref_worker_init():
    os.environ["OMP_NUM_THREADS"] = "1"


def _ref_scene(seed):
    from gsa_b200 import scenes
    from oracle import fps

    p, start = scenes.room(seed, n=SIZES[0])
    return p[fps.fps_order(p, start)]


def _ref_step(args):
    P, fraction = args
    from oracle import numpy_oracle as orc

    t0 = time.perf_counter()
    _, rows = orc.hierarchy_oracle(P, SIZES, RADII, K, fraction)
    return rows, time.perf_counter() - t0


def ref_session_calls(gsa, s, P, out):
    """The hierarchy's twelve calls on the reference's QuerySession, in the
    order a PointNeXt-style network issues them; yields each call's name
    after enqueueing it."""
    for st in range(4):
        ps, pn = P[: SIZES[st]], P[: SIZES[st + 1]]
        s.ball_into(ps, ps, RADII[st], K, out[f"ball{st}"])
        yield f"ball{st}"
        s.ball_into(pn, ps, RADII[st], K, out[f"hit{st}"])
        yield f"hit{st}"
    for st in range(3, -1, -1):
        s.nn_into(P[: SIZES[st]], P[: SIZES[st + 1]], out[f"nnd{st}"], out[f"nni{st}"])
        yield f"nn{st}"


def run_ref_cuda(args, total):
    """The reference's GPU path on the job's scenes (all on this GPU): per
    call CUDA-event time summed over scenes (host synchronisations inside
    the calls included), a standalone prefix-tree build per scene, and the
    end-to-end rate with pinned host buffers like our ``e2e``."""
    import torch

    from oracle import reference_gpu

    why = reference_gpu.available()
    if why:
        return {"unavailable": why}
    gsa = reference_gpu.load()
    from gsa_b200 import hierarchy as hz, scenes

    dev = torch.device("cuda", torch.cuda.current_device())
    X = scenes.room_batch(range(total))  # the same inputs as our arm
    flat, views = hz.session_outputs(SIZES, dev)
    steps = max(1, min(args.steps, 3))
    call_ms, build_ms = session_call_spans(gsa, X, views, steps)
    # end to end, as our e2e: pinned host points in, every row out (a scene's
    # rows on a copy stream while the next scene runs, two output buffers)
    host_x = X.cpu().pin_memory()
    bufs = [(flat, views), hz.session_outputs(SIZES, dev)]
    host_flat = torch.empty((total, flat.numel()), dtype=torch.int32, pin_memory=True)
    copy_stream = torch.cuda.Stream(dev)
    main = torch.cuda.current_stream()
    ms = 0.0
    for step in range(steps + 1):
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        free = [torch.cuda.Event(), torch.cuda.Event()]
        for ev in free:
            ev.record(main)
        for i in range(total):
            k = i % 2
            main.wait_event(free[k])
            x = host_x[i].to(dev, non_blocking=True)
            with gsa.QuerySession() as s:
                for _ in ref_session_calls(gsa, s, x, bufs[k][1]):
                    pass
            done = torch.cuda.Event()
            done.record(main)
            copy_stream.wait_event(done)
            with torch.cuda.stream(copy_stream):
                host_flat[i].copy_(bufs[k][0], non_blocking=True)
                free[k].record(copy_stream)
        main.wait_stream(copy_stream)
        t1.record()
        torch.cuda.synchronize()
        if step:
            ms += t0.elapsed_time(t1)
    ball, hit, nn = rows_per_scene()
    rows = ball + hit + nn
    step_ms = sum(call_ms.values())
    return {
        "what": "reference gsa.QuerySession + csrc/gsa_bvh.cu, csrc/reference_queries.cu built from source for sm_100a, one scene per session, threshold 1024",
        "scenes": total,
        "steps": steps,
        "value": total * rows / (step_ms / 1000.0),
        "ms_per_step": step_ms,
        "calls_ms_per_step": {k: round(v, 4) for k, v in call_ms.items()},
        "tree_build_ms_per_step": build_ms,
        "e2e": {"value": total * rows * steps / (ms / 1000.0), "unit": UNIT,
                "h2d_bytes_per_step": int(host_x.numel() * 4),
                "d2h_bytes_per_step": int(host_flat.numel() * 4)},
        "unit": UNIT,
        "note": "call times are CUDA-event spans around each session call, host synchronisations inside the calls included",
    }


def session_call_spans(mod, X, views, steps):
    """Per session call, the CUDA-event span around the call summed over the
    scenes (host synchronisations inside the call included), and a
    standalone prefix-tree build per scene; ``mod`` is the reference's
    ``gsa`` package or ``gsa_b200`` (the same QuerySession / Tree API), so
    both arms are timed the same way.  Milliseconds per pass over X."""
    import torch

    total = X.shape[0]
    per_call = {}
    for step in range(steps + 1):
        for i in range(total):
            with mod.QuerySession() as s:
                calls = ref_session_calls(mod, s, X[i], views)
                while True:
                    t0 = torch.cuda.Event(enable_timing=True)
                    t1 = torch.cuda.Event(enable_timing=True)
                    t0.record()
                    name = next(calls, None)
                    t1.record()
                    if name is None:
                        break
                    if step:
                        per_call.setdefault(name, []).append((t0, t1))
    torch.cuda.synchronize()
    call_ms = {k: sum(a.elapsed_time(b) for a, b in v) / steps for k, v in per_call.items()}
    spans = []
    for step in range(steps + 1):
        for i in range(total):
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record()
            tree = mod.Tree(X[i].clone(), prefix=True)
            t1.record()
            tree.close()
            if step:
                spans.append((t0, t1))
    torch.cuda.synchronize()
    build_ms = sum(a.elapsed_time(b) for a, b in spans) / steps
    return call_ms, build_ms


def run_reference(args, rank, world):
    import multiprocessing as mp

    if rank != 0:
        return
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    workers = max(1, min(cores, args.scenes))
    # each step answers the first 10 % of every hierarchy call's queries on
    # each worker's scene (~2.5 s of CPU work per step), so a 20-step run
    # ends in about a minute while the GPUs of the job are held
    fraction = 0.10
    ctx = mp.get_context("spawn")
    with ctx.Pool(workers, initializer=_ref_worker_init) as pool:
        # the scenes (CPU FPS order) once, untimed; every step then sends each
        # worker a scene's points, so no timed step generates a scene
        scenes_P = pool.map(_ref_scene, list(range(workers)), chunksize=1)
        tasks = [(P, fraction) for P in scenes_P]
        for _ in range(args.warmup):
            pool.map(_ref_step, tasks, chunksize=1)
        total_rows, total_t = 0, 0.0
        for _ in range(args.steps):
            t0 = time.perf_counter()
            res = pool.map(_ref_step, tasks, chunksize=1)
            total_t += time.perf_counter() - t0
            total_rows += sum(r for r, _ in res)
    value = total_rows / total_t
    sample = (
        f"{workers} scenes per step, one per process, each the first {fraction:.0%} of every "
        f"hierarchy call's queries (NumPy oracle port, spawn pool)"
    )
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * total_t / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": config(args.scenes, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": workers, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    try:
        import torch

        if torch.cuda.is_available():
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
            line["ref_cuda"] = run_ref_cuda(args, args.scenes)
    except Exception as e:  # the CPU line stands; say why the GPU leg is missing
        line["ref_cuda"] = {"unavailable": f"{type(e).__name__}: {e}"}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# our arm



class NvmlClocks:
    """NVML samples (every 5 ms, read-only) of this GPU's SM clock and
    clock-event reasons during the timed region."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}

    def __init__(self, torch, device):
        import pynvml

        self.nv = pynvml
        pynvml.nvmlInit()
        want = str(torch.cuda.get_device_properties(device).uuid).replace("GPU-", "")
        self.handle = None
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            uuid = pynvml.nvmlDeviceGetUUID(h)
            uuid = uuid.decode() if isinstance(uuid, bytes) else uuid
            if uuid.replace("GPU-", "") == want:
                self.handle = h
        if self.handle is None:
            raise RuntimeError("GPU not found in NVML")
        self.samples, self.reasons, self.stop_flag = [], set(), False

    def _poll(self):
        nv = self.nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop_flag:
            self.samples.append(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM))
            bits = get_reasons(self.handle)
            for bit, name in self.REASONS.items():
                if bits & bit:
                    self.reasons.add(name)
            time.sleep(0.005)

    def start(self):
        import threading

        self.thread = threading.Thread(target=self._poll, daemon=True)
        self.thread.start()

    def stop(self):
        self.stop_flag = True
        self.thread.join()
        mx = self.nv.nvmlDeviceGetMaxClockInfo(self.handle, self.nv.NVML_CLOCK_SM)
        if not self.samples:
            return {"error": "no samples"}
        return {
            "sm_mhz": statistics.median(self.samples),
            "sm_max_mhz": mx,
            "samples": len(self.samples),
            "reasons": sorted(self.reasons),
            "source": "NVML",
        }


class Clocks:
    """nvidia-smi samples of this GPU's clocks and throttle reasons."""

    FIELDS = [
        "uuid",
        "clocks.sm",
        "clocks.max.sm",
        "power.draw",
        "clocks_event_reasons.hw_slowdown",
        "clocks_event_reasons.hw_thermal_slowdown",
        "clocks_event_reasons.sw_thermal_slowdown",
        "clocks_event_reasons.sw_power_cap",
    ]

    def __init__(self, torch, device):
        self.uuid = str(torch.cuda.get_device_properties(device).uuid)
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + ",".join(self.FIELDS), "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file,
                stderr=subprocess.DEVNULL,
            )
        except OSError as e:
            self.proc = None
            self.error = str(e)

    def stop(self):
        if self.proc is None:
            return {"error": getattr(self, "error", "nvidia-smi unavailable")}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.seek(0)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.file.read().splitlines():
            cols = [c.strip() for c in line.split(",")]
            if len(cols) != len(self.FIELDS) or cols[0].replace("GPU-", "") not in self.uuid.replace("GPU-", ""):
                continue
            try:
                sm.append(float(cols[1]))
                mx.append(float(cols[2]))
            except ValueError:
                continue
            for name, val in zip(names, cols[4:]):
                if val.lower() == "active":
                    reasons.add(name)
        os.unlink(self.file.name)
        if not sm:
            return {"error": "no samples"}
        return {
            "sm_mhz": statistics.median(sm),
            "sm_max_mhz": max(mx),
            "samples": len(sm),
            "reasons": sorted(reasons),
        }




def hbm_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# Sources whose change invalidates a traffic profile: the query kernels and
# the tree layout they read.
TRAFFIC_SOURCES = ["query.cu", "common.cuh", "forest.cuh", "build.cu"]
TRAFFIC_COMMAND = (
    "ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,dram__bytes_write.sum,smsp__inst_executed.sum "
    "--clock-control none -k regex:frontier_kernel -c 6 --csv --log-file dram.csv "
    "python bench.py --steps 1 --warmup 3 --no-e2e --no-cpu-baseline --no-configs"
)


def write_traffic_profile(csv_path, out_path=None):
    """Per-query DRAM bytes of the frontier kernels from an ncu --csv capture
    of TRAFFIC_COMMAND (the first hierarchy run: each kernel's launches are
    stages 0, 1, 2 in order, over 64 scenes of SIZES[0..2] queries), written
    with the SHA-256 of TRAFFIC_SOURCES so that bench lines use it only for
    the code it was taken of."""
    import csv

    rows = []
    with open(csv_path, newline="") as fh:
        lines = [ln for ln in fh if ln.startswith('"')]
    for r in csv.DictReader(lines):
        rows.append(r)
    per = {}
    for r in rows:
        # "void <unnamed>::radius_frontier_kernel<128>(<unnamed>::QArgs)"
        name = r["Kernel Name"].split("(")[0]
        while name.endswith(">"):  # template arguments
            name = name[: name.rindex("<")]
        name = name.split("::")[-1].split()[-1]
        launch = per.setdefault(name, {}).setdefault(r["ID"], {})
        unit = r.get("Metric Unit", "")
        val = float(r["Metric Value"].replace(",", ""))
        scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "nsecond": 1, "usecond": 1e3,
                 "msecond": 1e6}.get(unit, 1)
        launch[r["Metric Name"]] = val * scale
    out = {"command": TRAFFIC_COMMAND, "sources": TRAFFIC_SOURCES,
           "sources_sha256": kernel_sources_sha(TRAFFIC_SOURCES), "kernels": {}}
    for name, launches in per.items():
        stages = [launches[k] for k in sorted(launches, key=int)][:3]
        queries = [SCENES * SIZES[i] for i in range(len(stages))]
        dram = [st["dram__bytes_read.sum"] + st["dram__bytes_write.sum"] for st in stages]
        out["kernels"][name] = {
            "dram_bytes_per_query": sum(dram) / sum(queries),
            "per_stage": [
                {"stage": i, "queries": q, "dram_bytes": d, "dram_bytes_per_query": d / q,
                 "ncu_ns": st.get("gpu__time_duration.sum"),
                 "warp_inst_per_32_queries": st.get("smsp__inst_executed.sum", 0) * 32 / q}
                for i, (q, d, st) in enumerate(zip(queries, dram, stages))
            ],
        }
    Path(out_path or TRAFFIC_PROFILE).write_text(json.dumps(out, indent=1) + "\n")
    print(json.dumps(out, indent=1))
    return out


def kernel_sources_sha(names):
    h = hashlib.sha256()
    for n in names:
        h.update((ROOT / "gsa_b200" / "csrc" / n).read_bytes())
    return h.hexdigest()


def measured_traffic(kernel):
    """ncu DRAM bytes per query of ``kernel`` from the committed profile,
    used only when the profile was taken of the kernel source built here
    (same SHA-256 of its source files); else None."""
    try:
        prof = json.loads(TRAFFIC_PROFILE.read_text())
        entry = prof["kernels"][kernel]
        if kernel_sources_sha(prof["sources"]) != prof["sources_sha256"]:
            return None, "profile taken of a different kernel source"
        return float(entry["dram_bytes_per_query"]), prof.get("command")
    except (OSError, KeyError, ValueError) as e:
        return None, f"no profile ({type(e).__name__})"


def timed_steps(fn, steps, flush, torch):
    """CUDA-event milliseconds of ``steps`` calls of ``fn`` (L2 flushed
    before each, outside the events)."""
    records = []
    for _ in range(steps):
        flush.zero_()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        records.append((start, end))
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in records]


class Step:
    """One hierarchy step over the rank's scenes: a captured CUDA graph or
    direct launches, whichever a calibration run finds faster (the graph
    removes ~40 host calls per step; with many scenes per GPU the step is
    device bound and direct launches schedule the concurrent stages a little
    better)."""

    def __init__(self, eng, X, out, flush, torch, calibrate=True):
        from gsa_b200._library import launch_counter

        self.eng, self.X, self.out = eng, X, out
        self.graph = eng.capture(X, out)
        self.mode = "graph"
        if calibrate:
            eager_fn = lambda: eng.run(X, out)
            for _ in range(3):
                eager_fn()
                self.graph.replay()
            torch.cuda.synchronize()
            eager = statistics.median(timed_steps(eager_fn, 7, flush, torch))
            graph = statistics.median(timed_steps(self.graph.replay, 7, flush, torch))
            self.calibration_ms = {"graph": graph, "eager": eager}
            if eager < graph:
                self.mode = "eager"
        if self.mode == "eager":
            before = launch_counter()
            eng.run(X, out)
            self.launches = launch_counter() - before
        else:
            self.launches = self.graph.launches

    def __call__(self):
        if self.mode == "graph":
            self.graph.replay()
        else:
            self.eng.run(self.X, self.out)

    def close(self):
        self.graph.close()


def run_ours(args, rank, world, local):
    import torch

    from gsa_b200 import distributed as gd, hierarchy as hz, scenes

    dev = torch.device("cuda", local)
    seeds = gd.shard_seeds(rank, world, args.scenes)
    S = len(seeds)
    X = scenes.room_batch(seeds)
    eng = hz.Batch(SIZES, RADII)
    out = eng.allocate(S, dev)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    step = Step(eng, X, out, flush, torch)
    warmup = max(3, args.warmup)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()

    try:
        clocks = NvmlClocks(torch, dev)
    except Exception:
        clocks = Clocks(torch, dev)
    if world > 1:
        gd.barrier()
    torch.cuda.synchronize()
    clocks.start()
    step_ms = timed_steps(step, args.steps, flush, torch)
    if world > 1:
        gd.barrier()
    clock_info = clocks.stop()
    launches = step.launches * args.steps

    total_ms = sum(step_ms)
    max_ms = gd.max_over_ranks(total_ms, dev)
    ball_rows, hit_rows, nn_rows = rows_per_scene()
    rows = ball_rows + hit_rows + nn_rows
    value = args.scenes * rows * args.steps / (max_ms / 1000.0)

    # Stage attribution and the roofline come from a second, serialized pass
    # of the same steps (direct launches, stages one after another on one
    # stream, CUDA events around each stage), because concurrent spans overlap.
    timer = hz.StageTimer()
    torch.cuda.synchronize()
    for _ in range(args.steps):
        flush.zero_()
        eng.run(X, out, timer, concurrent=False)
    torch.cuda.synchronize()
    stage = timer.totals()
    phase = {}
    for name, ms in stage.items():
        key = name.rstrip("0123456789")
        phase[key] = phase.get(key, 0.0) + ms
    serial_ms = sum(phase.values()) / args.steps

    # Roofline per query kernel (serialized pass): stages 0-2 of the radius
    # query and of 3NN walk the tree, stage 3 scans (support prefixes of at
    # most 512 / 128 points).  Algorithmic bytes per query: radius
    # 12 + 4K (query + K ids), 3NN 12 + 12 + 12 (query, 3 dists, 3 ids).
    peak, peak_kind = hbm_peak()
    radius_q = 12 + 4 * K

    def kernel_line(stages, sizes_idx, per_query):
        ms = sum(stage.get(s, 0.0) for s in stages)
        queries = args.steps * S * sum(SIZES[i] for i in sizes_idx)
        gbs = queries * per_query / (ms / 1000.0) / 1e9 if ms else 0.0
        return {"ms_per_step": ms / args.steps, "launches_per_step": len(stages),
                "queries_per_step": queries // args.steps, "achieved_gbs": gbs,
                "frac": gbs / peak}

    kernels = {
        "radius_frontier_kernel": kernel_line(["ball0", "ball1", "ball2"], [0, 1, 2], radius_q),
        "radius_scan_kernel": kernel_line(["ball3"], [3], radius_q),
        "knn3_frontier_kernel": kernel_line(["nn0", "nn1", "nn2"], [0, 1, 2], 36),
        "knn3_scan_kernel": kernel_line(["nn3"], [3], 36),
    }
    # Reuse check + row copy (reuse_stages_kernel, one launch for the four
    # stages of a large batch, else reuse_stage_kernel per stage): per scene
    # and stage the support prefix is read twice (input and snapshot, 12 B
    # per point each; the query prefix is its first rows, so one pass
    # answers both checks) and the hit rows are read and written once (4K B
    # each).
    reuse_ms = stage.get("reuse", 0.0) + sum(stage.get(f"reuse{s}", 0.0) for s in range(4))
    reuse_bytes = args.steps * S * sum(24 * SIZES[s] + 8 * K * SIZES[s + 1] for s in range(4))
    reuse_line = {
        "ms_per_step": reuse_ms / args.steps,
        "launches_per_step": 1 if "reuse" in stage else 4,
        "bytes_per_step": reuse_bytes // args.steps,
        "achieved_gbs": reuse_bytes / (reuse_ms / 1000.0) / 1e9 if reuse_ms else 0.0,
    }
    name = max(kernels, key=lambda k: kernels[k]["ms_per_step"])
    kl = kernels[name]
    achieved = kl["achieved_gbs"]
    dbq, traffic_src = measured_traffic(name)
    traffic = None if dbq is None else dbq * kl["queries_per_step"] / kl["launches_per_step"]
    roofline = {
        "bound": "hbm",
        "kernel": name,
        "achieved": achieved,
        "peak": peak,
        "unit": "GB/s",
        "frac": achieved / peak,
        "traffic": traffic,
        "traffic_source": traffic_src,
        "peak_source": f"{peak_kind} HBM copy bandwidth",
        "algorithmic_bytes_per_query": radius_q if name.startswith("radius") else 36,
        "note": "achieved = algorithmic bytes of the kernel's launches / their summed CUDA-event time (serialized pass); traffic = ncu DRAM bytes per launch",
        "kernels": kernels,
        "reuse_check_and_copy": reuse_line,
    }

    # the one data-path-free exchange: every rank's row count and checksum
    gathered = gd.gather_counts(S * rows, gd.output_checksum(out), dev)

    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": warmup,
        "ms_per_step": max_ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": config(args.scenes, world),
        "step_mode": step.mode,
        "step_calibration_ms": getattr(step, "calibration_ms", None),
        "roofline": roofline,
        "phases_ms_per_step": {k: v / args.steps for k, v in phase.items()},
        # per row type, from the serialized pass: computed radius rows over the
        # radius stages, reuse-hit rows over the reuse checks and copies, 3NN
        # rows over the 3NN stages
        "rates_per_s": {
            "radius_computed": S * ball_rows * args.steps / (phase["ball"] / 1000.0),
            "reuse_hit": S * hit_rows * args.steps / (phase["reuse"] / 1000.0),
            "nn3": S * nn_rows * args.steps / (phase["nn"] / 1000.0),
        },
        "stages_ms_per_step": {k: round(v / args.steps, 4) for k, v in stage.items()},
        "serialized_ms_per_step": serial_ms,
        "stage_note": (
            "timed steps run the 8 query stages concurrently on side streams after the build; "
            "stage times and the roofline come from a separate serialized pass of the same steps"
        ),
        "gpu_launches": launches,
        "gpu_launches_per_step": step.launches,
        "clocks": clock_info,
        "rank_rows_checksums": [list(g) for g in gathered],
    }

    if world > 1:
        line["weak"] = weak_run(args, rank, world, dev, flush)

    if not args.no_e2e:
        line["e2e"], line["e2e_fixed_graph"], line["e2e_batched"], line["e2e_concurrent_sessions"] = e2e(
            args, X, step, out, world, dev)
        import gsa_b200

        _, views = hz.session_outputs(SIZES, dev)
        calls, build = session_call_spans(gsa_b200, X, views, max(1, min(args.steps, 3)))
        line["session_calls"] = {
            "calls_ms_per_step": {k: round(v, 4) for k, v in calls.items()},
            "ms_per_step": sum(calls.values()),
            "tree_build_ms_per_step": build,
            "note": "CUDA-event span around each QuerySession call summed over the rank's scenes, "
                    "as the reference arm's ref_cuda times the reference's session",
        }

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(X[0].cpu().numpy(), out)
    if world == 1 and not args.no_configs:
        line["configs"] = other_configs(dev, flush)
    step.close()
    if rank == 0:
        print(json.dumps(line), flush=True)


def weak_run(args, rank, world, dev, flush):
    """Weak scaling: 64 scenes on every GPU (seeds rank*64 + i)."""
    import torch

    from gsa_b200 import distributed as gd, hierarchy as hz, scenes

    S = SCENES
    X = scenes.room_batch(gd.rank_seeds(rank, S))
    eng = hz.Batch(SIZES, RADII)
    out = eng.allocate(S, dev)
    step = Step(eng, X, out, flush, torch)
    for _ in range(3):
        step()
    torch.cuda.synchronize()
    gd.barrier()
    ms = sum(timed_steps(step, args.steps, flush, torch))
    gd.barrier()
    max_ms = gd.max_over_ranks(ms, dev)
    ball, hit, nn = rows_per_scene()
    step.close()
    return {
        "scenes_per_gpu": S,
        "value": world * S * (ball + hit + nn) * args.steps / (max_ms / 1000.0),
        "ms_per_step": max_ms / args.steps,
        "step_mode": step.mode,
        "unit": UNIT,
    }


def e2e(args, X, step, out, world, dev):
    """End-to-end rows/s through the public APIs with pinned host buffers."""
    import torch

    from gsa_b200 import QuerySession, distributed as gd, fixed_graph_forward, hierarchy as hz
    from gsa_b200 import reference as ops

    S = X.shape[0]
    host_x = X.cpu().pin_memory()
    ball_rows, hit_rows, nn_rows = rows_per_scene()
    rows = ball_rows + hit_rows + nn_rows
    steps = max(1, min(args.steps, 3))
    # two output buffers: scene i's rows leave the device on a copy stream
    # while scene i+1 runs (a scene's outputs are views of one device buffer,
    # copied back in one transfer)
    bufs = [hz.session_outputs(SIZES, dev) for _ in range(2)]
    words = bufs[0][0].numel()
    host_flat = torch.empty((S, words), dtype=torch.int32, pin_memory=True)
    d2h = S * words * 4
    copy_stream = torch.cuda.Stream(dev)

    def per_scene(run_scene):
        ms = 0.0
        main = torch.cuda.current_stream()
        for st in range(steps + 1):  # first pass warms allocator and pinned buffers
            torch.cuda.synchronize()
            if world > 1:
                gd.barrier()
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record()
            free = [torch.cuda.Event(), torch.cuda.Event()]
            for ev in free:
                ev.record(main)
            for i in range(S):
                k = i % 2
                main.wait_event(free[k])  # scene i-2's copy out of this buffer done
                x = host_x[i].to(dev, non_blocking=True)
                run_scene(x, k)
                done = torch.cuda.Event()
                done.record(main)
                copy_stream.wait_event(done)
                with torch.cuda.stream(copy_stream):
                    host_flat[i].copy_(bufs[k][0], non_blocking=True)
                    free[k].record(copy_stream)
            main.wait_stream(copy_stream)
            t1.record()
            torch.cuda.synchronize()
            if st:
                ms += t0.elapsed_time(t1)
        return world * S * rows * steps / (gd.max_over_ranks(ms, dev) / 1000.0)

    def session_scene(x, k):
        with QuerySession() as s:
            hz.run_session(s, x, SIZES, RADII, bufs[k][1])

    session = {
        "value": per_scene(session_scene),
        "unit": UNIT,
        "h2d_bytes_per_step": int(host_x.numel() * 4),
        "d2h_bytes_per_step": int(d2h),
        "api": "gsa_b200.QuerySession (drop-in for gsa.QuerySession), one scene per session, one session at a time, threshold 1024; each scene's rows copied out on a copy stream while the next scene runs",
        "steps": steps,
    }
    session_rows = host_flat.clone()

    models = [hz.graph_model(ops, SIZES, RADII, bufs[k][1]) for k in range(2)]

    def fixed_scene(x, k):
        fixed_graph_forward(models[k], {"pos": x[None]}, ops=ops, policy="prefix", verify=False)

    with torch.inference_mode():
        fixed_value = per_scene(fixed_scene)
    fixed = {
        "value": fixed_value,
        "unit": UNIT,
        "h2d_bytes_per_step": int(host_x.numel() * 4),
        "d2h_bytes_per_step": int(d2h),
        "api": "gsa_b200.fixed_graph_forward (drop-in for gsa.fixed_graph.forward), policy prefix, verify=False (the measured 'frozen' policy), one scene per forward",
        "steps": steps,
        "rows_equal_session": bool(torch.equal(host_flat, session_rows)),
    }
    concurrent = concurrent_sessions(host_x, host_flat, steps, world, dev, threads=2)
    concurrent.update({
        "h2d_bytes_per_step": int(host_x.numel() * 4),
        "d2h_bytes_per_step": int(d2h),
        "rows_equal_session": bool(torch.equal(host_flat, session_rows)),
    })
    session_rows0 = session_rows[0]

    # batched engine: the captured step reads X, so the host copy lands there
    keys = [k for k in out if k.startswith(("ball", "hit", "nn"))]
    host_b = {k: torch.empty(out[k].shape, dtype=out[k].dtype, pin_memory=True) for k in keys}
    ms = 0.0
    for st in range(steps + 1):
        torch.cuda.synchronize()
        if world > 1:
            gd.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        X.copy_(host_x, non_blocking=True)
        step()
        for k in keys:
            host_b[k].copy_(out[k], non_blocking=True)
        t1.record()
        torch.cuda.synchronize()
        if st:
            ms += t0.elapsed_time(t1)
    _, first = hz.session_outputs(SIZES, "cpu", session_rows0)
    session["rows_equal_batched_scene0"] = bool(
        all(torch.equal(v, host_b[k][: v.shape[0]]) for k, v in first.items() if k in host_b)
    )
    batched = {
        "value": world * S * rows * steps / (gd.max_over_ranks(ms, dev) / 1000.0),
        "unit": UNIT,
        "h2d_bytes_per_step": int(host_x.numel() * 4),
        "d2h_bytes_per_step": int(sum(v.numel() * v.element_size() for v in host_b.values())),
        "api": f"gsa_b200.hierarchy.Batch over gsa_b200.Forest (batched C ABI), step as {step.mode}",
        "steps": steps,
    }
    return session, fixed, batched, concurrent


def concurrent_sessions(host_x, host_flat, steps, world, dev, threads=2):
    """The session API from several host threads, one QuerySession per scene,
    each thread on its own CUDA stream (scenes t, t+T, ...): while one thread
    waits for its comparison flags, another enqueues its next call.  Device
    time from an event on the calling stream before the threads start to one
    after every thread's stream is joined back."""
    import threading

    import torch

    from gsa_b200 import QuerySession, distributed as gd, hierarchy as hz

    S = host_x.shape[0]
    ball_rows, hit_rows, nn_rows = rows_per_scene()
    rows = ball_rows + hit_rows + nn_rows
    streams = [torch.cuda.Stream(dev) for _ in range(threads)]
    bufs = [hz.session_outputs(SIZES, dev) for _ in range(threads)]
    errors = []

    def worker(t, start):
        try:
            torch.cuda.set_device(dev)
            st = streams[t]
            st.wait_event(start)
            flat, views = bufs[t]
            with torch.cuda.stream(st):
                for i in range(t, S, threads):
                    x = host_x[i].to(dev, non_blocking=True)
                    with QuerySession() as s:
                        hz.run_session(s, x, SIZES, RADII, views)
                    host_flat[i].copy_(flat, non_blocking=True)
        except Exception as e:  # reported after the join
            errors.append(e)

    ms = 0.0
    main = torch.cuda.current_stream()
    for it in range(steps + 1):
        torch.cuda.synchronize()
        if world > 1:
            gd.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        ths = [threading.Thread(target=worker, args=(t, t0)) for t in range(threads)]
        for th in ths:
            th.start()
        for th in ths:
            th.join()
        if errors:
            raise errors[0]
        for st in streams:
            main.wait_stream(st)
        t1.record()
        torch.cuda.synchronize()
        if it:
            ms += t0.elapsed_time(t1)
    return {
        "value": world * S * rows * steps / (gd.max_over_ranks(ms, dev) / 1000.0),
        "unit": UNIT,
        "api": f"gsa_b200.QuerySession from {threads} host threads, one session per scene, each thread on its own CUDA stream",
        "threads": threads,
        "steps": steps,
    }


def other_configs(dev, flush, steps=5):
    """The other device workloads, each timed on its own (CUDA events per
    step, L2 flushed between steps, inputs resident): the 1,000,000-point
    room (20 x 20 x 3 m, FPS-ordered, prefixes 1M/250k/62.5k/15.6k/3.9k,
    r = 0.05/0.1/0.2/0.4, K = 32) through the batched engine with one scene,
    and the 200,000-point clustered stress scene (50,000 radius queries at
    r = 0.25, K = 32, against all points; 3NN of all 200,000 points against
    the first 50,000) through the forest API.  Stage times from a
    serialized pass; `radius_gbs` = 140 algorithmic bytes per radius row
    over the radius stages' time."""
    import torch

    from gsa_b200 import hierarchy as hz, scenes
    from gsa_b200.forest import Forest

    res = {}
    # 1M-point room: scene generation (FPS order) outside any timing
    p, start = scenes.room(11, n=1_000_000, box=(20.0, 20.0, 3.0))
    x = torch.from_numpy(p).to(dev)
    order = scenes.fps_order(x, start)
    X = x[order.to(dev)].contiguous()[None]
    eng = hz.Batch(hz.LARGE_SIZES, hz.LARGE_RADII)
    out = eng.allocate(1, dev)
    for _ in range(2):
        eng.run(X, out)
    ms = statistics.median(timed_steps(lambda: eng.run(X, out), steps, flush, torch))
    timer = hz.StageTimer()
    for _ in range(steps):
        flush.zero_()
        eng.run(X, out, timer, concurrent=False)
    torch.cuda.synchronize()
    stage = {k: v / steps for k, v in timer.totals().items()}
    ball, hit, nn = hz.unit_counts(hz.LARGE_SIZES)
    radius_ms = sum(stage.get(f"ball{s}", 0.0) for s in range(4))
    res["large_room"] = {
        "workload": "1,000,000-point room (20 x 20 x 3 m), one scene, prefixes "
                    + "/".join(str(v) for v in hz.LARGE_SIZES) + ", r = "
                    + "/".join(str(v) for v in hz.LARGE_RADII) + ", K = 32, reuse rows, 3NN per stage",
        "rows_per_step": ball + hit + nn,
        "ms_per_step": ms,
        "rows_per_s": (ball + hit + nn) / (ms / 1000.0),
        "stages_ms": {k: round(v, 4) for k, v in stage.items()},
        "radius_gbs": 140 * ball / (radius_ms / 1000.0) / 1e9 if radius_ms else None,
    }
    del X, out, x
    # clustered stress scene
    pts, info = scenes.clustered(seed=0)
    xc = torch.from_numpy(pts).to(dev)
    n, nq = len(pts), info["queries"]
    f = Forest(xc, [0, n], prefix=True)
    rows = torch.empty((nq, 32), dtype=torch.int32, device=dev)
    d = torch.empty((n, 3), device=dev)
    ids = torch.empty((n, 3), dtype=torch.int32, device=dev)
    level = next(l for l in range(4) if n >> (2 * l) == nq)
    calls = {
        "build": lambda: f.rebuild(xc),
        "radius": lambda: f.ball_prefix(nq, 0, 0.25, 32, rows, m=n),
        "nn3": lambda: f.query_prefix(n, level, d, ids),
    }
    for _ in range(2):
        for c in calls.values():
            c()
    stage = {k: statistics.median(timed_steps(c, steps, flush, torch)) for k, c in calls.items()}
    total = sum(stage.values())
    res["clustered_stress"] = {
        "workload": f"{n} clustered points (50 clusters, sigma 1e-3, 20 % duplicates, 5 % at exactly r), "
                    f"{nq} radius queries r = 0.25 K = 32 against all points, 3NN of all points against the first {nq}",
        "rows_per_step": nq + n,
        "ms_per_step": total,
        "rows_per_s": (nq + n) / (total / 1000.0),
        "stages_ms": {k: round(v, 4) for k, v in stage.items()},
        "radius_gbs": 140 * nq / (stage["radius"] / 1000.0) / 1e9,
        "fallback_queries": int(f.fallback.item()),
    }
    f.close()
    torch.cuda.synchronize()
    res["query_order"] = query_order(dev, flush, steps)
    return res


def query_order(dev, flush, steps=5):
    """Query sets that are not the support's own rows, through the C ABI on
    one FPS-ordered 24,000-point room: the room's points shuffled and 24,000
    unrelated room points (another seed), radius r = 0.1 (K = 32) over all
    points and 3NN against the 6,000-point prefix, walked in the support's
    leaf order (`query_ball_bvh` / `query_bvh`) and in the queries' own
    Morton order (the `_unordered` entries, which sort them first; the sort
    is inside the timed call); the support's own points for reference.
    Microseconds per call, median of `steps`, L2 flushed between calls."""
    import ctypes

    import torch

    from gsa_b200 import runtime as er, scenes

    X = scenes.room_batch([5, 6], n=24000)
    x, other = X[0].contiguous(), X[1].contiguous()
    tree = er.Tree(x, prefix=True)
    lib, fb = er.lib, torch.zeros(1, dtype=torch.int32, device=dev)
    g = torch.Generator(device=dev).manual_seed(0)
    cases = {
        "support_points": x,
        "support_points_shuffled": x[torch.randperm(24000, device=dev, generator=g)].contiguous(),
        "unrelated_points": other,
    }
    out = torch.empty((24000, 32), dtype=torch.int32, device=dev)
    d = torch.empty((24000, 3), device=dev)
    ids = torch.empty((24000, 3), dtype=torch.int32, device=dev)
    st = er._stream()

    def us(fn):
        return round(1000.0 * statistics.median(timed_steps(fn, steps, flush, torch)), 1)

    res = {"workload": "one 24,000-point room, 24,000 queries: radius r = 0.1 K = 32 over all "
                       "points, 3NN against the 6,000-point prefix (microseconds per call)"}
    for name, q in cases.items():
        qp = q.data_ptr()
        row = {}
        for order, (ball, knn) in {
            "support_order": (lib.query_ball_bvh, lib.query_bvh),
            "morton_order": (lib.query_ball_bvh_unordered, lib.query_bvh_unordered),
        }.items():
            calls = {
                "radius": lambda: er.check(ball(tree.ptr, qp, 24000, 24000, 0, 0.1, 32, out.data_ptr(),
                                                fb.data_ptr(), st)),
                "nn3": lambda: er.check(knn(tree.ptr, qp, 24000, 6000, 1, d.data_ptr(), ids.data_ptr(),
                                            fb.data_ptr(), st)),
            }
            for c in calls.values():
                c()
            row[order] = {k: us(c) for k, c in calls.items()}
        res[name] = row
    tree.close()
    torch.cuda.synchronize()
    return res


def cpu_baseline(P, out):
    """The NumPy oracle on scene 0 (one core); also checks scene 0's rows."""
    import numpy as np

    from oracle import numpy_oracle as orc

    t0 = time.perf_counter()
    ref, rows = orc.hierarchy_oracle(P, SIZES, RADII, K)
    dt = time.perf_counter() - t0
    ok = True
    for key, v in ref.items():
        n = v.shape[0]
        ok &= bool(np.array_equal(out[key][:n].cpu().numpy(), v))
    return {
        "value": rows / dt,
        "unit": UNIT,
        "cores": 1,
        "kind": "port",
        "sample": f"one full scene (seed 0, {rows} rows), NumPy oracle port, single process",
        "seconds": dt,
        "gpu_rows_equal_oracle": ok,
    }


def main():
    args = parse()
    if args.write_traffic_profile:
        write_traffic_profile(args.write_traffic_profile)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        # stdout carries the one JSON line: NCCL_DEBUG is left unset here
        # (at WARN, NCCL prints its version line on stdout)
        dist.init_process_group(
            "nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local)
        )
    try:
        run_ours(args, rank, world, local)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
