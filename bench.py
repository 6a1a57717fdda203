#!/usr/bin/env python3
"""Benchmark of the B200 plan executor on YOLOv8n-pose 640x640 (batch 64 per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1).  Each rank runs its own executor on
its own batch (pure batch sharding, no data-path collective); torch.distributed
(gloo) is used only for the barrier and the max-over-ranks timing.  Rank 0
prints ONE JSON line.

  value  : images/s of the whole job with the fp16 input already resident in
           HBM: K CUDA-graph replays timed with CUDA events on the launching
           stream, max over ranks.
  e2e    : the same metric through the public C ABI call `ivc_infer_f32`
           (ClBackend::infer): pinned host f32 input -> H2D (batches of 32 or
           more: five eighths of the images cast to fp16 on the host first,
           with the reference's truncation) -> network -> f32 outputs D2H into pinned
           host memory, every step, all inside the timed region.
  roofline: the dominant kernel (the tcgen05 implicit-GEMM convolution) from a
           per-launch CUDA-event profile: algorithmic bytes / launch time vs the
           measured HBM copy bandwidth.  `network_roofline_frac` is the summed
           per-layer roofline time over the measured step time.
  cpu_baseline: the CPU oracle (restatement of the reference executor) on the
           host cores, a bounded sample of single images, rank 0 only.
`--impl reference` times the reference's CPU implementation of this path (the
oracle port; the reference's OpenCL executor cannot run here) on the same
workload and metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "YOLOv8n-pose 640² imgs/s per B200 (b=64) + b=1 p50 latency; % of roofline"
MODEL = "yolov8n-pose"
SEED = 1234
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


class RankGroup:
    """Timing plumbing of a multi-GPU run: a barrier and the max over ranks,
    over gloo on CPU tensors (no data-path collective; images are independent)."""

    def __init__(self, world: int):
        self.world = world
        if world > 1:
            import datetime
            import torch.distributed as dist
            if not dist.is_initialized():
                dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))

    def barrier(self) -> None:
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max(self, v: float) -> float:
        if self.world == 1:
            return v
        import torch
        import torch.distributed as dist
        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self) -> None:
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def make_plan(rank: int, workload: str = MODEL) -> str:
    """Model name, or a single op: conv3x3:CIN:COUT:HW:S / conv1x1:CIN:COUT:HW / dw:C:K:HW:S."""
    from infvino_b200 import plangen
    d = os.path.join(tempfile.gettempdir(), f"ivb_bench_{os.getuid()}_{rank}", workload.replace(":", "_"))
    if workload in plangen.MODELS:
        return plangen.MODELS[workload](d, seed=SEED)
    kind, *v = workload.split(":")
    v = [int(t) for t in v]
    # a 1x1 conv on each side, so the measured conv reads and writes channels-last
    # tensors as it does inside the network (its launch is the first conv_tc_kernel
    # of a run when the producer runs on the CUDA cores)
    if kind == "conv3x3":
        return plangen.op_conv(d, v[0], v[1], v[2], v[2], 3, v[3] if len(v) > 3 else 1, act=1, producer=True,
                               consumer=True)
    if kind == "conv1x1":
        return plangen.op_conv(d, v[0], v[1], v[2], v[2], 1, 1, act=1, producer=True, consumer=True)
    if kind == "dw":  # channels-last in and out, as inside MobileNet
        return plangen.op_conv(d, v[0], v[0], v[2], v[2], v[1], v[3] if len(v) > 3 else 1, act=3, groups=v[0],
                               producer=True, consumer=True)
    raise SystemExit(f"unknown workload {workload}")


def h2d_bytes(B: int, n_in: int) -> int:
    """Input bytes `ivc_infer_f32` copies per call: batches of 32 or more cast
    the first five eighths (rounded down to a multiple of 4 images) to fp16 on
    the host and copy the rest as f32; smaller batches copy f32."""
    n16 = B * 5 // 8 // 4 * 4 if B >= 32 else 0
    return n16 * n_in * 2 + (B - n16) * n_in * 4


def _t_roof(s, B, pk):
    """Per-step roofline time: max(FLOPs / tensor peak (burst), bytes / HBM)."""
    return max(s["flops_per_image"] * B / (pk["bf16_tflops"] * 1e12),
               (s["act_bytes_per_image"] * B + s["fixed_bytes"]) / (pk["hbm_gbs"] * 1e9))


def _graph_ms(m, B, reps):
    """CUDA-event time per graph replay (after warm-up), on the handle's stream."""
    import torch
    s = torch.cuda.Stream()
    m.set_stream(s.cuda_stream)
    for _ in range(5):
        m.run_async(B, s.cuda_stream)
    s.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(reps):
        m.run_async(B, s.cuda_stream)
    e1.record(s)
    e1.synchronize()
    return e0.elapsed_time(e1) / reps


def run_model(args, local: int) -> int:
    """Any model of the plan emitter (3, 4): batch-1 graph
    latency (p50 / p99 over 200 replays) and batch-B throughput (CUDA events
    around >= 200 replays, inputs resident), the summed per-layer roofline
    and the per-family launch times of an eager profile.  One JSON line."""
    import torch
    import infvino_b200 as ivb
    torch.cuda.set_device(local)
    pk, pk_src = peaks()
    B = args.batch
    m = ivb.PlanModel(make_plan(0, args.workload), device=local, max_batch=B)
    x = np.random.default_rng(SEED).random(B * m.inputNumel(), dtype=np.float32)
    m.setInput(ivb.f32_to_f16(x), B)
    m.run(B)
    m.run(1)
    s = torch.cuda.Stream()
    m.set_stream(s.cuda_stream)
    for _ in range(20):
        m.run_async(1, s.cuda_stream)
    s.synchronize()
    lat = []
    for _ in range(200):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        m.run_async(1, s.cuda_stream)
        b.record(s)
        b.synchronize()
        lat.append(a.elapsed_time(b))
    reps = max(args.min_replays, 20)
    ms = _graph_ms(m, B, reps)
    steps = m.steps()
    troof = sum(_t_roof(st, B, pk) for st in steps)
    troof1 = sum(_t_roof(st, 1, pk) for st in steps)
    prof = np.mean([np.array(m.profile(B)) for _ in range(3)], axis=0)
    fam = {}
    for st, t in zip(steps, prof):
        fam[st["family"]] = fam.get(st["family"], 0.0) + float(t)
    line = {"mode": "model", "workload": args.workload, "batch": B, "images_per_s": round(B / (ms / 1e3), 1),
            "ms_per_batch": round(ms, 4), "timed_replays": reps, "b1_p50_ms": round(float(np.median(lat)), 4),
            "b1_p99_ms": round(float(np.percentile(lat, 99)), 4),
            "gflop_per_image": round(sum(st["flops_per_image"] for st in steps) / 1e9, 4),
            "network_roofline_ms": round(troof * 1e3, 4), "network_roofline_frac": round(troof / (ms / 1e3), 4),
            "b1_roofline_us": round(troof1 * 1e6, 2), "launches_per_run": m.launch_count(B),
            "family_ms_eager": {k: round(v, 4) for k, v in sorted(fam.items(), key=lambda kv: -kv[1])},
            "peaks": f"{pk_src}: hbm_gbs {pk['hbm_gbs']}, bf16_tflops {pk['bf16_tflops']} (burst)"}
    print(json.dumps(line), flush=True)
    if args.layers:  # one line per step: its eager launch time against its own roofline
        import re
        geo = {ln.split()[2]: ln for ln in m.describe().splitlines() if ln.startswith("step ")}
        for st, t in zip(steps, prof):
            r = _t_roof(st, B, pk)
            print(json.dumps({"mode": "layer", "workload": args.workload, "batch": B, "step": st["name"],
                              "family": st["family"], "us": round(float(t) * 1e3, 2), "roofline_us": round(r * 1e6, 2),
                              "frac": round(r / (float(t) / 1e3), 4) if t > 0 else None,
                              "geometry": next(iter(re.findall(rf"\[(B={B} [^\]]*)\]", geo.get(st["name"], ""))),
                                               None)}), flush=True)
    m.close()
    return 0


def sweep_shapes():
    """1x1 convs as GEMMs (M = H*W in {6400, 1600, 400},
    K, N in {16 .. 256}), 3x3 s1 / s2 at 160..20 with Cin = Cout in
    {16 .. 128}, depthwise 3x3 / 5x5 s1 / s2 at 112..7 with C in
    {16, 72, 96, 240, 576}; each with fused bias + SiLU (depthwise: HardSwish,
    its MobileNet activation)."""
    out = []
    for hw in (80, 40, 20):
        for k in (16, 32, 64, 128, 256):
            for n in (16, 32, 64, 128, 256):
                out.append(f"conv1x1:{k}:{n}:{hw}")
    for hw in (160, 80, 40, 20):
        for c in (16, 32, 64, 128):
            for s in (1, 2):
                out.append(f"conv3x3:{c}:{c}:{hw}:{s}")
    for hw in (112, 56, 28, 14, 7):
        for c in (16, 72, 96, 240, 576):
            for k in (3, 5):
                for s in (1, 2):
                    out.append(f"dw:{c}:{k}:{hw}:{s}")
    return out


def run_sweep(args, local: int) -> int:
    """Config 2 op sweep: per op and batch (1 and 64) the op's own launch time
    (CUDA events around its launch in an eager profile, median of 5), its
    roofline time and the fraction; one JSON line per (op, batch)."""
    import torch
    import infvino_b200 as ivb
    torch.cuda.set_device(local)
    pk, pk_src = peaks()
    shapes = sweep_shapes() if args.workload in (MODEL, "sweep") else args.workload.split(",")
    for wl in shapes:
        plan = make_plan(0, wl)
        for B in (1, 64):
            m = ivb.PlanModel(plan, device=local, max_batch=B)
            x = np.random.default_rng(SEED).random(B * m.inputNumel(), dtype=np.float32)
            m.setInput(ivb.f32_to_f16(x), B)
            m.run(B)
            steps = m.steps()
            prof = np.median(np.array([m.profile(B) for _ in range(5)]), axis=0)
            # the measured op is the node named "op" (producer / consumer convs around it)
            i = next(j for j, st in enumerate(steps) if ":op" in st["name"] or st["name"].endswith("op.out"))
            t = float(prof[i]) / 1e3
            r = _t_roof(steps[i], B, pk)
            st = steps[i]
            print(json.dumps({"mode": "sweep", "op": wl, "batch": B, "family": st["family"], "us": round(t * 1e6, 2),
                              "roofline_us": round(r * 1e6, 2), "frac": round(r / t, 4),
                              "gflops": round(st["flops_per_image"] * B / 1e9, 4),
                              "mbytes": round((st["act_bytes_per_image"] * B + st["fixed_bytes"]) / 1e6, 3),
                              "bound": "tensor" if st["flops_per_image"] * B / (pk["bf16_tflops"] * 1e12) >
                              (st["act_bytes_per_image"] * B + st["fixed_bytes"]) / (pk["hbm_gbs"] * 1e9) else "hbm"}),
                  flush=True)
            m.close()
    return 0


def run_kernels_only(args, local: int) -> int:
    """Warm-up + K graph replays and nothing else (for launch lists and ncu captures)."""
    import infvino_b200 as ivb
    plan = make_plan(0, args.workload)
    m = ivb.PlanModel(plan, device=local, max_batch=args.batch)
    x = np.random.default_rng(SEED).random(args.batch * m.inputNumel(), dtype=np.float32)
    m.setInput(ivb.f32_to_f16(x), args.batch)
    for _ in range(args.warmup):  # the first run also tunes the conv geometries (eager launches)
        m.run(args.batch)
    m.synchronize()
    # the replays alone form the profiled range (ncu --profile-from-start off)
    cu = None
    try:
        import ctypes
        cu = ctypes.CDLL("libcuda.so.1")
        cu.cuProfilerStart()
    except OSError:
        cu = None
    t0 = time.perf_counter()
    for _ in range(args.steps):
        m.run_async(args.batch)
    m.synchronize()
    dt = (time.perf_counter() - t0) / max(1, args.steps)
    n_dets = None
    if args.decode:  # pose decode + NMS of the last replay's output, inside the profiled range
        n_dets = [len(d) for d in m.decodePose(args.batch)]
    if args.frames:  # one ivc_infer_bgr_u8 pass over 1280x720 BGR frames (device letterbox), in the range
        fr = np.random.default_rng(SEED + 100).integers(0, 256, (args.batch, 720, 1280, 3), dtype=np.uint8)
        m.inferBgr(fr, [np.empty(args.batch * m.outputNumel(0), dtype=np.float32)])
    if cu is not None:
        cu.cuProfilerStop()
    print(json.dumps({"mode": "kernels", "workload": args.workload, "batch": args.batch,
                      "launches_per_step": m.launch_count(args.batch), "wall_ms_per_step": round(dt * 1e3, 4),
                      "detections_per_image": n_dets}))
    m.close()
    return 0


class ClockSampler:
    """SM clock, power and clock-event reasons of one GPU while the timed
    region runs (read-only queries).  NVML from a thread every 5 ms, plus one
    sample when sampling starts and one when it stops, so that even a short
    timed region is covered; without NVML, nvidia-smi every 200 ms."""

    # NVML clock-event reason bits (nvmlClocksEventReason*)
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}

    def __init__(self, gpu_id: str):
        self.rows = []  # (sm MHz, max sm MHz, power W, reason bits)
        self.p = None
        self.nv = None
        try:
            import threading
            import pynvml as nv
            nv.nvmlInit()
            try:
                h = nv.nvmlDeviceGetHandleByPciBusId(gpu_id)
            except Exception:
                h = nv.nvmlDeviceGetHandleByIndex(int(gpu_id) if gpu_id.isdigit() else 0)
            reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self.nv, self.h, self._reasons = nv, h, reasons
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self._stop = threading.Event()
            self.sample()
            self.t = threading.Thread(target=self._loop, daemon=True)
            self.t.start()
            return
        except Exception:
            self.nv = None
        self.path = os.path.join(tempfile.gettempdir(), f"ivb_clocks_{os.getpid()}.csv")
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        self.f = open(self.path, "w")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={gpu_id}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def sample(self):
        nv, h = self.nv, self.h
        self.rows.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), self.max_mhz,
                          nv.nvmlDeviceGetPowerUsage(h) / 1000.0, int(self._reasons(h))))

    def _loop(self):
        while not self._stop.wait(0.005):
            try:
                self.sample()
            except Exception:
                return

    def stop(self):
        if self.nv is not None:
            self._stop.set()
            self.t.join(timeout=5)
            try:
                self.sample()
            except Exception:
                pass
            rows = self.rows
            load = [r[0] for r in rows if r[2] > 250.0] or [r[0] for r in rows]
            reasons = sorted({name for r in rows for bit, name in self.REASONS.items() if r[3] & bit})
            return {"sm_mhz": statistics.median(load), "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                    "samples": len(rows), "source": "nvml"}
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
        self.f.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        pw = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        load = [s for s, p in zip(sm, pw) if p > 250.0] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi"}


def gpu_pci_id(dev: int) -> str:
    import torch
    try:
        p = torch.cuda.get_device_properties(dev)
        return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
    except Exception:
        return str(dev)


def host_cores() -> int:
    """Threads this process may run on (its CPU affinity), not the OpenMP
    default, which torchrun sets to 1."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_baseline(plan: str, budget_s: float = 12.0):
    from oracle import ivref
    cores = ivref.set_threads(host_cores())
    o = ivref.OraclePlan(plan)
    x = np.random.default_rng(SEED).random(o.input_numel, dtype=np.float32)
    o.run(x, 1)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        o.run(x, 1)
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 4), "unit": "images/s", "cores": cores, "kind": "port",
            "sample": f"{n} single-image runs of {MODEL} (batch 1) in {dt:.1f} s, OpenMP over {cores} threads"}


def run_reference(args, rank: int, world: int) -> int:
    if rank != 0:
        return 0
    from oracle import ivref
    plan = make_plan(0)
    cores = ivref.set_threads(host_cores())
    o = ivref.OraclePlan(plan)
    x = np.random.default_rng(SEED).random(o.input_numel, dtype=np.float32)
    for _ in range(max(0, args.warmup)):
        o.run(x, 1)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        o.run(x, 1)
    dt = time.perf_counter() - t0
    value = args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "images/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"{MODEL} 640x640, 1 image per step (bounded CPU sample), random-init weights seed {SEED}",
                   "batch_per_step": 1, "parallelism": "host threads"},
        "cpu_baseline": {"value": round(value, 4), "unit": "images/s", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} timed single-image runs, OpenMP over {cores} threads; the reference's "
                                   "OpenCL executor needs an Intel iGPU / PoCL, absent here, so its CPU restatement "
                                   "(oracle/cpu_ref.cpp) is timed"},
        "e2e": {"value": round(value, 4), "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def bind_rank_cpus(local: int, local_world: int):
    """Multi-GPU runs: binds this rank to CPUs of its GPU's NUMA node, split
    evenly among the local ranks whose GPUs share that node, so that its
    host-cast threads and the pinned buffers it touches first sit next to its
    GPU and no two ranks share cores.  Without NUMA information the allowed
    CPUs are split evenly by local rank.  Returns the CPUs bound (or None)."""
    try:
        allowed = sorted(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return None

    def node_of(dev):
        try:
            import torch
            p = torch.cuda.get_device_properties(dev)
            path = f"/sys/bus/pci/devices/{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0/numa_node"
            with open(path) as f:
                return int(f.read().strip())
        except Exception:
            return -1

    def node_cpus(node):
        try:
            with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
                spec = f.read().strip()
        except OSError:
            return []
        cpus = []
        for part in spec.split(","):
            if "-" in part:
                a, b = part.split("-")
                cpus.extend(range(int(a), int(b) + 1))
            elif part:
                cpus.append(int(part))
        return [c for c in cpus if c in set(allowed)]

    nodes = [node_of(d) for d in range(local_world)]
    pool, peers = allowed, list(range(local_world))
    if nodes[local] >= 0:
        cand = node_cpus(nodes[local])
        if len(cand) >= sum(1 for n in nodes if n == nodes[local]):
            pool, peers = cand, [d for d in range(local_world) if nodes[d] == nodes[local]]
    k = peers.index(local)
    per = max(1, len(pool) // len(peers))
    mine = pool[k * per:(k + 1) * per] or pool
    try:
        os.sched_setaffinity(0, mine)
    except OSError:
        return None
    return mine


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default=MODEL)
    ap.add_argument("--mode", default="full", choices=["full", "kernels", "model", "sweep"],
                    help="full: the headline bench line; kernels: graph replays only (for launch lists and ncu); "
                         "model: latency / throughput of --workload (any emitted model); sweep: the config-2 op sweep")
    ap.add_argument("--layers", action="store_true", help="model mode: also one JSON line per step")
    ap.add_argument("--frames", action="store_true",
                    help="kernels mode: also one pass from 8-bit BGR frames (device letterbox) in the profiled range")
    ap.add_argument("--decode", action="store_true", help="kernels mode: also run the device pose decode + NMS")
    ap.add_argument("--min-replays", type=int, default=200,
                    help="device-resident timing: each step repeats the graph replay so that at least this many "
                         "replays are timed")
    args = ap.parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.mode == "kernels":
        return run_kernels_only(args, local)
    if args.mode == "model":
        return run_model(args, local)
    if args.mode == "sweep":
        return run_sweep(args, local)

    import torch
    import infvino_b200 as ivb

    group = RankGroup(world)
    torch.cuda.set_device(local)
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    bound_cpus = bind_rank_cpus(local, local_world) if world > 1 else None
    B = args.batch
    plan = make_plan(rank)
    model = ivb.PlanModel(plan, device=local, max_batch=B)
    stream = torch.cuda.Stream(device=local)
    model.set_stream(stream.cuda_stream)
    n_in = model.inputNumel()
    n_out = model.outputNumel(0)

    # synthetic input, per-rank seed; pinned host memory
    x_host = torch.empty(B * n_in, dtype=torch.float32, pin_memory=True)
    x_host.numpy()[:] = np.random.default_rng(SEED + rank).random(B * n_in, dtype=np.float32)
    y_host = torch.empty(B * n_out, dtype=torch.float32, pin_memory=True)
    x_dev = x_host.to(f"cuda:{local}", non_blocking=False)

    barrier = group.barrier
    max_over_ranks = group.max

    # ---- device-resident throughput: input converted once, then steps of R
    # graph replays each (R such that at least --min-replays are timed)
    y_dev = torch.empty(B * n_out, dtype=torch.float32, device=f"cuda:{local}")
    model.infer_f32_device(x_dev.data_ptr(), B, [y_dev.data_ptr()], stream.cuda_stream)
    for _ in range(max(3, args.warmup)):
        model.run_async(B, stream.cuda_stream)
    stream.synchronize()
    model.synchronize()
    launches = model.launch_count(B)
    reps = max(1, -(-args.min_replays // max(1, args.steps)))
    sampler = ClockSampler(gpu_pci_id(local))
    barrier()
    torch.cuda.synchronize(local)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        for _ in range(reps):
            model.run_async(B, stream.cuda_stream)
    ev1.record(stream)
    ev1.synchronize()
    torch.cuda.synchronize(local)
    barrier()
    clocks = sampler.stop()
    model.synchronize()  # raises if a kernel reported a bounded-wait timeout
    timed_replays = args.steps * reps
    region_ms = ev0.elapsed_time(ev1)
    ms = region_ms / timed_replays
    ms_max = max_over_ranks(ms)
    value = world * B / (ms_max / 1e3)

    # ---- end to end through the public API (ClBackend::infer equivalent),
    # from pinned host memory (the headline e2e) and from pageable memory
    # (what a std::vector / cv::Mat caller passes)
    outs = [y_host.numpy()]
    # the first eleven calls at a batch of 32 or more choose the host / device
    # cast split (the library times five splits twice each); then two more
    for _ in range(13 if B >= 32 else 2):
        model.infer_f32(x_host.numpy(), B, outs)
    e2e_steps = max(3, min(args.steps, 20))

    def time_e2e(src, dst, steps):
        barrier()
        torch.cuda.synchronize(local)
        t0 = time.perf_counter()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            model.infer_f32(src, B, dst)
        e1.record(stream)
        e1.synchronize()
        wall = (time.perf_counter() - t0) / steps * 1e3
        return max_over_ranks(max(e0.elapsed_time(e1) / steps, wall))

    e2e_ms = time_e2e(x_host.numpy(), outs, e2e_steps)
    e2e_val = world * B / (e2e_ms / 1e3)
    x_page = np.array(x_host.numpy(), copy=True)
    y_page = [np.empty(B * n_out, dtype=np.float32)]
    model.infer_f32(x_page, B, y_page)
    e2e_page_ms = time_e2e(x_page, y_page, max(3, e2e_steps // 2))
    del x_page, y_page

    # ---- end to end from 8-bit camera frames (1280x720 BGR, pinned): the
    # reference's host preprocessing (letterbox, resize, normalise, cast) runs
    # on the device, so 2.8 MB of bytes per image cross the link instead of a
    # 4.9 MB f32 blob (ivc_infer_bgr_u8)
    fh, fw = 720, 1280
    frames = torch.empty((B, fh, fw, 3), dtype=torch.uint8, pin_memory=True)
    frames.numpy()[:] = np.random.default_rng(SEED + 100 + rank).integers(0, 256, (B, fh, fw, 3), dtype=np.uint8)
    fr_outs = [y_host.numpy()]
    for _ in range(2):
        model.inferBgr(frames.numpy(), fr_outs)
    barrier()
    torch.cuda.synchronize(local)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        model.inferBgr(frames.numpy(), fr_outs)
    fr_ms = max_over_ranks((time.perf_counter() - t0) / e2e_steps * 1e3)
    e2e_frames = {"value": round(world * B / (fr_ms / 1e3), 1), "unit": "images/s", "ms_per_step": round(fr_ms, 3),
                  "frames": f"{B} x {fh}x{fw} BGR uint8, pinned host memory",
                  "h2d_bytes_per_step": B * fh * fw * 3, "d2h_bytes_per_step": B * n_out * 4,
                  "api": "ivc_infer_bgr_u8 (Preprocessor + ClBackend::infer with the preprocessing on the device)"}
    del frames

    # ---- the host link alone: the same bytes per step as the e2e path, as
    # plain pinned copies (H2D and D2H on two streams, all ranks at once); the
    # bound the e2e figure is measured against
    hb, db = h2d_bytes(B, n_in), B * n_out * 4
    src_h = x_host.view(torch.uint8)[:hb]
    dst_d = torch.empty(hb, dtype=torch.uint8, device=f"cuda:{local}")
    src_d = torch.empty(db, dtype=torch.uint8, device=f"cuda:{local}")
    dst_h = y_host.view(torch.uint8)[:db]
    s_in, s_out = torch.cuda.Stream(device=local), torch.cuda.Stream(device=local)
    for _ in range(2):
        dst_d.copy_(src_h, non_blocking=True)
        dst_h.copy_(src_d, non_blocking=True)
    torch.cuda.synchronize(local)
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        with torch.cuda.stream(s_in):
            dst_d.copy_(src_h, non_blocking=True)
        with torch.cuda.stream(s_out):
            dst_h.copy_(src_d, non_blocking=True)
    torch.cuda.synchronize(local)
    link_ms = max_over_ranks((time.perf_counter() - t0) / e2e_steps * 1e3)
    del src_h, dst_d, src_d, dst_h

    # ---- pose decode + NMS on the device (ivc_decode_pose) of the last e2e
    # batch: random-init class scores are all ~0.5, so every anchor is a
    # candidate and each image reaches the max_det cut (the worst case)
    model.infer_f32(x_host.numpy(), B, outs)
    model.decodePose(B)
    dec_t = []
    for _ in range(5):
        t0 = time.perf_counter()
        dets = model.decodePose(B)
        dec_t.append((time.perf_counter() - t0) * 1e3)
    pose_decode = {"ms_per_batch": round(float(np.median(dec_t)), 3), "batch": B, "conf": 0.25, "iou": 0.7,
                   "max_det": 300, "detections_per_image": int(np.median([len(d) for d in dets])),
                   "includes": "kernel + copy of the detections to host memory (synchronous call)"}

    # ---- batch-1 latency (device-resident graph replay and host round trip)
    lat, lat_e2e = [], []
    x1 = x_host.numpy()[:n_in]
    y1 = [np.empty(n_out, dtype=np.float32)]
    model.infer_f32(x1, 1, y1)
    for _ in range(20):
        model.run_async(1, stream.cuda_stream)
    stream.synchronize()
    for _ in range(200):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        model.run_async(1, stream.cuda_stream)
        b.record(stream)
        b.synchronize()
        lat.append(a.elapsed_time(b))
    for _ in range(50):
        t = time.perf_counter()
        model.infer_f32(x1, 1, y1)
        lat_e2e.append((time.perf_counter() - t) * 1e3)

    # ---- per-launch profile for the roofline (eager, CUDA events per launch)
    pk, pk_src = peaks()
    steps = model.steps()
    prof = np.zeros(len(steps))
    nprof = 3
    for _ in range(nprof):
        prof += np.array(model.profile(B))
    prof /= nprof
    bw = pk["hbm_gbs"] * 1e9
    # the step is milliseconds long, not seconds: the burst tensor peak applies
    tc = pk["bf16_tflops"] * 1e12

    def t_roof(s):
        return max(s["flops_per_image"] * B / tc, (s["act_bytes_per_image"] * B + s["fixed_bytes"]) / bw)

    conv = [i for i, s in enumerate(steps) if s["family"] in ("conv3x3_tc", "conv1x1_tc")]
    fam_ms = {}
    for i, s in enumerate(steps):
        fam_ms[s["family"]] = fam_ms.get(s["family"], 0.0) + prof[i]
    conv_ms = float(sum(prof[i] for i in conv))
    conv_bytes = float(sum(steps[i]["act_bytes_per_image"] * B + steps[i]["fixed_bytes"] for i in conv))
    conv_flops = float(sum(steps[i]["flops_per_image"] * B for i in conv))
    conv_troof = float(sum(t_roof(steps[i]) for i in conv))
    achieved = conv_bytes / (conv_ms / 1e3) / 1e9
    share = conv_ms / float(prof.sum())
    troof_total = sum(t_roof(s) for s in steps)
    net_frac = troof_total / (ms / 1e3)
    # DRAM bytes of the same launches from the committed ncu capture of this
    # workload (per network step, summed over the conv launches)
    traffic = None
    tpath = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles",
                         "conv_tc_dram_yolov8n-pose_b64.json")
    if B == 64 and args.workload == MODEL and os.path.exists(tpath):
        with open(tpath) as f:
            t = json.load(f)
        if t.get("launches_per_run") == len(conv):
            traffic = int(t["dram_bytes_read"] + t["dram_bytes_write"])
    # the conv share of the graph step (eager launch shares applied to the
    # measured graph replay time): an upper bound on the conv time inside the graph
    graph_conv_ms = share * ms
    roofline = {
        "kernel": "conv_tc_kernel (tcgen05 implicit-GEMM conv, %d launches/step)" % len(conv),
        "bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
        "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": traffic,
        "algorithmic_bytes": int(conv_bytes),
        "per": "network step (bytes over all conv launches of one step); launch times from CUDA events per launch",
        "peak_source": pk_src + " (hbm_gbs copy bandwidth)",
        "achieved_tflops": round(conv_flops / (conv_ms / 1e3) / 1e12, 1),
        "share_of_step": round(share, 3),
        "frac_graph_share": round(conv_bytes / (graph_conv_ms / 1e3) / 1e9 / pk["hbm_gbs"], 4),
        "frac_of_layer_roofline": round(conv_troof / (conv_ms / 1e3), 4),
    }
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline(plan)
        except Exception as e:  # reported, not fatal
            cpu = {"value": None, "error": repr(e)}
        try:  # the CPU restatement of the reference's pose decoder + NMS on one image of the same batch
            from oracle import decode
            y0 = outs[0].reshape(B, -1)[0].reshape(56, -1)
            t0 = time.perf_counter()
            decode.pose_decode(y0)
            pose_decode["cpu_port_ms_per_image"] = round((time.perf_counter() - t0) * 1e3, 2)
        except Exception as e:  # reported, not fatal
            pose_decode["cpu_port_error"] = repr(e)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": f"{MODEL} 640x640, batch {B} per GPU, random-init weights (seed {SEED}), "
                                   "f32 uniform[0,1) input (seed+rank)",
                       "batch_per_gpu": B, "parallelism": f"batch sharding x{world}, no collectives",
                       "l2": "inputs larger than L2 (157 MB fp16 input + >300 MB activations per step)",
                       "compute": "fp16 storage, fp32 accumulation"},
            "timed_replays": timed_replays, "replays_per_step": reps,
            "timed_region_ms": round(region_ms, 2),
            "step_definition": "one CUDA-graph replay of the network over one batch of 64 images; ms_per_step is per "
                               "replay (each of the K timed steps repeats the replay replays_per_step times)",
            "gpu_launches": launches * timed_replays,
            "e2e": {"value": round(e2e_val, 1), "unit": "images/s", "h2d_bytes_per_step": h2d_bytes(B, n_in),
                    "d2h_bytes_per_step": B * n_out * 4, "ms_per_step": round(e2e_ms, 3),
                    "host_memory": "pinned",
                    "h2d_gbs_per_rank": round(hb / (e2e_ms / 1e3) / 1e9, 2),
                    "d2h_gbs_per_rank": round(db / (e2e_ms / 1e3) / 1e9, 2),
                    "pageable": {"value": round(world * B / (e2e_page_ms / 1e3), 1), "ms_per_step": round(e2e_page_ms, 3)},
                    "link_bound": {"ms_per_step": round(link_ms, 3),
                                   "value": round(world * B / (link_ms / 1e3), 1),
                                   "what": "the same H2D and D2H bytes as plain pinned copies on two streams, all "
                                           "ranks at once (max over ranks)",
                                   "frac_achieved": round(link_ms / e2e_ms, 4)},
                    "rank_cpus": len(bound_cpus) if bound_cpus else host_cores()},
            "e2e_frames": e2e_frames,
            "b1_p50_ms": round(float(np.median(lat)), 4), "b1_p99_ms": round(float(np.percentile(lat, 99)), 4),
            "b1_e2e_p50_ms": round(float(np.median(lat_e2e)), 4),
            "roofline": roofline,
            "network_roofline_frac": round(net_frac, 4),
            "network_roofline_ms": round(troof_total * 1e3, 4),
            "network_roofline_peaks": f"{pk_src}: hbm_gbs {pk['hbm_gbs']}, bf16_tflops {pk['bf16_tflops']} (burst)",
            "family_ms": {k: round(v, 4) for k, v in sorted(fam_ms.items(), key=lambda kv: -kv[1])},
            "cpu_baseline": cpu,
            "pose_decode": pose_decode,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    model.close()
    group.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
