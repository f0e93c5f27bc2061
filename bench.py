#!/usr/bin/env python3
"""Benchmark of the attention forward engine (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c2|c3|c4|c5]
                    [--impl ours|reference]

A step is one attention forward over one batch of synthetic inputs (seeded
N(0, sigma^2)).  Default workload C2 = B=1, H=16, S=4096, D=128 fp16 per GPU,
the configuration the north-star metric is quoted on; with N GPUs the global
batch is B=N and each GPU owns its (batch, head) units -- no collective on the
data path (weak scaling).  C4/C5 are the strong-scaling sharded shapes.

Metric: attn fwd TFLOP/s = 4*B*H*S^2*D / t, whole job, t = max over ranks of
the device time (CUDA events) of exactly K steps.  Every line of our arm also
carries sub-records timed the same way in the same run: `sharded.c4` and
`sharded.c5`, the sharded configurations strong-scaled over the N GPUs
(aggregate TFLOP/s, per-rank units, achieved TFLOP/s and SM clocks), and at
N = 1 `c3` (D = 64).  `e2e` repeats the metric
through the public API with pinned host buffers and the H2D/D2H copies inside
the timed region.  `cpu_baseline` times the reference's own host attention
(oracle/_ref, the reference's verify_attn compiled from its sources) on this
host.  `--impl reference` is the reference arm: the reference's CPU attention
algorithm (oracle port, bit-identical to the reference's output on the golden
fixtures) on all host threads, one bounded sample of the workload per step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {
    # name: (B, H, S, D, dtype, sigma, scaling)
    "c2": dict(B=1, H=16, S=4096, D=128, dtype="f16", sigma=1.0, scaling="weak"),
    "c3": dict(B=1, H=16, S=4096, D=64, dtype="f16", sigma=1.0, scaling="weak"),
    "c4": dict(B=8, H=32, S=8192, D=128, dtype="bf16", sigma=1.0, scaling="strong"),
    "c5": dict(B=1, H=64, S=32768, D=128, dtype="f16", sigma=0.5, scaling="strong"),
}
# The reference's published figures for the same metric and shape (Hopper,
# 114 SMs; the reference project's README.md:333-337 for C2 and
# README.md:265-270 for C3).  None for the other shapes.
PUBLISHED = {"c2": 309.022, "c3": 296.931}
L2_BYTES = 126 * 1024 * 1024
METRIC = "attn fwd TFLOP/s (4*B*H*S^2*D/t)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="c2", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--bm", type=int, default=None, help="default: the workload's best tile")
    ap.add_argument("--bn", type=int, default=None, help="default: the workload's best tile")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--gather", action="store_true",
                    help="N > 1: after timing, collect the sharded O on rank 0 over NCCL "
                         "point-to-point and report its time separately")
    ap.add_argument("--preroll-s", type=float, default=0.02,
                    help="untimed back-to-back launches before timing: 20 ms bring the SM "
                         "clock to its boost, the regime of the burst bf16 peak (the "
                         "`sustained` record repeats the timing after SUSTAINED_PREROLL_S)")
    ap.add_argument("--schedule", type=int, default=0, choices=[0, 1, 2],
                    help="attn_set_schedule mode: 0 automatic (default), 1 classic, 2 persistent")
    ap.add_argument("--correction", type=int, default=0, choices=[0, 1],
                    help="attn_set_correction mode: 1 runs the tiles that have it with a "
                         "correction warpgroup (default 0)")
    ap.add_argument("--no-sub", action="store_true",
                    help="skip the sub-records (C4/C5 strong scaling at every N, C3 at N=1)")
    a = ap.parse_args()
    best = best_tile(a.workload)
    a.bm = best[0] if a.bm is None else a.bm
    a.bn = best[1] if a.bn is None else a.bn
    return a


def best_tile(wl):
    """Fastest tile measured on B200 per workload (BM x BN sweep): 256 x 128,
    except D = 64 where 256 x 96 keeps two S buffers per Q tile in TMEM."""
    return {"c3": (256, 96)}.get(wl, (256, 128))


# Sub-records of every line of our arm: the sharded configurations C4 and C5
# (strong scaling: the whole job split over the N GPUs), and C3 at N = 1.
# Timed steps per sub-record: a few tens to a few hundreds of ms at N = 1.
SUB_STEPS = {"c3": 50, "c4": 10, "c5": 4}
SUB_WARMUP = 3
SUB_PREROLL_S = 0.3
# The headline workload timed again after this long a run of back-to-back
# launches: by then the 1 kW power limit has settled the SM clock (about
# 1.7 GHz for C2 on a B200), the regime of the sustained bf16 peak.
SUSTAINED_PREROLL_S = 0.5


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), "measured"
    return 1590.0, 1400.0, "fallback"


def flops(units, S, D):
    return 4.0 * units * float(S) * S * D


def config_of(wl, args, n):
    w = WORKLOADS[wl]
    if w["scaling"] == "weak":
        B = w["B"] * n
        desc = (f"{wl.upper()}: per GPU B={w['B']},H={w['H']},S={w['S']},D={w['D']} {w['dtype']}; "
                f"global B={B} sharded by (batch, head), no collective")
    else:
        B = w["B"]
        desc = (f"{wl.upper()}: B={w['B']},H={w['H']},S={w['S']},D={w['D']} {w['dtype']} "
                f"sharded by (batch, head) over {n} GPU(s), no collective")
    return {"workload": desc, "B": B, "H": w["H"], "S": w["S"], "D": w["D"],
            "BM": args.bm, "BN": args.bn, "inputs": f"N(0,{w['sigma']}^2) seeded {args.seed}",
            "accumulate": "fp32", "causal": False}


# ---------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clock, its maximum, board power and the throttle reasons of one GPU,
    sampled while a region runs: through NVML in a thread every 5 ms (so a
    region of a few ms still gets samples), else an `nvidia-smi -lms 100`
    loop.  It only reads the GPU's state."""
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    PERIOD_S = 0.005

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.lines = []
        self.samples = []  # NVML: (sm MHz, max MHz, watts or None, set of reasons)
        self.nvml = None
        self.stop_ev = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
            get = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.get_reasons = get
            self.bits = [0x8, 0x40, 0x20, 0x4]  # NVML's bits for NAMES
        except Exception:
            self.nvml = None

    def _sample_nvml(self):
        nv = self.nvml
        sm = float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
        try:
            watts = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
        except Exception:
            watts = None
        try:
            r = int(self.get_reasons(self.h))
            reasons = {nm for nm, b in zip(self.NAMES, self.bits) if r & b}
        except Exception:
            reasons = set()
        self.samples.append((sm, self.max_mhz, watts, reasons))

    def _loop_nvml(self):
        while not self.stop_ev.is_set():
            try:
                self._sample_nvml()
            except Exception:
                return
            self.stop_ev.wait(self.PERIOD_S)

    def start(self):
        if self.nvml is not None:
            self.stop_ev.clear()
            self.t = threading.Thread(target=self._loop_nvml, daemon=True)
            self.t.start()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def mark(self):
        """The timed region starts now: the summary keeps the samples from
        here on and the one just before (the sampler runs from before the
        pre-roll so that it is up when the region starts)."""
        self.mark_at = max(0, (len(self.samples) if self.nvml is not None else len(self.lines)) - 1)

    def stop(self):
        if self.nvml is not None:
            self.stop_ev.set()
            self.t.join(timeout=2)
            try:
                self._sample_nvml()  # the state at the end of the region
            except Exception:
                pass
            rows = list(self.samples[getattr(self, "mark_at", 0):])
            self.samples = []
        elif self.proc is None:
            return None
        else:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.t.join(timeout=2)
            rows = []
            for ln in self.lines[getattr(self, "mark_at", 0):]:
                parts = [x.strip() for x in ln.split(",")]
                if len(parts) < 7:
                    continue
                try:
                    sm, mx = float(parts[0]), float(parts[1])
                except ValueError:
                    continue
                try:
                    pw = float(parts[2])
                except ValueError:
                    pw = None
                rows.append((sm, mx, pw, {nm for nm, val in zip(self.NAMES, parts[3:7])
                                          if val.lower() == "active"}))
            self.lines = []
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        pw = [r[2] for r in rows if r[2] is not None]
        return {"sm_mhz": statistics.median(r[0] for r in rows),
                "sm_max_mhz": max(r[1] for r in rows),
                "sm_mhz_min": min(r[0] for r in rows),
                "reasons": sorted(set().union(*(r[3] for r in rows))), "samples": len(rows),
                "power_w": statistics.median(pw) if pw else None,
                "how": "NVML every 5 ms" if self.nvml is not None else "nvidia-smi -lms 100"}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own host attention (oracle/_ref)
# ---------------------------------------------------------------------------
def cpu_baseline_reference(wl):
    from oracle import oracle
    exe = oracle.ref_binary()
    cfg = {"c2": "c2head", "c3": "c3head"}.get(wl, "c2head")
    threads = max(1, min(len(os.sched_getaffinity(0)), 16))
    if not exe.exists():
        return None
    r = subprocess.run([str(exe), "time", cfg, str(threads)], capture_output=True, text=True,
                       timeout=600)
    line = [ln for ln in r.stderr.splitlines() if ln.startswith("{")]
    if r.returncode != 0 or not line:
        return None
    d = json.loads(line[-1])
    D = 128 if cfg == "c2head" else 64
    out = {"value": d["tflops"], "unit": "TFLOP/s", "cores": threads, "kind": "reference",
           "sample": (f"{d['heads']} heads of 1x1x4096x{D} fp16 (one C2/C3 head per thread), "
                      f"the reference's verify_attn host oracle (tuning/utils.cuh:139-198) "
                      f"compiled from its sources; {d['seconds']:.2f} s wall")}
    # C1 (1x1x512x128), the reference's CPU-runnable case: one thread as the
    # reference runs it, and one C1 problem per host thread at once.
    c1 = {}
    for key, t in (("gflops_1_thread", 1), ("gflops_all_threads", threads)):
        r = subprocess.run([str(exe), "time", "c1", str(t)], capture_output=True, text=True,
                           timeout=120)
        ln = [x for x in r.stderr.splitlines() if x.startswith("{")]
        if r.returncode == 0 and ln:
            c1[key] = json.loads(ln[-1])["tflops"] * 1e3
    if c1:
        out["c1"] = dict(c1, threads=threads, shape="1x1x512x128 fp16")
    return out


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np
    import torch
    from oracle import oracle
    w = WORKLOADS[args.workload]
    n = args.gpus
    cfg = config_of(args.workload, args, n)
    B, H, S, D = cfg["B"], w["H"], w["S"], w["D"]
    dt = 0 if w["dtype"] == "f16" else 1
    tdt = torch.float16 if dt == 0 else torch.bfloat16
    # Inputs of one C-unit group (the rows sampled per step come from them).
    Bs = min(B, 1)
    g = torch.Generator().manual_seed(args.seed)
    q, k, v = ((torch.randn(Bs, H, S, D, generator=g) * w["sigma"]).to(tdt)
               .view(torch.int16).numpy().view(np.uint16) for _ in range(3))
    # every host core (torchrun sets OMP_NUM_THREADS=1 per rank; override it)
    threads = len(os.sched_getaffinity(0))
    rows_per_step = 1024
    rng = np.random.default_rng(args.seed)

    def step(i):
        rows = rng.choice(Bs * H * S, size=rows_per_step, replace=False).astype(np.int64)
        oracle.attention_rows(q, k, v, rows, bn_tile=args.bn, dtype=dt, nthreads=threads)

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(i)
    sec = time.perf_counter() - t0
    f = 4.0 * rows_per_step * S * D * args.steps
    val = f / sec / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": n,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec / args.steps * 1e3,
        "higher_is_better": True, "scaling": w["scaling"], "vs_baseline": None,
        "dtype": w["dtype"], "data": "synthetic", "config": cfg,
        "cpu_baseline": {
            "value": val, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": (f"{rows_per_step} query rows of the {args.workload.upper()} workload per "
                       f"step ({S} keys, D={D}), the reference's host attention algorithm "
                       "(oracle/attn_oracle.c, bit-identical to the reference's verify_attn on "
                       "tests/golden) on all host threads")},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
class Ctx:
    """This rank's place in the job: rank, world size, device, barrier."""

    def __init__(self):
        import torch
        import torch.distributed as dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=self.dev)

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()


def measure(ctx, wl, bm, bn, steps, warmup, preroll_s, seed, keep_sets=False):
    """Times exactly `steps` launches of workload `wl` on this rank's (batch,
    head) units, between CUDA events on the launching stream, with a barrier
    and a synchronize on both sides; the job time is the MAX over ranks.
    Inputs rotate over enough sets to exceed the L2 (or one set when a set is
    already larger).  Every rank takes the same collective steps."""
    import torch
    import attnprofile_b200 as ap
    from attnprofile_b200 import shard
    n = ctx.world
    w = WORKLOADS[wl]
    S, D, H = w["S"], w["D"], w["H"]
    tdt = torch.float16 if w["dtype"] == "f16" else torch.bfloat16
    B = w["B"] * n if w["scaling"] == "weak" else w["B"]
    units_total = B * H
    u0, u1 = shard.shard_range(units_total, n, ctx.rank)
    units = u1 - u0
    set_bytes = 4 * units * S * D * 2
    n_sets = 1 if set_bytes >= L2_BYTES else min(4, max(2, math.ceil(2 * L2_BYTES / set_bytes)))
    # Seeded inputs, generated per global unit so a unit's data does not
    # depend on the number of GPUs.
    sets = [shard.generate_units(u0, u1, S, D, tdt, ctx.dev, seed, si, w["sigma"])
            for si in range(n_sets)]
    torch.cuda.synchronize()

    def launch(i):
        if units:
            Q, K, V, O = sets[i % n_sets]
            ap.attn(Q, K, V, O, BM=bm, BN=bn)

    for i in range(max(warmup, 3)):
        launch(i)
    torch.cuda.synchronize()
    rc, site = ap.get_status(ctx.local)
    if rc != 0:
        raise SystemExit(f"{wl}: device status after warm-up: {rc} site {site:#x}")

    # A first barrier before the pre-roll: it also sets up the collectives
    # (NCCL creates its communicator on the first one, which can idle the
    # GPUs long enough for their clocks to drop), so the barrier right before
    # timing is a short one and the pre-roll runs directly ahead of the
    # timed steps.
    ctx.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(ctx.local)
    sampler.start()
    t_end = time.perf_counter() + preroll_s
    i = 0
    while time.perf_counter() < t_end:
        launch(i)
        i += 1
        if i % 16 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx.barrier()
    torch.cuda.synchronize()
    sampler.mark()
    ev0.record(stream)
    for i in range(steps):
        launch(i)
    ev1.record(stream)
    torch.cuda.synchronize()
    ctx.barrier()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    rc, site = ap.get_status(ctx.local)
    if rc != 0:
        raise SystemExit(f"{wl}: device status after timing: {rc} site {site:#x}")
    ms_max = shard.max_over_ranks(ms, ctx.dev)
    out = {"ms": ms, "ms_max": ms_max, "units": units, "units_total": units_total, "S": S,
           "D": D, "n_sets": n_sets, "set_bytes": set_bytes, "clocks": clocks, "tdt": tdt,
           "launches": shard.sum_over_ranks(steps if units else 0, ctx.dev)}
    if keep_sets:
        out["sets"] = sets
    else:
        del sets
        torch.cuda.empty_cache()
    return out


def sub_record(ctx, wl, args, preroll_s=SUB_PREROLL_S):
    """One sub-record: workload `wl` on its best tile, timed like the main
    line; value = the whole job's FLOPs / the MAX over ranks of the time."""
    from attnprofile_b200 import shard
    bm, bn = best_tile(wl)
    steps = SUB_STEPS[wl]
    m = measure(ctx, wl, bm, bn, steps, SUB_WARMUP, preroll_s, args.seed)
    S, D = m["S"], m["D"]
    achieved = flops(m["units"], S, D) / (m["ms"] / steps * 1e-3) / 1e12 if m["units"] else 0.0
    clk = m["clocks"] or {}
    reasons = clk.get("reasons") or []
    bits = sum(1 << k for k, nm in enumerate(("hw_slowdown", "hw_thermal_slowdown",
                                              "sw_thermal_slowdown", "sw_power_cap"))
               if nm in reasons)
    per_rank = [shard.gather_over_ranks(x, ctx.dev) for x in
                (m["units"], achieved, m["ms"], clk.get("sm_mhz") or 0.0, float(bits))]
    ns = argparse.Namespace(bm=bm, bn=bn, seed=args.seed)
    cfg = config_of(wl, ns, ctx.world)
    cfg["l2"] = (f"{m['n_sets']} rotating input sets vs 126 MiB L2" if m["n_sets"] > 1
                 else "inputs larger than the 126 MiB L2")
    names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    return {
        "value": flops(m["units_total"], S, D) * steps / (m["ms_max"] * 1e-3) / 1e12,
        "unit": "TFLOP/s", "scaling": WORKLOADS[wl]["scaling"], "n_gpus": ctx.world,
        "steps": steps, "warmup": SUB_WARMUP, "ms_per_step": m["ms_max"] / steps,
        "dtype": WORKLOADS[wl]["dtype"], "config": cfg,
        "units_per_gpu": [int(x) for x in per_rank[0]],
        "achieved_per_rank": per_rank[1], "ms_per_rank": per_rank[2],
        "gpu_launches": m["launches"],
        "clocks": clk,
        "sm_mhz_per_rank": per_rank[3],
        "reasons_per_rank": [[nm for k, nm in enumerate(names) if int(b) >> k & 1]
                             for b in per_rank[4]],
    }


def sustained_record(ctx, args):
    """The headline workload and tile, timed like the main line but after
    SUSTAINED_PREROLL_S of untimed launches (power-limited clock), with its
    fraction of the sustained bf16 peak."""
    m = measure(ctx, args.workload, args.bm, args.bn, args.steps, args.warmup,
                SUSTAINED_PREROLL_S, args.seed)
    S, D = m["S"], m["D"]
    value = flops(m["units_total"], S, D) * args.steps / (m["ms_max"] * 1e-3) / 1e12
    achieved = flops(m["units"], S, D) / (m["ms"] / args.steps * 1e-3) / 1e12
    _, sustained, kind = peaks()
    return {"value": value, "unit": "TFLOP/s", "steps": args.steps,
            "ms_per_step": m["ms_max"] / args.steps, "preroll_s": SUSTAINED_PREROLL_S,
            "clocks": m["clocks"], "gpu_launches": m["launches"],
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": sustained,
                         "unit": "TFLOP/s", "frac": achieved / sustained,
                         "peak_source": f"{kind} sustained bf16 cuBLAS (MEASURED_PEAKS.json)"}}


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference_arm(args)

    import torch
    import attnprofile_b200 as ap
    from attnprofile_b200 import shard

    ctx = Ctx()
    n, rank, dev = ctx.world, ctx.rank, ctx.dev
    ap.set_schedule(args.schedule)
    ap.set_correction(args.correction)
    w = WORKLOADS[args.workload]
    cfg = config_of(args.workload, args, n)
    m = measure(ctx, args.workload, args.bm, args.bn, args.steps, args.warmup, args.preroll_s,
                args.seed, keep_sets=True)
    S, D = m["S"], m["D"]
    units, units_total, sets, n_sets = m["units"], m["units_total"], m["sets"], m["n_sets"]
    tdt, ms, ms_max, clocks = m["tdt"], m["ms"], m["ms_max"], m["clocks"]
    elt = 2
    stream = torch.cuda.current_stream()
    total_flops = flops(units_total, S, D) * args.steps
    value = total_flops / (ms_max * 1e-3) / 1e12

    # roofline of the (only) kernel: algorithmic FLOPs per launch / mean launch time
    per_launch_ms = ms / args.steps
    achieved = flops(units, S, D) / (per_launch_ms * 1e-3) / 1e12
    burst, sustained, kind = peaks()
    peak = sustained if ms > 1000.0 else burst
    # Every rank's own rate and clock (the job time is the slowest rank's).
    ranks = None
    if n > 1:
        per = [shard.gather_over_ranks(x, dev) for x in
               (ms, achieved, (clocks or {}).get("sm_mhz") or 0.0)]
        ranks = {"ms": per[0], "achieved_tflops": per[1], "sm_mhz": per[2]}
    traffic = None
    tf = ROOT / "profiles" / "ncu_traffic.json"
    if tf.exists():
        try:
            traffic = json.loads(tf.read_text()).get(args.workload, {}).get(
                f"bm{args.bm}_bn{args.bn}")
        except Exception:
            traffic = None

    # End to end through the public API with host buffers: every step copies
    # its Q, K, V from pinned host memory, runs attnprofile_b200.attn and reads
    # O back.  Steps are pipelined over two device buffer sets and three
    # streams (H2D / compute / D2H) so the copy engines of step i+1 and i-1 run
    # while step i computes; all of it is inside the timed region.
    e2e = None
    if not args.no_e2e:
        Q0 = sets[0][0]
        steps_e = max(2, min(args.steps, 20))
        hq = [[x.cpu().pin_memory() for x in sets[0][:3]] for _ in range(2)]
        ho = [torch.empty(Q0.shape, dtype=tdt).pin_memory() for _ in range(2)]
        dbuf = [tuple(torch.empty_like(Q0) for _ in range(4)) for _ in range(2)]
        s_h2d, s_cmp, s_d2h = (torch.cuda.Stream(dev) for _ in range(3))
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_cmp = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]

        def e2e_steps(k):
            for i in range(k):
                b = i % 2
                Qd, Kd, Vd, Od = dbuf[b]
                with torch.cuda.stream(s_h2d):
                    if i >= 2:
                        s_h2d.wait_event(ev_cmp[b])  # buffer b's previous compute done
                    for dst, src in zip((Qd, Kd, Vd), hq[b]):
                        dst.copy_(src, non_blocking=True)
                    ev_in[b].record(s_h2d)
                with torch.cuda.stream(s_cmp):
                    s_cmp.wait_event(ev_in[b])
                    if i >= 2:
                        s_cmp.wait_event(ev_out[b])  # O of buffer b read back
                    if units:
                        ap.attn(Qd, Kd, Vd, Od, BM=args.bm, BN=args.bn, stream=s_cmp)
                    ev_cmp[b].record(s_cmp)
                with torch.cuda.stream(s_d2h):
                    s_d2h.wait_event(ev_cmp[b])
                    ho[b].copy_(Od, non_blocking=True)
                    ev_out[b].record(s_d2h)

        e2e_steps(2)
        torch.cuda.synchronize()
        ctx.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s_h2d)
        e2e_steps(steps_e)
        s_h2d.wait_stream(s_d2h)
        e1.record(s_h2d)
        torch.cuda.synchronize()
        ctx.barrier()
        te = shard.max_over_ranks(e0.elapsed_time(e1), dev)
        e2e = {"value": flops(units_total, S, D) * steps_e / (te * 1e-3) / 1e12,
               "unit": "TFLOP/s", "h2d_bytes_per_step": 3 * Q0.numel() * elt,
               "d2h_bytes_per_step": Q0.numel() * elt, "steps": steps_e,
               "api": "attnprofile_b200.attn -> attn_fwd (C ABI)",
               "pipelining": "2 buffer sets, H2D / compute / D2H streams"}
        del dbuf, hq, ho

    launches = m["launches"]

    # Optional consumer-side step, outside the metric: the last step's O
    # shards gathered on rank 0 (NVLink point-to-point through NCCL).
    gather = None
    if args.gather and n > 1:
        O_last = sets[(args.steps - 1) % n_sets][3]
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for rep in range(2):  # the first call sets up NCCL's point-to-point channels
            ctx.barrier()
            torch.cuda.synchronize()
            g0.record(stream)
            shard.gather_output(O_last, units_total, dst=0)
            g1.record(stream)
            torch.cuda.synchronize()
        g_ms = shard.max_over_ranks(g0.elapsed_time(g1), dev)
        g_bytes = units_total * S * D * elt * (n - 1) // n
        gather = {"ms": g_ms, "bytes_to_rank0": g_bytes, "GB_per_s": g_bytes / (g_ms * 1e-3) / 1e9,
                  "how": "torch.distributed send / batch_isend_irecv (NCCL) into rank 0's [1, B*H, S, D]"}
    del sets, m
    torch.cuda.empty_cache()

    # Sub-records, after the main line's timing.  First C3 on one GPU, in
    # the main line's clock regime (its short pre-roll, before anything long
    # has run); then the same workload under the power limit (after a long
    # pre-roll); then the sharded configurations (C4, C5) strong-scaled over
    # the N GPUs, long enough to sit under the power limit themselves.
    subs = {}
    if not args.no_sub and n == 1 and args.workload != "c3":
        subs["c3"] = sub_record(ctx, "c3", args, preroll_s=args.preroll_s)
    sustained = None
    if not args.no_sub:
        sustained = sustained_record(ctx, args)
    if not args.no_sub:
        for wl in ("c4", "c5"):
            if wl != args.workload:
                subs.setdefault("sharded", {})[wl] = sub_record(ctx, wl, args)

    cpu = None
    if rank == 0 and n == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_reference(args.workload)

    if rank == 0:
        set_bytes = 4 * units * S * D * elt
        cfg["l2"] = (f"{n_sets} rotating input sets ({n_sets * set_bytes / 2**20:.0f} MiB) vs "
                     f"126 MiB L2" if n_sets > 1 else "inputs larger than the 126 MiB L2")
        pub = PUBLISHED.get(args.workload)
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": n,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": w["scaling"],
            "vs_baseline": (value / pub) if pub else None,
            "dtype": w["dtype"], "data": "synthetic", "config": cfg,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
                         "peak_source": f"{kind} {'sustained' if peak == sustained else 'burst'}"
                                        " bf16 cuBLAS (MEASURED_PEAKS.json)",
                         "kernel": "attn_fwd_kernel"},
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
            "clocks": clocks,
            "ranks": ranks,
            "plan": dict(ap.query_split(cfg["B"], w["H"], S, D, BM=args.bm, BN=args.bn,
                                        dtype=0 if w["dtype"] == "f16" else 1),
                         schedule={0: "automatic (classic)", 1: "classic",
                                   2: "persistent"}[args.schedule],
                         correction_warpgroup=bool(args.correction)),
        }
        if sustained is not None:
            line["sustained"] = sustained
        line.update(subs)
        if gather is not None:
            line["gather"] = gather
        print(json.dumps(line), flush=True)
    if n > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
