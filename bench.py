"""Benchmark of the Q4_K decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

Default workload (the headline): the fused Q4_K x fp16
decode GEMV y = W x with W = 14336 x 4096 Q4_K (Llama-3-8B FFN up/gate shape),
x = 4096 fp16 ~ N(0,1), fp32 accumulation.  A step is one GEMV.  Six seeded
weight copies (198 MB > the 126 MB L2) rotate between steps, so every step
streams its weights from HBM.  The reported value is algorithmic bytes
(packed weights + x + y) per second, timed with CUDA events on the launch
stream; ``e2e`` is the same metric through the C ABI with the step's x
copied in from pinned host memory and y copied back, inside the timed
region.  The GEMV does not shard (one 33 MB matrix), so with --gpus N every
rank runs an independent replica (weak scaling) and the value is the sum of
all ranks' bytes over the slowest rank's time.

``--impl reference`` times the reference's own CPU implementation of the same
workload on the host cores: the reference's Metal dequantization kernel
compiled for the host (oracle/_ref) feeding an fp32 dot product, with every
host thread.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4_K GEMV HBM GB/s (% of peak); Llama-3-8B-shape Q4_K decode tokens/s"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0

WORKLOADS = {
    # name: (rows, cols, description)
    "gemv_up": (14336, 4096, "Q4_K x fp16 GEMV 14336x4096 (Llama-3-8B FFN up/gate), batch 1"),
    "gemv_down": (4096, 14336, "Q4_K x fp16 GEMV 4096x14336 (Llama-3-8B FFN down), batch 1"),
    "dequant": (4096, 4096, "Q4_K -> fp32 dequantization of one 4096x4096 tensor "
                            "(65,536 super-blocks)"),
}


def gemv_bytes(rows: int, cols: int) -> int:
    return rows * (cols // 256) * 144 + 2 * cols + 4 * rows


def dequant_bytes(rows: int, cols: int) -> int:
    return rows * (cols // 256) * 144 + 4 * rows * cols


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        try:
            d = json.load(open(p))
            return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                    "source": "measured"}
        except Exception:
            pass
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS,
            "source": "fallback"}


# committed ncu summary of each workload's dominant kernel (named kernel + shape)
PROFILES = {
    "gemv_up": "q4k_gemv_14336x4096.md",
    "gemv_down": "q4k_gemv_4096x14336.md",
    "dequant": "q4k_dequant_f32_4096x4096.md",
}


def ncu_traffic(workload: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", PROFILES[workload])
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.rows: list[list[str]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
                for k, name in enumerate(names):
                    if r[5 + k].lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        pg = dist
    return world, rank, local, pg


def max_over_ranks(v: float, pg, local: int) -> float:
    if pg is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local}")
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def barrier(pg, local):
    if pg is not None:
        import torch
        torch.cuda.synchronize(local)
        pg.barrier()


# ----------------------------------------------------------------------------
# CPU legs
# ----------------------------------------------------------------------------

def cpu_gemv_rate(rows: int, cols: int, budget_s: float, threads: int, kind: str) -> dict:
    """GEMV GB/s of the CPU implementation on one seeded matrix, time-bounded."""
    from oracle import oracle as O
    W = O.gen_q4k(11, 1, rows * cols // 256)
    x = O.gen_f16(11, 2, cols)
    use_ref = kind == "reference" and O.ref_lib() is not None
    fn = (lambda: O.ref_q4k_matvec(W, rows, cols, x, threads)) if use_ref else \
        (lambda: O.q4k_matvec(W, rows, cols, x, acc64=False, nthreads=threads))
    fn()  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 1000:
            break
    gbs = gemv_bytes(rows, cols) * reps / el / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
            "kind": "reference" if use_ref else "port",
            "sample": f"{reps} full {rows}x{cols} GEMVs in {el:.1f} s "
                      f"({'reference Metal dequant kernel compiled for the host' if use_ref else 'C restatement'}"
                      f" + fp32 dot, {threads} threads)"}


def cpu_dequant_rate(rows: int, cols: int, budget_s: float, threads: int, kind: str) -> dict:
    from oracle import oracle as O
    nb = rows * cols // 256
    W = O.gen_q4k(1234, 0, nb)
    use_ref = kind == "reference" and O.ref_lib() is not None
    n = nb * 256
    fn = (lambda: O.ref_q4k_dequant_f32(W, n, threads)) if use_ref else \
        (lambda: O.q4k_dequant_f32(W, n, threads))
    fn()
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 1000:
            break
    return {"value": round(dequant_bytes(rows, cols) * reps / el / 1e9, 3), "unit": "GB/s",
            "cores": threads, "kind": "reference" if use_ref else "port",
            "sample": f"{reps} dequantizations of {nb} blocks in {el:.1f} s, {threads} threads"}


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ----------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------

def run_gpu(args, world, rank, local, pg) -> dict:
    import torch

    from metallm_b200 import Context
    rows, cols, desc = WORKLOADS[args.workload]
    ctx = Context(local)
    torch.cuda.set_device(local)
    stream_ptr = ctx.stream()
    tstream = torch.cuda.ExternalStream(stream_ptr, device=f"cuda:{local}")
    nb = rows * cols // 256
    copies = args.copies
    is_gemv = args.workload.startswith("gemv")
    Ws = []
    for c in range(copies):
        W = ctx.alloc(nb * 144)
        ctx.gen_q4k(1000 + c, 1, nb, W)
        Ws.append(W)
    x = ctx.alloc(2 * cols)
    ctx.gen_f16(7, 2, cols, x)
    out_elems = rows if is_gemv else nb * 256
    outs = [ctx.alloc(4 * out_elems) for _ in range(2 if not is_gemv else 1)]
    ctx.wait()

    def step(i: int):
        if is_gemv:
            ctx.q4k_gemv(Ws[i % copies], rows, cols, x, outs[0])
        else:
            ctx.q4k_dequant_f32(Ws[i % copies], outs[i % len(outs)], nb * 256)

    # The timed region replays a CUDA graph of K consecutive steps, the way a
    # decode loop replays its captured step: launches cost no host time.
    ctx.graph_begin()
    for i in range(args.steps):
        step(i)
    graph = ctx.graph_end()
    for _ in range(max(1, args.warmup // max(1, min(args.steps, args.warmup)))):
        graph.launch()
    for i in range(args.warmup):
        step(i)
    ctx.wait()
    barrier(pg, local)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(tstream)
    graph.launch()
    ev1.record(tstream)
    ev1.synchronize()
    dev_ms = ev0.elapsed_time(ev1)
    clocks = sampler.stop()
    graph.destroy()
    barrier(pg, local)
    ms_max = max_over_ranks(dev_ms, pg, local)
    per_step_ms = ms_max / args.steps
    alg_bytes = gemv_bytes(rows, cols) if is_gemv else dequant_bytes(rows, cols)
    value = alg_bytes * args.steps * world / (ms_max * 1e-3) / 1e9
    kernel_gbs = alg_bytes / (per_step_ms * 1e-3) / 1e9

    # ---- end to end through the C ABI with host buffers ----------------------
    # Each step: x copied in from pinned host memory, the op, y copied back to
    # pinned host memory, then a wait so the host can read y.  The three are
    # one captured graph per weight copy.
    lib, h = ctx.lib, ctx.handle
    hx = ctypes.c_void_p()
    hy = ctypes.c_void_p()
    lib.mlm_host_alloc(h, 2 * cols, ctypes.byref(hx))
    lib.mlm_host_alloc(h, 4 * out_elems, ctypes.byref(hy))
    from oracle import oracle as O  # host input only (the x the caller owns)
    xin = O.gen_f16(7, 2, cols)
    ctypes.memmove(hx, xin.ctypes.data, xin.nbytes)
    h2d = 2 * cols if is_gemv else 0
    d2h = 4 * out_elems
    e2e_graphs = []
    for c in range(copies):
        ctx.graph_begin()
        if is_gemv:
            ctx._check(lib.mlm_upload_async(h, ctypes.c_void_p(x.ptr), hx, 2 * cols), "upload")
        step(c)
        ctx._check(lib.mlm_download_async(h, hy, ctypes.c_void_p(outs[0].ptr), d2h), "download")
        e2e_graphs.append(ctx.graph_end())

    def e2e_step(i: int):
        e2e_graphs[i % copies].launch()
        ctx.wait()

    for i in range(args.warmup):
        e2e_step(i)
    barrier(pg, local)
    t0 = time.perf_counter()
    for i in range(args.steps):
        e2e_step(i)
    e2e_s = time.perf_counter() - t0
    barrier(pg, local)
    for g in e2e_graphs:
        g.destroy()
    e2e_s = max_over_ranks(e2e_s, pg, local)
    e2e_value = alg_bytes * args.steps * world / e2e_s / 1e9
    lib.mlm_host_free(h, hx)
    lib.mlm_host_free(h, hy)

    peaks = measured_peaks()
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(per_step_ms, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "q4k x f16 -> f32" if is_gemv else "q4k -> f32",
        "data": "synthetic (seeded Q4_K blocks generated on device, as BASELINE config 0)",
        "config": {"workload": desc, "rows": rows, "cols": cols,
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "weight_copies": copies,
                   "l2": f"inputs larger than L2: {copies} rotating weight copies "
                         f"({copies * nb * 144 / 1e6:.0f} MB)",
                   "algorithmic_bytes_per_step": alg_bytes},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": args.steps,
        "launch": "CUDA graph of K steps (programmatic dependent launch between GEMVs)",
        "roofline": {"bound": "hbm", "achieved": round(kernel_gbs, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(kernel_gbs / peaks["hbm_gbs"], 4),
                     "peak_source": peaks["source"],
                     "traffic": ncu_traffic(args.workload)},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        th = host_threads()
        if is_gemv:
            line["cpu_baseline"] = cpu_gemv_rate(rows, cols, args.cpu_seconds, th, "reference")
        else:
            line["cpu_baseline"] = cpu_dequant_rate(rows, cols, args.cpu_seconds, th, "reference")
    ctx.close()
    return line


def run_reference(args, world, rank) -> dict | None:
    if rank != 0:
        return None
    rows, cols, desc = WORKLOADS[args.workload]
    is_gemv = args.workload.startswith("gemv")
    th = host_threads()
    per = max(2.0, args.cpu_seconds / max(args.steps, 1))
    vals = []
    for _ in range(max(1, min(args.steps, 5))):
        r = (cpu_gemv_rate if is_gemv else cpu_dequant_rate)(rows, cols, per, th, "reference")
        vals.append(r)
    v = statistics.median([r["value"] for r in vals])
    alg = gemv_bytes(rows, cols) if is_gemv else dequant_bytes(rows, cols)
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": v,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(alg / (v * 1e9) * 1e3, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "q4k x f16 -> f32" if is_gemv else "q4k -> f32",
        "data": "synthetic (seeded Q4_K blocks)",
        "config": {"workload": desc, "rows": rows, "cols": cols},
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": th, "kind": vals[0]["kind"],
                         "sample": vals[0]["sample"]},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default="gemv_up", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--copies", type=int, default=6, help="rotating weight copies (> L2)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    world, rank, local, pg = dist_setup(args)
    try:
        line = run_gpu(args, world, rank, local, pg)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if pg is not None:
            pg.destroy_process_group()


if __name__ == "__main__":
    main()
