"""Benchmark of the Q4_K decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

Default workload (the headline GEMV): the fused Q4_K x fp16
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


# decoder workloads on the Llama-3-8B shape (hidden 4096, 32/8 heads of 128,
# FFN 14336, vocab 128256, RoPE theta 500000)
LLAMA_WORKLOADS = {
    "layer": "one Llama-3-8B-shape decoder layer, single-token decode at position 2047 over a "
             "2047-token fp16 cache",
    "decode": "Llama-3-8B-shape Q4_K model, batch 1: 512 prompt tokens then greedy decode",
    "prefill": "Llama-3-8B-shape Q4_K model, batch 1: the 512-token prompt pass (tcgen05 Q4_K "
               "GEMM, bf16 activations) up to the first generated token",
    "tp70b": "Llama-3-70B-shape Q4_K model (80 layers, hidden 8192, 64/8 heads of 128, FFN 28672, "
             "vocab 128256), a batch of 8 sequences: each a 2048-token prompt, then greedy "
             "decode of all 8 together, tensor-parallel over the N GPUs",
}

L70 = dict(n_layers=80, dim=8192, n_heads=64, n_kv_heads=8, ffn_dim=28672, vocab=128256)


def llama70_rank_bytes(tp: int, pos: int, batch: int = 1) -> int:
    """Algorithmic HBM bytes one rank reads and writes in a decode step of the
    70B shape at position pos: its shard of every weight once (for the whole
    batch), every sequence's KV heads up to pos, the appended K/V rows."""
    d, hd, ffn, vocab = 8192, 128, 28672, 128256
    nh, nkv = 64 // tp, 8 // tp
    blk = lambda rows, cols: rows * (cols // 256) * 144
    layer = (blk((nh + 2 * nkv) * hd, d) + blk(d, nh * hd) + blk(2 * ffn // tp, d)
             + blk(d, ffn // tp))
    kv = 2 * (pos + 1) * nkv * hd * 2 * batch
    return 80 * (layer + kv) + blk(vocab // tp, d) + 2 * d * batch


def llama_prefill_flops(n_layers: int, T: int) -> int:
    """Algorithmic FLOPs of a T-token prompt pass from position 0: every linear
    on every token, causal attention (QK^T and PV over the keys at or before
    each query), the output head on the last token."""
    d, kvd, ffn, vocab, heads, hd = 4096, 1024, 14336, 128256, 32, 128
    linear = 2 * T * (d * (d + 2 * kvd) + d * d + 2 * ffn * d + ffn * d)
    attn = 2 * 2 * heads * hd * (T * (T + 1) // 2)
    return n_layers * (linear + attn) + 2 * vocab * d


def llama_token_bytes(n_layers: int, pos: int, with_head: bool = True) -> int:
    """Algorithmic HBM bytes of one decode step at position pos (weights read
    once, the KV cache read up to pos, K/V written, the embedding row)."""
    d, kvd, ffn, vocab = 4096, 1024, 14336, 128256
    rb = d // 256 * 144
    layer = (d + 2 * kvd) * rb + d * rb + 2 * ffn * rb + d * (ffn // 256 * 144)
    kv = 2 * (pos + 1) * kvd * 2
    head = vocab * rb if with_head else 0
    return n_layers * (layer + kv) + head + 2 * d


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
    "dequant": "q4k_dequant_f32_4096x4096.md",
    "prefill": "q4k_gemm_28672x4096x512.md",
    "gemm": "q4k_gemm_28672x4096x512.md",
    "gemv_batch": "q4k_gemv_batch_57344x8192x8.md",
    "gemv_q6k": "q6k_gemv_128256x4096.md",
    "repack": "q4k_repack_4096x4096.md",
}


def ncu_traffic(workload: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    if workload not in PROFILES:
        return None
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


class nvtx_range:
    """An NVTX range around a timed region, so a profiler can select its
    kernels (ncu --nvtx --nvtx-include "timed/"); no effect otherwise."""

    def __init__(self, name: str):
        self.name = name

    def __enter__(self):
        import torch
        torch.cuda.nvtx.range_push(self.name)

    def __exit__(self, *exc):
        import torch
        torch.cuda.nvtx.range_pop()


L2_BYTES = 126 * 1024 * 1024


def rotation_copies(steps: int, nbytes: int, requested: int = 0) -> int:
    """Weight copies rotated through the K-step graph: a divisor of K (so a
    replayed graph reuses each copy only after every other one) whose total
    is at least 1.25x the L2; `requested` > 0 forces a count."""
    if requested > 0:
        return requested
    need = -(-int(1.25 * L2_BYTES) // max(nbytes, 1))
    for c in range(max(need, 1), steps + 1):
        if steps % c == 0:
            return c
    return max(need, 1)


def gemv_config(args, world: int, rows: int, cols: int, desc: str) -> dict:
    """config of the GEMV / dequant workloads (the same keys in both arms)."""
    nb = rows * cols // 256
    is_gemv = args.workload.startswith("gemv")
    copies = rotation_copies(args.steps, nb * 144, args.copies)
    outs = 1 if is_gemv else 4
    alg = gemv_bytes(rows, cols) if is_gemv else dequant_bytes(rows, cols)
    return {"workload": desc, "rows": rows, "cols": cols,
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
            "weight_copies": copies,
            "l2": (f"inputs larger than L2: {copies} rotating weight copies "
                   f"({copies * nb * 144 / 1e6:.0f} MB)" if is_gemv else
                   f"outputs larger than L2: {outs} rotating fp32 outputs "
                   f"({outs * 4 * nb * 256 / 1e6:.0f} MB)"),
            "algorithmic_bytes_per_step": alg}


TP70_PROMPT, TP70_GEN = 2048, 128


def tp70b_steps(args) -> int:
    return min(args.steps, TP70_GEN - args.warmup - 2)


def tp70b_config(args, world: int) -> dict:
    """config of the tensor-parallel 70B workload (the same keys in both arms);
    timed steps start after the prompt and the warm-up steps."""
    steps = tp70b_steps(args)
    alg = llama70_rank_bytes(world, TP70_PROMPT + args.warmup + steps // 2, args.batch)
    return {"workload": LLAMA_WORKLOADS["tp70b"], "batch": args.batch,
            "prompt_tokens": TP70_PROMPT, "decode_steps_timed": steps,
            "parallelism": f"tp{world}",
            "l2": "inputs larger than L2: Q4_K weights of 39.1 GB / N per step",
            "algorithmic_bytes_per_step_per_rank": alg}


def replay_timed(graph_launch, tstream, target_s: float = 1.0, min_reps: int = 10,
                 max_reps: int = 20000) -> dict:
    """Replays a captured K-step graph R times back to back, each replay
    bracketed by CUDA events on the launch stream, long enough (about
    target_s) that the clock sampler sees the GPU under load; returns the
    median replay time and the spread."""
    import torch
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record(tstream)
    graph_launch()
    ev[1].record(tstream)
    ev[1].synchronize()
    one = max(ev[0].elapsed_time(ev[1]) * 1e-3, 1e-6)
    reps = int(min(max_reps, max(min_reps, target_s / one)))
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    evs[0].record(tstream)
    for i in range(reps):
        graph_launch()
        evs[i + 1].record(tstream)
    evs[-1].synchronize()
    ms = sorted(evs[i].elapsed_time(evs[i + 1]) for i in range(reps))
    return {"median_ms": ms[reps // 2], "min_ms": ms[0], "max_ms": ms[-1], "replays": reps,
            "total_ms": evs[0].elapsed_time(evs[-1])}


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
    copies = rotation_copies(args.steps, nb * 144, args.copies)
    is_gemv = args.workload.startswith("gemv")
    Ws = []
    for c in range(copies):
        W = ctx.alloc(nb * 144)
        ctx.gen_q4k(1000 + c, 1, nb, W)
        Ws.append(W)
    x = ctx.alloc(2 * cols)
    ctx.gen_f16(7, 2, cols, x)
    out_elems = rows if is_gemv else nb * 256
    # the dequant writes 67 MB per step: four rotating outputs (268 MB, twice
    # the L2) so each step's stores go out to HBM
    outs = [ctx.alloc(4 * out_elems) for _ in range(4 if not is_gemv else 1)]
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
    rt = replay_timed(graph.launch, tstream)
    dev_ms = rt["median_ms"]
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
    xin = x.download(np.float16, cols)  # the caller's host copy of x
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
        "data": "synthetic (seeded Q4_K blocks generated on device)",
        "config": gemv_config(args, world, rows, cols, desc),
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": args.steps,
        "launch": "CUDA graph of K steps (programmatic dependent launch between GEMVs)",
        "timing": {"replays": rt["replays"], "statistic": "median over replays of the K-step "
                   "graph, each bracketed by CUDA events", "replay_ms_min": round(rt["min_ms"], 5),
                   "replay_ms_median": round(rt["median_ms"], 5),
                   "replay_ms_max": round(rt["max_ms"], 5),
                   "timed_region_s": round(rt["total_ms"] * 1e-3, 3)},
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


def cpu_decode_rate(budget_s: float, threads: int, big: bool = False) -> dict:
    """The reference's Q4_K kernels compiled for the host (oracle/_ref) on one
    decoder layer's seven linears plus the output head, at all host threads;
    tokens/s = 1 / (L x layer + head) with L = 32 (the 8B shape) or 80 (the
    70B shape, big=True).  Norms, RoPE and attention (under 1 % of the
    bytes) are left out of the sample."""
    from oracle import oracle as O
    if big:
        nl, d, shapes = 80, 8192, [(10240, 8192), (8192, 8192), (57344, 8192), (8192, 28672)]
    else:
        nl, d, shapes = 32, 4096, [(6144, 4096), (4096, 4096), (28672, 4096), (4096, 14336)]
    Ws = [O.gen_q4k(3, i, r * c // 256) for i, (r, c) in enumerate(shapes)]
    head = O.gen_q4k(3, 9, 128256 * d // 256)
    xs = {c: O.gen_f16(3, 20 + c, c) for c in {c for _, c in shapes}}
    mv = (lambda W, r, c: O.ref_q4k_matvec(W, r, c, xs[c], threads)) if O.ref_lib() is not None \
        else (lambda W, r, c: O.q4k_matvec(W, r, c, xs[c], acc64=False, nthreads=threads))
    reps, t_layer, t_head = 0, 0.0, 0.0
    t0 = time.perf_counter()
    while reps == 0 or time.perf_counter() - t0 < budget_s:
        a = time.perf_counter()
        for W, (r, c) in zip(Ws, shapes):
            mv(W, r, c)
        b = time.perf_counter()
        mv(head, 128256, d)
        t_layer += b - a
        t_head += time.perf_counter() - b
        reps += 1
    per_token = nl * t_layer / reps + t_head / reps
    return {"value": round(1.0 / per_token, 4), "unit": "tokens/s", "cores": threads,
            "layer_s": t_layer / reps, "head_s": t_head / reps,
            "kind": "reference" if O.ref_lib() is not None else "port",
            "sample": f"{reps} x (one layer's 7 Q4_K matvecs + the 128256x{d} head) in "
                      f"{time.perf_counter() - t0:.1f} s, {threads} threads; tokens/s = "
                      f"1 / ({nl} x layer + head)"}


GEMM_SHAPE = (28672, 4096, 512)
GEMM_DESC = ("Q4_K x bf16 GEMM on tcgen05: the fused gate/up weights of a Llama-3-8B layer "
             "(28672 x 4096 Q4_K) on a 512-token prompt of the 8B shape")


def cpu_gemm_rate(budget_s: float, threads: int) -> dict:
    """CPU matvec rate on the GEMM's weights, as TFLOP/s: the GEMM is T
    independent matvecs, so a bounded sample of them gives its rate."""
    rows, cols, _ = GEMM_SHAPE
    r = cpu_gemv_rate(rows, cols, budget_s, threads, "reference")
    tflops = r["value"] * 1e9 / gemv_bytes(rows, cols) * 2 * rows * cols / 1e12
    return {"value": round(tflops, 6), "unit": "TFLOP/s", "cores": threads, "kind": r["kind"],
            "sample": r["sample"] + "; TFLOP/s = 2 x rows x cols per matvec"}


GEMV_BATCH_SHAPE = (57344, 8192, 8)
GEMV_BATCH_DESC = ("Q4_K batched decode GEMV: the fused gate/up weights of a Llama-3-70B layer "
                   "(57344 x 8192 Q4_K) on the 8 tokens of a 70B-shape decode batch")


def run_gemv_batch(args, world, rank, local, pg) -> dict:
    """The batched decode linear alone: each step is one 57344 x 8192 launch
    over 8 bf16 tokens, rotating over two weight copies (528 MB > L2)."""
    import torch

    from metallm_b200 import Context
    rows, cols, T = GEMV_BATCH_SHAPE
    ctx = Context(local)
    torch.cuda.set_device(local)
    tstream = torch.cuda.ExternalStream(ctx.stream(), device=f"cuda:{local}")
    peaks = measured_peaks()
    nb = rows * cols // 256
    Ws = []
    for c in range(2):
        W = ctx.alloc(nb * 144)
        ctx.gen_q4k(1000 + c, 1, nb, W)
        Ws.append(W)
    x = ctx.alloc(2 * T * cols)
    ctx.gen_f16(7, 2, T * cols, x)  # fp16 normals read as bf16: finite, small
    y = ctx.alloc(4 * T * rows)
    step = lambda i: ctx.call("mlm_q4k_gemv_batch", Ws[i % 2], rows, cols, x, T, y, None)
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
    for i in range(args.steps):
        step(i)
    ev1.record(tstream)
    ev1.synchronize()
    dev_ms = ev0.elapsed_time(ev1)
    clocks = sampler.stop()
    ms_max = max_over_ranks(dev_ms, pg, local)
    per_ms = ms_max / args.steps
    alg = nb * 144 + 2 * T * cols + 4 * T * rows
    gbs = alg / (per_ms * 1e-3) / 1e9
    # e2e: the tokens from pinned host memory, the product back to it
    lib, h = ctx.lib, ctx.handle
    hx, hy = ctypes.c_void_p(), ctypes.c_void_p()
    lib.mlm_host_alloc(h, 2 * T * cols, ctypes.byref(hx))
    lib.mlm_host_alloc(h, 4 * T * rows, ctypes.byref(hy))
    e2e_steps = min(args.steps, 20)
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        ctx._check(lib.mlm_upload_async(h, ctypes.c_void_p(x.ptr), hx, 2 * T * cols), "up")
        step(i)
        ctx._check(lib.mlm_download_async(h, hy, ctypes.c_void_p(y.ptr), 4 * T * rows), "dn")
        ctx.wait()
    e2e_s = max_over_ranks(time.perf_counter() - t0, pg, local)
    lib.mlm_host_free(h, hx)
    lib.mlm_host_free(h, hy)
    line = {
        "metric": METRIC, "value": round(gbs * world, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q4k x bf16 (as fp16 with per-sub-block scales) -> f32",
        "data": "synthetic (seeded Q4_K blocks, fp16 normals read as bf16, generated on device)",
        "config": {"workload": GEMV_BATCH_DESC, "rows": rows, "cols": cols, "tokens": T,
                   "parallelism": "replicas" if world > 1 else "single GPU",
                   "l2": f"2 rotating weight copies ({2 * nb * 144 / 1e6:.0f} MB > L2)",
                   "algorithmic_bytes_per_step": alg},
        "e2e": {"value": round(alg * e2e_steps * world / e2e_s / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": 2 * T * cols, "d2h_bytes_per_step": 4 * T * rows},
        "gpu_launches": args.steps,
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                     "peak_source": peaks["source"], "traffic": ncu_traffic("gemv_batch")},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        r = cpu_gemv_rate(rows, cols, args.cpu_seconds, host_threads(), "reference")
        line["cpu_baseline"] = dict(r, sample=r["sample"] + "; one token per matvec, GB/s of "
                                    "the weights streamed per token")
    ctx.close()
    return line


def run_gemm(args, world, rank, local, pg) -> dict:
    """The prefill GEMM alone: each step is one 28672 x 4096 x 512 launch,
    rotating over weight copies larger than L2 together."""
    import torch

    from metallm_b200 import Context
    rows, cols, T = GEMM_SHAPE
    ctx = Context(local)
    torch.cuda.set_device(local)
    tstream = torch.cuda.ExternalStream(ctx.stream(), device=f"cuda:{local}")
    peaks = measured_peaks()
    nb = rows * cols // 256
    copies = args.copies if args.copies > 0 else 4  # 4 x 66 MB > L2
    Ws = []
    for c in range(copies):
        W = ctx.alloc(nb * 144)
        ctx.gen_q4k(1000 + c, 1, nb, W)
        Ws.append(W)
    x = ctx.alloc(2 * T * cols)
    ctx.gen_f16(7, 2, T * cols, x)  # fp16 normals read as bf16: finite, small
    y = ctx.alloc(4 * T * rows)
    step = lambda i: ctx.call("mlm_q4k_gemm", Ws[i % copies], rows, cols, x, T, y, None)
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
    for i in range(args.steps):
        step(i)
    ev1.record(tstream)
    ev1.synchronize()
    dev_ms = ev0.elapsed_time(ev1)
    clocks = sampler.stop()
    ms_max = max_over_ranks(dev_ms, pg, local)
    per_ms = ms_max / args.steps
    flops = 2 * rows * cols * T
    tflops = flops / (per_ms * 1e-3) / 1e12
    # e2e: X from pinned host memory, the GEMM, Y back to pinned host memory
    lib, h = ctx.lib, ctx.handle
    hx, hy = ctypes.c_void_p(), ctypes.c_void_p()
    lib.mlm_host_alloc(h, 2 * T * cols, ctypes.byref(hx))
    lib.mlm_host_alloc(h, 4 * T * rows, ctypes.byref(hy))
    e2e_steps = min(args.steps, 20)
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        ctx._check(lib.mlm_upload_async(h, ctypes.c_void_p(x.ptr), hx, 2 * T * cols), "up")
        step(i)
        ctx._check(lib.mlm_download_async(h, hy, ctypes.c_void_p(y.ptr), 4 * T * rows), "dn")
        ctx.wait()
    e2e_s = max_over_ranks(time.perf_counter() - t0, pg, local)
    lib.mlm_host_free(h, hx)
    lib.mlm_host_free(h, hy)
    line = {
        "metric": METRIC, "value": round(tflops * world, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q4k -> bf16 x bf16 -> f32 (tcgen05)",
        "data": "synthetic (seeded Q4_K blocks, fp16 normals read as bf16, generated on device)",
        "config": {"workload": GEMM_DESC, "rows": rows, "cols": cols, "tokens": T,
                   "parallelism": "replicas" if world > 1 else "single GPU",
                   "l2": f"{copies} rotating weight copies ({copies * nb * 144 / 1e6:.0f} MB > L2)",
                   "algorithmic_flops_per_step": flops},
        "e2e": {"value": round(flops * e2e_steps * world / e2e_s / 1e12, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": 2 * T * cols, "d2h_bytes_per_step": 4 * T * rows},
        "gpu_launches": args.steps,
        "roofline": {"bound": "tensor", "achieved": round(tflops, 1),
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(tflops / peaks["bf16_tflops"], 4),
                     "peak_source": peaks["source"] + " (bf16 burst)",
                     "traffic": ncu_traffic("gemm")},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_gemm_rate(args.cpu_seconds, host_threads())
    ctx.close()
    return line


def gemm_kernel_time(ctx, m, n_layers: int, T: int, reps: int, tstream) -> dict:
    """Device time of the dominant prefill kernel alone: the fused gate/up
    Q4_K GEMM (28672 x 4096) on T bf16 tokens, rotating over the layers'
    weights (66 MB each) so every launch streams its weights from HBM."""
    import torch
    x = ctx.alloc(2 * T * 4096)
    ctx.gen_f16(1, 11, T * 4096, x)  # fp16 normals read as bf16: finite, small
    y = ctx.alloc(4 * T * 28672)
    ws = [m.layer_tensors(l)["w_gate"] for l in range(n_layers)]
    call = lambda i: ctx.call("mlm_q4k_gemm", ws[i % n_layers], 28672, 4096, x, T, y, None)
    for i in range(3):
        call(i)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(tstream)
    for i in range(reps):
        call(i)
    ev1.record(tstream)
    ev1.synchronize()
    ms = ev0.elapsed_time(ev1) / reps
    flops = 2 * 28672 * 4096 * T
    return {"ms": ms, "flops": flops, "tflops": flops / (ms * 1e-3) / 1e12}


def run_llama(args, world, rank, local, pg) -> dict:
    """The 8B-shape decoder workloads: one layer, and the model (prompt pass, greedy decode)."""
    import torch

    from metallm_b200 import Context, Llama
    from metallm_b200.synthetic import fill_llama, llama_config
    ctx = Context(local)
    torch.cuda.set_device(local)
    tstream = torch.cuda.ExternalStream(ctx.stream(), device=f"cuda:{local}")
    peaks = measured_peaks()

    def timed(fn):
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(tstream)
        fn()
        ev1.record(tstream)
        ev1.synchronize()
        return ev0.elapsed_time(ev1)

    extra = {}
    if args.workload == "layer":
        cfg = llama_config(n_layers=1, vocab=256, max_seq=2048)
        m = Llama(ctx, cfg)
        pos = 2047
        fill_llama(m, 1, cache_positions=pos)
        hidden = ctx.alloc(4 * cfg.dim)
        ctx.gen_f32(1, 7, cfg.dim, hidden)
        m.set_position(pos)
        ctx.graph_begin()
        for _ in range(args.steps):
            m.forward_layer(0, hidden)
        graph = ctx.graph_end()
        for _ in range(args.warmup):
            m.forward_layer(0, hidden)
        ctx.wait()
        barrier(pg, local)
        sampler = ClockSampler(local)
        sampler.start()
        time.sleep(0.3)
        dev_ms = timed(graph.launch)
        clocks = sampler.stop()
        graph.destroy()
        ms_max = max_over_ranks(dev_ms, pg, local)
        per_step_ms = ms_max / args.steps
        alg = llama_token_bytes(1, pos, with_head=False) - 2 * 4096
        value = alg * args.steps * world / (ms_max * 1e-3) / 1e9
        unit, metric_value_desc = "GB/s", "one decoder layer per step"
        launches = args.steps * 6  # state, QKV GEMV, RoPE + append + attention, 3 GEMVs
        # e2e: hidden state in from pinned host memory, the layer, out again
        lib, h = ctx.lib, ctx.handle
        hbuf = ctypes.c_void_p()
        lib.mlm_host_alloc(h, 4 * cfg.dim, ctypes.byref(hbuf))
        t0 = time.perf_counter()
        for _ in range(args.steps):
            ctx._check(lib.mlm_upload_async(h, ctypes.c_void_p(hidden.ptr), hbuf, 4 * cfg.dim), "up")
            m.forward_layer(0, hidden)
            ctx._check(lib.mlm_download_async(h, hbuf, ctypes.c_void_p(hidden.ptr), 4 * cfg.dim), "dn")
            ctx.wait()
        e2e_s = max_over_ranks(time.perf_counter() - t0, pg, local)
        lib.mlm_host_free(h, hbuf)
        e2e = {"value": round(alg * args.steps * world / e2e_s / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": 4 * cfg.dim, "d2h_bytes_per_step": 4 * cfg.dim}
        config = {"workload": LLAMA_WORKLOADS["layer"], "hidden": 4096, "heads": "32/8 x 128",
                  "ffn": 14336, "position": pos, "parallelism": "single GPU",
                  "l2": "inputs larger than L2: 122.7 MB of Q4_K weights + 8.4 MB of KV per layer",
                  "algorithmic_bytes_per_step": alg}
        cpu = None
    elif args.workload == "prefill":
        T = 512
        steps = min(args.steps, 16)
        cfg = llama_config(n_layers=32, vocab=128256, max_seq=T)
        m = Llama(ctx, cfg)
        fill_llama(m, 1)
        prompt = np.random.default_rng(512).integers(0, 128000, size=T).tolist()
        nxt = ctx.alloc(16)
        for _ in range(args.warmup):
            m.reset()
            m.prefill(prompt, nxt)
        ctx.wait()
        barrier(pg, local)
        sampler = ClockSampler(local)
        sampler.start()
        time.sleep(0.3)

        def passes():
            for _ in range(steps):
                m.reset()
                m.prefill(prompt, nxt)
        dev_ms = timed(passes)
        clocks = sampler.stop()
        ms_max = max_over_ranks(dev_ms, pg, local)
        per_step_ms = ms_max / steps
        value = T * steps * world / (ms_max * 1e-3)
        unit = "tokens/s"
        flops = llama_prefill_flops(32, T)
        alg = llama_token_bytes(32, 0)  # weights streamed once per pass
        launches = steps * (1 + 32 * 9 + 2)  # embed, 9 per layer, head GEMV + argmax
        # e2e: the prompt ids from host memory through mlm_llama_prefill, the
        # first generated token read back
        lib, h = ctx.lib, ctx.handle
        htok = ctypes.c_void_p()
        lib.mlm_host_alloc(h, 16, ctypes.byref(htok))
        e2e_steps = min(steps, 4)
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            m.reset()
            m.prefill(prompt, nxt)
            ctx._check(lib.mlm_download_async(h, htok, ctypes.c_void_p(nxt.ptr), 4), "dn")
            ctx.wait()
        e2e_s = max_over_ranks(time.perf_counter() - t0, pg, local)
        lib.mlm_host_free(h, htok)
        e2e = {"value": round(T * e2e_steps * world / e2e_s, 2), "unit": "tokens/s",
               "h2d_bytes_per_step": 4 * T, "d2h_bytes_per_step": 4}
        gk = gemm_kernel_time(ctx, m, 32, T, 64, tstream)
        config = {"workload": LLAMA_WORKLOADS["prefill"], "layers": 32, "hidden": 4096,
                  "heads": "32/8 x 128", "ffn": 14336, "vocab": 128256, "batch": 1,
                  "prompt_tokens": T, "parallelism": "single GPU",
                  "l2": "inputs larger than L2: 4.2 GB of Q4_K weights per pass",
                  "algorithmic_flops_per_step": flops}
        extra = {"tflops": round(flops / (per_step_ms * 1e-3) / 1e12, 1),
                 "roofline": {"bound": "tensor", "achieved": round(gk["tflops"], 1),
                              "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                              "frac": round(gk["tflops"] / peaks["bf16_tflops"], 4),
                              "peak_source": peaks["source"] + " (bf16 burst)",
                              "traffic": ncu_traffic("prefill"),
                              "kernel": "q4k_gemm_kernel, gate/up 28672x4096 x 512 tokens",
                              "kernel_ms": round(gk["ms"], 4),
                              "algorithmic_flops_per_launch": gk["flops"]}}
        cpu = None
    else:
        prompt_len, gen_len = 512, 256
        steps = min(args.steps, gen_len - args.warmup)
        cfg = llama_config(n_layers=32, vocab=128256, max_seq=prompt_len + gen_len)
        m = Llama(ctx, cfg)
        fill_llama(m, 1)
        prompt = np.random.default_rng(512).integers(0, 128000, size=prompt_len).tolist()
        nxt = ctx.alloc(16)
        ctx.wait()
        barrier(pg, local)
        m.prefill(prompt, nxt)  # first pass loads the kernels
        m.reset()
        prefill_ms = max_over_ranks(timed(lambda: m.prefill(prompt, nxt)), pg, local)
        first = int(nxt.download(np.int32)[0])
        out = ctx.alloc(4 * gen_len)
        m.decode_greedy(first, args.warmup, out)  # captures the step graph
        last = int(out.download(np.int32, args.warmup)[-1])
        ctx.wait()
        barrier(pg, local)
        sampler = ClockSampler(local)
        sampler.start()
        time.sleep(0.3)
        pos0 = m.position
        with nvtx_range("timed"):
            dev_ms = timed(lambda: m.decode_greedy(last, steps, out))
        clocks = sampler.stop()
        toks = out.download(np.int32, steps)
        ms_max = max_over_ranks(dev_ms, pg, local)
        per_step_ms = ms_max / steps
        value = steps * world / (ms_max * 1e-3)
        unit = "tokens/s"
        alg = llama_token_bytes(32, pos0 + steps // 2)
        launches = steps * (1 + 32 * 5 + 3)  # embed, 5 per layer, head, argmax, advance
        # e2e: forward(tokenID:) per token through the C ABI, the argmax read back
        m.set_position(prompt_len)
        lib, h = ctx.lib, ctx.handle
        htok = ctypes.c_void_p()
        lib.mlm_host_alloc(h, 16, ctypes.byref(htok))
        tok_dev = ctx.alloc(16)
        logits = ctx.alloc(4 * cfg.vocab)
        tok = first
        e2e_steps = min(steps, 32)
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            m.forward(tok, logits)
            ctx.call("mlm_argmax_f32", logits, cfg.vocab, tok_dev)
            ctx._check(lib.mlm_download_async(h, htok, ctypes.c_void_p(tok_dev.ptr), 4), "dn")
            ctx.wait()
            tok = ctypes.c_int32.from_address(htok.value).value
        e2e_s = max_over_ranks(time.perf_counter() - t0, pg, local)
        lib.mlm_host_free(h, htok)
        e2e = {"value": round(e2e_steps * world / e2e_s, 2), "unit": "tokens/s",
               "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 4}
        config = {"workload": LLAMA_WORKLOADS["decode"], "layers": 32, "hidden": 4096,
                  "heads": "32/8 x 128", "ffn": 14336, "vocab": 128256, "batch": 1,
                  "prompt_tokens": prompt_len, "decode_steps_timed": steps,
                  "parallelism": "single GPU",
                  "l2": "inputs larger than L2: 4.2 GB of Q4_K weights per token",
                  "algorithmic_bytes_per_step": alg}
        extra = {"prefill": {"value": round(prompt_len / (prefill_ms * 1e-3), 2),
                             "unit": "tokens/s",
                             "path": "batched prompt pass: tcgen05 Q4_K GEMM, bf16 activations"},
                 "first_tokens": [int(t) for t in toks[:8]]}
        cpu = "decode"
    kernel_gbs = alg / (per_step_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": unit, "n_gpus": world,
        "steps": args.steps if args.workload == "layer" else steps, "warmup": args.warmup,
        "ms_per_step": round(per_step_ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q4k x f16 -> f32 (fp16 KV cache)",
        "data": "synthetic (seeded Q4_K weights, fp16 embedding, fp32 norms generated on "
                "device)",
        "config": config, "e2e": e2e, "gpu_launches": launches,
        "launch": ("stream-ordered launches, one per kernel" if args.workload == "prefill" else
                   "CUDA graph (one decode step captured, replayed per token)"),
        "roofline": {"bound": "hbm", "achieved": round(kernel_gbs, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(kernel_gbs / peaks["hbm_gbs"], 4),
                     "peak_source": peaks["source"], "traffic": None},
        "clocks": clocks,
    }
    line.update(extra)
    if args.workload == "prefill":
        line["dtype"] = "q4k -> bf16 x bf16 -> f32 (tcgen05), fp16 KV cache"
    if rank == 0 and world == 1 and not args.no_cpu and cpu == "decode":
        line["cpu_baseline"] = cpu_decode_rate(args.cpu_seconds, host_threads())
    ctx.close()
    return line


def run_tp70b(args, world, rank, local, pg) -> dict:
    """The 70B shape tensor-parallel over the launch's ranks (one process and
    one NCCL rank per GPU): every sequence's prompt pass, then timed batched
    greedy decode."""
    import torch

    from metallm_b200 import Context, Llama
    from metallm_b200.synthetic import fill_llama, llama_config
    from metallm_b200.tp import bootstrap
    ctx = Context(local)
    torch.cuda.set_device(local)
    tstream = torch.cuda.ExternalStream(ctx.stream(), device=f"cuda:{local}")
    peaks = measured_peaks()
    if world > 1:
        bootstrap(ctx)
    B, prompt_len, gen_len = args.batch, TP70_PROMPT, TP70_GEN
    steps = tp70b_steps(args)
    cfg = llama_config(max_seq=prompt_len + gen_len, **L70)
    m = Llama(ctx, cfg, batch=B)
    fill_llama(m, 1)
    prompts = [np.random.default_rng(2048 + b).integers(0, 128000, size=prompt_len).tolist()
               for b in range(B)]
    nxt = ctx.alloc(16)

    def timed(fn):
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(tstream)
        fn()
        ev1.record(tstream)
        ev1.synchronize()
        return ev0.elapsed_time(ev1)

    m.prefill(prompts[0][:256], nxt)  # loads the kernels
    m.reset()
    ctx.wait()
    barrier(pg, local)
    firsts = []

    def prompt_pass():
        for b in range(B):
            m.prefill(prompts[b], nxt, None, seq=b)
            firsts.append(int(nxt.download(np.int32)[0]))
    prefill_ms = max_over_ranks(timed(prompt_pass), pg, local)
    out = ctx.alloc(4 * gen_len * B)
    m.decode_greedy_batch(firsts, args.warmup, out)  # captures the batched step
    last = out.download(np.int32, args.warmup * B).reshape(args.warmup, B)[-1].tolist()
    ctx.wait()
    barrier(pg, local)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    pos0 = m.seq_position(0)
    with nvtx_range("timed"):
        dev_ms = timed(lambda: m.decode_greedy_batch(last, steps, out))
    clocks = sampler.stop()
    toks = out.download(np.int32, steps * B).reshape(steps, B)
    ms_max = max_over_ranks(dev_ms, pg, local)
    per_step_ms = ms_max / steps
    alg = llama70_rank_bytes(world, pos0 + steps // 2, B)
    kernel_gbs = alg / (per_step_ms * 1e-3) / 1e9
    # e2e: one greedy batched step per call through the C ABI, the batch's
    # tokens in from host memory and out again
    tok = toks[-1].tolist()
    e2e_steps = 2
    barrier(pg, local)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        m.decode_greedy_batch(tok, 1, out)
        tok = out.download(np.int32, B).tolist()
    e2e_s = max_over_ranks(time.perf_counter() - t0, pg, local)
    line = {
        "metric": METRIC, "value": round(B * steps / (ms_max * 1e-3), 2), "unit": "tokens/s",
        "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(per_step_ms, 5), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None,
        "dtype": "q4k -> bf16 x bf16 -> f32 (tcgen05 GEMM over the batch), fp16 KV cache",
        "data": "synthetic (seeded Q4_K weights, fp16 embedding, fp32 norms generated on device; "
                "every rank its shard of one model; uniform random prompt ids)",
        "config": dict(tp70b_config(args, world), algorithmic_bytes_per_step_per_rank=alg),
        "e2e": {"value": round(B * e2e_steps / e2e_s, 2), "unit": "tokens/s",
                "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B},
        # per step: embedding; per layer 2 RMSNorm rows, 4 batched GEMVs, the
        # fused attention, SwiGLU rows (+ 2 one-shot all-reduces with TP);
        # head: RMSNorm, GEMV, B argmaxes (+ the key reduce with TP); advance
        "gpu_launches": steps * (1 + 80 * (8 + (2 if world > 1 else 0)) + 2 + B
                                 + (1 if world > 1 else 0) + 1),
        "launch": "CUDA graph (one batched decode step, all-reduces included, replayed per step)",
        "roofline": {"bound": "hbm", "achieved": round(kernel_gbs, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(kernel_gbs / peaks["hbm_gbs"], 4),
                     "peak_source": peaks["source"], "traffic": None,
                     "note": "per rank: its weight shard once per step and its KV heads of "
                             "every sequence"},
        "prefill": {"value": round(B * prompt_len / (prefill_ms * 1e-3), 2), "unit": "tokens/s",
                    "path": "batched prompt pass per sequence: tcgen05 Q4_K GEMM, all-reduce per "
                            "projection"},
        "first_tokens": [int(t) for t in toks[:4, 0]],
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_decode_rate(args.cpu_seconds, host_threads(), big=True)
    m.close()
    ctx.close()
    return line



FORMAT_WORKLOADS = {
    # name: (rows, cols, description)
    "gemv_q6k": (128256, 4096, "Q6_K x fp16 GEMV 128256x4096 (the Llama-3-8B output head as "
                               "Q4_K_M files store it), batch 1"),
    "repack": (4096, 4096, "GGUF-order Q4_K -> kernel-order repack of one 4096x4096 tensor "
                           "(65,536 super-blocks, in place)"),
}


def q6k_gemv_bytes(rows: int, cols: int) -> int:
    return rows * (cols // 256) * 210 + 2 * cols + 4 * rows


def cpu_q6k_gemv_rate(rows: int, cols: int, budget_s: float, threads: int) -> dict:
    """The reference's path for a Q6_K linear on the host: its own
    kernel_dequantize_q6_K_f32 (oracle/_ref) over the matrix, then the fp32
    product with x (the reference hands the dequantized matrix to MPS), on a
    bounded row sample; GB/s of packed weights."""
    import numpy as np

    from oracle import oracle as O
    sample = min(rows, 8192)
    W = O.gen_q6k(11, 1, sample * cols // 256)
    x = O.gen_f16(11, 2, cols).astype(np.float32)
    use_ref = O.ref_lib() is not None
    deq = (lambda: O.ref_q6k_dequant_f32(W, sample * cols, threads)) if use_ref else \
        (lambda: O.q6k_dequant_f32(W, sample * cols, threads))
    fn = lambda: deq().reshape(sample, cols) @ x  # noqa: E731
    fn()
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(q6k_gemv_bytes(sample, cols) / dt / 1e9, 4), "unit": "GB/s",
            "cores": threads, "kind": "reference" if use_ref else "port",
            "sample": f"{reps} x ({sample} rows x {cols} Q6_K dequantized by the reference kernel "
                      f"+ fp32 product) in {time.perf_counter() - t0:.1f} s, {threads} threads"}


def cpu_repack_rate(nblocks: int, budget_s: float) -> dict:
    """The oracle's repack (a plain C loop, one thread): the reference has no
    repack at all (it reads GGUF blocks in its own order)."""
    from oracle import oracle as O
    b = O.gen_q4k(5, 1, nblocks)
    O.q4k_canonical_to_interleaved(b)
    reps, t0 = 0, time.perf_counter()
    while True:
        O.q4k_canonical_to_interleaved(b)
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(2 * 144 * nblocks / dt / 1e9, 4), "unit": "GB/s", "cores": 1,
            "kind": "port",
            "sample": f"{reps} x {nblocks} blocks in {time.perf_counter() - t0:.1f} s, 1 thread"}


def run_formats(args, world, rank, local, pg) -> dict:
    """The Q6_K GEMV (the output head of a Q4_K_M file) and the GGUF-order
    Q4_K repack, each step one launch over rotating inputs larger than L2."""
    import torch

    from metallm_b200 import Context
    rows, cols, desc = FORMAT_WORKLOADS[args.workload]
    ctx = Context(local)
    torch.cuda.set_device(local)
    tstream = torch.cuda.ExternalStream(ctx.stream(), device=f"cuda:{local}")
    peaks = measured_peaks()
    nb = rows * cols // 256
    q6 = args.workload == "gemv_q6k"
    bb = 210 if q6 else 144
    copies = max(2, -(-400_000_000 // (nb * bb)))  # > 3x the 126 MB L2
    Ws = []
    for c in range(copies):
        W = ctx.alloc(nb * bb)
        (ctx.gen_q6k if q6 else ctx.gen_q4k)(1000 + c, 1, nb, W)
        Ws.append(W)
    x = ctx.alloc(2 * cols)
    ctx.gen_f16(7, 2, cols, x)
    y = ctx.alloc(4 * rows)
    if q6:
        step = lambda i: ctx.q6k_gemv(Ws[i % copies], rows, cols, x, y)  # noqa: E731
        alg = q6k_gemv_bytes(rows, cols)
    else:  # in place: each pass shuffles a copy again (a bijection, same traffic)
        step = lambda i: ctx.q4k_repack_canonical(Ws[i % copies], Ws[i % copies], nb)  # noqa: E731
        alg = 2 * 144 * nb
    ctx.graph_begin()
    for i in range(args.steps):
        step(i)
    graph = ctx.graph_end()
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
    ms_max = max_over_ranks(dev_ms, pg, local)
    per_ms = ms_max / args.steps
    gbs = alg / (per_ms * 1e-3) / 1e9
    # e2e through the C ABI with host buffers: x in (GEMV) or the GGUF blocks
    # in and the repacked blocks out (repack), from/to pinned host memory
    lib, h = ctx.lib, ctx.handle
    in_bytes = 2 * cols if q6 else nb * 144
    out_bytes = 4 * rows if q6 else nb * 144
    hin, hout = ctypes.c_void_p(), ctypes.c_void_p()
    lib.mlm_host_alloc(h, in_bytes, ctypes.byref(hin))
    lib.mlm_host_alloc(h, out_bytes, ctypes.byref(hout))
    dst_in = x if q6 else Ws[0]
    dst_out = y if q6 else Ws[0]
    e2e_steps = min(args.steps, 20)
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        ctx._check(lib.mlm_upload_async(h, ctypes.c_void_p(dst_in.ptr), hin, in_bytes), "up")
        step(i if q6 else 0)
        ctx._check(lib.mlm_download_async(h, hout, ctypes.c_void_p(dst_out.ptr), out_bytes), "dn")
        ctx.wait()
    e2e_s = max_over_ranks(time.perf_counter() - t0, pg, local)
    lib.mlm_host_free(h, hin)
    lib.mlm_host_free(h, hout)
    line = {
        "metric": METRIC, "value": round(gbs * world, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q6k x f16 -> f32" if q6 else "u8 (nibble shuffle)",
        "data": "synthetic (seeded blocks generated on device)",
        "config": {"workload": desc, "rows": rows, "cols": cols,
                   "parallelism": "replicas" if world > 1 else "single GPU",
                   "l2": f"{copies} rotating copies ({copies * nb * bb / 1e6:.0f} MB > L2)",
                   "algorithmic_bytes_per_step": alg},
        "e2e": {"value": round(alg * e2e_steps * world / e2e_s / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": out_bytes},
        "gpu_launches": args.steps,
        "launch": "CUDA graph of K steps",
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                     "peak_source": peaks["source"], "traffic": ncu_traffic(args.workload)},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = (cpu_q6k_gemv_rate(rows, cols, args.cpu_seconds, host_threads())
                                if q6 else cpu_repack_rate(nb, args.cpu_seconds))
    ctx.close()
    return line

def run_reference(args, world, rank) -> dict | None:
    if rank != 0:
        return None
    if args.workload in FORMAT_WORKLOADS:
        rows, cols, desc = FORMAT_WORKLOADS[args.workload]
        q6 = args.workload == "gemv_q6k"
        r = (cpu_q6k_gemv_rate(rows, cols, args.cpu_seconds, host_threads()) if q6
             else cpu_repack_rate(rows * cols // 256, args.cpu_seconds))
        v = r["value"]
        alg = q6k_gemv_bytes(rows, cols) if q6 else 2 * 144 * (rows * cols // 256)
        return {"impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(alg / (v * 1e9) * 1e3, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None,
                "dtype": "q6k x f16 -> f32" if q6 else "u8 (nibble shuffle)",
                "data": "synthetic (seeded blocks)",
                "config": {"workload": desc, "rows": rows, "cols": cols}, "cpu_baseline": r,
                "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
    if args.workload == "gemv_batch":
        rows, cols, T = GEMV_BATCH_SHAPE
        r = cpu_gemv_rate(rows, cols, args.cpu_seconds, host_threads(), "reference")
        v = r["value"]
        return {"impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(gemv_bytes(rows, cols) / (v * 1e9) * 1e3 * T, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "q4k x f16 -> f32", "data": "synthetic (seeded Q4_K blocks)",
                "config": {"workload": GEMV_BATCH_DESC, "rows": rows, "cols": cols, "tokens": T},
                "cpu_baseline": dict(r, sample=r["sample"] + "; one token per matvec"),
                "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
    if args.workload == "gemm":
        r = cpu_gemm_rate(args.cpu_seconds, host_threads())
        rows, cols, T = GEMM_SHAPE
        v = r["value"]
        return {"impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(2 * rows * cols * T / (v * 1e12) * 1e3, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "q4k x f16 -> f32", "data": "synthetic (seeded Q4_K blocks)",
                "config": {"workload": GEMM_DESC, "rows": rows, "cols": cols, "tokens": T},
                "cpu_baseline": r,
                "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
    if args.workload in LLAMA_WORKLOADS:
        th = host_threads()
        r = cpu_decode_rate(args.cpu_seconds, th, big=args.workload == "tp70b")
        if args.workload in ("decode", "tp70b"):
            v, unit = r["value"], "tokens/s"
            ms = 1e3 / v
        elif args.workload == "prefill":  # every prompt token through 32 layers, one head
            T = 512
            ms = (T * 32 * r["layer_s"] + r["head_s"]) * 1e3
            v, unit = round(T / (ms * 1e-3), 4), "tokens/s"
            r = dict(r, sample=r["sample"] + "; prompt tokens/s = 512 / (512 x 32 x layer + head)")
        else:  # one layer: its bytes over a 32nd of the token time without the head
            alg = llama_token_bytes(1, 2047, with_head=False) - 2 * 4096
            ms = 1e3 / r["value"] / 33.0
            v, unit = round(alg / (ms * 1e-3) / 1e9, 3), "GB/s"
        return {"impl": "reference", "metric": METRIC, "value": v, "unit": unit, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "q4k x f16 -> f32", "data": "synthetic (seeded Q4_K blocks)",
                "config": (tp70b_config(args, world) if args.workload == "tp70b" else
                           {"workload": LLAMA_WORKLOADS[args.workload]}),
                "cpu_baseline": dict(r, value=v, unit=unit),
                "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
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
        "config": gemv_config(args, world, rows, cols, desc),
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": th, "kind": vals[0]["kind"],
                         "sample": vals[0]["sample"]},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


SUB_KEYS = ("value", "unit", "ms_per_step", "steps", "warmup", "dtype", "config", "e2e",
            "gpu_launches", "launch", "roofline", "prefill", "first_tokens", "clocks",
            "cpu_baseline", "scaling", "n_gpus")


def sub_measurements(args, local: int) -> dict:
    """The second half of the metric and the sharded workload at one GPU,
    measured in the same run as the headline: 'decode' = the Llama-3-8B-shape
    model (512-token prompt pass, then timed greedy decode, tokens/s) and
    'tp70b' = the 70B-shape batch of 8 on this one GPU through the same code
    the multi-GPU lines run (the base of the scaling curve)."""
    import copy
    out = {}
    sub = copy.copy(args)
    sub.workload, sub.steps, sub.default_line = "decode", 128, False
    d = run_llama(sub, 1, 0, local, None)
    out["decode"] = {k: d[k] for k in SUB_KEYS if k in d}
    sub = copy.copy(args)
    sub.workload, sub.default_line = "tp70b", False
    t = run_tp70b(sub, 1, 0, local, None)
    out["tp70b"] = {k: t[k] for k in SUB_KEYS if k in t}
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default=None,
                    choices=sorted(WORKLOADS) + sorted(LLAMA_WORKLOADS) + sorted(FORMAT_WORKLOADS)
                    + ["gemm", "gemv_batch"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--copies", type=int, default=0,
                    help="rotating weight copies (default: a divisor of --steps totalling > L2)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--batch", type=int, default=8, help="sequences of the tp70b workload")
    ap.add_argument("--no-extras", action="store_true",
                    help="default line without its decode / tp70b sub-measurements")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    # No --workload: one GPU measures the headline GEMV (with the 8B decode and
    # the one-GPU 70B batch as sub-objects); under torchrun the ranks run the
    # 70B model tensor-parallel, the workload that shards.
    args.default_line = args.workload is None
    if args.workload is None:
        args.workload = "tp70b" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else "gemv_up"

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    world, rank, local, pg = dist_setup(args)
    try:
        run = {"gemm": run_gemm, "gemv_batch": run_gemv_batch, "tp70b": run_tp70b,
               "gemv_q6k": run_formats, "repack": run_formats}.get(
            args.workload, run_llama if args.workload in LLAMA_WORKLOADS else run_gpu)
        line = run(args, world, rank, local, pg)
        if args.default_line and world == 1 and not args.no_extras:
            line.update(sub_measurements(args, local))
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if pg is not None:
            pg.destroy_process_group()


if __name__ == "__main__":
    main()
