#!/usr/bin/env python
"""Benchmark of the batch-invariant bf16 linear path.

Workload ("config2-bf16-linear-sweep"): Y = X[:M] @ W_N^T + b_N through the
reference-compatible ``linear_batch_invariant`` for K = 4096,
N in {4096, 11008, 16384} and M in {1, 8, 32, 128, 512, 2048, 8192};
X ~ N(0, 1), W ~ N(0, 1/4096), b ~ N(0, 0.02), bf16, synthetic, seeded.
One step = one pass over the 21 (M, N) points.

Reported (one JSON line from rank 0):
  value     whole-job TFLOP/s = sum of 2*M*N*K over all points and ranks /
            max over ranks of the summed device time of the GEMM launches.
            Each launch is replayed from a CUDA graph and bracketed by CUDA
            events on its stream; between launches (outside the events) a
            512 MiB write flushes L2 and a 256 MiB read then evicts the dirty
            lines, so no operand is L2-resident and the timed kernel does not
            pay for the flush's write-backs.
  e2e       the same metric through the public Python API with the step's
            activations copied host->device from pinned memory and the
            outputs copied back, inside the timed region.
  roofline  the dominant launch (largest share of device time) against the
            measured peaks of MEASURED_PEAKS.json; per-point figures in
            "sweep".
  bitwise   B=1 vs slice-of-B=N checks over the sweep (must be 0).
  cpu_baseline  stock PyTorch CPU F.linear in bf16 on a bounded sample of
            the same points, all host threads (rank 0, N=1 only): the path a
            reference user gets for CPU tensors; cpu_fp64_oracle is the fp64
            parity checker timed the same way.

``--impl reference`` times that stock CPU path on the host cores, on the same
metric and config.  Multi-GPU (torchrun): every rank runs the whole sweep on
its own GPU (weak scaling, no collective on the hot path);
NCCL is used only for the barrier, the max-time reduction and the final
bitwise cross-check of the ranks' outputs.
"""

from __future__ import annotations

import argparse
import contextlib
import csv
import io
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG_ROOT = ROOT / "robotics-batch-invariant-ops_b200"

METRIC = "BI bf16 mm/bmm TFLOP/s & %roofline at M=1–8192; B1-vs-BN bit diffs = 0"
UNIT = "TFLOP/s"
WORKLOAD = "config2-bf16-linear-sweep"
SWEEP_N = (4096, 11008, 16384)
SWEEP_M = (1, 8, 32, 128, 512, 2048, 8192)
K = 4096
FLUSH_BYTES = 512 << 20
EVICT_BYTES = 256 << 20

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def _peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def _points():
    return [(m, n) for n in SWEEP_N for m in SWEEP_M]


def _flops(m, n):
    return 2.0 * m * n * K


def _bytes(m, n):
    return 2.0 * (m * K + n * K + m * n + n)


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during timing."""

    QUERY = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, index: int):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"samples": 0, "note": "nvidia-smi unavailable"}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = []
        with open(self.file.name) as fh:
            for rec in csv.reader(fh):
                if len(rec) < 9:
                    continue
                try:
                    rows.append([r.strip() for r in rec])
                except ValueError:
                    continue
        os.unlink(self.file.name)
        if not rows:
            return {"samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "reasons": reasons,
            "samples": len(rows),
        }


class _Flusher:
    """L2 flush between timed launches: write FLUSH_BYTES, then read EVICT_BYTES
    of another buffer so the written lines are evicted (written back) before
    the next timed launch starts."""

    def __init__(self, dev):
        import torch

        self.w = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.r = torch.ones(EVICT_BYTES // 4, dtype=torch.float32, device=dev)

    def __call__(self):
        self.w.zero_()
        self.r.sum()


# ---------------------------------------------------------------------------
# distributed helpers
# ---------------------------------------------------------------------------
def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---------------------------------------------------------------------------
# CPU baselines on the box's host cores
# ---------------------------------------------------------------------------
STOCK_CPU_WHAT = (
    "stock PyTorch CPU F.linear in bf16, all host threads: the path a user of "
    "the reference gets for CPU tensors (its overrides are registered on the "
    "accelerator's dispatch key only, batch_invariant_ops.py:1666-1684)")


def _cpu_points(gen):
    """Sweep points ordered by work, with their CPU operands."""
    import torch

    weights = {}
    for n in SWEEP_N:
        w = (torch.randn(n, K, generator=gen) / 64).to(torch.bfloat16)
        b = (torch.randn(n, generator=gen) * 0.02).to(torch.bfloat16)
        weights[n] = (w, b)
    x_all = torch.randn(max(SWEEP_M), K, generator=gen).to(torch.bfloat16)
    return sorted(_points(), key=lambda p: _flops(*p)), weights, x_all


def cpu_stock_linear(budget_s: float = 20.0) -> dict:
    """Stock bf16 F.linear on the host cores over a bounded sample of the
    sweep: points in order of work, each run once (after one warm-up call),
    skipping a point whose predicted time would exceed the budget."""
    import torch
    import torch.nn.functional as F

    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator().manual_seed(0)
    points, weights, x_all = _cpu_points(gen)
    F.linear(x_all[:8], *weights[SWEEP_N[0]])  # warm-up (thread pool, kernels)
    done, flops, elapsed, rate = [], 0.0, 0.0, None
    for m, n in points:
        if rate is not None and elapsed + _flops(m, n) / rate > budget_s:
            continue
        w, b = weights[n]
        t0 = time.perf_counter()
        F.linear(x_all[:m], w, b)
        dt = time.perf_counter() - t0
        elapsed += dt
        flops += _flops(m, n)
        rate = flops / elapsed
        done.append(f"{m}x{n}")
    # the CPU path's own batch invariance (first row alone vs in the batch)
    w, b = weights[SWEEP_N[0]]
    full = F.linear(x_all[:512], w, b)
    cpu_diffs = int((F.linear(x_all[:1], w, b) != full[:1]).sum().item())
    return {
        "value": flops / elapsed / 1e12 if elapsed > 0 else None,
        "unit": UNIT,
        "cores": torch.get_num_threads(),
        "kind": "reference",
        "what": STOCK_CPU_WHAT,
        "sample": f"{len(done)} of 21 sweep points ({', '.join(done)}), {elapsed:.1f} s of CPU work",
        "b1_vs_bn_bit_diffs_m512_n4096": cpu_diffs,
    }


def cpu_fp64_oracle(budget_s: float = 5.0) -> dict:
    """The fp64 CPU oracle (the parity checker) on a bounded sample of the sweep."""
    import torch

    sys.path.insert(0, str(ROOT))
    from oracle import bio_oracle

    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator().manual_seed(0)
    points, weights, x_all = _cpu_points(gen)
    done, flops, elapsed = [], 0.0, 0.0
    for m, n in points:
        if elapsed > budget_s:
            break
        w, b = weights[n]
        t0 = time.perf_counter()
        bio_oracle.linear(x_all[:m], w, b)
        elapsed += time.perf_counter() - t0
        flops += _flops(m, n)
        done.append(f"{m}x{n}")
    return {
        "value": flops / elapsed / 1e12 if elapsed > 0 else None,
        "unit": UNIT,
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": f"fp64 oracle linear on {len(done)} of 21 sweep points, {elapsed:.1f} s",
    }


def _config(world: int) -> dict:
    """The workload description both arms print (identical by construction)."""
    return {
        "workload": WORKLOAD,
        "K": K,
        "N": list(SWEEP_N),
        "M": list(SWEEP_M),
        "layout": "F.linear: weight [N,K] K-contiguous",
        "l2": "flushed before every timed launch (512 MiB write + 256 MiB read), outside the events",
        "parallelism": f"replica{world} (each rank runs the full sweep)",
    }


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(PKG_ROOT))
    from batch_invariant_ops import _gemm, linear_batch_invariant, sharding

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    peaks, peak_kind = _peaks()

    gen = torch.Generator(device=dev).manual_seed(0)
    x_all = torch.randn(max(SWEEP_M), K, device=dev, generator=gen).to(torch.bfloat16)
    weights = {}
    for n in SWEEP_N:
        w = (torch.randn(n, K, device=dev, generator=gen) / 64).to(torch.bfloat16)
        b = (torch.randn(n, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        weights[n] = (w, b)
    flush = _Flusher(dev)
    points = _points()
    stream = torch.cuda.current_stream(dev)

    # One CUDA graph per point: the replay launches exactly the library's GEMM
    # kernel (no host work inside the timed events).
    graphs, outs = {}, {}
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for m, n in points:
            w, b = weights[n]
            linear_batch_invariant(x_all[:m], w, b)
    stream.wait_stream(side)
    torch.cuda.synchronize(dev)
    for m, n in points:
        w, b = weights[n]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            outs[(m, n)] = linear_batch_invariant(x_all[:m], w, b)
        graphs[(m, n)] = g
    torch.cuda.synchronize(dev)

    def device_step(record):
        evs = []
        for p in points:
            flush()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            graphs[p].replay()
            e1.record(stream)
            evs.append((p, e0, e1))
        if record is not None:
            record.append(evs)

    sampler = ClockSampler(local)
    sampler.start()
    t_warm = time.perf_counter()
    for i in range(max(args.warmup, 3)):
        device_step(None)
    torch.cuda.synchronize(dev)
    while time.perf_counter() - t_warm < 0.5:  # let clocks settle
        device_step(None)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    records = []
    wall0 = time.perf_counter()
    for _ in range(args.steps):
        device_step(records)
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - wall0
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()

    per_point = {p: [] for p in points}
    for evs in records:
        for p, e0, e1 in evs:
            per_point[p].append(e0.elapsed_time(e1) * 1e-3)
    dev_time = sum(sum(v) for v in per_point.values())
    step_flops = sum(_flops(m, n) for m, n in points)

    # ---- end to end through the public API with host buffers.  Each step
    # copies every point's activations in from pinned host memory, runs the
    # linear and copies the output back to pinned host memory; the three
    # stages run on their own streams so the 21 points pipeline (copy-in of
    # point i+1 and copy-out of point i-1 overlap the GEMM of point i).
    host_x = torch.empty((max(SWEEP_M), K), dtype=torch.bfloat16, pin_memory=True)
    host_x.copy_(x_all.cpu())
    host_y = {p: torch.empty((p[0], p[1]), dtype=torch.bfloat16, pin_memory=True) for p in points}
    dev_x = {p: torch.empty((p[0], K), dtype=torch.bfloat16, device=dev) for p in points}
    h2d = sum(m * K * 2 for m, _ in points)
    d2h = sum(m * n * 2 for m, n in points)
    s_in = torch.cuda.Stream(device=dev)
    s_out = torch.cuda.Stream(device=dev)

    def e2e_step(record):
        flush()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        s_in.wait_stream(stream)
        s_out.wait_stream(stream)
        for m, n in points:
            w, b = weights[n]
            with torch.cuda.stream(s_in):
                dev_x[(m, n)].copy_(host_x[:m], non_blocking=True)
            stream.wait_stream(s_in)
            y = linear_batch_invariant(dev_x[(m, n)], w, b)
            s_out.wait_stream(stream)
            with torch.cuda.stream(s_out):
                host_y[(m, n)].copy_(y, non_blocking=True)
            y.record_stream(s_out)
        stream.wait_stream(s_out)
        e1.record(stream)
        if record is not None:
            record.append((e0, e1))

    for _ in range(max(args.warmup, 3)):
        e2e_step(None)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e2e_records = []
    for _ in range(args.steps):
        e2e_step(e2e_records)
    torch.cuda.synchronize(dev)
    e2e_time = sum(e0.elapsed_time(e1) * 1e-3 for e0, e1 in e2e_records)

    # ---- bitwise batch invariance over the sweep (B=1 .. 8192 rows)
    bit_diffs = 0
    checks = 0
    for n in SWEEP_N:
        w, b = weights[n]
        full = linear_batch_invariant(x_all, w, b)
        for m in SWEEP_M:
            part = linear_batch_invariant(x_all[:m], w, b)
            bit_diffs += int((part != full[:m]).sum().item())
            checks += 1
        other = torch.cat([x_all[:1], torch.randn(300, K, device=dev, generator=gen).to(torch.bfloat16)])
        bit_diffs += int((linear_batch_invariant(other, w, b)[:1] != full[:1]).sum().item())
        checks += 1
    # identical seeds on every rank: the ranks' outputs must agree bitwise
    cross_rank_equal = None
    if world > 1:
        cross_rank_equal = sharding.ranks_agree(
            sharding.bit_digest(outs[(SWEEP_M[-1], SWEEP_N[-1])]))

    # ---- max over ranks
    dev_time = sharding.max_over_ranks(dev_time, dev)
    e2e_time = sharding.max_over_ranks(e2e_time, dev)

    if rank == 0:
        total_flops = step_flops * args.steps * world
        value = total_flops / dev_time / 1e12
        sweep = []
        ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
        dominant, dom_time = None, -1.0
        for p in points:
            m, n = p
            t = statistics.mean(per_point[p])
            tf = _flops(m, n) / t / 1e12
            gbs = _bytes(m, n) / t / 1e9
            bound = "tensor" if _flops(m, n) / _bytes(m, n) >= ridge else "hbm"
            frac = tf / peaks["bf16_tflops"] if bound == "tensor" else gbs / peaks["hbm_gbs"]
            sweep.append({"m": m, "n": n, "us": round(t * 1e6, 2), "tflops": round(tf, 1),
                          "gbs": round(gbs, 1), "bound": bound, "frac": round(frac, 3)})
            if sum(per_point[p]) > dom_time:
                dominant, dom_time = p, sum(per_point[p])
        dm, dn = dominant
        dt = statistics.mean(per_point[dominant])
        achieved = _flops(dm, dn) / dt / 1e12
        traffic = None
        tfile = ROOT / "profiles" / "gemm_tc_dram_traffic.json"
        if tfile.exists():
            tinfo = json.loads(tfile.read_text())
            traffic = tinfo.get("dram_bytes_per_launch", {}).get(f"{dm}x{dn}")
        roofline = {
            "bound": "tensor",
            "achieved": round(achieved, 1),
            "peak": peaks["bf16_tflops"],
            "unit": "TFLOP/s",
            "frac": round(achieved / peaks["bf16_tflops"], 3),
            "traffic": traffic,
            "kernel": f"bio::gemm_tc2_kernel (CTA pair) tile {_gemm.tile_config(dn, K, torch.bfloat16)} at M={dm} N={dn} K={K}",
            "peak_source": f"{peak_kind} bf16_tflops (burst); sustained {peaks.get('bf16_tflops_sustained')}",
            "algorithmic_flops_per_launch": _flops(dm, dn),
        }
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(dev_time / args.steps * 1e3, 4),
            "wall_ms_per_step": round(wall / args.steps * 1e3, 3),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) activations, N(0,1/4096) weights, N(0,0.02) bias)",
            "config": _config(world),
            "timing": "CUDA graph replay per point, CUDA events on the launch stream",
            "bitwise": {"bit_diffs": bit_diffs, "checks": checks, "cross_rank_equal": cross_rank_equal},
            "e2e": {
                "value": round(total_flops / e2e_time / 1e12, 2),
                "unit": UNIT,
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "api": "batch_invariant_ops.linear_batch_invariant (eager); pinned host buffers, "
                "copy-in / GEMM / copy-out pipelined across the 21 points on 3 streams",
            },
            "gpu_launches": len(points) * args.steps,
            "roofline": roofline,
            "sweep": sweep,
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_stock_linear(args.cpu_budget)
            line["cpu_fp64_oracle"] = cpu_fp64_oracle(min(5.0, args.cpu_budget))
        if world == 1 and not args.no_triton_ref:
            line["reference_triton_b200"] = _triton_reference(args)
    graphs.clear()
    del outs
    torch.cuda.empty_cache()
    if not args.no_vla:
        # every rank takes part (sharded step, NCCL gather); rank 0 reports
        vla = vla_sharded(world, rank, dev, args.vla_global_batch, args.vla_steps, args.warmup)
        if rank == 0:
            line["vla"] = vla
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _triton_reference(args) -> dict:
    """Time the reference's own Triton matmul_persistent on the same sweep
    (same method) in a child process; requires baseline/_ref."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "batch_invariant_ops").exists():
        return {"unavailable": "reference package not installed in baseline/_ref"}
    try:
        proc = subprocess.run([sys.executable, str(Path(__file__).resolve()), "--triton-ref-worker",
                               "--steps", str(args.steps), "--warmup", str(args.warmup)],
                              capture_output=True, text=True, timeout=900)
        lines = [l for l in proc.stdout.splitlines() if l.startswith("{")]
        if proc.returncode != 0 or not lines:
            return {"unavailable": (proc.stderr.strip().splitlines() or ["failed"])[-1][:300]}
        return json.loads(lines[-1])
    except subprocess.TimeoutExpired:
        return {"unavailable": "timed out"}


def run_triton_ref_worker(args) -> None:
    import torch

    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
    import batch_invariant_ops as ref  # the reference package

    assert "baseline" in ref.__file__
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(0)
    x_all = torch.randn(max(SWEEP_M), K, device=dev, generator=gen).to(torch.bfloat16)
    weights = {}
    for n in SWEEP_N:
        w = (torch.randn(n, K, device=dev, generator=gen) / 64).to(torch.bfloat16)
        b = (torch.randn(n, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        weights[n] = (w, b)
    flush = _Flusher(dev)
    points = _points()
    stream = torch.cuda.current_stream(dev)
    for m, n in points:
        ref.linear_batch_invariant(x_all[:m], *weights[n])
    torch.cuda.synchronize()
    graphs = {}
    for m, n in points:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ref.linear_batch_invariant(x_all[:m], *weights[n])
        graphs[(m, n)] = g
    per_point = {p: [] for p in points}
    for step in range(max(args.warmup, 3) + args.steps):
        evs = []
        for p in points:
            flush()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            graphs[p].replay()
            e1.record(stream)
            evs.append((p, e0, e1))
        torch.cuda.synchronize()
        if step >= max(args.warmup, 3):
            for p, e0, e1 in evs:
                per_point[p].append(e0.elapsed_time(e1) * 1e-3)
    total = sum(sum(v) for v in per_point.values())
    flops = sum(_flops(m, n) for m, n in points) * args.steps
    print(json.dumps({
        "value": round(flops / total / 1e12, 2),
        "unit": UNIT,
        "what": "reference Triton matmul_persistent (baseline/_ref) on this B200, same sweep and timing",
        "sweep_us": {f"{m}x{n}": round(statistics.mean(per_point[(m, n)]) * 1e6, 2) for m, n in points},
    }), flush=True)


# ---------------------------------------------------------------------------
# reference arm: the reference's CPU restatement on the host cores
# ---------------------------------------------------------------------------
def run_reference(args) -> None:
    """The reference arm: the reference's CPU path for this workload (stock
    bf16 F.linear on CPU tensors, all host threads) on the same metric; each
    step is a bounded sample of the sweep."""
    world, rank, _ = _dist()
    if rank != 0:
        return
    per_step = max(2.0, min(20.0, 60.0 / max(args.steps + args.warmup, 1)))
    for _ in range(args.warmup):
        cpu_stock_linear(per_step / 4)
    vals = [cpu_stock_linear(per_step) for _ in range(args.steps)]
    good = [v["value"] for v in vals if v["value"]]
    value = statistics.median(good) if good else None
    cb = dict(vals[-1])
    cb["value"] = value
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,1/4096) weights, N(0,0.02) bias)",
        "config": _config(world),
        "cpu_baseline": cb,
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# per-operator table (--ops): every operator family of the path on a
# representative BASELINE shape, ours vs stock PyTorch vs the reference's
# Triton implementation, with algorithmic flops / bytes and roofline fractions
# ---------------------------------------------------------------------------
def _ops_cases(api, dev):
    """[(name, fn, flops, bytes, stock_fn)] built against the module ``api``
    (this package or the reference package: same public names)."""
    import torch
    import torch.nn.functional as F

    g = torch.Generator(device=dev).manual_seed(0)

    def rn(*shape, dtype=torch.bfloat16, scale=1.0):
        return (torch.randn(*shape, device=dev, generator=g) * scale).to(dtype)

    cases = []
    # GEMM (config 2 extremes)
    x1, x8k = rn(1, 4096), rn(8192, 4096)
    w, b = rn(16384, 4096, scale=1 / 64), rn(16384, scale=0.02)
    cases.append(("linear M=1 N=16384 K=4096 bf16", lambda: api.linear_batch_invariant(x1, w, b),
                  2 * 16384 * 4096, 2 * (4096 + 16384 * 4096 + 16384 + 16384),
                  lambda: F.linear(x1, w, b)))
    cases.append(("linear M=8192 N=16384 K=4096 bf16", lambda: api.linear_batch_invariant(x8k, w, b),
                  2 * 8192 * 16384 * 4096, 2 * (8192 * 4096 + 16384 * 4096 + 8192 * 16384),
                  lambda: F.linear(x8k, w, b)))
    # fp32 mm (config 1)
    a32 = torch.linspace(-100, 100, 2048 * 4096, device=dev).reshape(2048, 4096)
    w32 = torch.linspace(-100, 100, 4096 * 4096, device=dev).reshape(4096, 4096)
    cases.append(("mm fp32 2048x4096x4096 (config 1)", lambda: api.matmul_persistent(a32, w32),
                  2 * 2048 * 4096 * 4096, 4 * (2 * 2048 * 4096 + 4096 * 4096),
                  lambda: torch.mm(a32, w32)))
    # attention (config 3)
    for bsz, seq, causal in ((4, 4096, True), (16, 1024, False)):
        q = rn(bsz, 16, seq, 128)
        k, v = rn(bsz, 4, seq, 128), rn(bsz, 4, seq, 128)
        fl = 4 * bsz * 16 * seq * seq * 128 // (2 if causal else 1)
        by = 2 * (2 * bsz * 16 * seq * 128 + 2 * bsz * 4 * seq * 128)
        cases.append((f"sdpa B={bsz} S={seq} H16/4 D128 {'causal' if causal else 'full'} bf16",
                      lambda q=q, k=k, v=v, c=causal: api.scaled_dot_product_attention_batch_invariant(
                          q, k, v, is_causal=c, enable_gqa=True),
                      fl, by,
                      lambda q=q, k=k, v=v, c=causal: F.scaled_dot_product_attention(
                          q, k, v, is_causal=c, enable_gqa=True)))
    q = rn(2, 16, 1024, 128)
    k, v = rn(2, 4, 1024, 128), rn(2, 4, 1024, 128)
    keep = torch.rand(2, 1, 1024, 1024, device=dev, generator=g) > 0.1
    cases.append(("sdpa B=2 S=1024 bool mask p=0.1 bf16",
                  lambda: api.scaled_dot_product_attention_batch_invariant(q, k, v, attn_mask=keep,
                                                                          enable_gqa=True),
                  4 * 2 * 16 * 1024 * 1024 * 128, 2 * (2 * 2 * 16 * 1024 * 128 + 2 * 2 * 4 * 1024 * 128)
                  + 2 * 1024 * 1024,
                  lambda: F.scaled_dot_product_attention(q, k, v, attn_mask=keep, enable_gqa=True)))
    lens = torch.randint(16, 2049, (32,), generator=torch.Generator().manual_seed(0)).tolist()
    cu = torch.tensor([0] + list(__import__("itertools").accumulate(lens)), device=dev,
                      dtype=torch.int32)
    tot = int(cu[-1])
    vq, vk, vv = rn(1, tot, 16, 128), rn(1, tot, 4, 128), rn(1, tot, 4, 128)
    vfl = sum(4 * 16 * L * (L + 1) // 2 * 128 for L in lens)
    cases.append(("varlen 32 seqs U[16,2048] H16/4 D128 top-left causal bf16",
                  lambda: api.varlen_scaled_dot_product_attention_batch_invariant(
                      vq, vk, vv, cu, cu, is_causal=True, causal_type="TopLeft"),
                  vfl, 2 * tot * (16 + 4 + 4 + 16) * 128, None))
    # MoE (config 4)
    hid = rn(1024, 2048)
    gw, uw = rn(8, 5632, 2048, scale=0.02), rn(8, 5632, 2048, scale=0.02)
    dw = rn(8, 2048, 5632, scale=0.02)
    logits = torch.randn(1024, 8, device=dev, generator=g)
    top, sel = torch.topk(logits, 2)
    rw = torch.softmax(top, -1)
    sel64 = sel.contiguous()
    cases.append(("moe T=1024 E=8 top-2 2048->5632 bf16 (routed rows only; flops of the routed "
                  "rows)",
                  lambda: api.deterministic_token_choice_moe(hid, rw, sel, gw, uw, dw),
                  6 * 1024 * 2 * 2048 * 5632, 2 * 3 * 8 * 2048 * 5632, None))
    cases.append(("moe T=1024 E=8 top-2 2048->5632 bf16 (every expert on every token, the "
                  "reference's schedule; same bits)",
                  lambda: api.moe._dense_moe(hid, rw, sel64, gw, uw, dw),
                  6 * 1024 * 8 * 2048 * 5632, 2 * 3 * 8 * 2048 * 5632, None))
    # convolutions
    img = rn(32, 3, 224, 224)
    pw = rn(1152, 3, 14, 14, scale=0.02)
    cases.append(("conv2d SigLIP patch14 B=32 bf16",
                  lambda: api.conv2d_batch_invariant(img, pw, None, (14, 14), (0, 0), (1, 1), False,
                                                     (0, 0), 1),
                  2 * 32 * 256 * 1152 * 588, 2 * (img.numel() + pw.numel() + 32 * 1152 * 256),
                  lambda: F.conv2d(img, pw, stride=14)))
    sig = rn(8, 6144, 650)
    dwk = rn(6144, 1, 4)
    cases.append(("conv1d depthwise [8,6144,650] k4 p3 bf16",
                  lambda: api.conv1d_batch_invariant(sig, dwk, None, (1,), (3,), (1,), False, (0,), 6144),
                  2 * 8 * 6144 * 653 * 4, 2 * (sig.numel() + 8 * 6144 * 653),
                  lambda: F.conv1d(sig, dwk, padding=3, groups=6144)))
    lat = rn(8, 256, 24, 24)
    tw = rn(256, 256, 4, 4, scale=0.05)
    cases.append(("conv_transpose2d [8,256,24,24] 4x4 s4 bf16",
                  lambda: api.conv_transpose2d_batch_invariant(lat, tw, None, (4, 4), (0, 0), (1, 1),
                                                               (0, 0), 1),
                  2 * 8 * 576 * 256 * 4096, 2 * (lat.numel() + tw.numel() + 8 * 256 * 96 * 96),
                  lambda: F.conv_transpose2d(lat, tw, stride=4)))
    # row kernels
    sc = rn(65536, 4096)
    cases.append(("softmax [65536,4096] bf16", lambda: api.softmax(sc, -1), 0, 4 * sc.numel(),
                  lambda: torch.softmax(sc, -1)))
    lm = rn(64, 257152)
    cases.append(("log_softmax [64,257152] bf16", lambda: api.log_softmax(lm, -1), 0, 4 * lm.numel(),
                  lambda: torch.log_softmax(lm, -1)))
    hs = rn(4096, 2048)
    cases.append(("mean dim -1 [4096,2048] bf16", lambda: api.mean_dim(hs, -1), 0,
                  2 * hs.numel() + 2 * 4096, lambda: hs.mean(-1)))
    # VLA (config 5) shapes: head-dim-256 GQA attention of the action expert
    # (8 query heads on one KV head, 50 queries over 354 keys) and the
    # vision tower's head dim 72, both at 128 samples, token-major like the
    # model's projections
    for tag, (bsz, h, hk, lq, lk, d) in (("VLA action expert", (128, 8, 1, 50, 354, 256)),
                                         ("VLA vision tower", (128, 16, 16, 256, 256, 72))):
        aq = rn(bsz, lq, h, d).transpose(1, 2)
        ak, av = rn(bsz, lk, hk, d).transpose(1, 2), rn(bsz, lk, hk, d).transpose(1, 2)
        gq = h != hk
        cases.append((f"sdpa {tag} B={bsz} H{h}/{hk} Lq={lq} Lk={lk} D{d} bf16",
                      lambda q=aq, k=ak, v=av, gq=gq:
                      api.scaled_dot_product_attention_batch_invariant(q, k, v, enable_gqa=gq),
                      4 * bsz * h * lq * lk * d, 2 * (2 * bsz * h * lq * d + 2 * bsz * hk * lk * d),
                      lambda q=aq, k=ak, v=av, gq=gq: F.scaled_dot_product_attention(
                          q, k, v, enable_gqa=gq)))
    # additions (not in the reference): fused normalisations and the fused
    # GeGLU projection, against the stock torch ops they replace
    ln_x, ln_w, ln_b = rn(32768, 1152), rn(1152, scale=0.1) + 1, rn(1152, scale=0.1)
    cases.append(("layer_norm [32768,1152] bf16 (addition)",
                  lambda: api.layer_norm_batch_invariant(ln_x, (1152,), ln_w, ln_b), 0,
                  4 * ln_x.numel(), lambda: F.layer_norm(ln_x, (1152,), ln_w, ln_b)))
    rm_x, rm_w = rn(38912, 2048), rn(2048, scale=0.1) + 1
    cases.append(("rms_norm [38912,2048] bf16 (addition)",
                  lambda: api.rms_norm_batch_invariant(rm_x, (2048,), rm_w, eps=1e-6), 0,
                  4 * rm_x.numel(), lambda: F.rms_norm(rm_x, (2048,), rm_w, 1e-6)))
    gx, gw2 = rn(4864, 2048), rn(2 * 16384, 2048, scale=1 / 45)

    def geglu_stock():
        gate, up = F.linear(gx, gw2).split(16384, dim=-1)
        return F.gelu(gate, approximate="tanh") * up

    cases.append(("gated_linear GeGLU 4864x2048 -> 16384 bf16 (addition)",
                  lambda: api.gated_linear_batch_invariant(gx, gw2),
                  2 * 4864 * 2048 * 2 * 16384, 2 * (gx.numel() + gw2.numel() + 4864 * 16384),
                  geglu_stock))
    vol = rn(8, 1024, 4, 132, 160)
    cases.append(("vector_norm dim 1 [8,1024,4,132,160] bf16",
                  lambda: api.linalg_vector_norm_batch_invariant(vol, dim=1), 0,
                  2 * vol.numel() + 2 * vol.numel() // 1024,
                  lambda: torch.linalg.vector_norm(vol, dim=1)))
    return cases


def _time_op(fn, flush, reps=5):
    import torch

    fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e-3)
    return statistics.median(times)


def run_ops(args) -> None:
    import torch

    dev = torch.device("cuda", 0)
    if args.ops_reference:
        sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
        import batch_invariant_ops as api

        assert "baseline" in api.__file__
    else:
        sys.path.insert(0, str(PKG_ROOT))
        import batch_invariant_ops as api
    flush = _Flusher(dev)
    peaks, _ = _peaks()
    rows = []
    for name, fn, fl, by, stock in _ops_cases(api, dev):
        if args.ops_filter and args.ops_filter not in name:
            continue
        try:
            t = _time_op(fn, flush)
        except Exception as exc:  # the reference may not support a case
            rows.append({"op": name, "error": f"{type(exc).__name__}: {str(exc)[:120]}"})
            continue
        row = {"op": name, "us": round(t * 1e6, 1)}
        if fl:
            row["tflops"] = round(fl / t / 1e12, 1)
        row["gbs"] = round(by / t / 1e9, 1)
        ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
        if fl and fl / by >= ridge:
            row["bound"], row["frac"] = "tensor", round(fl / t / 1e12 / peaks["bf16_tflops"], 3)
        else:
            row["bound"], row["frac"] = "hbm", round(by / t / 1e9 / peaks["hbm_gbs"], 3)
        if stock is not None and not args.ops_reference:
            row["stock_us"] = round(_time_op(stock, flush) * 1e6, 1)
        rows.append(row)
        del fn
    print(json.dumps({"impl": "reference-triton" if args.ops_reference else "ours", "ops": rows}),
          flush=True)


def _vla_inputs(cfg, dev, indices):
    """Per-global-sample synthetic inputs (image ~ U[0,1], ids uniform over the
    vocabulary, noise ~ N(0,1)), seeded by the global sample index so that a
    shard holds exactly the samples the whole batch holds at those rows."""
    import torch

    imgs, ids, noise = [], [], []
    for i in indices:
        g = torch.Generator(device=dev).manual_seed(1000 + i)
        imgs.append(torch.rand(3, cfg.image_size, cfg.image_size, generator=g, device=dev))
        ids.append(torch.randint(0, cfg.vocab, (cfg.text_tokens,), generator=g, device=dev))
        noise.append(torch.randn(cfg.chunk, cfg.action_dim, generator=g, device=dev))
    return torch.stack(imgs), torch.stack(ids), torch.stack(noise)


def vla_sharded(world: int, rank: int, dev, global_batch: int, steps: int, warmup: int) -> dict:
    """Config 5: the random-init pi0-style VLA step with a fixed global batch
    sharded contiguously over the ranks (strong scaling, no collective in the
    step).  Each rank captures its shard's step in a CUDA graph (one capture
    with set_batch_invariant_mode, one stock), replays it ``steps`` times
    between CUDA events, and the max over ranks is the step time.  The
    sharded outputs are then gathered to rank 0 over NCCL and compared bit
    for bit with rank 0's own run of the whole global batch (and, at one GPU,
    with a run of the first sample alone).  Returns the record on rank 0."""
    import torch
    import torch.distributed as dist

    from batch_invariant_ops import set_batch_invariant_mode, sharding
    from batch_invariant_ops.vla import PiZeroStyleVLA, VLAConfig

    cfg = VLAConfig.full()
    model = PiZeroStyleVLA(cfg, dev, seed=0).eval()
    start, end = sharding.shard_range(global_batch, world, rank)
    imgs, ids, noise = _vla_inputs(cfg, dev, range(start, end))
    stream = torch.cuda.current_stream(dev)

    def graphed(mode: bool):
        ctx = set_batch_invariant_mode() if mode else contextlib.nullcontext()
        with torch.inference_mode(), ctx:
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                for _ in range(2):
                    model(imgs, ids, noise)
            stream.wait_stream(side)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                out = model(imgs, ids, noise)
        return graph, out

    def timed(graph) -> float:
        for _ in range(max(warmup, 1)):
            graph.replay()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return sharding.max_over_ranks(e0.elapsed_time(e1) / steps, dev)

    sampler = ClockSampler(dev.index)
    sampler.start()
    graph, out = graphed(True)
    ms_mode = timed(graph)
    clocks = sampler.stop()
    actions, prefix = out["actions"].clone(), out["prefix"].clone()
    del graph, out
    graph, out = graphed(False)
    ms_stock = timed(graph)
    del graph, out
    torch.cuda.empty_cache()

    # verification: gather the shards and compare with one run of the whole batch
    all_actions = sharding.gather_rows(actions, global_batch)
    all_prefix = sharding.gather_rows(prefix, global_batch)
    record = None
    if rank == 0:
        with torch.inference_mode(), set_batch_invariant_mode():
            f_imgs, f_ids, f_noise = _vla_inputs(cfg, dev, range(global_batch))
            whole = model(f_imgs, f_ids, f_noise)
            alone = model(f_imgs[:1], f_ids[:1], f_noise[:1])
        bitwise = bool(torch.equal(all_actions, whole["actions"]) and
                       torch.equal(all_prefix, whole["prefix"]))
        first_alone = bool(torch.equal(alone["actions"], whole["actions"][:1]) and
                           torch.equal(alone["prefix"], whole["prefix"][:1]))
        per_sample = _vla_flops(cfg)
        record = {
            "metric": "pi0-style VLA step samples/s under set_batch_invariant_mode",
            "value": round(global_batch / (ms_mode * 1e-3), 2),
            "unit": "samples/s",
            "n_gpus": world,
            "scaling": "strong",
            "global_batch": global_batch,
            "batch_per_gpu": f"{end - start} (rank 0)",
            "steps": steps,
            "ms_per_step": round(ms_mode, 3),
            "achieved_tflops": round(per_sample * global_batch / (ms_mode * 1e-3) / 1e12, 1),
            "stock_samples_per_s": round(global_batch / (ms_stock * 1e-3), 2),
            "stock_ms_per_step": round(ms_stock, 3),
            "gathered_shards_bitwise_equal_whole_batch_run": bitwise,
            "first_sample_alone_bitwise_equal": first_alone,
            "timing": "each rank replays its shard's step from a CUDA graph between CUDA events; "
                      "max over ranks; stock = the same graph captured with the mode off "
                      "(cuBLAS, flash attention)",
            "config": {"workload": "config5-pi0-style-vla", "vision": "27 x 1152 (SigLIP-like)",
                       "prefix_lm": "18 x 2048, GQA 8/1, head 256, GeGLU 16384",
                       "action_expert": "18 x 1024, 10 flow steps, chunk 50x32",
                       "parallelism": f"dp{world} (global batch sharded, no collective in the "
                                      "step; NCCL gather for verification only)"},
            "clocks": clocks,
        }
    if world > 1:
        dist.barrier()
    del model
    torch.cuda.empty_cache()
    return record


def _extended_cases(dev):
    """(id, kind, ours, stock) for the 54 extended shapes of
    tests/golden/extended_shapes.json (the operator shapes the reference
    benchmarked on real VLA models, research/*/benchmarks.json), with inputs
    built as in tests/test_extended_shapes_gpu.py; stock is the plain torch
    op (None where torch has no direct counterpart: varlen, MoE)."""
    import zlib

    import torch
    import torch.nn.functional as F

    import batch_invariant_ops as bio
    from batch_invariant_ops.batch_invariant_ops import addmm_batch_invariant, mm_batch_invariant

    dt = {"torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16,
          "torch.float32": torch.float32}
    cases = json.loads((ROOT / "tests" / "golden" / "extended_shapes.json").read_text())["cases"]
    for case in cases:
        kind, sh = case["kind"], case["shape"]
        dtype = dt[sh["dtype"]]
        gen = torch.Generator(device=dev).manual_seed(zlib.crc32(case["id"].encode()))

        def rnd(shape, scale=1.0):
            return (torch.randn(*shape, device=dev, generator=gen) * scale).to(dtype)

        ours = stock = None
        if kind in ("mm", "addmm"):
            a, b = rnd(sh["left"]), rnd(sh["right"], sh["right"][-2] ** -0.5)
            if a.ndim == 3:
                b = b[: a.shape[0]] if b.ndim == 3 else b
                ours = lambda a=a, b=b: bio.bmm_persistent(a, b)  # noqa: E731
                stock = lambda a=a, b=b: torch.bmm(a, b)  # noqa: E731
            elif kind == "addmm":
                bias = rnd(sh["bias"], 0.1)
                ours = lambda a=a, b=b, c=bias: addmm_batch_invariant(c, a, b)  # noqa: E731
                stock = lambda a=a, b=b, c=bias: torch.addmm(c, a, b)  # noqa: E731
            else:
                ours = lambda a=a, b=b: mm_batch_invariant(a, b)  # noqa: E731
                stock = lambda a=a, b=b: torch.mm(a, b)  # noqa: E731
        elif kind == "linear":
            x, w = rnd(sh["input"]), rnd(sh["weight"], sh["weight"][1] ** -0.5)
            b = rnd(sh["bias"], 0.1) if sh.get("bias") else None
            ours = lambda x=x, w=w, b=b: bio.linear_batch_invariant(x, w, b)  # noqa: E731
            stock = lambda x=x, w=w, b=b: F.linear(x, w, b)  # noqa: E731
        elif kind == "sdpa":
            q, k, v = rnd(sh["query"]), rnd(sh["key"]), rnd(sh["value"])
            gqa, causal = q.shape[1] != k.shape[1], bool(sh["causal"])
            ours = lambda q=q, k=k, v=v: bio.scaled_dot_product_attention_batch_invariant(  # noqa: E731
                q, k, v, is_causal=causal, enable_gqa=gqa)
            stock = lambda q=q, k=k, v=v: F.scaled_dot_product_attention(  # noqa: E731
                q, k, v, is_causal=causal, enable_gqa=gqa)
        elif kind == "varlen":
            lq, lk = sh["logical_query_length"], sh["logical_kv_length"]
            nseq = max(2, sh["query"][1] // lq)
            q = rnd((1, nseq * lq, sh["query_heads"], sh["head_dim"]))
            k = rnd((1, nseq * lk, sh["kv_heads"], sh["head_dim"]))
            v = rnd((1, nseq * lk, sh["kv_heads"], sh["head_dim"]))
            cq = torch.arange(nseq + 1, device=dev, dtype=torch.int32) * lq
            ck = torch.arange(nseq + 1, device=dev, dtype=torch.int32) * lk
            ours = lambda q=q, k=k, v=v, cq=cq, ck=ck: (  # noqa: E731
                bio.varlen_scaled_dot_product_attention_batch_invariant(
                    q, k, v, cq, ck, is_causal=bool(sh["causal"])))
        elif kind in ("conv", "depthwise_conv1d", "conv_transpose"):
            x, w = rnd(sh["input"]), rnd(sh["weight"], 0.05)
            b = rnd(sh["bias"], 0.1) if sh.get("bias") else None
            nd = x.ndim - 2
            stride = tuple(sh.get("stride", [1] * nd))
            padding = tuple(sh.get("padding", [0] * nd))
            groups = int(sh.get("groups", 1))
            if kind == "conv_transpose":
                fn = {2: bio.conv_transpose2d_batch_invariant, 3: bio.conv_transpose3d_batch_invariant}[nd]
                tfn = {2: F.conv_transpose2d, 3: F.conv_transpose3d}[nd]
                ours = lambda x=x, w=w, b=b: fn(x, w, b, stride, padding, (1,) * nd, (0,) * nd,  # noqa: E731
                                                groups)
            else:
                fn = {1: bio.conv1d_batch_invariant, 2: bio.conv2d_batch_invariant,
                      3: bio.conv3d_batch_invariant}[nd]
                tfn = {1: F.conv1d, 2: F.conv2d, 3: F.conv3d}[nd]
                ours = lambda x=x, w=w, b=b: fn(x, w, b, stride, padding, (1,) * nd, False,  # noqa: E731
                                                (0,) * nd, groups)
            stock = lambda x=x, w=w, b=b: tfn(x, w, b, stride=stride, padding=padding,  # noqa: E731
                                              groups=groups)
        elif kind == "mean":
            x = rnd(sh["input"])
            dim = sh.get("dimension", sh.get("dim"))
            keep = bool(sh.get("keepdim", False))
            ours = lambda x=x: bio.mean_dim(x, dim, keep)  # noqa: E731
            stock = lambda x=x: x.mean(dim, keepdim=keep)  # noqa: E731
        elif kind == "vector_norm":
            x = rnd(sh["input"])
            ours = lambda x=x: bio.linalg_vector_norm_batch_invariant(x, dim=sh["dim"])  # noqa: E731
            stock = lambda x=x: torch.linalg.vector_norm(x, dim=sh["dim"])  # noqa: E731
        elif kind == "moe":
            t, dmodel = sh["hidden"]
            e, topk, inter = sh["experts"], sh["top_k"], sh["intermediate"]
            hid = rnd((t, dmodel))
            gate, up = rnd((e, inter, dmodel), 0.02), rnd((e, inter, dmodel), 0.02)
            down = rnd((e, dmodel, inter), 0.02)
            logits = torch.randn(t, e, device=dev, generator=gen)
            top, sel = torch.topk(logits, topk)
            rw = torch.softmax(top, -1).to(dtype)
            ours = lambda: bio.deterministic_token_choice_moe(hid, rw, sel, gate, up, down)  # noqa: E731
        yield case["id"], kind, sh["dtype"].split(".")[-1], ours, stock


def run_extended(args) -> None:
    """``--extended``: time every extended shape (ours and stock torch, L2
    flushed before each call, CUDA events, median of 5) with the call's
    algorithmic flops / bytes from the library's launch records and the
    roofline fraction against MEASURED_PEAKS.json; the per-model benchmark
    pattern of the reference (scripts/benchmark_batch_invariant_ops.py)."""
    import torch

    from batch_invariant_ops import tracing

    dev = torch.device("cuda", 0)
    flush = _Flusher(dev)
    peaks, _ = _peaks()
    rows = []
    for cid, kind, dtype, ours, stock in _extended_cases(dev):
        ours()
        torch.cuda.synchronize()
        with tracing.record_launches() as rec:
            ours()
        flops = sum(next((v for k, v in r.items() if k.startswith("flops")), 0.0) for r in rec)
        nbytes = sum(r["bytes"] for r in rec)
        t = _time_op(ours, flush)
        row = {"id": cid, "kind": kind, "dtype": dtype, "us": round(t * 1e6, 1),
               "launches": len(rec)}
        if flops:
            row["tflops"] = round(flops / t / 1e12, 1)
        row["gbs"] = round(nbytes / t / 1e9, 1)
        tensor_peak = peaks["bf16_tflops"] if dtype != "float32" else None
        if flops and tensor_peak and flops / max(nbytes, 1) >= tensor_peak * 1e12 / (peaks["hbm_gbs"] * 1e9):
            row["bound"], row["frac"] = "tensor", round(flops / t / 1e12 / tensor_peak, 3)
        else:
            row["bound"], row["frac"] = "hbm", round(nbytes / t / 1e9 / peaks["hbm_gbs"], 3)
        if stock is not None:
            ts = _time_op(stock, flush)
            row["stock_us"] = round(ts * 1e6, 1)
            row["speedup_vs_stock"] = round(ts / t, 3)
        rows.append(row)
        print(json.dumps(row), flush=True)
    print(json.dumps({"extended": len(rows), "impl": "ours"}), flush=True)


def run_vla(args) -> None:
    """``--vla``: only the config-5 VLA step (see vla_sharded)."""
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(PKG_ROOT))
    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    rec = vla_sharded(world, rank, dev, args.vla_global_batch, args.vla_steps, args.warmup)
    if rank == 0:
        print(json.dumps(rec), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _vla_flops(cfg) -> float:
    """Matmul flops of one VLA sample (2 per multiply-add; attention scores
    and values included, elementwise work excluded)."""
    p_img = (cfg.image_size // cfg.patch) ** 2
    t_pre = p_img + cfg.text_tokens
    hd = cfg.lm_head_dim
    qkv = (cfg.lm_heads + 2 * cfg.lm_kv_heads) * hd
    vis = p_img * 3 * cfg.patch * cfg.patch * cfg.vis_width + cfg.vis_layers * (
        p_img * (4 * cfg.vis_width ** 2 + 2 * cfg.vis_width * cfg.vis_mlp)
        + 2 * p_img * p_img * cfg.vis_width)
    vis += p_img * cfg.vis_width * cfg.lm_width
    lm = cfg.lm_layers * (t_pre * (cfg.lm_width * qkv + cfg.lm_heads * hd * cfg.lm_width
                                   + 3 * cfg.lm_width * cfg.lm_mlp)
                          + 2 * t_pre * t_pre * cfg.lm_heads * hd)
    t_act, t_kv = cfg.chunk, cfg.chunk + t_pre
    act = cfg.flow_steps * (
        t_act * (cfg.action_dim + cfg.act_width) * cfg.act_width
        + cfg.act_layers * (t_act * (cfg.act_width * qkv + cfg.lm_heads * hd * cfg.act_width
                                     + 3 * cfg.act_width * cfg.act_mlp)
                            + 2 * t_act * t_kv * cfg.lm_heads * hd)
        + t_act * cfg.act_width * cfg.action_dim)
    return 2.0 * (vis + lm + act)


def run_profile_point(args) -> None:
    """Minimal launch sequence for ncu captures: one GEMM point (MxN) or one
    attention shape (attn:B,S,causal), 1 + steps launches."""
    import torch

    sys.path.insert(0, str(PKG_ROOT))
    from batch_invariant_ops import linear_batch_invariant, scaled_dot_product_attention_batch_invariant

    if args.profile_point.startswith("gated:"):
        # fused GeGLU GEMM and the plain GEMM of the same operands, per round
        from batch_invariant_ops import gated_linear_batch_invariant

        m, f, k = (int(v) for v in args.profile_point[6:].split("x"))
        dev = torch.device("cuda", 0)
        gen = torch.Generator(device=dev).manual_seed(0)
        x = torch.randn(m, k, device=dev, generator=gen).to(torch.bfloat16)
        w = (torch.randn(2 * f, k, device=dev, generator=gen) / math.sqrt(k)).to(torch.bfloat16)
        for _ in range(1 + args.steps):
            y = gated_linear_batch_invariant(x, w)
            linear_batch_invariant(x, w)
        torch.cuda.synchronize()
        print(json.dumps({"profile_point": args.profile_point, "launches": 2 * (1 + args.steps),
                          "checksum": float(y.float().sum().item())}))
        return
    if args.profile_point.startswith("attn:"):
        bsz, seq, causal = (int(v) for v in args.profile_point[5:].split(","))
        dev = torch.device("cuda", 0)
        gen = torch.Generator(device=dev).manual_seed(0)
        q = torch.randn(bsz, 16, seq, 128, device=dev, generator=gen).to(torch.bfloat16)
        k = torch.randn(bsz, 4, seq, 128, device=dev, generator=gen).to(torch.bfloat16)
        v = torch.randn(bsz, 4, seq, 128, device=dev, generator=gen).to(torch.bfloat16)
        for _ in range(1 + args.steps):
            y = scaled_dot_product_attention_batch_invariant(q, k, v, is_causal=bool(causal),
                                                             enable_gqa=True)
        torch.cuda.synchronize()
        print(json.dumps({"profile_point": args.profile_point, "launches": 1 + args.steps,
                          "checksum": float(y.float().sum().item())}))
        return
    # MxN (K = 4096, library tile) or MxNxK@TMxTN (explicit output tile)
    spec, _, tile = args.profile_point.partition("@")
    dims = [int(v) for v in spec.split("x")]
    m, n = dims[0], dims[1]
    k = dims[2] if len(dims) > 2 else K
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(m, k, device=dev, generator=gen).to(torch.bfloat16)
    w = (torch.randn(n, k, device=dev, generator=gen) / 64).to(torch.bfloat16)
    b = (torch.randn(n, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
    if tile:
        from batch_invariant_ops import _gemm

        t = tuple(int(v) for v in tile.split("x"))
        for _ in range(1 + args.steps):
            y = _gemm.mm(x, w.t(), b, tile=t)
    else:
        for _ in range(1 + args.steps):
            y = linear_batch_invariant(x, w, b)
    torch.cuda.synchronize()
    print(json.dumps({"profile_point": args.profile_point, "launches": 1 + args.steps,
                      "checksum": float(y.float().sum().item())}))


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--cpu-budget", type=float, default=20.0)
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-triton-ref", action="store_true")
    parser.add_argument("--triton-ref-worker", action="store_true", help=argparse.SUPPRESS)
    parser.add_argument("--profile-point", default=None, help="MxN: run one GEMM point (for ncu)")
    parser.add_argument("--ops", action="store_true", help="per-operator roofline table")
    parser.add_argument("--extended", action="store_true",
                        help="time the 54 extended VLA operator shapes (ours vs stock)")
    parser.add_argument("--vla", action="store_true",
                        help="config 5: pi0-style VLA step samples/s under the mode")
    parser.add_argument("--vla-global-batch", type=int, default=256,
                        help="VLA samples per step over all GPUs (sharded)")
    parser.add_argument("--vla-steps", type=int, default=3, help="timed VLA graph replays")
    parser.add_argument("--no-vla", action="store_true", help="skip the VLA step in the default run")
    parser.add_argument("--ops-filter", default="", help="only --ops cases whose name has this")
    parser.add_argument("--ops-reference", action="store_true",
                        help="with --ops: time the reference package from baseline/_ref")
    args = parser.parse_args()
    if args.vla:
        run_vla(args)
    elif args.extended:
        sys.path.insert(0, str(PKG_ROOT))
        run_extended(args)
    elif args.ops:
        run_ops(args)
    elif args.profile_point:
        run_profile_point(args)
    elif args.triton_ref_worker:
        run_triton_ref_worker(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
