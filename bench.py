#!/usr/bin/env python3
"""Benchmark of the tierk frozen-weight linear path on B200.

Default workload (the metric's single-GPU configuration):
  Q4_K weight W[14336, 4096] (SwiGLU up-proj), X bf16 [4096, 4096], dY bf16
  [4096, 14336]; one step = forward Y = X.W^T plus input gradient dX = dY.W,
  both through the C ABI (tk_linear_fwd / tk_linear_dx): bit-exact dequant of
  W to fp16, activation conversion, tcgen05 GEMM with fp32 accumulation.
  Useful work per step: 2 x 2*M*N*K = 962.1 GFLOP.

Multi-GPU (torchrun, one process per GPU, NCCL): W is split by output rows;
each rank computes its Y columns and its partial
dX; Y shards are all-gathered and dX partials all-reduced inside the step.
Total work is fixed (strong scaling); value = total FLOP / max-over-ranks time.

--impl reference: the reference's CPU implementation of the same operation
(its quant.h q_val dequant compiled from its sources in oracle/_ref, with the
cpu_gemm_fwd/cpu_gemm_dx loop structure), timed on this host's cores on a
bounded sample of the workload (a slice of weight rows), rank 0 only.

Data: synthetic, seeded (tests/gen.py); no dataset exists for this path.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

METRIC = "dequant/x3 GEMM TFLOP/s + decode GEMV HBM GB/s (% B200 peak) at 1/2/4/8 GPU"
M_TOK, N_OUT, K_IN = 4096, 14336, 4096
FLOP_DIR = 2.0 * M_TOK * N_OUT * K_IN            # one direction (fwd or dX)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None

    def stop(self):
        if not self.p:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        out, _ = self.p.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def make_inputs(seed=1):
    import numpy as np
    from gen import q4_k_blocks
    rng = np.random.default_rng(seed)
    Wq = q4_k_blocks(rng, N_OUT, K_IN)
    X = rng.standard_normal((M_TOK, K_IN), dtype=np.float32)
    dY = rng.standard_normal((M_TOK, N_OUT), dtype=np.float32)
    return Wq, X, dY


# ---------------------------------------------------------------------------
def run_reference(args):
    """The reference's CPU path on a bounded sample (rank 0 only)."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    import numpy as np
    from oracle.oracle import RefOracle, Oracle
    threads = os.cpu_count() or 1
    Wq, X, dY = make_inputs()
    kind = "reference" if RefOracle.available() else "port"
    eng = RefOracle() if kind == "reference" else None
    if eng is None:
        return print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref not built and no port timing"}))
    per_step = min(args.ref_seconds, 150.0 / (args.steps + args.warmup))   # whole run within a few minutes
    rows = calibrate_rows(eng, Wq, X, dY, threads, target_s=per_step)
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        eng.qgemm_fwd(Wq, 12, 0, rows, K_IN, X, threads)
        eng.qgemm_dx(Wq, 12, 0, rows, K_IN, dY[:, :rows], threads)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
    t = statistics.median(times)
    flop = 2 * 2.0 * M_TOK * rows * K_IN
    v = flop / t / 1e12
    sample = (f"Q4_K rows 0..{rows} of {N_OUT} (K={K_IN}), M={M_TOK} fp32 tokens, fwd+dX per step; "
              f"reference quant.h q_val + cpu_gemm_fwd/dx loop structure, {threads} threads")
    line = {"metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, tests/gen.py)", "impl": "reference",
            "config": {"workload": "C2 Q4_K 14336x4096 fwd+dX, M=4096 (sampled rows)", "rows_sampled": rows},
            "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def calibrate_rows(eng, Wq, X, dY, threads, target_s):
    rows = 16
    t0 = time.perf_counter()
    eng.qgemm_fwd(Wq, 12, 0, rows, K_IN, X, threads)
    eng.qgemm_dx(Wq, 12, 0, rows, K_IN, dY[:, :rows], threads)
    dt = max(time.perf_counter() - t0, 1e-3)
    want = int(rows * target_s / dt) // 16 * 16
    return max(16, min(N_OUT, want))


def cpu_baseline(Wq, X, dY, seconds):
    from oracle.oracle import RefOracle
    threads = os.cpu_count() or 1
    if not RefOracle.available():
        return None
    eng = RefOracle()
    rows = calibrate_rows(eng, Wq, X, dY, threads, target_s=seconds)
    t0 = time.perf_counter()
    eng.qgemm_fwd(Wq, 12, 0, rows, K_IN, X, threads)
    eng.qgemm_dx(Wq, 12, 0, rows, K_IN, dY[:, :rows], threads)
    t = time.perf_counter() - t0
    v = 2 * 2.0 * M_TOK * rows * K_IN / t / 1e12
    return {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "reference",
            "sample": f"Q4_K rows 0..{rows} of {N_OUT}, M={M_TOK}, fwd+dX, one pass ({t:.1f} s); reference quant.h "
                      f"q_val row expansion + cpu_gemm_fwd/dx loop structure on {threads} threads"}


# ---------------------------------------------------------------------------
def run_ours(args):
    import numpy as np
    import torch

    import tier_b200 as tk
    from tier_b200.host import shard_rows

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    group = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        group = dist.group.WORLD
    ctx = tk.Context(local)
    Wq, X, dY = make_inputs()
    r0, r1 = shard_rows(N_OUT, world, rank)
    n_loc = r1 - r0
    dev = torch.device("cuda", local)
    Wd = torch.from_numpy(Wq[r0:r1].copy()).to(dev)
    w = tk.make_weight(tk.Q4_K, n_loc, K_IN, Wd)
    Xb = torch.from_numpy(X).to(torch.bfloat16)
    dYb = torch.from_numpy(np.ascontiguousarray(dY[:, r0:r1])).to(torch.bfloat16)
    Xd, dYd = Xb.to(dev), dYb.to(dev)
    Y = torch.empty(M_TOK, n_loc, dtype=torch.float32, device=dev)
    dX = torch.empty(M_TOK, K_IN, dtype=torch.float32, device=dev)
    Yfull = torch.empty(world, M_TOK, n_loc, dtype=torch.float32, device=dev) if world > 1 else None
    stream = torch.cuda.current_stream(dev)

    def step(Xin, dYin):
        ctx.linear(w, Xin, M_TOK, Y, x_dtype=tk.DT_BF16)
        ctx.linear_dx(w, dYin, M_TOK, dX, dy_dtype=tk.DT_BF16)
        if world > 1:
            import torch.distributed as dist
            dist.all_gather_into_tensor(Yfull, Y, group=group)
            dist.all_reduce(dX, group=group)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier(group=group)
        torch.cuda.synchronize(dev)

    # ---- device-resident timing ----
    # Clocks are sampled from before the warm-up to after the timed steps; the
    # warm-up is extended to >= 1 s of load so the 100 ms samples see the GPU busy.
    clocks = Clocks(local)
    clocks.start()
    t0 = time.perf_counter()
    for _ in range(args.warmup):
        step(Xd, dYd)
    barrier()
    while time.perf_counter() - t0 < 1.0:
        for _ in range(10):
            step(Xd, dYd)
        barrier()
    n0 = ctx.launches()
    ctx.profile(True)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev0.record(stream)
    for _ in range(args.steps):
        step(Xd, dYd)
    ev1.record(stream)
    barrier()
    t_ms = ev0.elapsed_time(ev1)
    gemm_ms, gemm_n = ctx.profile_read(tk.PROF_GEMM)
    deq_ms, deq_n = ctx.profile_read(tk.PROF_DEQUANT)
    spl_ms, spl_n = ctx.profile_read(tk.PROF_SPLIT)
    ctx.profile(False)
    launches = ctx.launches() - n0
    clk = clocks.stop()
    t_max = t_ms
    if world > 1:
        import torch.distributed as dist
        tt = torch.tensor([t_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX, group=group)
        t_max = float(tt.item())
    ms_step = t_max / args.steps
    flop_step = 2 * FLOP_DIR
    value = flop_step / (ms_step * 1e-3) / 1e12

    # ---- end to end through the C ABI with host buffers ----
    Xh = Xb.pin_memory()
    dYh = dYb.pin_memory()
    Yh = torch.empty(M_TOK, n_loc, dtype=torch.float32).pin_memory()
    dXh = torch.empty(M_TOK, K_IN, dtype=torch.float32).pin_memory()
    Xs = torch.empty_like(Xd)
    dYs = torch.empty_like(dYd)

    def e2e_step():
        Xs.copy_(Xh, non_blocking=True)
        dYs.copy_(dYh, non_blocking=True)
        step(Xs, dYs)
        Yh.copy_(Y, non_blocking=True)
        dXh.copy_(dX, non_blocking=True)

    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    barrier()
    e_steps = max(2, args.steps // 4)
    ev0.record(stream)
    for _ in range(e_steps):
        e2e_step()
    ev1.record(stream)
    barrier()
    te = ev0.elapsed_time(ev1)
    if world > 1:
        import torch.distributed as dist
        tt = torch.tensor([te], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX, group=group)
        te = float(tt.item())
    e2e_val = flop_step / (te / e_steps * 1e-3) / 1e12
    h2d = Xh.numel() * 2 + dYh.numel() * 2
    d2h = Yh.numel() * 4 + dXh.numel() * 4

    if rank == 0:
        hbm, tf_burst, tf_sus, src = peaks()
        gemm_avg_ms = gemm_ms / max(gemm_n, 1)
        gemm_flop_launch = flop_step / 2 / world      # one direction on this rank's rows
        achieved = gemm_flop_launch / (gemm_avg_ms * 1e-3) / 1e12
        traffic = None   # dram read+write bytes per GEMM launch from the committed ncu summary
        tf = ROOT / "profiles" / "gemm_tc_kernel_c2_q4k_m4096.md"
        if tf.exists():
            for ln in tf.read_text().splitlines():
                if ln.startswith("traffic_bytes_per_launch:"):
                    traffic = float(ln.split(":")[1].split()[0])
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp16 tensor-core products, fp32 accumulate (Q4_K -> fp16 exact dequant)",
            "data": "synthetic (seeded, tests/gen.py)",
            "config": {"workload": "C2 Q4_K 14336x4096, M=4096 tokens, fwd + dX per step",
                       "x_dtype": "bf16", "partition": f"W rows split over {world} GPU(s)" if world > 1 else "1 GPU",
                       "l2": "working set per step ~0.5 GB > 126 MB L2 (no explicit flush)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tf_burst, "unit": "TFLOP/s",
                         "frac": achieved / tf_burst, "traffic": traffic,
                         "kernel": "gemm_tc_kernel", "peak_source": f"{src} bf16 burst (MEASURED_PEAKS.json)",
                         "sustained_peak": tf_sus},
            "kernels_ms_per_step": {"gemm": gemm_ms / args.steps, "dequant": deq_ms / args.steps,
                                    "act_split": spl_ms / args.steps},
            "e2e": {"value": e2e_val, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "clocks": clk,
        }
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = cpu_baseline(Wq, X, dY, args.ref_seconds)
        print(json.dumps(line))
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-seconds", type=float, default=10.0, help="CPU baseline sample size (seconds)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
