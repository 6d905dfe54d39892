#!/usr/bin/env python3
"""Benchmark of the tierk frozen-weight linear path on B200.

Default workload (the metric's single-GPU configuration):
  Q4_K weight W[14336, 4096] (SwiGLU up-proj), X bf16 [4096, 4096], dY bf16
  [4096, 14336]; one step = forward Y = X.W^T plus input gradient dX = dY.W,
  both through the C ABI in one call (tk_linear_fwd_dx; --step-call separate:
  tk_linear_fwd then tk_linear_dx): bit-exact dequant of W to fp16 once,
  activation conversion, one tcgen05 GEMM launch for both products with fp32
  accumulation.  Useful work per step: 2 x 2*M*N*K = 962.1 GFLOP.

Multi-GPU (torchrun, one process per GPU): W is split by output rows; each
rank computes its Y columns (kept sharded, as a column-parallel layer's
consumer takes them; --gather-y all-gathers the full Y) and its partial dX,
whose tiles the GEMM stores into the owner rank's memory over NVLink
(tk_linear_fwd_dx_rs; --dx-mode chooses NCCL variants or the dY reshard).
Total work is fixed (strong scaling); value = total FLOP / max-over-ranks time.
Timing: CUDA events around the timed steps, max over ranks; per-launch events
(kernel breakdown, roofline) on one timed step in four.

--impl reference: the reference's CPU implementation of the same operation
(the engine's own cpu_gemm_fwd / cpu_gemm_dx and thread pool, extracted and
compiled from its sources into oracle/_ref, over its quant.h q_val rows
rounded to bf16), timed on this host's cores on a bounded sample of the
workload (a slice of weight rows), rank 0 only; gguf-py + numpy (the
reference test's oracle) is timed beside it.

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
PROF_EVERY = 4          # timed steps per step with per-launch events
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

METRIC = "dequant/x3 GEMM TFLOP/s + decode GEMV HBM GB/s (% B200 peak) at 1/2/4/8 GPU"
M_TOK, N_OUT, K_IN = 4096, 14336, 4096
FLOP_DIR = 2.0 * M_TOK * N_OUT * K_IN            # one direction (fwd or dX)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained") or d["bf16_tflops"], "measured"
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
class RefCPU:
    """The reference's CPU path for one sampled slice of the C2 step.

    engine (kind "reference"): the reference engine's own CPU GEMMs,
      cpu_gemm_fwd / cpu_gemm_dx with the thread pool they run on
      (tier/tier.cpp:1015-1099, AVX2 FMA over bf16 weight rows), extracted and
      compiled from the reference's sources into oracle/_ref/libtkref.so, fed
      the reference's q_val expansion (tier/quant.h:59-121) of the sampled
      weight rows rounded to bf16 -- the expansion is inside every step.
    numpy (the reference test's oracle, tier/check_quant.py:71): gguf-py's
      quants.dequantize of the sampled rows, then numpy float32 matmuls (BLAS
      threads = all cores)."""

    def __init__(self, threads):
        from oracle.oracle import RefOracle
        self.threads = threads
        self.eng = RefOracle()
        self.eng.engine_pool(threads)

    @staticmethod
    def available() -> bool:
        from oracle.oracle import RefOracle
        return RefOracle.available()

    def prepare(self, Wq, X, dY, rows):
        import numpy as np
        self.rows = rows
        self.Wq = Wq
        self.X = X
        self.dY = np.ascontiguousarray(dY[:, :rows])
        self.Wb = np.empty((rows, K_IN), np.uint16)
        self.Y = np.empty((M_TOK, rows), np.float32)
        self.dX = np.empty((M_TOK, K_IN), np.float32)

    def step(self):
        self.eng.dequant_bf16(self.Wq, 12, 0, self.rows, K_IN, out=self.Wb)
        self.eng.cpu_gemm_fwd(self.X, self.Wb, out=self.Y)
        self.eng.cpu_gemm_dx(self.dY, self.Wb, out=self.dX)

    def calibrate(self, Wq, X, dY, target_s):
        """Rows of the workload whose step takes about target_s on the host.
        Probes grow (at most 8x at a time) until one takes a quarter of the
        target; the run is sized from it."""
        rows = 64
        self.prepare(Wq, X, dY, rows)
        self.step()           # pool start-up and the GEMMs' first-touch of their buffers, untimed
        while True:
            self.prepare(Wq, X, dY, rows)
            t0 = time.perf_counter()
            self.step()
            dt = max(time.perf_counter() - t0, 1e-3)
            want = max(16, min(N_OUT, int(rows * target_s / dt) // 16 * 16))
            if dt >= target_s / 4 or rows == N_OUT:
                return want
            rows = max(16, min(N_OUT, want, rows * 8))

    def sample_text(self, rows):
        return (f"Q4_K rows 0..{rows} of {N_OUT} (K={K_IN}), M={M_TOK} fp32 tokens, fwd + dX per step: the "
                f"reference engine's cpu_gemm_fwd / cpu_gemm_dx (tier/tier.cpp:1015-1099, extracted, AVX2) on "
                f"its q_val rows rounded to bf16, {self.threads} pool threads; rate scaled to the unit by FLOPs")


def numpy_baseline(Wq, X, dY, seconds):
    """gguf-py dequantize + numpy matmuls on a row sample sized to ~seconds."""
    import numpy as np
    try:
        from gguf import GGMLQuantizationType, quants
        import gguf
    except ImportError:
        return None
    rows = 64
    while True:
        t0 = time.perf_counter()
        W = quants.dequantize(Wq[:rows], GGMLQuantizationType.Q4_K)
        Y = X @ W.T
        dX = np.ascontiguousarray(dY[:, :rows]) @ W
        dt = time.perf_counter() - t0
        if dt >= seconds / 4 or rows >= N_OUT:
            break
        rows = min(N_OUT, rows * 4)
    v = 2 * 2.0 * M_TOK * rows * K_IN / dt / 1e12
    del Y, dX
    return {"value": v, "unit": "TFLOP/s", "cores": os.cpu_count() or 1, "kind": "reference-test oracle",
            "sample": f"Q4_K rows 0..{rows} of {N_OUT}, M={M_TOK}: gguf-py {getattr(gguf, '__version__', '?')} "
                      f"quants.dequantize + numpy float32 X.W^T and dY.W (tier/check_quant.py:71), one pass "
                      f"({dt:.1f} s)"}


def reference_gpu(steps=5):
    """The reference engine's own GPU path on this box (oracle/ref_gpu.cu:
    tier.cpp compiled whole with cuBLAS / cuBLASLt, as its build.sh does),
    on the configurations the repository's arm measures:
      C1  gemv_q, q8_0 4096x4096 and 14336x4096, one token (as chat_lin
          launches it), rotating weight copies over 4x the L2;
      C3  fp3gemm (split3_fp_k + three cuBLASLt GEMMs) forward + dX of the
          seven 12B-class projections, fp16 W, fp32 X, M = 4096;
      C2  the training path for a Q4_K weight: dq_launch to fp16, then
          fp3gemm forward and dX on fp32 X / dY (the engine's activations are
          fp32), M = 4096.
    Every record carries an fp64 check of its output.  CUDA events on the
    legacy default stream, which the reference launches on."""
    import numpy as np
    import torch
    from oracle.oracle import RefGPU
    from gen import blocks_for
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    if not RefGPU.available():
        return {"unavailable": "oracle/_ref/libtierref_gpu.so not built (reference tree absent at build time)"}
    ref = RefGPU()
    hbm, tf_burst = peaks()[0], peaks()[1]
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn, n):
        fn()
        ref.sync()
        ev0.record()
        for _ in range(n):
            fn()
        ev1.record()
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1) / n

    out = {}
    rng = np.random.default_rng(0)
    for (N, K) in ((4096, 4096), (14336, 4096)):
        b = blocks_for(rng, 8, N, K)
        rb = b.shape[1]
        copies = int(np.ceil(4 * 126e6 / b.nbytes))
        W = torch.from_numpy(b).cuda()
        pool = [W.clone() for _ in range(copies)]
        x = torch.from_numpy(rng.standard_normal(K).astype(np.float32)).cuda()
        y = torch.empty(N, device="cuda")
        ref.gemv_q(W, 8, rb, x, y, N, K)
        ref.sync()
        Wd = torch.from_numpy(np.ascontiguousarray(b)).cuda()
        W16 = torch.empty(N, K, dtype=torch.float16, device="cuda")
        ref.dequant_f16(Wd, 8, rb, N, K, W16)
        ref.sync()
        want = W16.double() @ x.double()
        err = float((y.double() - want).norm() / want.norm())

        def run():
            for w in pool:
                ref.gemv_q(w, 8, rb, x, y, N, K)
        ms = timed(run, max(2, steps)) / copies
        gbs = (b.nbytes + 4 * (N + K)) / (ms * 1e-3) / 1e9
        out[f"gemv_q q8_0 {N}x{K} M=1"] = {"us_per_launch": ms * 1e3, "GB_s": gbs, "frac_of_hbm": gbs / hbm,
                                           "check_rel_err": err}
        del pool, W, Wd, W16
    # C3: seven projections, fp3gemm fwd + dX
    M, H, I = 4096, 5120, 14336
    shapes = [(4096, H), (1024, H), (1024, H), (H, 4096), (I, H), (I, H), (H, I)]
    g = torch.Generator(device="cuda").manual_seed(2)
    Ws, xs, dys = [], {}, []
    for (n, k) in shapes:
        Ws.append((torch.randn(n, k, device="cuda", generator=g) * 0.02).half())
        if k not in xs:
            xs[k] = torch.randn(M, k, device="cuda", generator=g)
        dys.append(torch.randn(M, n, device="cuda", generator=g))
    ys = [torch.empty(M, n, device="cuda") for n, _ in shapes]
    dxs = [torch.empty(M, k, device="cuda") for _, k in shapes]

    def c3():
        for W16, (n, k), y, dy, dx in zip(Ws, shapes, ys, dys, dxs):
            ref.fp3gemm_fwd(W16, xs[k], y, M, k, n)
            ref.fp3gemm_dx(W16, dy, dx, M, k, n)
    ms = timed(c3, steps)
    want = xs[H][1].double() @ Ws[0].double().T
    err = float((ys[0][1].double() - want).norm() / want.norm())
    useful = 2 * 2.0 * M * sum(n * k for n, k in shapes)
    out["C3 fp3gemm 12B layer fwd+dX"] = {"ms_per_step": ms, "tflops_useful": useful / (ms * 1e-3) / 1e12,
                                          "tflops_executed": 3 * useful / (ms * 1e-3) / 1e12,
                                          "frac_of_bf16_burst_executed": 3 * useful / (ms * 1e-3) / 1e12 / tf_burst,
                                          "check_rel_err": err}
    del Ws, xs, dys, ys, dxs
    # C2 the reference's way: dq_k to fp16 + fp3gemm on fp32 activations
    Wq, X, dY = make_inputs()
    Wd = torch.from_numpy(Wq).cuda()
    W16 = torch.empty(N_OUT, K_IN, dtype=torch.float16, device="cuda")
    Xd = torch.from_numpy(X).cuda()
    dYd = torch.from_numpy(dY).cuda()
    Y = torch.empty(M_TOK, N_OUT, device="cuda")
    dX = torch.empty(M_TOK, K_IN, device="cuda")

    def c2():
        ref.dequant_f16(Wd, 12, Wq.shape[1], N_OUT, K_IN, W16)
        ref.fp3gemm_fwd(W16, Xd, Y, M_TOK, K_IN, N_OUT)
        ref.fp3gemm_dx(W16, dYd, dX, M_TOK, K_IN, N_OUT)
    ms = timed(c2, steps)
    want = Xd[7].double() @ W16.double().T
    err = float((Y[7].double() - want).norm() / want.norm())
    out["C2 Q4_K fp32 activations: dq_k + fp3gemm fwd+dX"] = {
        "ms_per_step": ms, "tflops_useful": 2 * FLOP_DIR / (ms * 1e-3) / 1e12, "check_rel_err": err}
    del Wd, W16, Xd, dYd, Y, dX
    torch.cuda.empty_cache()
    return out


def run_reference(args):
    """The reference's CPU path on a bounded sample (rank 0 only)."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    if not RefCPU.available():
        return print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref (the reference's CPU code built "
                                                                     "from its sources) is not present"}))
    Wq, X, dY = make_inputs()
    ref = RefCPU(threads)
    per_step = min(args.ref_seconds, 120.0 / (args.steps + args.warmup))   # whole run within a few minutes
    rows = ref.calibrate(Wq, X, dY, target_s=per_step)
    ref.prepare(Wq, X, dY, rows)
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        ref.step()
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
    t = statistics.median(times)
    flop = 2 * 2.0 * M_TOK * rows * K_IN
    v = flop / t / 1e12
    line = {"metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32 (bf16 weights)", "data": "synthetic (seeded, tests/gen.py)",
            "impl": "reference",
            "config": {"workload": "C2 Q4_K 14336x4096 fwd+dX, M=4096 (sampled weight rows)", "rows_sampled": rows},
            "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "reference",
                             "sample": ref.sample_text(rows)},
            "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "numpy_baseline": numpy_baseline(Wq, X, dY, 8.0)}
    if not args.no_extra:
        try:
            line["reference_gpu"] = reference_gpu()
        except Exception as e:            # the CPU arm stands on its own
            line["reference_gpu"] = {"unavailable": f"{type(e).__name__}: {e}"}
    print(json.dumps(line))


def cpu_baseline(Wq, X, dY, seconds):
    threads = os.cpu_count() or 1
    if not RefCPU.available():
        return None
    ref = RefCPU(threads)
    rows = ref.calibrate(Wq, X, dY, target_s=seconds)
    ref.prepare(Wq, X, dY, rows)
    t0 = time.perf_counter()
    ref.step()
    t = time.perf_counter() - t0
    v = 2 * 2.0 * M_TOK * rows * K_IN / t / 1e12
    return {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "reference",
            "sample": ref.sample_text(rows) + f"; one pass ({t:.1f} s)"}


CHECK_TOL = 2e-3        # the stated bound of the bf16-activation quant GEMM (relative, vs fp64)


def check_outputs(ctx, Wq, Xb, dY, Y, r0, r1, dX_part, dx_row0, dev, group):
    """Sampled rows of this rank's timed outputs against fp64.

    The reference weight is the library's own fp32 expansion of the whole
    Q4_K matrix (tk_dequant, which the tests pin bit for bit to the
    reference's q_val); the products are fp64 matmuls of the same bf16
    inputs.  Y rows cover this rank's output columns [r0, r1); dX rows are
    the token rows this rank holds (dx_row0 onwards: its reduce-scatter shard,
    or the whole matrix on one GPU).  The worst per-row relative error over
    all ranks is returned with the bound it is held to."""
    import numpy as np
    import torch
    import tier_b200 as tk
    Wfull = torch.from_numpy(Wq).to(dev)
    W32 = torch.empty(N_OUT, K_IN, dtype=torch.float32, device=dev)
    ctx.dequant(tk.Q4_K, Wfull, N_OUT, K_IN, W32)
    torch.cuda.synchronize(dev)
    W64 = W32.double()
    m_loc = dX_part.shape[0]
    rows_y = sorted({0, 1, 255, 256, M_TOK // 2 + 7, M_TOK - 1})
    rows_dx = sorted({0, 255, 256, m_loc // 2 + 3, m_loc - 1})
    errs = []
    Xr = Xb[rows_y].double().to(dev)
    want = Xr @ W64[r0:r1].T
    got = Y[rows_y].double()
    errs += ((got - want).norm(dim=1) / want.norm(dim=1)).tolist()
    g_rows = [dx_row0 + r for r in rows_dx]
    dYr = torch.from_numpy(np.ascontiguousarray(dY[g_rows])).to(torch.bfloat16).double().to(dev)
    want = dYr @ W64
    got = dX_part[rows_dx].double()
    errs += ((got - want).norm(dim=1) / want.norm(dim=1)).tolist()
    e = torch.tensor([max(errs)], dtype=torch.float64, device=dev)
    bad = torch.tensor([0 if all(np.isfinite(errs)) else 1], device=dev)
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(e, op=dist.ReduceOp.MAX, group=group)
        dist.all_reduce(bad, op=dist.ReduceOp.MAX, group=group)
    del Wfull, W32, W64
    err = float(e.item())
    return {"rel_err": err, "tol": CHECK_TOL, "ok": bool(err < CHECK_TOL and not int(bad.item())),
            "rows": {"y": rows_y, "dx_local": rows_dx},
            "against": "fp64 matmul of the same bf16 inputs and tk_dequant's fp32 W (bit-exact to q_val in "
                       "tests/test_gpu_fullsize.py); worst per-row relative L2 error over all ranks"}


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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
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
    Yfull = torch.empty(world, M_TOK, n_loc, dtype=torch.float32, device=dev) if (world > 1 and args.gather_y) else None
    stream = torch.cuda.current_stream(dev)

    chunks = args.dx_chunks if world > 1 else 1
    mc = M_TOK // chunks
    dx_mode = args.dx_mode if world > 1 else "local"
    dXr = None
    if dx_mode in ("fused", "rs-nccl", "reshard"):
        dXr = torch.empty(M_TOK // world, K_IN, dtype=torch.float32, device=dev)
    w_full = dYrows = side = None
    if dx_mode == "reshard":
        # the frozen weight is held whole by every rank (33 MB of Q4_K); the
        # forward still uses this rank's rows of it (a view), and the dX GEMM
        # takes this rank's token rows of dY against the whole weight
        Wfull_d = torch.from_numpy(Wq).to(dev)
        w_full = tk.make_weight(tk.Q4_K, N_OUT, K_IN, Wfull_d)
        w = tk.make_weight(tk.Q4_K, n_loc, K_IN, Wfull_d[r0:r1])
        dYrows = torch.empty(M_TOK // world, N_OUT, dtype=torch.bfloat16, device=dev)
        side = torch.cuda.Stream(dev)
    if dx_mode in ("fused", "reshard"):
        # peer buffers for the reduce-scatter inside the dX GEMM: exchange the
        # IPC handles once, outside the timed region.  If any rank cannot map
        # its peers, every rank falls back to GEMM + NCCL reduce-scatter.
        import torch.distributed as dist
        ok = torch.ones(1, dtype=torch.int32, device=dev)
        h = b"\0" * tk.IPC_HANDLE_BYTES
        try:
            h = ctx.comm_init(rank, world, M_TOK * K_IN * 4)
        except tk.TierkError:
            ok.zero_()
        mine = torch.tensor(list(h), dtype=torch.uint8, device=dev)
        allh = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allh, mine, group=group)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if int(ok.item()):
            try:
                ctx.comm_connect(bytes(torch.cat(allh).cpu().tolist()))
            except tk.TierkError:
                ok.zero_()
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if not int(ok.item()):
            if dx_mode == "reshard":
                raise SystemExit("--dx-mode reshard: the peer buffers could not be set up")
            dx_mode = "rs-nccl"
        dist.barrier(group=group)

    pair = args.step_call == "pair"

    def step(Xin, dYin, Yo=None, dXo=None):
        if dx_mode == "reshard":
            # dY's column shards become token-row shards over NVLink on a side
            # stream while the forward GEMM runs; then the local dX GEMM
            side.wait_stream(torch.cuda.current_stream(dev))
            ctx.reshard_cols_send(dYin, stream=side)
            ctx.linear(w, Xin, M_TOK, Y if Yo is None else Yo, x_dtype=tk.DT_BF16)
            torch.cuda.current_stream(dev).wait_stream(side)
            ctx.reshard_cols_recv(dYrows)
            ctx.linear_dx(w_full, dYrows, M_TOK // world, dXr if dXo is None else dXo, dy_dtype=tk.DT_BF16)
            return
        if pair and dx_mode in ("local", "fused"):
            # forward and dX GEMMs in one launch (tiles interleaved); W
            # expanded once; at N > 1 the dX tiles go to their owners over NVLink
            if world == 1:
                ctx.linear_fwd_dx(w, Xin, M_TOK, Y if Yo is None else Yo, dYin, M_TOK, dX if dXo is None else dXo,
                                  x_dtype=tk.DT_BF16)
                return
            ctx.linear_fwd_dx_rs(w, Xin, M_TOK, Y if Yo is None else Yo, dYin, M_TOK, dXr if dXo is None else dXo,
                                 x_dtype=tk.DT_BF16)
            if args.gather_y:
                import torch.distributed as dist
                dist.all_gather_into_tensor(Yfull, Y if Yo is None else Yo, group=group)
            return
        ctx.linear(w, Xin, M_TOK, Y if Yo is None else Yo, x_dtype=tk.DT_BF16)
        # the dX GEMM reuses the forward's fp16 expansion of W (same frozen
        # weight, same step): one dequant per step
        if world == 1:
            ctx.linear_dx(w, dYin, M_TOK, dX if dXo is None else dXo, dy_dtype=tk.DT_BF16, products=tk.WREUSE)
            return
        import torch.distributed as dist
        works = []
        if args.gather_y:
            works.append(dist.all_gather_into_tensor(Yfull, Y, group=group, async_op=True))
        if dx_mode == "fused":
            # one kernel: dX tiles go to their owner rank over NVLink as they finish
            ctx.linear_dx_rs(w, dYin, M_TOK, dXr if dXo is None else dXo, dy_dtype=tk.DT_BF16, products=tk.WREUSE)
        elif dx_mode == "rs-nccl":
            ctx.linear_dx(w, dYin, M_TOK, dX, dy_dtype=tk.DT_BF16, products=tk.WREUSE)
            works.append(dist.reduce_scatter_tensor(dXr, dX, group=group, async_op=True))
        else:
            # NCCL on its own stream: each dX chunk's all-reduce overlaps the next GEMM
            for c in range(chunks):
                ctx.linear_dx(w, dYin[c * mc:(c + 1) * mc], mc, dX[c * mc:(c + 1) * mc], dy_dtype=tk.DT_BF16,
                              products=tk.WREUSE)
                works.append(dist.all_reduce(dX[c * mc:(c + 1) * mc], group=group, async_op=True))
        for wk in works:
            wk.wait()

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
    for _ in range(args.warmup):
        step(Xd, dYd)
    barrier()
    # extra untimed steps up to ~1 s of load; every rank runs the same count
    # (agreed with an all-reduce) so all ranks issue the same collectives.
    t0 = time.perf_counter()
    step(Xd, dYd)
    barrier()
    n_extra = torch.tensor([int(1.0 / max(time.perf_counter() - t0, 1e-4))], device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(n_extra, op=dist.ReduceOp.MAX, group=group)
    for _ in range(int(n_extra.item())):
        step(Xd, dYd)
    barrier()
    n0 = ctx.launches()
    # Per-launch CUDA events (the kernel breakdown and the roofline's GEMM
    # time) bracket every launch of one timed step in PROF_EVERY: an event
    # between two kernels holds the second back until the first has ended,
    # which on every step would add ~35 us to a 0.95 ms step.
    ctx.profile(True)
    ctx.profile(False)
    n_prof = 0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev0.record(stream)
    for i in range(args.steps):
        sample = i % PROF_EVERY == PROF_EVERY - 1 or (i == args.steps - 1 and n_prof == 0)
        if sample:
            ctx.profile(True, resume=True)
            n_prof += 1
        step(Xd, dYd)
        if sample:
            ctx.profile(False)
    ev1.record(stream)
    barrier()
    t_ms = ev0.elapsed_time(ev1)
    gemm_ms, gemm_n = ctx.profile_read(tk.PROF_GEMM)
    deq_ms, deq_n = ctx.profile_read(tk.PROF_DEQUANT)
    spl_ms, spl_n = ctx.profile_read(tk.PROF_SPLIT)
    comm_ms, comm_n = ctx.profile_read(tk.PROF_COMM)
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

    # ---- correctness of the timed outputs (every rank, every N) ----
    if dx_mode in ("fused", "rs-nccl", "reshard"):
        dx_check, dx_row0 = dXr, rank * (M_TOK // world)
    else:
        dx_check, dx_row0 = dX, 0
    check = check_outputs(ctx, Wq, Xb, dY, Y, r0, r1, dx_check, dx_row0, dev, group)

    # ---- where a step's time goes: each phase alone, max over ranks ----
    def phase_ms(fn, n=5):
        fn()
        barrier()
        ev0.record(stream)
        for _ in range(n):
            fn()
        ev1.record(stream)
        barrier()
        v = torch.tensor([ev0.elapsed_time(ev1) / n], device=dev)
        if world > 1:
            import torch.distributed as dist
            dist.all_reduce(v, op=dist.ReduceOp.MAX, group=group)
        return float(v.item())

    phases = {"fwd": phase_ms(lambda: ctx.linear(w, Xd, M_TOK, Y, x_dtype=tk.DT_BF16))}
    if world == 1:
        phases["dx"] = phase_ms(lambda: ctx.linear_dx(w, dYd, M_TOK, dX, dy_dtype=tk.DT_BF16, products=tk.WREUSE))
    elif dx_mode == "reshard":
        phases["dy_reshard"] = phase_ms(lambda: ctx.reshard_cols(dYd, dYrows))
        phases["dx_local_rows"] = phase_ms(
            lambda: ctx.linear_dx(w_full, dYrows, M_TOK // world, dXr, dy_dtype=tk.DT_BF16))
    elif dx_mode == "fused":
        phases["dx_reduce_scatter"] = phase_ms(
            lambda: ctx.linear_dx_rs(w, dYd, M_TOK, dXr, dy_dtype=tk.DT_BF16, products=tk.WREUSE))
        phases["dx_local_no_exchange"] = phase_ms(
            lambda: ctx.linear_dx(w, dYd, M_TOK, dX, dy_dtype=tk.DT_BF16, products=tk.WREUSE))
    if pair and dx_mode in ("local", "fused"):
        phases["fwd_dx_one_launch"] = phase_ms(lambda: step(Xd, dYd))

    # ---- end to end through the C ABI with host buffers ----
    Xh = Xb.pin_memory()
    dYh = dYb.pin_memory()
    Yh = torch.empty(M_TOK, n_loc, dtype=torch.float32).pin_memory()
    dX_out = dXr if dXr is not None else dX        # this rank's dX: token-row shard or the full matrix
    dXh = torch.empty(dX_out.shape, dtype=torch.float32).pin_memory()
    Xs = torch.empty_like(Xd)
    dYs = torch.empty_like(dYd)

    def e2e_step():
        Xs.copy_(Xh, non_blocking=True)
        dYs.copy_(dYh, non_blocking=True)
        step(Xs, dYs)
        Yh.copy_(Y, non_blocking=True)
        dXh.copy_(dX_out, non_blocking=True)

    # the step's work stays on the compute stream at one GPU and with the dX
    # reduce-scatter fused into the GEMM (no NCCL call inside the step)
    pipelined = world == 1 or (dx_mode in ("fused", "reshard") and not args.gather_y)
    if pipelined:
        # copy-in, compute and copy-out on three streams with two buffer sets:
        # step i's inputs come in while step i-1 computes and step i-2's
        # outputs go out (PCIe carries both directions at once).  Every step
        # still moves all of its inputs and outputs inside the timed region.
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        Xs2, dYs2 = [Xs, torch.empty_like(Xs)], [dYs, torch.empty_like(dYs)]
        Y2, dX2 = [Y, torch.empty_like(Y)], [dX_out, torch.empty_like(dX_out)]
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_cmp = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]

        def e2e_pipe(i, start=None):
            b = i & 1
            if start is not None:
                s_in.wait_event(start)
            if i >= 2:
                s_in.wait_event(ev_cmp[b])        # step i-2 has finished reading this input set
            with torch.cuda.stream(s_in):
                Xs2[b].copy_(Xh, non_blocking=True)
                dYs2[b].copy_(dYh, non_blocking=True)
            ev_in[b].record(s_in)
            stream.wait_event(ev_in[b])
            if i >= 2:
                stream.wait_event(ev_out[b])      # step i-2's outputs have left this set
            step(Xs2[b], dYs2[b], Y2[b], dX2[b])
            ev_cmp[b].record(stream)
            s_out.wait_event(ev_cmp[b])
            with torch.cuda.stream(s_out):
                Yh.copy_(Y2[b], non_blocking=True)
                dXh.copy_(dX2[b], non_blocking=True)
            ev_out[b].record(s_out)

        def e2e_run(n):
            ev0.record(stream)
            for i in range(n):
                e2e_pipe(i, ev0 if i == 0 else None)
            for b in range(min(n, 2)):
                stream.wait_event(ev_out[b])
            ev1.record(stream)

        e2e_run(max(2, args.warmup))
        barrier()
        e_steps = max(4, args.steps // 2)
        e2e_run(e_steps)
        barrier()
    else:
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
        # this rank's GEMM FLOPs per step (fwd + dX over its rows) over its GEMM
        # time per step; launches per step vary (dX may run in M-chunks)
        gemm_ms_step = gemm_ms / n_prof
        achieved = flop_step / world / (gemm_ms_step * 1e-3) / 1e12
        # dram read+write bytes per GEMM launch from the committed ncu summary of
        # the launch the step runs (one pair launch, or the fwd and dX launches)
        traffic = None
        one_launch = pair and dx_mode in ("local", "fused")
        tf = ROOT / "profiles" / ("gemm_pair_kernel_c2_q4k_m4096.md" if one_launch else "gemm_tc_kernel_c2_q4k_m4096.md")
        if tf.exists() and world == 1:   # the summaries are of the one-GPU shape
            for ln in tf.read_text().splitlines():
                if ln.startswith("traffic_bytes_per_launch:"):
                    traffic = float(ln.split(":")[1].split()[0])
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp16 tensor-core products, fp32 accumulate (Q4_K -> fp16 exact dequant)",
            "data": "synthetic (seeded, tests/gen.py)",
            "config": {"workload": "C2 Q4_K 14336x4096, M=4096 tokens, fwd + dX per step",
                       "x_dtype": "bf16",
                       "dequant": ("W expanded to fp16 once per step; forward and dX GEMMs in one launch, their "
                                   "tiles interleaved (tk_linear_fwd_dx" + ("_rs)" if world > 1 else ")")
                                   if pair and dx_mode in ("local", "fused") else
                                   "W expanded to fp16 once per step by the forward; the dX GEMM reuses it "
                                   "(TK_WREUSE)"),
                       "partition": (f"W rows split over {world} GPUs; Y " + ("all-gathered" if args.gather_y else
                                     "kept row-sharded (column-parallel: consumed where produced)") +
                                     {"fused": "; dX reduce-scattered by token rows inside the dX GEMM "
                                               "(tiles stored into the owner GPU's memory over NVLink)",
                                      "rs-nccl": "; dX reduce-scattered by token rows (NCCL after the GEMM)",
                                      "allreduce": f"; dX all-reduced in {chunks} M-chunks overlapped with the GEMMs",
                                      "reshard": ("; dY's column shards turned into token-row shards over NVLink "
                                                  "(tk_reshard_cols, overlapping the forward GEMM) and each rank's "
                                                  "dX rows computed against the whole frozen weight, which every "
                                                  "rank holds (dequantized to fp16 by that dX GEMM every step)")
                                      }[dx_mode])
                       if world > 1 else "1 GPU",
                       "l2": "working set per step ~0.5 GB > 126 MB L2 (no explicit flush)"},
            # the timed steps run back to back after >= 1 s of load, at the 1 kW
            # power cap (clocks below): the sustained GEMM figure is the peak
            # the timed region is tens of milliseconds: the burst GEMM figure is the peak
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tf_burst, "unit": "TFLOP/s",
                         "frac": achieved / tf_burst, "traffic": traffic,
                         "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of the step's one "
                                            "GEMM launch (fwd + dX) at this shape on one GPU, from "
                                            "profiles/gemm_pair_kernel_c2_q4k_m4096.md; not measured in this run"
                                            if one_launch else
                                            "ncu dram__bytes_read.sum + dram__bytes_write.sum per GEMM launch "
                                            "(mean of the fwd and dX launches at this shape on one GPU), from "
                                            "profiles/gemm_tc_kernel_c2_q4k_m4096.md; not measured in this run"),
                         "kernel": "gemm_pair_kernel" if one_launch else "gemm_tc_kernel",
                         "peak_source": f"{src} bf16 burst (MEASURED_PEAKS.json)",
                         "sustained_peak": tf_sus, "frac_of_sustained": achieved / tf_sus},
            "check": check,
            "kernels_ms_per_step": {"gemm": gemm_ms / n_prof, "dequant": deq_ms / n_prof,
                                    "act_split": spl_ms / n_prof,
                                    # the owner's reduce of the dX reduce-scatter, its wait for the
                                    # peers' tiles included (N > 1, fused and reshard modes)
                                    "rs_reduce_and_collectives": comm_ms / n_prof,
                                    "sampled": (f"CUDA events around every launch of {n_prof} of the "
                                                f"{args.steps} timed steps (1 in {PROF_EVERY})")},
            "phases_ms": phases,
            "e2e": {"value": e2e_val, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e_steps,
                    "schedule": ("pinned host X, dY in and Y, dX out every step; copy-in, compute and copy-out "
                                 "on three streams with two buffer sets (step k+1's inputs and step k-1's "
                                 "outputs cross PCIe while step k computes)" if pipelined else
                                 "pinned host X, dY in and Y, dX (this rank's part) out every step, one stream")},
            "gpu_launches": launches,
            "clocks": clk,
        }
        if world == 1 and not args.no_extra:
            # the other configurations, each timed on its own after the headline
            del Xh, dYh, Yh, dXh
            torch.cuda.empty_cache()
            line["configs"] = {
                "C1 q8_0 4096x4096 M=1": measure_c1(ctx, tk.Q8_0, 4096, 4096, [1], 50),
                "decode q8_0 14336x4096 M=1": measure_c1(ctx, tk.Q8_0, 14336, 4096, [1], 50),
                "C3 x3 layer (fp32 W hi/lo)": measure_c3(ctx, 5, "hhl"),
                "C4 LM head single pass": measure_c4(ctx, 3),
            }
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = cpu_baseline(Wq, X, dY, args.ref_seconds)
        print(json.dumps(line))
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# Secondary configurations (not the driver's headline line): --config c1|c3|c4
def _timed_graph(fn, steps):
    """One step captured as a CUDA graph (how a serving engine issues a decode
    step: no host launch cost per kernel), replayed `steps` times."""
    import torch
    fn()                                   # workspace growth and attributes outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < 0.5:
        g.replay()
        torch.cuda.synchronize()
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    time.sleep(0.25)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(steps):
        g.replay()
    ev1.record()
    torch.cuda.synchronize()
    t_ms = ev0.elapsed_time(ev1)
    del g
    return t_ms, clocks.stop()


def _timed(ctx, fn, steps, warmup, kind):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < 0.5:
        fn()
        torch.cuda.synchronize()
    clocks = Clocks(torch.cuda.current_device())
    clocks.start()
    time.sleep(0.25)
    ctx.profile(True)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(steps):
        fn()
    ev1.record()
    torch.cuda.synchronize()
    t_ms = ev0.elapsed_time(ev1)
    k_ms, k_n = ctx.profile_read(kind)
    ctx.profile(False)
    return t_ms, k_ms, k_n, clocks.stop()


C1_TYPES = {"q8_0": 8, "q4_k": 12, "q5_k": 13, "q6_k": 14}


def measure_c1(ctx, qt, N, K, Ms, steps, seed=0):
    """Decode GEMV W[N, K] of block type qt for each token count in Ms,
    rotating over distinct weight copies (>= 4x the 126 MB L2) so every
    launch reads HBM.  The launches are captured in one CUDA graph and the
    graph is replayed, so the timing measures back-to-back kernels, not the
    host's launch rate.  Two graphs per M:
      isolated  each GEMV starts after the previous one has finished;
      frozen    the weights are flagged TK_WFROZEN (never written by earlier
                kernels, as every projection of a decode step is), so each
                GEMV is launched as a programmatic dependent of the previous
                one and fetches its weight while that one finishes; x and y
                are still read and written only after it.
    The first M's output is checked against an fp64 matmul of tk_dequant's
    fp32 weight, from both graphs."""
    import numpy as np
    import torch
    import tier_b200 as tk
    from gen import blocks_for
    rng = np.random.default_rng(seed)
    out = {}
    check = None
    clk = None
    for M in Ms:
        b = blocks_for(rng, qt, N, K)
        wbytes = b.nbytes
        copies = int(np.ceil(4 * 126e6 / wbytes))
        W = torch.from_numpy(b).cuda()
        pool = [W.clone() for _ in range(copies)]
        x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
        y = torch.empty(M, N, device="cuda")
        bytes_launch = wbytes + 4 * K * M + 4 * N * M
        res = {}
        for mode, t in (("isolated", qt), ("frozen", qt | tk.WFROZEN)):
            ctx.gemv(t, pool[0], N, K, x, y, M=M)                 # module load / attributes outside capture
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for w in pool:
                    ctx.gemv(t, w, N, K, x, y, M=M)
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            clocks = Clocks(torch.cuda.current_device())
            clocks.start()
            t0 = time.perf_counter()
            while time.perf_counter() - t0 < 0.4:
                g.replay()
                torch.cuda.synchronize()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
            for _ in range(steps):
                g.replay()
            ev1.record()
            torch.cuda.synchronize()
            res[mode] = (ev0.elapsed_time(ev1) / (steps * copies), clocks.stop())
            if M == Ms[0]:
                W32 = torch.empty(N, K, device="cuda")
                ctx.dequant(qt, W, N, K, W32)
                want = x.double() @ W32.double().T
                err = float((y.double() - want).norm() / want.norm())   # y of the last replayed launch
                if check is None or err > check["rel_err"]:
                    check = {"rel_err": err, "tol": 2e-3, "ok": bool(err < 2e-3), "M": M,
                             "against": "fp64 matmul of tk_dequant's fp32 W (bit-exact to q_val in the tests); "
                                        "worst of the isolated and frozen graphs"}
                del W32, want
            del g
        out[M] = {mode: (v[0], bytes_launch / (v[0] * 1e-3) / 1e9) for mode, v in res.items()}
        if clk is None:
            clk = res["frozen"][1]
        out[M]["copies"] = copies
        out[M]["bytes"] = bytes_launch
        del pool, W
    hbm = peaks()[0]
    m0 = Ms[0]
    per_launch, gbs = out[m0]["frozen"]
    iso_launch, iso_gbs = out[m0]["isolated"]
    name = {8: "q8_0", 12: "q4_k", 13: "q5_k", 14: "q6_k"}.get(qt, str(qt))
    shape = f"{name} {N}x{K}"
    return {"metric": f"decode GEMV HBM GB/s ({shape}, M={m0})", "value": gbs, "unit": "GB/s",
            "n_gpus": 1, "steps": steps, "higher_is_better": True, "us_per_launch": per_launch * 1e3,
            "isolated": {"us_per_launch": iso_launch * 1e3, "GB_s": iso_gbs, "frac": iso_gbs / hbm},
            "by_M": {m: {"us_per_launch": v["frozen"][0] * 1e3, "GB_s": v["frozen"][1], "frac": v["frozen"][1] / hbm,
                         "isolated_us_per_launch": v["isolated"][0] * 1e3, "isolated_GB_s": v["isolated"][1],
                         "isolated_frac": v["isolated"][1] / hbm} for m, v in out.items()},
            "config": {"workload": f"{'C1' if shape == 'q8_0 4096x4096' else 'decode'} GEMV {shape}",
                       "rotating_copies": out[m0]["copies"], "bytes_per_launch": out[m0]["bytes"],
                       "timing": ("CUDA graph replay of one launch per weight copy, CUDA events; value: frozen "
                                  "weights (TK_WFROZEN: each GEMV fetches its weight while the previous one "
                                  "finishes, as a decode step's projections run); 'isolated': each launch "
                                  "after the previous one ends")},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "peak_source": "measured hbm_gbs (MEASURED_PEAKS.json)"},
            "check": check, "clocks": clk}


def run_c1(args):
    """C1: q8_0 decode GEMV W[4096, 4096], M = 1 (measure_c1).  --c1-type /
    --c1-shape / --c1-m run the same measurement for the other block types
    and the decode shapes of the 40-layer sweep."""
    import tier_b200 as tk
    ctx = tk.Context(0)
    N, K = (int(v) for v in args.c1_shape.lower().split("x"))
    print(json.dumps(measure_c1(ctx, C1_TYPES[args.c1_type], N, K, [int(m) for m in args.c1_m.split(",")],
                                args.steps)))


def measure_c3(ctx, steps, products="hhl"):
    """C3: the seven projections of one 12B-class layer (hidden 5120, q 4096,
    k/v 1024, o, SwiGLU 14336), M = 4096 fp32 tokens, forward + dX of every
    projection per step.  products "hhl": fp32 W split into fp16 hi/lo,
    Xh.Wh + Xh.Wl + Xl.Wh (<= 1e-5 against fp32 W); "ref": the reference's
    fp3gemm products W.xl + W.xm + W.xh on fp16 W.  Two rows of every
    projection's outputs are checked against fp64 after the timed steps."""
    import torch
    import tier_b200 as tk
    from tier_b200.host import LinearPath
    M, H, I = 4096, 5120, 14336
    shapes = [(4096, H), (1024, H), (1024, H), (H, 4096), (I, H), (I, H), (H, I)]   # q k v o gate up down
    g = torch.Generator(device="cuda").manual_seed(2)
    ws, wref, xs, dys = [], [], {}, []
    prod = tk.X3_HHL if products == "hhl" else tk.X3_REF
    for (n, k) in shapes:
        W = torch.randn(n, k, device="cuda", generator=g) * 0.02
        if products == "hhl":
            lp = LinearPath.from_f32_split(ctx, W)
            ws.append((lp.W, lp.data))
            wref.append(W)                         # fp32, the weight the products approximate
        else:
            W16 = W.half()
            ws.append((tk.make_weight(tk.F16, n, k, W16), W16))
            wref.append(W16)
        del W
        if k not in xs:
            xs[k] = torch.randn(M, k, device="cuda", generator=g)
        dys.append(torch.randn(M, n, device="cuda", generator=g))
    outs = [torch.empty(M, n, device="cuda") for (n, _) in shapes]
    dxs = [torch.empty(M, k, device="cuda") for (_, k) in shapes]

    def fn():
        for (w, _), (n, k), y, dy, dx in zip(ws, shapes, outs, dys, dxs):
            ctx.linear(w, xs[k], M, y, products=prod)
            ctx.linear_dx(w, dy, M, dx, products=prod)

    t_ms, k_ms, k_n, clk = _timed(ctx, fn, steps, 3, tk.PROF_GEMM)
    # check: whole rows 1 and M-1 of every projection's Y and dX against fp64
    errs = []
    for (n, k), y, dy, dx, wr in zip(shapes, outs, dys, dxs, wref):
        w64 = wr.double()
        for r in (1, M - 1):
            want = xs[k][r].double() @ w64.T
            errs.append(float((y[r].double() - want).norm() / want.norm()))
            wdx = dy[r].double() @ w64
            errs.append(float((dx[r].double() - wdx).norm() / wdx.norm()))
        del w64
    err = max(errs)
    snk = sum(n * k for n, k in shapes)
    useful = 2 * 2.0 * M * snk
    ms = t_ms / steps
    tf_burst = peaks()[1]
    gemm_tf_exec = 3 * useful / (k_ms / steps * 1e-3) / 1e12
    return {"metric": "fp16 x3 split GEMM TFLOP/s (12B layer, fwd + dX)", "value": useful / (ms * 1e-3) / 1e12,
            "unit": "TFLOP/s (fp32-equivalent useful)", "executed_tflops": 3 * useful / (ms * 1e-3) / 1e12,
            "ms_per_step": ms, "steps": steps, "n_gpus": 1,
            "config": {"workload": ("C3 12B layer x3, M=4096, fp32 X; " +
                                    ("fp32 W as fp16 hi/lo, Xh.Wh+Xh.Wl+Xl.Wh" if products == "hhl" else
                                     "fp16 W, the reference's W.xl+W.xm+W.xh")),
                       "useful_tflop_per_step": useful / 1e12},
            "roofline": {"bound": "tensor", "achieved": gemm_tf_exec, "peak": tf_burst, "unit": "TFLOP/s",
                         "frac": gemm_tf_exec / tf_burst, "kernel": "gemm_tc_kernel (executed products)",
                         "peak_source": "measured bf16 burst (MEASURED_PEAKS.json)",
                         "sustained_peak": peaks()[2], "frac_of_sustained": gemm_tf_exec / peaks()[2]},
            "gemm_ms_per_step": k_ms / steps,
            "check": {"rel_err": err, "tol": 1e-5, "ok": bool(err < 1e-5),
                      "against": "fp64 matmul of the same fp32 X / dY and the unsplit weight: whole rows 1 and "
                                 "M-1 of every projection's Y and dX, worst per-row relative L2 error"},
            "clocks": clk}


def run_c3(args):
    import tier_b200 as tk
    ctx = tk.Context(0)
    print(json.dumps(measure_c3(ctx, args.steps, args.c3_products)))


def _c5_blocks(qt, n, k, g):
    """Seeded random blocks of type qt [n rows, K = k] on the GPU with finite,
    small fp16 scales (d, dmin): synthetic weights of the 40-layer sweep."""
    import torch
    import tier_b200 as tk
    rb = tk.row_bytes(qt, k)
    B = torch.randint(0, 256, (n, rb), dtype=torch.uint8, device="cuda", generator=g)
    if qt == tk.Q8_0:
        v = B.view(n, k // 32, 34)
        d = (torch.rand(n, k // 32, device="cuda", generator=g) * 3e-4 + 5e-5).half()
        v[:, :, 0:2] = d.view(torch.uint8).view(n, k // 32, 2)
    elif qt == tk.Q6_K:
        v = B.view(n, k // 256, 210)
        d = (torch.rand(n, k // 256, device="cuda", generator=g) * 2e-4 + 1e-5).half()
        v[:, :, 208:210] = d.view(torch.uint8).view(n, k // 256, 2)
    else:
        sb = 144 if qt == tk.Q4_K else 176
        v = B.view(n, k // 256, sb)
        dd = (torch.rand(n, k // 256, 2, device="cuda", generator=g) * 2e-3 + 1e-4).half()
        v[:, :, 0:4] = dd.view(torch.uint8).view(n, k // 256, 4)
    return B


def run_c5(args):
    """C5: 40 layers x the 7 projections of a 12B-class layer (hidden 5120,
    q 4096, k/v 1024, o, SwiGLU 14336), every layer its own weights (so every
    read comes from HBM), in q8_0, the Q4_K_S recipe (Q4_K; Q5_K for v_proj of
    layers 0-3 and down_proj of layers < 40/8), the Q4_K_M recipe (Q4_K; Q6_K
    for the v_proj / down_proj layers quant_main gives more bits), or fp32
    weights split into fp16 hi/lo.  M >= 512: forward + dX of every projection (fp32 activations, x3
    products); M <= 16 (decode): the forward GEMV of every projection (frozen
    weights).  One JSON line per (weights, M)."""
    import torch
    import tier_b200 as tk
    from tier_b200.host import LinearPath
    ctx = tk.Context(0)
    H, I, L = 5120, 14336, 40
    shapes = [(4096, H), (1024, H), (1024, H), (H, 4096), (I, H), (I, H), (H, I)]
    names = ["q", "k", "v", "o", "gate", "up", "down"]
    hbm, tf_burst = peaks()[0], peaks()[1]
    kinds = args.c5_kinds.split(",")
    Ms = [int(m) for m in args.c5_m.split(",")]
    snk = sum(n * k for n, k in shapes)
    from tier_b200.tq import recipe_types
    slots = ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]
    rtypes = {}
    for kind in kinds:
        if kind in ("q4_k_s", "q4_k_m"):
            for l, slot, qt in recipe_types(kind.upper(), [slots] * L):
                rtypes[(kind, l, slots.index(slot))] = qt
    for kind in kinds:
        g = torch.Generator(device="cuda").manual_seed(4)
        layers, wbytes = [], 0
        for l in range(L):
            ws = []
            for j, (n, k) in enumerate(shapes):
                if kind == "fp16x3":
                    W32 = torch.randn(n, k, device="cuda", generator=g) * 0.02
                    lp = LinearPath.from_f32_split(ctx, W32)
                    del W32
                    ws.append((lp.W, tk.F16X2, lp.data))
                    wbytes += n * k * 4
                else:
                    qt = tk.Q8_0 if kind == "q8_0" else rtypes[(kind, l, j)]
                    B = _c5_blocks(qt, n, k, g)
                    ws.append((tk.make_weight(qt, n, k, B), qt, B))
                    wbytes += B.numel()
            layers.append(ws)
        torch.cuda.synchronize()
        for M in Ms:
            xs = {k: torch.randn(M, k, device="cuda", generator=g) for k in {k for _, k in shapes}}
            ys = {n: torch.empty(M, n, device="cuda") for n in {n for n, _ in shapes}}
            decode = M <= 16
            if not decode:
                dys = {n: torch.randn(M, n, device="cuda", generator=g) for n in {n for n, _ in shapes}}
                dxs = {k: torch.empty(M, k, device="cuda") for k in {k for _, k in shapes}}

            # decode: the projections that read the same x (q/k/v, gate/up) go in one
            # tk_gemv_multi launch when their block types match
            yp = [torch.empty(M, n, device="cuda") for n, _ in shapes] if decode else None

            def fn():
                for ws in layers:
                    if decode and kind != "fp16x3":
                        for grp in ((0, 1, 2), (3,), (4, 5), (6,)):
                            runs = []
                            for j in grp:
                                if runs and ws[runs[-1][-1]][1] == ws[j][1]:
                                    runs[-1].append(j)
                                else:
                                    runs.append([j])
                            for run in runs:
                                qt, k = ws[run[0]][1], shapes[run[0]][1]
                                if len(run) == 1:
                                    j = run[0]
                                    ctx.gemv(qt | tk.WFROZEN, ws[j][2], shapes[j][0], k, xs[k], yp[j], M=M)
                                else:
                                    ctx.gemv_multi(qt | tk.WFROZEN, [ws[j][2] for j in run], [shapes[j][0] for j in run],
                                                   [yp[j] for j in run], k, xs[k], M=M)
                        continue
                    for (w, qt, data), (n, k) in zip(ws, shapes):
                        if decode:
                            ctx.linear(w, xs[k], M, ys[n])
                        else:
                            ctx.linear(w, xs[k], M, ys[n])
                            ctx.linear_dx(w, dys[n], M, dxs[k])

            steps = 1 if M >= 4096 else max(1, min(args.steps, 5))
            # quantized decode (GEMVs only) replays as one CUDA graph; the fp16-x3 weights
            # decode through tk_linear_fwd, whose split-K stamps advance per launch, so
            # those steps launch eagerly
            graph = decode and kind != "fp16x3"
            if graph:
                steps = max(steps, 20)
                t_ms, clk = _timed_graph(fn, steps)
                k_ms = None
            else:
                t_ms, k_ms, k_n, clk = _timed(ctx, fn, steps, 1, tk.PROF_GEMV if decode else tk.PROF_GEMM)
            ms = t_ms / steps
            line = {"metric": "C5 40-layer sweep", "kind": kind, "M": M, "ms_per_step": ms, "steps": steps,
                    "n_gpus": 1, "weight_bytes": wbytes, "clocks": clk,
                    "config": {"workload": f"C5 40 layers x 7 projections (12B-class), {kind} weights, M={M}, " +
                               (("forward GEMV (decode; q/k/v and gate/up of one type share a tk_gemv_multi "
                                 "launch), a step's launches replayed as one CUDA graph" if graph
                                 else "forward (decode) through tk_linear_fwd, eager launches")
                                if decode else "forward + dX, fp32 activations, x3 products")}}
            if decode:
                gbs = wbytes / (ms * 1e-3) / 1e9
                line.update({"value": gbs, "unit": "GB/s", "higher_is_better": True,
                             "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                                          "frac": gbs / hbm, "note": "whole step, weight bytes / step time"}})
            else:
                useful = 2 * 2.0 * M * snk * L
                gemm_exec = 3 * useful / (k_ms / steps * 1e-3) / 1e12
                line.update({"value": useful / (ms * 1e-3) / 1e12, "unit": "TFLOP/s (fp32-equivalent useful)",
                             "higher_is_better": True, "executed_tflops": 3 * useful / (ms * 1e-3) / 1e12,
                             "roofline": {"bound": "tensor", "achieved": gemm_exec, "peak": tf_burst,
                                          "unit": "TFLOP/s", "frac": gemm_exec / tf_burst,
                                          "kernel": "gemm_tc_kernel (executed products)"}})
            print(json.dumps(line), flush=True)
            del xs, ys
            if not decode:
                del dys, dxs
        del layers
        torch.cuda.empty_cache()


def measure_c4(ctx, steps, two_pass=False):
    """C4: chunked-vocab LM head + CE: W fp16 [262144, 3840], hidden fp32
    [8192, 3840], labels uniform, chunk 16384.  Default: the single pass
    (one logits GEMM per chunk with the x3 split of X, then the dX GEMM with
    the hi/lo probabilities); two_pass runs the reference's two passes
    (logits recomputed in pass 2, dlogit split in three).  After the timed
    steps the loss terms and dX of two rows are checked against fp64
    (vocabulary in chunks, on the GPU)."""
    import torch
    import tier_b200 as tk
    from tier_b200.host import LMHead
    V, H, T, chunk = 262144, 3840, 8192, 16384
    g = torch.Generator(device="cuda").manual_seed(3)
    W = (torch.randn(V, H, device="cuda", generator=g) * 0.02).half()
    X = torch.randn(T, H, device="cuda", generator=g)
    labels = torch.randint(0, V, (T,), device="cuda", generator=g, dtype=torch.int32)
    mask = torch.ones(T, dtype=torch.uint8, device="cuda")
    head = LMHead(ctx, W, 0, chunk=chunk, products=tk.X3_REF)
    dX = torch.zeros(T, H, device="cuda")
    n_loss = T - 1
    res = {}

    def fn():
        if two_pass:
            rmax, rsum, amax, tgt = head.stats(X, labels, mask)
            res["loss"] = head.loss(T, labels, mask, rmax, rsum, amax, tgt)[0]
            dX.zero_()                     # pass 2 accumulates (the reference's dX += per chunk)
            head.grad(X, labels, mask, n_loss, rmax, rsum, dX=dX)
            res["dX"] = dX
        else:
            out = head.step_fused(X, labels, mask, n_loss=n_loss)
            res["loss"], res["dX"] = out[0], out[4]

    steps = max(1, min(steps, 5))
    t_ms, k_ms, k_n, clk = _timed(ctx, fn, steps, 1, tk.PROF_GEMM)
    # fp64 check of rows 0 and T-2: lse - target and the dX row
    rows = [0, T - 2]
    Xr = X[rows].double()
    lab = labels[[r + 1 for r in rows]].long()
    m = torch.full((2,), -float("inf"), dtype=torch.float64, device="cuda")
    ssum = torch.zeros(2, dtype=torch.float64, device="cuda")
    for v0 in range(0, V, chunk):
        L = (Xr @ W[v0:v0 + chunk].double().T).float().double()   # logits rounded to fp32, as the GEMM stores them
        nm = torch.maximum(m, L.max(1).values)
        ssum = ssum * torch.exp(m - nm) + torch.exp(L - nm[:, None]).sum(1)
        m = nm
    lse = m + torch.log(ssum)
    d = torch.zeros(2, H, dtype=torch.float64, device="cuda")
    for v0 in range(0, V, chunk):
        Wc = W[v0:v0 + chunk].double()
        P = torch.exp((Xr @ Wc.T).float().double() - lse[:, None])
        for i in range(2):
            if v0 <= int(lab[i]) < v0 + chunk:
                P[i, int(lab[i]) - v0] -= 1.0
        d += (P / n_loss) @ Wc
    got = res["dX"][rows].double()
    err = float(((got - d).norm(dim=1) / d.norm(dim=1)).max())
    ms = t_ms / steps
    useful = 2 * 2.0 * T * V * H
    # executed products: logits x3 (+ x3 recompute + x3 dX in two passes;
    # + hi/lo dX in the single pass)
    executed = (3 + 3 + 3 if two_pass else 3 + 2) * 2.0 * T * V * H
    tf_burst = peaks()[1]
    gemm_exec = executed / (k_ms / steps * 1e-3) / 1e12
    rec = {"metric": "LM head + CE TFLOP/s (useful: logits + dX GEMMs)", "value": useful / (ms * 1e-3) / 1e12,
           "unit": "TFLOP/s", "executed_tflops": executed / (ms * 1e-3) / 1e12, "ms_per_step": ms,
           "steps": steps, "n_gpus": 1,
           "config": {"workload": "C4 V=262144 H=3840 T=8192 chunk=16384, " +
                      ("two-pass, x3 split of X and dlogit" if two_pass else
                       "single pass, x3 split of X, hi/lo probabilities")},
           "roofline": {"bound": "tensor", "achieved": gemm_exec, "peak": tf_burst, "unit": "TFLOP/s",
                        "frac": gemm_exec / tf_burst, "kernel": "gemm_tc_kernel (executed products)",
                        "peak_source": "measured bf16 burst (MEASURED_PEAKS.json)",
                        # steps of ~0.1 s back to back run at the power cap, as the sustained figure does
                        "sustained_peak": peaks()[2], "frac_of_sustained": gemm_exec / peaks()[2]},
           "gemm_ms_per_step": k_ms / steps,
           "check": {"rel_err": err, "tol": 1e-5, "ok": bool(err < 1e-5),
                     "against": "fp64 two-pass LM head (logits rounded to fp32) on rows 0 and T-2: dX rows"},
           "clocks": clk}
    del W, X, dX, head
    torch.cuda.empty_cache()
    return rec


def run_c4(args):
    import tier_b200 as tk
    ctx = tk.Context(0)
    print(json.dumps(measure_c4(ctx, args.steps, args.c4_two_pass)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-seconds", type=float, default=10.0, help="CPU baseline sample size (seconds)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--gather-y", action="store_true", help="multi-GPU: all-gather the full Y every step")
    ap.add_argument("--dx-chunks", type=int, default=4, help="multi-GPU allreduce mode: dX GEMM / all-reduce chunks")
    ap.add_argument("--step-call", default="pair", choices=["pair", "separate"],
                    help="pair: forward and dX in one call and one GEMM launch (tk_linear_fwd_dx[_rs]); "
                         "separate: tk_linear_fwd then tk_linear_dx[_rs]")
    ap.add_argument("--dx-mode", default="fused", choices=["fused", "rs-nccl", "allreduce", "reshard"],
                    help="multi-GPU dX: reduce-scatter by token rows inside the GEMM over NVLink (fused), "
                         "GEMM then NCCL reduce-scatter (rs-nccl), chunked NCCL all-reduce of the full dX "
                         "(allreduce), or dY resharded to token rows and dX computed locally (reshard)")
    ap.add_argument("--c1-type", default="q8_0", choices=sorted(C1_TYPES), help="c1: weight block type")
    ap.add_argument("--c1-shape", default="4096x4096", help="c1: N x K of the weight")
    ap.add_argument("--c1-m", default="1,4,16", help="c1: token counts (the first is the headline)")
    ap.add_argument("--c4-two-pass", action="store_true", help="c4: the reference's two passes")
    ap.add_argument("--c3-products", default="hhl", choices=["hhl", "ref"],
                    help="c3: fp32 W as hi/lo planes (hhl) or the reference's products on fp16 W (ref)")
    ap.add_argument("--no-extra", action="store_true",
                    help="headline only: skip the C1/C3/C4 sub-records measured after it on one GPU")
    ap.add_argument("--c5-kinds", default="q8_0,q4_k_s,fp16x3", help="c5: weight kinds")
    ap.add_argument("--c5-m", default="1,16,512,4096,16384", help="c5: token counts")
    ap.add_argument("--config", default="c2", choices=["c1", "c2", "c3", "c4", "c5"],
                    help="c2 (default, the headline) or a secondary configuration on one GPU")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "ours" and args.config != "c2":
        return {"c1": run_c1, "c3": run_c3, "c4": run_c4, "c5": run_c5}[args.config](args)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
