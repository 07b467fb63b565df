"""Benchmark: Sinkhorn ms per iteration (one f half-step + one g half-step) on the fused CUDA half-step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload auto|cfg2|cfg5|weak]

Workloads (synthetic, seeded; trnopt.synthetic):
  cfg2  n = m = 10,000, d = 64, x, y ~ U[0,1]^64, eps 0.1, raw cost (the N = 1 default)
  weak  the N > 1 default: n = 10,000 N rows, m = 10,000, d = 64 (config 2's per-GPU work at every N)
  cfg5  n = m = 262,144, d = 64, x, y ~ N(0, I)/8, mean-normalised cost, eps 0.01 (strong
        scaling over N)
  cfg3  one wot transport map, 7,355 x 8,962 cells in d = 30 (median cost, eps 0.05, lambda (1, 50), 3 growth
        iterations, tol 1e-8): a step is the whole map through the public API, reported in seconds
  cfg4  the 38-pair trajectory pipeline (175k cells) with cfg3's settings: a step is the whole pipeline, seconds
  cfg2conv  config 2 to convergence: one sinkhorn() call from pinned host arrays, balanced marginal error below
        tol 1e-6 checked every 10 iterations; a step is the whole solve, seconds (iterations in `config`)
  cfg5conv  config 5's schedule: eps 1.0 -> 0.01 over 8 geometric values, at most 50 iterations per intermediate
        value (a stage also ends when its potential change falls below the float32 stage floor), 400 iterations
        in all, mean-normalised cost; a step is the whole solve, seconds
A step is one Sinkhorn iteration with the inputs resident in HBM; L2 (126 MB) is flushed between timed steps by
writing a 256 MB buffer (outside the timed region). Under torchrun each rank drives one GPU and rows of every
half-step are split across the ranks; each GPU's new rows reach the others through peer stores from the half-step
kernel (--exchange peer, the default on the tensor-core path) or one NCCL all-gather per half-step (--exchange
nccl); the reported time is the max over ranks.

--impl reference times the reference's CPU solver on this host's cores (the CPU port in oracle/, float32, all
threads) on the same workload; under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "trainium-sinkhorn_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "Sinkhorn ms/iter (10k^2 d=64; 262k^2 d=64 @1/2/4/8 B200)"
SMS = 148


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="auto", choices=["auto", "cfg2", "cfg5", "weak", "cfg3", "cfg4", "cfg2conv", "cfg5conv"])
    ap.add_argument("--path", default="auto", choices=["auto", "ffma", "tc"])
    ap.add_argument("--exchange", default="auto", choices=["auto", "peer", "nccl"],
                    help="N > 1: peer stores from the half-step kernels (tc path) or an NCCL all-gather per half-step")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--no-flush", action="store_true", help="(profiling runs only) do not flush L2 between steps")
    return ap.parse_args()


def workload(name: str, world: int):
    from trnopt import synthetic
    if name == "auto":
        name = "cfg2" if world == 1 else "weak"
    if name == "cfg2":
        x, y = synthetic.cfg2()
        return name, x, y, dict(eps=0.1, normalize=False), {"n": 10_000, "m": 10_000, "d": 64, "eps": 0.1}
    if name == "weak":
        x, y = synthetic.cfg2(n=10_000 * world, m=10_000)
        return name, x, y, dict(eps=0.1, normalize=False), {"n": 10_000 * world, "m": 10_000, "d": 64, "eps": 0.1}
    x, y = synthetic.cfg5()
    return name, x, y, dict(eps=0.01, normalize="mean"), {"n": len(x), "m": len(y), "d": 64, "eps": 0.01}


class NvmlClocks:
    """SM clock and throttle-reason samples every ~1 ms through NVML while the timed region runs (the region can be a
    few milliseconds, shorter than nvidia-smi's sampling period). Falls back to nvidia-smi when NVML is missing."""
    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, dev: int, enabled: bool):
        self.enabled, self.samples, self.reasons, self.max_mhz = enabled, [], set(), None
        self.stop, self.thread, self.fallback = threading.Event(), None, None
        if not enabled:
            return
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(dev).uuid)
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            self.nv, self.h = pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
        except Exception:
            self.nv, self.fallback = None, Clocks(dev, enabled)

    def _run(self):
        while True:
            self._sample()
            if self.stop.wait(0.001):
                self._sample()
                return

    def _sample(self):
        try:
            self.samples.append(float(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)))
            mask = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            self.reasons.update(k for k, b in self.REASONS.items() if mask & b)
        except Exception:
            pass

    def __enter__(self):
        if self.fallback is not None:
            self.fallback.__enter__()
        elif self.enabled:
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        return self

    def __exit__(self, *a):
        if self.fallback is not None:
            self.fallback.__exit__(*a)
        elif self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)

    def summary(self):
        if self.fallback is not None:
            return self.fallback.summary()
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples), "source": "nvml"}


class Clocks:
    """nvidia-smi samples of this GPU's SM clock and throttle reasons while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, dev: int, enabled: bool):
        self.proc, self.lines, self.enabled = None, [], enabled
        self.target = None
        try:
            self.target = str(torch.cuda.get_device_properties(dev).uuid)
            if not self.target.startswith("GPU-"):
                self.target = "GPU-" + self.target
        except Exception:
            self.target = None

    def __enter__(self):
        if self.enabled:
            cmd = ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200"]
            if self.target:
                cmd += ["-i", self.target]
            try:
                self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.reader = threading.Thread(target=self._read, daemon=True)
                self.reader.start()
            except OSError:
                self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [s.strip() for s in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_oracle_iteration_ms(x, y, kw, max_seconds: float, threads: int | None = None):
    """The reference's CPU solver (oracle port, torch float32, all threads) on a bounded sample of the workload:
    whole iterations when they fit the time budget, else the f and g half-steps over a subset of rows, scaled."""
    from oracle import trnopt_oracle as O
    torch.set_num_threads(threads or os.cpu_count() or 1)
    eps = kw["eps"]
    if kw["normalize"]:
        center, scale = O.normalization(x, y, how="mean")
    else:
        center, scale = np.zeros(x.shape[1]), 1.0
    xs, ys = (x - center) / np.sqrt(scale), (y - center) / np.sqrt(scale)
    n, m = len(xs), len(ys)
    t = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float32)
    X, Y = t(xs), t(ys)
    XT, YT = X.T.contiguous(), Y.T.contiguous()
    xsq, ysq = t((xs * xs).sum(1)), t((ys * ys).sum(1))
    la, lb = torch.full((n,), float(-np.log(n))), torch.full((m,), float(-np.log(m)))
    zx, zy = torch.zeros(n), torch.zeros(m)
    gh = torch.zeros(m)
    inv, e, k = (torch.tensor(v, dtype=torch.float32) for v in (1.0 / eps, eps, 1.0))

    blk = max(n, m) if n * m <= 150_000_000 else 4096   # the reference's default block=None where it fits

    def iteration(rows_x, rows_y):
        fh = torch.cat([O.half_step(X[s:s + blk], xsq[s:s + blk], zx[s:s + blk], YT, gh, lb, inv, e, k)
                        for s in range(0, rows_x, blk)])
        gg = torch.cat([O.half_step(Y[s:s + blk], ysq[s:s + blk], zy[s:s + blk], XT, fh if rows_x == n else zx, la,
                                    inv, e, k) for s in range(0, rows_y, blk)])
        return gg

    t0 = time.perf_counter()
    iteration(min(n, 4096), min(m, 4096))                     # warm-up on one block of rows each way
    t_blk = time.perf_counter() - t0
    est_full = t_blk * (n / min(n, 4096) + m / min(m, 4096)) / 2
    if est_full * 2 <= max_seconds:
        reps, frac = 2, 1.0
        t0 = time.perf_counter()
        for _ in range(reps):
            iteration(n, m)
        dt = (time.perf_counter() - t0) / reps
        sample = f"{reps} full iterations ({n}x{m}, d {x.shape[1]}) after a 4096-row warm-up"
    else:
        frac = max(4096 / max(n, m), min(1.0, max_seconds / (2 * est_full)))
        rx, ry = max(1, int(n * frac)), max(1, int(m * frac))
        t0 = time.perf_counter()
        iteration(rx, ry)
        dt = (time.perf_counter() - t0) * (n + m) / (rx + ry)
        sample = f"f and g half-steps over {rx} + {ry} of {n} + {m} rows, scaled to a full iteration"
    return dt * 1e3, torch.get_num_threads(), sample


def run_reference(args, rank, world):
    if rank != 0:
        return
    name, x, y, kw, cfg = workload(args.workload, world)
    budget_per_step = max(0.5, 150.0 / max(1, args.steps + args.warmup))
    # Each step is one bounded sample of an iteration, timed on the host's cores.
    vals, cores, sample = [], 0, ""
    for i in range(args.warmup + args.steps):
        ms, cores, sample = cpu_oracle_iteration_ms(x, y, kw, budget_per_step)
        if i >= args.warmup:
            vals.append(ms)
    v = float(np.mean(vals))
    line = {"metric": METRIC, "value": v, "unit": "ms/iter", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": v, "higher_is_better": False, "scaling": "weak" if name == "weak"
            else "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)", "impl": "reference",
            "config": {"workload": name, **cfg, "l2": "inputs resident in host memory"},
            "cpu_baseline": {"value": v, "unit": "ms/iter", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "ms/iter", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_pipeline(args, rank, world, dev):
    """cfg3 / cfg4: wot transport maps through the public API (trnopt.singlecell), wall time per map / pipeline;
    cfg2conv: one config-2 solve to convergence through sinkhorn()."""
    from trnopt import Backend, SinkhornOptions, sinkhorn, synthetic
    from trnopt.singlecell import wot_trajectory, wot_transport_map
    opts = SinkhornOptions(backend=Backend.preset("cuda-fused", device=str(dev)), cores=world)
    last = {}
    def pinned(a):
        t = torch.empty(a.shape, dtype=torch.float64, pin_memory=True)
        t.numpy()[...] = a
        return t.numpy()
    if args.workload == "cfg2conv":
        xc, yc = (pinned(a) for a in synthetic.cfg2())
        conv = SinkhornOptions(eps=0.1, tol=1e-6, check_every=10, max_iters=20_000, normalize=False,
                               backend=opts.backend, cores=world)
        cfg = {"workload": "cfg2conv", "n": 10_000, "m": 10_000, "d": 64, "eps": 0.1, "tol": 1e-6, "check_every": 10,
               "input": "host float64 arrays in pinned memory, f and g returned to the host"}
    elif args.workload == "cfg5conv":
        xc, yc = (pinned(a) for a in synthetic.cfg5())
        stages = synthetic.cfg5_eps_stages()
        conv = SinkhornOptions(eps=0.01, eps_stages=stages, stage_max_iters=50, max_iters=400, fixed_iters=True,
                               normalize="mean", backend=opts.backend, cores=world)
        cfg = {"workload": "cfg5conv", "n": len(xc), "m": len(yc), "d": 64, "eps": 0.01,
               "eps_stages": [round(e, 6) for e in stages], "stage_max_iters": 50, "iterations_in_all": 400,
               "input": "host float64 arrays in pinned memory, f and g returned to the host"}
    elif args.workload == "cfg3":
        x0, x1, g = synthetic.cfg3()
        pairs = [(x0, x1, g)]
        cfg = {"workload": "cfg3", "n": len(x0), "m": len(x1), "d": 30, "eps": 0.05, "lambda": [1.0, 50.0],
               "growth_iters": 3, "tol": 1e-8}
    else:
        tr = synthetic.cfg4()
        pairs = [(tr.cohorts[t], tr.cohorts[t + 1], tr.growth[t]) for t in range(len(tr.cohorts) - 1)]
        cfg = {"workload": "cfg4", "pairs": len(pairs), "cells": int(sum(len(c) for c in tr.cohorts)), "d": 30,
               "eps": 0.05, "lambda": [1.0, 50.0], "growth_iters": 3, "tol": 1e-8}

    kw = dict(eps=0.05, lambda1=1.0, lambda2=50.0, growth_iters=3, tol=1e-8, opts=opts)

    def one():
        if args.workload in ("cfg2conv", "cfg5conv"):
            r = sinkhorn(xc, yc, opts=conv)
            last.update(converged=bool(r.converged), error=float(r.error))
            return r.iterations
        if args.workload == "cfg4":          # the whole time course through the public pipeline loop
            return sum(tm.iterations for tm in wot_trajectory(tr.cohorts, None, tr.growth, **kw))
        return sum(wot_transport_map(x0, x1, g, **kw).iterations for x0, x1, g in pairs)

    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize(dev)
    times, iters = [], 0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        iters = one()
        torch.cuda.synchronize(dev)
        times.append(time.perf_counter() - t0)
    v = float(np.mean(times))
    if rank == 0:
        metric = {"cfg3": "wot transport map seconds", "cfg4": "38-pair pipeline seconds",
                  "cfg2conv": "config 2 time to convergence seconds",
                  "cfg5conv": "config 5 eps-staged solve seconds"}[args.workload]
        line = {"metric": metric,
                "value": v, "unit": "s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": v * 1e3, "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic (seeded generators in trnopt.synthetic)",
                "config": {**cfg, "sinkhorn_iterations": iters, "ms_per_iteration": v * 1e3 / max(1, iters), **last},
                "gpu_launches": 2 * iters}
        print(json.dumps(line), flush=True)


def run_ours(args, rank, world, dev):
    import trnopt.sinkhorn  # noqa: F401
    from trnopt import Backend, SinkhornOptions, _capi, sinkhorn
    S = sys.modules["trnopt.sinkhorn"]
    name, x, y, kw, cfg = workload(args.workload, world)
    eps = kw["eps"]
    path = S._resolve_path(args.path, x.shape[1])
    if kw["normalize"]:
        center, scale = S.normalization(x, y, how="mean")
    else:
        center, scale = np.zeros(x.shape[1]), 1.0
    xs, ys = (x - center) / np.sqrt(scale), (y - center) / np.sqrt(scale)
    shift = np.concatenate([xs, ys]).mean(axis=0)
    xi, yi = xs - shift, ys - shift
    n, m = len(x), len(y)
    la, lb = np.full(n, -np.log(n)), np.full(m, -np.log(m))
    X = S._Cloud(xi, la, world, dev)
    Y = S._Cloud(yi, lb, world, dev)
    S._prepare_path(path, X, Y)
    ws = S._workspace(X, Y, world, dev, path)
    step = S._CudaStep(dev, world, rank, ws, path=path)
    exchange = S._exchange(args.exchange, path) if world > 1 else "none"
    peer = None
    if exchange == "peer":
        from trnopt import _comm
        peer = _comm.region(4 * (X.npad + 2 * Y.npad))
        fh = peer.tensor(0, X.npad)
        G = [peer.tensor(4 * X.npad, Y.npad), peer.tensor(4 * (X.npad + Y.npad), Y.npad)]
        G[0].zero_()
        fh.zero_()
        peer.arrive()
    else:
        G = [torch.zeros(Y.npad, dtype=torch.float32, device=dev) for _ in range(2)]
        fh = torch.zeros(X.npad, dtype=torch.float32, device=dev)
    tc = path == "tc"
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    counter = [0]

    def iteration(ev=None):
        # one iteration = f half-step then g half-step, through the same run entries the solver uses
        i = counter[0]
        counter[0] += 1
        if ev is not None:
            ev[0].record(stream)
        if peer is not None:
            _capi.sinkhorn_run_sharded(peer.comm, X.packed, X.sq, None, X.log_w, X.npad, X.sexp, Y.packed, Y.sq, None,
                                       Y.log_w, Y.npad, Y.sexp, X.d, G[0], G[1], fh, i % 2, 1, eps, 1.0, 1.0, ws)
        elif world > 1:
            step(X, Y, G[i % 2], eps, 1.0, out=fh)
            step(Y, X, fh, eps, 1.0, out=G[(i + 1) % 2])
        else:
            _capi.sinkhorn_run(_capi.PATH_TC if tc else _capi.PATH_FFMA, X.packed if tc else X.xT, X.npad, X.sq, None,
                               X.log_w, X.npad, X.sexp, Y.packed if tc else Y.xT, Y.npad, Y.sq, None, Y.log_w, Y.npad,
                               Y.sexp, X.d, G[0], G[1], fh, i % 2, 1, eps, 1.0, 1.0, ws)
        if ev is not None:
            ev[1].record(stream)

    for _ in range(args.warmup):
        iteration()
    torch.cuda.synchronize(dev)
    steps = []
    with NvmlClocks(dev.index, enabled=not args.no_clocks and rank == 0) as clk:
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)
        for _ in range(args.steps):
            if not args.no_flush:
                flush.zero_()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            iteration(ev)
            steps.append(ev)
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier()
    if peer is not None:
        peer.wait()
    step_ms = [a.elapsed_time(b) for a, b in steps]
    total = torch.tensor([sum(step_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(total, op=torch.distributed.ReduceOp.MAX)
    ms_per_step = float(total.item()) / args.steps
    clocks = clk.summary() if rank == 0 else None
    if _capi.device_error_flags():
        raise RuntimeError("a kernel reported device error flags during the timed region")

    # Roofline of the dominant kernel (the fused half-step): per launch, useful FLOPs 2 rows m d, exps rows m. A step
    # is two launches of it (f then g, the second allowed to start its prologue early), so a launch is half a step.
    rows_f, rows_g = X.npad // world, Y.npad // world
    launch_ms = statistics.mean(step_ms) / 2
    flops = (2.0 * rows_f * Y.npad * X.d + 2.0 * rows_g * X.npad * X.d) / 2
    exps = (rows_f * Y.npad + rows_g * X.npad) / 2.0
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    bf16 = peaks.get("bf16_tflops", 1590.0)
    peak_src = "measured" if peaks else "fallback"
    mhz = (clocks or {}).get("sm_mhz") or peaks.get("sm_max_mhz", 1965.0)
    tflops = flops / (launch_ms * 1e-3) / 1e12
    ffma_peak = SMS * 128 * 2 * mhz * 1e6 / 1e12
    sfu_rate = exps / (launch_ms * 1e-3)
    sfu_peak = SMS * 16 * mhz * 1e6
    traffic = None
    tfile = ROOT / "profiles" / f"traffic_{path}_{name}.json"
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get("bytes_per_launch")
    roof = {"bound": "tensor", "achieved": round(tflops, 2), "peak": bf16, "unit": "TFLOP/s",
            "frac": round(tflops / bf16, 4), "traffic": traffic, "peak_source": peak_src,
            "kernel": f"half-step ({path})", "launch_ms": round(launch_ms, 5),
            "sfu": {"achieved_exp_per_s": sfu_rate, "peak_exp_per_s": sfu_peak, "frac": round(sfu_rate / sfu_peak, 4),
                    "clock_mhz": mhz}}
    if path == "ffma":
        roof["ffma"] = {"achieved_tflops": round(tflops, 2), "peak_tflops": round(ffma_peak, 2),
                        "frac": round(tflops / ffma_peak, 4)}
    # The north star's roofline: the slowest of the contraction at its pipe's peak (useful FLOPs), the exps at the
    # MUFU rate and the algorithmic bytes at the measured HBM copy rate (both clouds once, 4 bytes per coordinate
    # in FP32 or as an FP16 hi/lo pair, plus the vectors: (n + m)(4d + 12) per launch); frac = that
    # bound's time over the measured launch time.
    hbm = peaks.get("hbm_gbs", 6650.0)
    bounds_us = {"contraction": flops / ((ffma_peak if path == "ffma" else bf16) * 1e12) * 1e6,
                 "exp": exps / sfu_peak * 1e6,
                 "hbm": (X.npad + Y.npad) * (4 * X.d + 12) / (hbm * 1e9) * 1e6}
    slow = max(bounds_us, key=bounds_us.get)
    roof["slowest_bound"] = {"name": slow, "bound_us": {k: round(v, 3) for k, v in bounds_us.items()},
                             "launch_us": round(launch_ms * 1e3, 3), "frac": round(bounds_us[slow] / (launch_ms * 1e3), 4)}

    # End to end through the public API: host arrays in, potentials out, K iterations.
    e2e = None
    if not args.no_e2e:
        opts = SinkhornOptions(max_iters=args.steps, fixed_iters=True, backend=Backend.preset("cuda-fused", device=str(dev)),
                               cores=world, cuda_path=path, cuda_exchange=args.exchange, **kw)
        # the clouds in pinned (page-locked) host memory, as a caller feeding a GPU solver keeps them: the upload
        # inside sinkhorn() is then one DMA per cloud
        def pinned(a):
            t = torch.empty(a.shape, dtype=torch.float64, pin_memory=True)
            t.numpy()[...] = a
            return t.numpy()
        xh, yh = pinned(x), pinned(y)
        for _ in range(max(1, min(args.warmup, 3))):      # warm-up solves of the same problem, untimed
            sinkhorn(xh, yh, opts=SinkhornOptions(max_iters=2, fixed_iters=True, backend=opts.backend, cores=world,
                                                  cuda_path=path, cuda_exchange=args.exchange, **kw))
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        r = sinkhorn(xh, yh, opts=opts)
        torch.cuda.synchronize(dev)
        dt = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
        if world > 1:
            torch.distributed.all_reduce(dt, op=torch.distributed.ReduceOp.MAX)
        h2d = X.h2d_bytes + Y.h2d_bytes                 # x, y and their log weights in float64
        d2h = 8 * (n + m)                                 # f and g in float64
        e2e = {"value": float(dt.item()) * 1e3 / r.iterations, "unit": "ms/iter",
               "h2d_bytes_per_step": h2d / r.iterations, "d2h_bytes_per_step": d2h / r.iterations,
               "note": "one public sinkhorn() call on host float64 arrays (pinned memory) after untimed 2-iteration warm-up calls of "
                       "the same problem (upload, normalisation, padding, "
                       f"{r.iterations} fixed iterations, f and g back to the host), divided by the iterations"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ms, cores, sample = cpu_oracle_iteration_ms(x, y, kw, 20.0)
        cpu = {"value": ms, "unit": "ms/iter", "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {"metric": METRIC, "value": ms_per_step, "unit": "ms/iter", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": False,
                "scaling": "strong" if name in ("cfg2", "cfg5") else "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded generators in trnopt.synthetic)",
                "config": {"workload": name, **cfg, "path": path, "shards": world, "exchange": exchange,
                           "l2": "flushed between timed steps (256 MB write)"},
                "gpu_launches": 2 * args.steps, "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks}
        print(json.dumps(line), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit("--gpus N > 1 needs torchrun --nproc-per-node N")
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    try:
        if args.workload in ("cfg3", "cfg4", "cfg2conv", "cfg5conv"):
            run_pipeline(args, rank, world, dev)
        else:
            run_ours(args, rank, world, dev)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
