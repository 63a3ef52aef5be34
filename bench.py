#!/usr/bin/env python3
"""bench.py -- the headline measurement of the B200 MLP GEMM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--dtype D --N n --K k --M m]

Workload (default): the i8i8 -> int32 square GEMM, N = K = M = 4096, seeded
int8 operands U{-127..127}, bit-exact against an int64 dot product.  A step
is one GEMM.  W untimed warm-up steps, then exactly K timed steps, each
bracketed by its own CUDA-event pair on the launching stream; a 256 MiB
buffer (> the 126 MB L2) is read before every timed step, outside the
event pair, so every step starts with a cold L2 (of clean lines: no dirty
write-back competes with the timed GEMM).  Under torchrun each
rank runs its own M-slice of a G-times wider GEMM (weak scaling, no data
collective); the time is the max over ranks.

One JSON line on rank 0 with value (whole-job TOPS), e2e (the same metric
through the C ABI from pinned host buffers, copies inside the timed
region), roofline (the GEMM kernel against the measured peak), cpu_baseline
(the reference's CPU dot product, re-run as an OpenMP host GEMM on a bounded
sample), clocks (NVML samples during the timed region) and gpu_launches.

--impl reference times the reference's CPU implementation of the path (the
oracle's restatement of its host dot product, main.swift:563-583) on all host
cores, for the same workload and metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "fp8-mlp-metal41-bench_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

FLUSH_BYTES = 256 << 20
BASELINE_METRIC = "TFLOPS/TOPS per dtype×shape at 1/2/4/8 B200; % of tensor-peak or HBM roofline"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--dtype", default="i8i8")
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--M", type=int, default=4096)
    ap.add_argument("--tile", default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def unit_of(dtype):
    return "TOPS" if dtype == "i8i8" else "TFLOPS"


def workload_name(dtype, N, K, M):
    sq = N == K == M
    shape = "square" if sq else ("thin" if N == 1 else "custom")
    return f"{dtype} {shape} GEMM N={N} K={K} M={M}"


def peaks():
    """Roofline denominators from MEASURED_PEAKS.json (driver-measured), else
    the recipe's fallback.  Non-bf16 kinds scale the measured bf16 burst by
    the B200's dense-rate ratio (i8 / f8f6f4 2x, mxf4 4x)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    src = "measured"
    try:
        with open(path) as f:
            mp = json.load(f)
        hbm, bf16 = float(mp["hbm_gbs"]), float(mp["bf16_tflops"])
    except (OSError, ValueError, KeyError):
        hbm, bf16, src = 6650.0, 1590.0, "fallback"
    return hbm, bf16, src


KIND_RATIO = {"f16": 1.0, "i8": 2.0, "f8f6f4": 2.0, "mxf4": 4.0}


class ClockSampler:
    """NVML SM clock / throttle-reason samples while the timed region runs."""

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.err = None

    def __enter__(self):
        try:
            import pynvml as N
            N.nvmlInit()
            self._N = N
            self._h = N.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self._h, N.NVML_CLOCK_SM)
        except Exception as e:   # NVML missing: report it, never fail the bench
            self.err = str(e)
            return self
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def _run(self):
        N = self._N
        names = {
            "gpu_idle": getattr(N, "nvmlClocksEventReasonGpuIdle", 0x1),
            "applications_clocks_setting": getattr(N, "nvmlClocksEventReasonApplicationsClocksSetting", 0x2),
            "sw_power_cap": getattr(N, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_slowdown": getattr(N, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "sync_boost": getattr(N, "nvmlClocksEventReasonSyncBoost", 0x10),
            "sw_thermal_slowdown": getattr(N, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "hw_thermal_slowdown": getattr(N, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "hw_power_brake_slowdown": getattr(N, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        while not self._stop.is_set():
            try:
                self.samples.append(N.nvmlDeviceGetClockInfo(self._h, N.NVML_CLOCK_SM))
                r = N.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for k, bit in names.items():
                    if r & bit and k != "gpu_idle":
                        self.reasons.add(k)
            except Exception as e:
                self.err = str(e)
                break
            time.sleep(0.0005)

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=2)

    def summary(self):
        d = {"sm_mhz": statistics.median(self.samples) if self.samples else None,
             "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
             "samples": len(self.samples), "source": "nvml, polled every 0.5 ms during the timed steps"}
        if self.err:
            d["error"] = self.err
        return d


# ---------------------------------------------------------------------------------
# CPU side: the reference's CPU dot product as a multithreaded host GEMM
# ---------------------------------------------------------------------------------
def cpu_sample(dtype, N, K, M, seconds, seed=0):
    """Time the oracle's host GEMM on rows of the same workload for about
    `seconds`; returns (TOPS-or-TFLOPS, rows, threads, elapsed)."""
    import oracle
    from mlpgemm import formats as F
    from mlpgemm.data import Operands
    ops = Operands(N, K, M, "seeded", seed)
    threads = oracle.num_threads()
    if dtype == "i8i8":
        X, W = ops.X(dtype), ops.W(dtype)

        def go(r0, nr):
            return oracle.host_gemm_i32(X, W, K, M, r0, nr, threads)
    else:
        xf = oracle.decode_x(dtype, ops.X(dtype), ops.xscale(dtype), N, K).astype(np.float32)
        wf = oracle.decode_w(dtype, ops.W(dtype), ops.wscale(dtype), K, M).astype(np.float32)

        def go(r0, nr):
            return oracle.host_gemm_f32(xf, wf, r0, nr, threads)
    del F
    # calibrate on a few rows, then size the sample to ~`seconds`
    nr = min(N, 4)
    t0 = time.perf_counter()
    go(0, nr)
    dt = max(time.perf_counter() - t0, 1e-4)
    rows = int(max(1, min(N, nr * seconds / dt)))
    t0 = time.perf_counter()
    go(0, rows)
    el = time.perf_counter() - t0
    return 2.0 * rows * K * M / el / 1e12, rows, threads, el


def reference_arm(a):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    dtype, N, K, M = a.dtype, a.N, a.K, a.M
    import oracle
    from mlpgemm.data import Operands
    ops = Operands(N, K, M, "seeded", 0)
    threads = oracle.num_threads()
    X, W = ops.X(dtype), ops.W(dtype)
    if dtype != "i8i8":
        xf = oracle.decode_x(dtype, X, ops.xscale(dtype), N, K).astype(np.float32)
        wf = oracle.decode_w(dtype, W, ops.wscale(dtype), K, M).astype(np.float32)

    def step(nr):
        if dtype == "i8i8":
            oracle.host_gemm_i32(X, W, K, M, 0, nr, threads)
        else:
            oracle.host_gemm_f32(xf, wf, 0, nr, threads)

    # rows per step: ~1 s of work, so warmup + steps stays within a few minutes
    t0 = time.perf_counter()
    step(min(N, 4))
    dt = max(time.perf_counter() - t0, 1e-4)
    budget = max(0.05, min(1.0, 150.0 / max(1, a.steps + a.warmup)))
    rows = int(max(1, min(N, min(N, 4) * budget / dt)))
    for _ in range(a.warmup):
        step(rows)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        step(rows)
    el = time.perf_counter() - t0
    v = 2.0 * rows * K * M * a.steps / el / 1e12
    unit = unit_of(dtype)
    sample = f"{rows} of {N} output rows per step (all {M} columns, K={K}), OpenMP over {threads} threads"
    line = {
        "impl": "reference", "metric": BASELINE_METRIC, "value": v, "unit": unit,
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": el / a.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8" if dtype == "i8i8" else "f32", "data": "synthetic",
        "config": {"workload": workload_name(dtype, N, K, M), "N": N, "K": K, "M": M,
                   "impl_detail": "the reference's host dot product (main.swift:563-583) run as a "
                                  "multithreaded host GEMM (oracle/mlp_oracle.c)"},
        "cpu_baseline": {"value": v, "unit": unit, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


# ---------------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------------
def traffic_for(kernel_key):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            t = json.load(f)
        return t.get(kernel_key, {}).get("dram_bytes_per_launch")
    except (OSError, ValueError):
        return None


def ours(a):
    from mlpgemm import dist_util as DU
    from mlpgemm import formats as F
    from mlpgemm import lib as G
    from mlpgemm.data import Operands

    world, rank, local = dist_env()
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    G.init(local)
    dtype, N, K, M = a.dtype, a.N, a.K, a.M
    dt = F.CODE[dtype]
    tile = a.tile or G.tile_names()[G.default_tile(dt, N, K, M)]
    ti = G.tile_index(tile)
    # weak scaling: rank r owns columns [r*M, (r+1)*M) of a world*M-wide GEMM;
    # its W slice is generated with its own seed (independent column block)
    ops = Operands(N, K, M, "seeded", seed=rank)
    X = G.DeviceBuffer(local, ops.X(dtype).nbytes).upload(ops.X(dtype))
    W = G.DeviceBuffer(local, ops.W(dtype).nbytes).upload(ops.W(dtype))
    xs, ws = ops.xscale(dtype), ops.wscale(dtype)
    XS = G.DeviceBuffer(local, xs.nbytes).upload(xs) if xs is not None else None
    WS = G.DeviceBuffer(local, ws.nbytes).upload(ws) if ws is not None else None
    Y = G.DeviceBuffer(local, N * M * 4).zero()
    wsb = G.workspace_size(dt, ti, N, K, M)
    WSP = G.DeviceBuffer(local, wsb).zero() if wsb else None
    FL = G.DeviceBuffer(local, FLUSH_BYTES).zero()

    # parity gate on this rank's own output before timing (sample rows)
    G.run(local, dt, ti, X, W, Y, N, K, M, XS, WS, WSP, wsb)
    G.sync(local)
    ok = check_rows(G, ops, dtype, Y, N, M)

    def barrier():
        if dist is not None:
            dist.barrier()

    barrier()
    with ClockSampler(local) as clk:
        ms = G.time(local, dt, ti, X, [W], Y, N, K, M, xscale=XS, wscales=[WS] if WS else None,
                    workspace=WSP, workspace_bytes=wsb, warmup=a.warmup, iters=a.steps,
                    flush=FL, flush_bytes=FLUSH_BYTES)
    barrier()
    total_ms = float(sum(ms))
    if dist is not None:
        total_ms = DU.reduce_max(dist, total_ms, "cuda")
        ok = DU.reduce_all(dist, ok, "cuda")
    flops = 2.0 * N * K * M
    value = DU.weak_scaling_rate(flops, world, a.steps, total_ms)

    # end to end through the C ABI: pinned host X in, device GEMM, host Y out,
    # every rank at once (they share the host's memory); the job's rate is set
    # by the slowest rank, as for `value`
    if dist is not None:
        dist.barrier()
    e2e = e2e_measure(G, local, dtype, dt, ti, ops, X, W, XS, WS, Y, WSP, wsb, N, K, M, a)
    if dist is not None:
        t_max = DU.reduce_max(dist, e2e["ms_per_step"], "cuda")
        t_ser = DU.reduce_max(dist, e2e["serial"]["ms_per_step"], "cuda")
        dist.barrier()
        dist.destroy_process_group()
    else:
        t_max, t_ser = e2e["ms_per_step"], e2e["serial"]["ms_per_step"]
    flops_job = 2.0 * N * K * M * world
    e2e.update({"value": flops_job / (t_max / 1e3) / 1e12, "ms_per_step": t_max,
                "h2d_bytes_per_step": e2e["h2d_bytes_per_step"] * world,
                "d2h_bytes_per_step": e2e["d2h_bytes_per_step"] * world, "ranks": world})
    e2e["serial"].update({"value": flops_job / (t_ser / 1e3) / 1e12, "ms_per_step": t_ser})
    if rank != 0:
        return 0 if ok else 3

    hbm, bf16, src = peaks()
    kind = F.TC_KIND[dtype] if not tile.startswith("gemv") else "hbm"
    per_launch_s = statistics.mean(ms) / 1e3
    if kind == "hbm":
        achieved = F.algorithmic_bytes(dtype, N, K, M) / per_launch_s / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "peak_source": f"{src} hbm_gbs (MEASURED_PEAKS.json)" if src == "measured" else "fallback 6650 GB/s"}
    else:
        peak = bf16 * KIND_RATIO[kind]
        achieved = flops / per_launch_s / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak,
                "unit": "TOPS" if dtype == "i8i8" else "TFLOP/s",
                "peak_source": (f"{src}: bf16_tflops burst {bf16} x {KIND_RATIO[kind]:g} "
                                f"(dense kind::{kind} : bf16 rate of B200)")}
    roof["frac"] = roof["achieved"] / roof["peak"]
    key = f"{dtype} {tile} N={N} K={K} M={M}"
    roof["traffic"] = traffic_for(key)
    roof["algorithmic_bytes"] = F.algorithmic_bytes(dtype, N, K, M)
    roof["kernel_ms_mean"] = per_launch_s * 1e3
    roof["kernel_ms_median"] = statistics.median(ms)

    line = {
        "metric": BASELINE_METRIC, "value": value, "unit": unit_of(dtype), "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": total_ms / a.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8" if dtype == "i8i8" else dtype, "data": "synthetic",
        "config": {"workload": workload_name(dtype, N, K, M), "N": N, "K": K, "M": M,
                   "tile": tile, "per_gpu": f"each rank computes its own [{N},{M}] column block "
                                             f"of a [{N},{M * world}] output",
                   "l2": "flushed: a 256 MiB buffer is read before every timed step, outside its events",
                   "operands": "seeded i.i.d. int8 U{-127..127}" if dtype == "i8i8" else "seeded",
                   "accumulate": "int32" if dtype == "i8i8" else "f32",
                   "parity": "bit-exact vs int64 dot product" if dtype == "i8i8" else "rel<=1e-3 vs fp64",
                   "parity_ok": ok},
        "e2e": e2e,
        "roofline": roof,
        "gpu_launches": a.steps * G.launches_per_run(dt, ti, N, K, M),
        "clocks": clk.summary(),
    }
    if not a.no_cpu_baseline and world == 1:
        v, rows, thr, el = cpu_sample(dtype, N, K, M, seconds=10.0)
        line["cpu_baseline"] = {"value": v, "unit": unit_of(dtype), "cores": thr, "kind": "port",
                                "sample": f"{rows} of {N} output rows (all {M} columns, K={K}) in "
                                          f"{el:.1f} s: the reference's host dot product "
                                          f"(main.swift:563-583) as an OpenMP host GEMM"}
    print(json.dumps(line))
    return 0 if ok else 3


def check_rows(G, ops, dtype, Y, N, M, nrows=4):
    host = np.empty((N, M), dtype=np.int32 if dtype == "i8i8" else np.float32)
    Y.download(host)
    rows = sorted({0, N - 1, N // 2, min(N - 1, 129)})[:nrows]
    ref = ops.x_rows(dtype, rows) @ ops.w_cols(dtype, np.arange(M))
    got = host[rows].astype(np.float64)
    if dtype == "i8i8":
        return bool(np.array_equal(got, ref))
    rms = float(np.sqrt(np.mean(ref * ref)))
    return bool(np.all(np.abs(got - ref) <= 1e-3 * np.maximum(np.abs(ref), 1e-2 * rms)))


def e2e_measure(G, dev, dtype, dt, ti, ops, X, W, XS, WS, Y, WSP, wsb, N, K, M, a):
    import ctypes
    xh = ops.X(dtype)
    hX = G.lib().gemm_host_alloc(xh.nbytes)
    hY = G.lib().gemm_host_alloc(N * M * 4)
    hXS = None
    xs = ops.xscale(dtype)
    try:
        ctypes.memmove(hX, xh.ctypes.data, xh.nbytes)
        if xs is not None:
            hXS = G.lib().gemm_host_alloc(xs.nbytes)
            ctypes.memmove(hXS, xs.ctypes.data, xs.nbytes)
        iters = max(5, min(a.steps, 30))
        # each step alone: copy in, GEMM, copy out back to back
        ms = G.time_e2e(dev, dt, ti, hX, X, W, Y, hY, N, K, M, hXS, XS, WS, WSP, wsb,
                        warmup=max(3, a.warmup), iters=iters)
        # the serving loop: consecutive steps overlapped two deep (second X / Y set)
        X2 = G.DeviceBuffer(dev, xh.nbytes)
        Y2 = G.DeviceBuffer(dev, N * M * 4)
        XS2 = G.DeviceBuffer(dev, xs.nbytes) if xs is not None else None
        total = G.time_e2e_pipelined(dev, dt, ti, hX, (X, X2), W, (Y, Y2), hY, N, K, M, hXS, (XS, XS2), WS,
                                     WSP, wsb, warmup=max(3, a.warmup), iters=iters)
    finally:
        G.lib().gemm_host_free(hX)
        G.lib().gemm_host_free(hY)
        if hXS:
            G.lib().gemm_host_free(hXS)
    t_serial = statistics.mean(ms) / 1e3
    t = total / iters / 1e3
    h2d = xh.nbytes + (xs.nbytes if xs is not None else 0)
    return {"value": 2.0 * N * K * M / t / 1e12, "unit": unit_of(dtype),
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": N * M * 4,
            "ms_per_step": t * 1e3, "steps": iters,
            "path": "gemm_time_e2e_pipelined: per step pinned host X -> device, gemm_run, device Y -> "
                    "pinned host, consecutive steps overlapped two deep on three streams",
            "serial": {"value": 2.0 * N * K * M / t_serial / 1e12, "ms_per_step": t_serial * 1e3,
                       "path": "gemm_time_e2e: the same three steps back to back"}}


def main():
    a = parse()
    if a.impl == "reference":
        return reference_arm(a)
    return ours(a)


if __name__ == "__main__":
    sys.exit(main())
