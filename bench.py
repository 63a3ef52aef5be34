#!/usr/bin/env python3
"""bench.py -- the headline measurement of the B200 MLP GEMM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--dtype D --N n --K k --M m --tile T]
                    [--no-suite] [--no-gathers] [--no-cpu-baseline]

Workload (default): the fat row of the reference's suite, f8f8 (E4M3 x
E4M3 -> f32), N=2048, K=4096, M=11008, operands RNE-rounded from N(0,1) with
a fixed seed, M-sharded across the GPUs of the job (strong scaling): X is
broadcast once over NCCL, rank g computes the columns [m0_g, m0_g + w_g) of
Y from its column block of W (32-column aligned), and N=1 is the whole GEMM.
A step is one GEMM on every rank.  W untimed warm-up steps, then exactly K
timed steps, each between its own CUDA-event pair on the launching stream;
a 256 MiB buffer (> the 126 MB L2) is read before every timed step, outside
its events, so every step starts with a cold L2 holding only clean lines.
The step time of the job is the max over ranks; value = 2*N*K*M per step /
that time.

The JSON line (rank 0) carries, besides the contract's keys:
  parity     this rank's block checked on whole rows against an fp64 numpy
             dot product of the decoded operands (max rel <= 1e-3), every rank
  e2e        the same metric through the C ABI from pinned host buffers: every
             step copies X in, runs the GEMM and copies the rank's Y block out
  roofline   the GEMM kernel against the measured peak (MEASURED_PEAKS.json)
  clocks     NVML SM clock and throttle reasons sampled every 0.5 ms while any
             timed GPU region runs (warm-up, timed steps and the suite), per rank
  sharded_suite (N > 1) every dtype at the fat shape, M-sharded like the
             headline, cold L2, max over ranks, parity on every rank
  sharded    (N > 1) the collectives beside the GEMM, timed separately: NCCL
             broadcast of X, NCCL all-gather of the M-sharded Y + permute, the
             N-sharded GEMM with its in-place NCCL all-gather, and the fused
             GEMM + all-gather over NVLink peer stores (gemm_run_gather), whose
             Y must equal the NCCL-gathered Y bit for bit on every rank
  suite      (N = 1) all 30 dtype x shape rows of the reference's suite
             (main.swift:156-160) on their default tiles, cold L2, with time,
             rate, fraction of the measured per-kind peak (thin row: of HBM),
             fraction of the tcgen05 probe peak, parity and clocks per row
  probe      (N = 1) gemm_peak_probe per tcgen05 kind (operands resident in
             shared memory)
  cpu_baseline (N = 1) the reference's CPU dot product as an OpenMP host GEMM

--impl reference times the reference's CPU implementation of the path (the
oracle's restatement of its host dot product, main.swift:577-583) on all host
cores, for the same workload, metric and config (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "fp8-mlp-metal41-bench_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

FLUSH_BYTES = 256 << 20
BASELINE_METRIC = "TFLOPS/TOPS per dtype×shape at 1/2/4/8 B200; % of tensor-peak or HBM roofline"
# the reference's suite shapes (main.swift:156-160); iterations per suite row
SUITE = [("square", 4096, 4096, 4096, 50), ("fat", 2048, 4096, 11008, 50), ("thin", 1, 4096, 11008, 100)]
KIND_RATIO = {"f16": 1.0, "i8": 2.0, "f8f6f4": 2.0, "mxf4": 4.0}
PROBE_KIND = {"f16": 0, "i8": 1, "f8f6f4": 2, "mxf8f6f4": 3, "mxf4": 4,
              "f16_pair_bmn": 8, "i8_pair_bmn": 9, "f8f6f4_pair_bmn": 10,
              "mxf8f6f4_pair": 11, "mxf4_pair": 12, "mxf8f6f4_pair_cp": 13, "mxf4_pair_cp": 14}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--dtype", default="f8f8")
    ap.add_argument("--N", type=int, default=2048)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--M", type=int, default=11008)
    ap.add_argument("--tile", default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-suite", action="store_true",
                    help="skip the 30-row suite and the peak probe (N = 1) or the sharded fat-row suite (N > 1)")
    ap.add_argument("--no-gathers", action="store_true")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def unit_of(dtype):
    return "TOPS" if dtype == "i8i8" else "TFLOPS"


def shape_name(N, K, M):
    for name, n, k, m, _ in SUITE:
        if (n, k, m) == (N, K, M):
            return name
    return "custom"


OPERANDS = {
    "fp16": "X, W half U[-1,1]", "int8": "X half N(0,1), W int8 U{-127..127}",
    "i8i8": "X, W int8 U{-127..127}", "fp8": "X half N(0,1), W RNE_E4M3(N(0,1))",
    "f8f8": "X, W RNE_E4M3(N(0,1))", "f4f4": "X, W E2M1 codes U{0..15} (unscaled)",
    "mxfp4": "X half N(0,1), W E2M1 U{0..15} [M,K] with UE8M0 U{124..130} per 32",
    "mxfp4/a4": "X, W E2M1 U{0..15} with UE8M0 U{124..130} per 32, W [M,K]",
    "mxfp4/a8": "X RNE_E4M3(N(0,1)) with UE8M0 U{124..130} per 32, W E2M1 [M,K] with UE8M0",
    "mxfp4/f8": "X RNE_E4M3(N(0,1)), W E2M1 [M,K] with UE8M0 U{124..130} per 32",
}


def workload_config(dtype, N, K, M, world):
    """The workload, identical in both arms (no arm-specific keys)."""
    return {"workload": f"{dtype} {shape_name(N, K, M)} GEMM N={N} K={K} M={M}, M-sharded across {world} GPU(s)",
            "dtype": dtype, "N": N, "K": K, "M": M, "gpus": world,
            "operands": f"seeded i.i.d.: {OPERANDS.get(dtype, 'seeded')} (numpy PCG64, seed 0)",
            "accumulate": "int32" if dtype == "i8i8" else "f32",
            "sharding": "W column blocks of 32-column multiples per GPU, X replicated (NCCL broadcast once); "
                        "strong scaling: the same GEMM at every GPU count",
            "l2": "flushed: a 256 MiB buffer is read before every timed step, outside its events"}


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


def nvml_index(local):
    """NVML index of CUDA device `local` (CUDA_VISIBLE_DEVICES may renumber)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    if vis:
        ids = [v.strip() for v in vis.split(",")]
        if local < len(ids) and ids[local].isdigit():
            return int(ids[local])
    return local


REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
               "applications_clocks_setting": 0x2, "sync_boost": 0x10}


# The sampler runs in its own process: it polls NVML every 0.2 ms and writes
# "monotonic-time sm_mhz reason-bits" lines to a file, independently of this
# process's threads (a Python thread would be starved by the interpreter lock
# during short timed regions).  Windows are matched by CLOCK_MONOTONIC, which
# is system-wide on Linux.
_SAMPLER = r"""
import sys, time
try:
    import pynvml as N
    N.nvmlInit()
    h = N.nvmlDeviceGetHandleByIndex(int(sys.argv[1]))
    print("max", N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM), flush=True)
    while True:
        t = time.monotonic()
        m = N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)
        b = N.nvmlDeviceGetCurrentClocksEventReasons(h)
        print("%.6f %d %d" % (t, m, b), flush=True)
        time.sleep(0.0002)
except Exception as e:
    print("error", str(e).replace(chr(10), " "), flush=True)
"""


class ClockSampler:
    """NVML SM clock and throttle reasons of one GPU, sampled by a child
    process every 0.2 ms for the whole run; `window()` marks a timed region
    and summarises the samples taken inside it."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None
        self.err = None

    def __enter__(self):
        import subprocess
        import tempfile
        fd, self.path = tempfile.mkstemp(prefix="clk", suffix=".txt")
        try:
            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER, str(self.index)], stdout=fd,
                                         stderr=subprocess.DEVNULL)
        except OSError as e:
            self.err = str(e)
        os.close(fd)
        # wait (bounded) for the first sample so the first window is covered
        t0 = time.monotonic()
        while self.proc is not None and time.monotonic() - t0 < 20.0:
            if len(self._lines()) >= 2 or self.proc.poll() is not None:
                break
            time.sleep(0.01)
        return self

    def __exit__(self, *a):
        if self.proc is not None and self.proc.poll() is None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def _lines(self):
        try:
            with open(self.path) as f:
                return f.read().splitlines()
        except OSError:
            return []

    def _parse(self):
        mx, samples, err = None, [], self.err
        for ln in self._lines():
            parts = ln.split()
            if not parts:
                continue
            if parts[0] == "max":
                mx = int(parts[1])
            elif parts[0] == "error":
                err = ln[6:]
            elif len(parts) == 3:
                try:
                    samples.append((float(parts[0]), int(parts[1]), int(parts[2])))
                except ValueError:
                    pass   # a line still being written
        return mx, samples, err

    class _Window:
        def __init__(self, clk):
            self.clk = clk
            self.t0 = self.t1 = None

        def __enter__(self):
            self.t0 = time.monotonic()
            return self

        def __exit__(self, *a):
            self.t1 = time.monotonic()

        def summary(self):
            return self.clk.summary(self.t0, self.t1)

    def window(self):
        return ClockSampler._Window(self)

    def summary(self, t0=None, t1=None, windows=None):
        """Samples between t0 and t1 (the whole run when both are None), or
        inside any of `windows` (a list of (t0, t1))."""
        mx, samples, err = self._parse()
        if windows is not None:
            s = [(m, b) for t, m, b in samples if any(a <= t <= z for a, z in windows)]
        else:
            s = [(m, b) for t, m, b in samples if (t0 is None or t >= t0) and (t1 is None or t <= t1)]
        bits = 0
        for _, b in s:
            bits |= b
        d = {"sm_mhz": statistics.median([m for m, _ in s]) if s else None,
             "sm_min_mhz": min((m for m, _ in s), default=None), "sm_max_mhz": mx,
             "reasons": sorted(k for k, v in REASON_BITS.items() if bits & v), "samples": len(s),
             "source": "NVML in a sampler process, every 0.2 ms, samples inside the timed region"}
        if err:
            d["error"] = err
        return d


# ---------------------------------------------------------------------------------
# CPU side: the reference's CPU dot product as a multithreaded host GEMM
# ---------------------------------------------------------------------------------
def _cpu_gemm(dtype, ops):
    import oracle
    N, K, M = ops.N, ops.K, ops.M
    threads = oracle.num_threads()
    if dtype == "i8i8":
        X, W = ops.X(dtype), ops.W(dtype)

        def go(nr):
            return oracle.host_gemm_i32(X, W, K, M, 0, nr, threads)
    else:
        xf = oracle.decode_x(dtype, ops.X(dtype), ops.xscale(dtype), N, K).astype(np.float32)
        wf = oracle.decode_w(dtype, ops.W(dtype), ops.wscale(dtype), K, M).astype(np.float32)

        def go(nr):
            return oracle.host_gemm_f32(xf, wf, 0, nr, threads)
    return go, threads


def cpu_sample(dtype, ops, seconds):
    """The oracle's host GEMM on output rows of the same workload for about
    `seconds`; returns (rate, rows, threads, elapsed)."""
    go, threads = _cpu_gemm(dtype, ops)
    N, K, M = ops.N, ops.K, ops.M
    nr = min(N, 4)
    t0 = time.perf_counter()
    go(nr)
    dt = max(time.perf_counter() - t0, 1e-4)
    rows = int(max(1, min(N, nr * seconds / dt)))
    t0 = time.perf_counter()
    go(rows)
    el = time.perf_counter() - t0
    return 2.0 * rows * K * M / el / 1e12, rows, threads, el


def reference_arm(a):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    from mlpgemm.data import Operands
    dtype, N, K, M = a.dtype, a.N, a.K, a.M
    ops = Operands(N, K, M, "seeded", 0)
    go, threads = _cpu_gemm(dtype, ops)
    # rows per step: about 1 s of work, so warm-up + steps stays within a few minutes
    t0 = time.perf_counter()
    go(min(N, 4))
    dt = max(time.perf_counter() - t0, 1e-4)
    budget = max(0.05, min(1.0, 150.0 / max(1, a.steps + a.warmup)))
    rows = int(max(1, min(N, min(N, 4) * budget / dt)))
    for _ in range(a.warmup):
        go(rows)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        go(rows)
    el = time.perf_counter() - t0
    v = 2.0 * rows * K * M * a.steps / el / 1e12
    unit = unit_of(dtype)
    sample = (f"{rows} of {N} output rows per step (all {M} columns, K={K}): the reference's host dot "
              f"product (main.swift:577-583) as an OpenMP host GEMM over {threads} threads "
              f"(oracle/mlp_oracle.c), on rank 0 only")
    line = {
        "impl": "reference", "metric": BASELINE_METRIC, "value": v, "unit": unit,
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": el / a.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8" if dtype == "i8i8" else "f32", "data": "synthetic",
        "config": workload_config(dtype, N, K, M, world),
        "cpu_baseline": {"value": v, "unit": unit, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    sys.stdout.flush()
    return 0


# ---------------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------------
def traffic_for(key):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            t = json.load(f)
        return t.get(key)
    except (OSError, ValueError):
        return None


def check_rows_of(ops, dtype, Yhost, rows, m0, width, wdec=None):
    """Whole rows [rows, m0:m0+width] of Y against an fp64 numpy dot product of
    the decoded operands (mlpgemm.data).  i8i8 bit-exact, float dtypes
    max rel <= 1e-3 (denominator max(|ref|, 1e-2 rms)).  Returns (ok, max rel)."""
    ref = ops.x_rows(dtype, rows) @ (wdec if wdec is not None else ops.w_cols(dtype, np.arange(m0, m0 + width)))
    got = Yhost[rows].astype(np.float64)
    if dtype == "i8i8":
        return bool(np.array_equal(got, ref)), 0.0
    if not np.all(np.isfinite(got)):
        return False, float("inf")
    rms = float(np.sqrt(np.mean(ref * ref)))
    rel = float(np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1e-2 * rms + 1e-30)))
    return rel <= 1e-3, rel


def parity_rows(N):
    return sorted({0, min(N - 1, 127), min(N - 1, 128), min(N - 1, 255), min(N - 1, 256), N // 2, N - 1})


class Dev:
    """Device buffers of one rank: DeviceBuffer (gemm_alloc) on one GPU,
    torch tensors under torchrun (NCCL needs them)."""

    def __init__(self, G, local, torch=None):
        self.G, self.local, self.torch = G, local, torch
        self.keep = []

    def empty(self, nbytes):
        if self.torch is None:
            b = self.G.DeviceBuffer(self.local, max(1, nbytes))
        else:
            b = self.torch.empty(max(1, nbytes), dtype=self.torch.uint8, device=f"cuda:{self.local}")
        self.keep.append(b)
        return b

    def zeros(self, nbytes):
        b = self.empty(nbytes)
        if self.torch is None:
            b.zero()
        else:
            b.zero_()
        return b

    def upload(self, arr):
        if arr is None:
            return None
        if self.torch is None:
            b = self.G.DeviceBuffer(self.local, arr.nbytes).upload(arr)
        else:
            b = self.torch.from_numpy(np.ascontiguousarray(arr).view(np.uint8).reshape(-1).copy()).to(
                f"cuda:{self.local}")
        self.keep.append(b)
        return b

    def download(self, buf, arr):
        if self.torch is None:
            return buf.download(arr)
        arr.view(np.uint8).reshape(-1)[:] = buf[:arr.nbytes].cpu().numpy()
        return arr


def run_suite(G, clk, FL, probe, hbm, bf16, src):
    """All dtype x shape rows of the suite on device 0, default tiles, cold L2."""
    from mlpgemm import formats as F
    from mlpgemm.data import Operands
    names = G.tile_names()
    rows = []
    windows = []
    shared_w = {}
    read_ceiling = {}   # bytes -> median ms of a plain streaming read of that many bytes
    for sname, N, K, M, iters in SUITE:
        ops = Operands(N, K, M, "seeded", 0)
        # the thin and fat rows share K and M, hence the very same seeded W planes
        for k, v in shared_w.items():
            ops._cache[k] = v
        wdec_cache = {}
        for dtype in F.DTYPES:
            dt = F.CODE[dtype]
            ti = G.default_tile(dt, N, K, M)
            tile = names[ti]
            d = Dev(G, 0)
            X, W = d.upload(ops.X(dtype)), d.upload(ops.W(dtype))
            XS, WS = d.upload(ops.xscale(dtype)), d.upload(ops.wscale(dtype))
            Y = d.zeros(N * M * 4)
            wsb = G.workspace_size(dt, ti, N, K, M)
            WSP = d.zeros(wsb) if wsb else None
            G.run(0, dt, ti, X, W, Y, N, K, M, XS, WS, WSP, wsb)
            G.sync(0)
            host = d.download(Y, np.empty((N, M), np.int32 if dtype == "i8i8" else np.float32))
            wkey = ops.w_name(dtype)
            if wkey not in wdec_cache:
                wdec_cache[wkey] = ops.w_cols(dtype, np.arange(M))
            ok, rel = check_rows_of(ops, dtype, host, parity_rows(N), 0, M, wdec_cache[wkey])
            with clk.window() as w:
                ms = G.time(0, dt, ti, X, [W], Y, N, K, M, xscale=XS, wscales=[WS] if WS is not None else None,
                            workspace=WSP, workspace_bytes=wsb, warmup=3, iters=iters, flush=FL,
                            flush_bytes=FLUSH_BYTES)
            med = statistics.median(ms)
            flops = 2.0 * N * K * M
            kind = F.TC_KIND[dtype]
            if dtype in ("mxfp4/a8", "mxfp4/f8"):
                kind_probe = "mxf8f6f4"
            else:
                kind_probe = kind
            if kind_probe in ("mxf8f6f4", "mxf4") and tile.startswith("256x"):
                kind_probe += "_pair"   # block-scaled MMAs on CTA pairs
            windows.append((w.t0, w.t1))
            row = {"shape": sname, "dtype": dtype, "N": N, "K": K, "M": M, "tile": tile,
                   "ms_median": med, "ms_mean": statistics.mean(ms), "iters": iters,
                   "value": flops / (med / 1e3) / 1e12, "unit": unit_of(dtype),
                   "parity_ok": ok, "max_rel": rel, "clocks": w.summary()}
            if N <= 16:
                nb = F.algorithmic_bytes(dtype, N, K, M)
                gbs = nb / (med / 1e3) / 1e9
                nb16 = (nb + 15) // 16 * 16
                if nb16 not in read_ceiling:
                    rbuf = d.zeros(nb16)
                    read_ceiling[nb16] = statistics.median(
                        G.read_probe(0, rbuf, nb16, warmup=3, iters=iters, flush=FL, flush_bytes=FLUSH_BYTES))
                    del rbuf
                rms = read_ceiling[nb16]
                row.update({"bound": "hbm", "achieved_gbs": gbs, "frac": gbs / hbm,
                            "peak": hbm, "peak_source": f"{src} hbm_gbs",
                            "read_ceiling": {"bytes": nb16, "ms_median": rms, "gbs": nb16 / (rms / 1e3) / 1e9,
                                             "frac": nb16 / (rms / 1e3) / 1e9 / hbm,
                                             "what": "gemm_read_probe: plain 16-byte streaming read of the "
                                                     "same byte count, cold L2"},
                            "of_read_ceiling": rms / med})
            else:
                peak = bf16 * KIND_RATIO[kind]
                pp = probe.get(kind_probe)
                row.update({"bound": "tensor", "kind": kind, "frac": row["value"] / peak, "peak": peak,
                            "peak_source": f"{src} bf16 burst x {KIND_RATIO[kind]:g} (dense kind::{kind})",
                            "probe_kind": kind_probe, "probe_peak": pp,
                            "probe_frac": (row["value"] / pp) if pp else None})
            rows.append(row)
            del d
        if sname == "fat":
            shared_w = {k: v for k, v in ops._cache.items() if k.startswith("w")}
    return rows, windows


def run_sharded_suite(G, torch, dist, world, rank, local, clk, FL, bf16, src, iters=20):
    """Every dtype at the suite's fat shape (N=2048, K=4096, M=11008), M-sharded
    across the job's GPUs as the headline is: each rank runs its column block
    (shard_columns, 32-column aligned) on its default tile with a cold L2 and
    takes the median of `iters` event-timed launches; the job's time is the
    max over ranks and value = 2NKM / that time.  Whole rows of every rank's
    block are checked against an fp64 numpy dot product.  Every rank takes the
    same single all-reduce per dtype whatever happened on it, so an error on
    one rank is reported in the row instead of leaving the others waiting."""
    from mlpgemm import dist_util as DU
    from mlpgemm import formats as F
    from mlpgemm.data import Operands, shard_columns
    from mlpgemm.shard import shard_plan
    N, K, M = 2048, 4096, 11008
    plan = shard_plan(M, world)
    m0, width = plan[rank]
    names = G.tile_names()
    ops = Operands(N, K, M, "seeded", 0)
    windows, tiles = [], {}

    def measure(dtype):
        dt = F.CODE[dtype]
        ti = G.default_tile(dt, N, K, width)
        tiles[dtype] = names[ti]
        d = Dev(G, local, torch)
        X, XS = d.upload(ops.X(dtype)), d.upload(ops.xscale(dtype))
        Wsh, wsc, _, w = shard_columns(ops, dtype, rank, world)
        assert w == width
        W, WS = d.upload(Wsh), d.upload(wsc)
        Y = d.zeros(N * width * 4)
        wsb = G.workspace_size(dt, ti, N, K, width)
        WSP = d.zeros(wsb) if wsb else None
        G.run(local, dt, ti, X, W, Y, N, K, width, XS, WS, WSP, wsb)
        G.sync(local)
        host = d.download(Y, np.empty((N, width), np.int32 if dtype == "i8i8" else np.float32))
        ok, rel = check_rows_of(ops, dtype, host, parity_rows(N), m0, width)
        with clk.window() as win:
            ms = G.time(local, dt, ti, X, [W], Y, N, K, width, xscale=XS,
                        wscales=[WS] if WS is not None else None, workspace=WSP, workspace_bytes=wsb,
                        warmup=3, iters=iters, flush=FL, flush_bytes=FLUSH_BYTES)
        windows.append((win.t0, win.t1))
        return statistics.median(ms), ok, rel

    rows = []
    for dtype, (ms_max, rel_max, ok, err) in zip(F.DTYPES, DU.reduce_rows(dist, f"cuda:{local}", F.DTYPES,
                                                                          measure)):
        kind = F.TC_KIND[dtype]
        peak = bf16 * KIND_RATIO[kind]
        value = 2.0 * N * K * M / (ms_max / 1e3) / 1e12 if ms_max < float("inf") else None
        row = {"shape": "fat", "dtype": dtype, "N": N, "K": K, "M": M, "tile": tiles.get(dtype, ""),
               "width": width, "ms_median_max_over_ranks": ms_max, "iters": iters, "value": value,
               "unit": unit_of(dtype), "kind": kind, "frac_per_gpu": (value / (world * peak)) if value else None,
               "peak_per_gpu": peak, "peak_source": f"{src} bf16 burst x {KIND_RATIO[kind]:g} (dense kind::{kind})",
               "parity_ok": ok, "max_rel": rel_max}
        if err:
            row["error_rank_%d" % rank] = err
        rows.append(row)
    return rows, windows


def e2e_measure(G, dev, dt, ti, ops, dtype, W, WS, Y, WSP, wsb, N, K, width, a, d):
    """Pinned host X in, GEMM of this rank's block, its Y block out, per step."""
    import ctypes
    xh = ops.X(dtype)
    xs = ops.xscale(dtype)
    L = G.lib()
    hX, hY = L.gemm_host_alloc(xh.nbytes), L.gemm_host_alloc(N * width * 4)
    hXS = L.gemm_host_alloc(xs.nbytes) if xs is not None else None
    try:
        ctypes.memmove(hX, xh.ctypes.data, xh.nbytes)
        if xs is not None:
            ctypes.memmove(hXS, xs.ctypes.data, xs.nbytes)
        iters = max(5, min(a.steps, 30))
        X1, X2 = d.empty(xh.nbytes), d.empty(xh.nbytes)
        Y2 = d.empty(N * width * 4)
        XS1 = d.empty(xs.nbytes) if xs is not None else None
        XS2 = d.empty(xs.nbytes) if xs is not None else None
        ms = G.time_e2e(dev, dt, ti, hX, X1, W, Y, hY, N, K, width, hXS, XS1, WS, WSP, wsb,
                        warmup=max(3, a.warmup), iters=iters)
        total = G.time_e2e_pipelined(dev, dt, ti, hX, (X1, X2), W, (Y, Y2), hY, N, K, width, hXS, (XS1, XS2), WS,
                                     WSP, wsb, warmup=max(3, a.warmup), iters=iters)
    finally:
        L.gemm_host_free(hX)
        L.gemm_host_free(hY)
        if hXS:
            L.gemm_host_free(hXS)
    h2d = xh.nbytes + (xs.nbytes if xs is not None else 0)
    return {"ms_per_step": total / iters, "serial_ms_per_step": statistics.mean(ms), "steps": iters,
            "h2d": h2d, "d2h": N * width * 4}


def ours(a):
    from mlpgemm import dist_util as DU
    from mlpgemm import formats as F
    from mlpgemm import lib as G
    from mlpgemm.data import Operands, shard_columns
    from mlpgemm.shard import shard_plan

    world, rank, local = dist_env()
    torch = dist = None
    if world > 1:
        import datetime
        # NCCL's banner would otherwise share stdout with the JSON line
        os.environ.setdefault("NCCL_DEBUG", "WARN")

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    G.init(local)
    dtype, N, K, M = a.dtype, a.N, a.K, a.M
    dt = F.CODE[dtype]
    names = G.tile_names()
    plan = shard_plan(M, world)
    m0, width = plan[rank]
    tile = a.tile or names[G.default_tile(dt, N, K, width)]
    ti = G.tile_index(tile)
    d = Dev(G, local, torch)
    ops = Operands(N, K, M, "seeded", 0)
    hbm, bf16, src = peaks()

    # X: replicated.  Under torchrun rank 0 uploads it and NCCL broadcasts it once.
    xh = ops.X(dtype)
    bcast_ms = None
    if dist is None:
        X = d.upload(xh)
    else:
        # set the communicator up before the timed broadcast (NCCL connects lazily)
        warm = torch.zeros(1 << 20, dtype=torch.uint8, device=f"cuda:{local}")
        dist.broadcast(warm, src=0)
        dist.all_reduce(torch.zeros(1, device=f"cuda:{local}"))
        torch.cuda.synchronize()
        X = d.empty(xh.nbytes)
        if rank == 0:
            X.copy_(torch.from_numpy(xh.view(np.uint8).reshape(-1).copy()))
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dist.broadcast(X, src=0)
        e1.record()
        torch.cuda.synchronize()
        bcast_ms = e0.elapsed_time(e1)
    XS = d.upload(ops.xscale(dtype))
    # this rank's column block of W (and of its scale plane)
    Wsh, wsc, _, w = shard_columns(ops, dtype, rank, world)
    assert w == width
    W = d.upload(Wsh)
    WS = d.upload(wsc)
    Y = d.zeros(N * width * 4)
    wsb = G.workspace_size(dt, ti, N, K, width)
    WSP = d.zeros(wsb) if wsb else None
    FL = d.zeros(FLUSH_BYTES)

    # parity gate on this rank's own block before timing: whole rows, all its columns
    G.run(local, dt, ti, X, W, Y, N, K, width, XS, WS, WSP, wsb)
    G.sync(local)
    host = d.download(Y, np.empty((N, width), np.int32 if dtype == "i8i8" else np.float32))
    prow = parity_rows(N)
    ok, rel = check_rows_of(ops, dtype, host, prow, m0, width)

    def barrier():
        if dist is not None:
            dist.barrier()

    with ClockSampler(nvml_index(local)) as clk:
        barrier()
        with clk.window() as win:
            ms = G.time(local, dt, ti, X, [W], Y, N, K, width, xscale=XS, wscales=[WS] if WS is not None else None,
                        workspace=WSP, workspace_bytes=wsb, warmup=a.warmup, iters=a.steps,
                        flush=FL, flush_bytes=FLUSH_BYTES)
        barrier()
        clocks = win.summary()
        total_ms = float(sum(ms))
        per_launch_ms = statistics.mean(ms)
        if dist is not None:
            total_ms = DU.reduce_max(dist, total_ms, "cuda")
            ok = DU.reduce_all(dist, ok, "cuda")
            rel = DU.reduce_max(dist, rel, "cuda")
        flops = 2.0 * N * K * M
        value = DU.strong_scaling_rate(flops * a.steps, total_ms)

        # end to end through the C ABI, every rank at once (they share the host)
        barrier()
        e = e2e_measure(G, local, dt, ti, ops, dtype, W, WS, Y, WSP, wsb, N, K, width, a, d)
        t_pipe, t_ser = e["ms_per_step"], e["serial_ms_per_step"]
        if dist is not None:
            t_pipe = DU.reduce_max(dist, t_pipe, "cuda")
            t_ser = DU.reduce_max(dist, t_ser, "cuda")
        e2e = {"value": flops / (t_pipe / 1e3) / 1e12, "unit": unit_of(dtype),
               "h2d_bytes_per_step": e["h2d"] * world, "d2h_bytes_per_step": N * M * 4,
               "ms_per_step": t_pipe, "steps": e["steps"], "ranks": world,
               "path": "gemm_time_e2e_pipelined on every rank: per step pinned host X -> device, gemm_run on the "
                       "rank's column block, its Y block -> pinned host; consecutive steps overlapped two deep "
                       "on three streams; the job's step is the slowest rank's",
               "serial": {"value": flops / (t_ser / 1e3) / 1e12, "ms_per_step": t_ser,
                          "path": "gemm_time_e2e: the same three steps back to back"}}

        sharded = None
        if dist is not None and not a.no_gathers:
            sharded = gathers(a, torch, dist, world, rank, local, ops, dtype, N, K, M)
            sharded.update({"bcast_ms": bcast_ms, "plan": [list(p) for p in plan]})
        sharded_suite = None
        if dist is not None and not a.no_suite:
            srows, swin = run_sharded_suite(G, torch, dist, world, rank, local, clk, FL, bf16, src)
            sharded_suite = {"rows": srows, "n": len(srows), "gpus": world,
                             "parity_ok": all(r["parity_ok"] for r in srows),
                             "what": ("every dtype at the fat shape, M-sharded across the job's GPUs like the "
                                      "headline (column blocks of 32-column multiples), default tile per block, "
                                      "L2 flushed before every timed launch; ms = the max over ranks of each "
                                      "rank's median; value = 2NKM / ms for the whole job; frac_per_gpu = "
                                      "value / (gpus x the measured per-kind peak); parity: whole rows of every "
                                      "rank's block against fp64 numpy"),
                             "clocks": clk.summary(windows=swin)}
            ok = ok and sharded_suite["parity_ok"]

        line = None
        if rank == 0:
            kind = F.TC_KIND[dtype]
            achieved = 2.0 * N * K * width / (per_launch_ms / 1e3) / 1e12
            if tile.startswith("gemv") or tile == "16x128" or tile == "stream":
                gbs = F.algorithmic_bytes(dtype, N, K, width) / (per_launch_ms / 1e3) / 1e9
                roof = {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                        "peak_source": f"{src} hbm_gbs (MEASURED_PEAKS.json)"}
            else:
                peak = bf16 * KIND_RATIO[kind]
                roof = {"bound": "tensor", "achieved": achieved, "peak": peak,
                        "unit": "TOPS" if dtype == "i8i8" else "TFLOP/s",
                        "peak_source": (f"{src}: bf16_tflops burst {bf16} x {KIND_RATIO[kind]:g} "
                                        f"(dense kind::{kind} : bf16 rate of B200)")}
            roof["frac"] = roof["achieved"] / roof["peak"]
            tr = traffic_for(f"{dtype} {tile} N={N} K={K} M={width}")
            roof["traffic"] = tr.get("dram_bytes_per_launch") if tr else None
            if tr:
                roof["traffic_note"] = tr.get("note", "")
            roof["algorithmic_bytes"] = F.algorithmic_bytes(dtype, N, K, width)
            roof["kernel_ms_mean"] = per_launch_ms
            roof["kernel_ms_median"] = statistics.median(ms)
            roof["kernel"] = f"{dtype} tile {tile} on rank 0's [{N},{width}] block"
            line = {
                "metric": BASELINE_METRIC, "value": value, "unit": unit_of(dtype), "n_gpus": world,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": total_ms / a.steps,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": {"i8i8": "int8", "f8f8": "e4m3"}.get(dtype, dtype), "data": "synthetic",
                "config": workload_config(dtype, N, K, M, world),
                "tile": tile,
                "parity": {"ok": ok, "max_rel": rel, "rows": prow,
                           "check": ("bit-exact vs an exact dot product" if dtype == "i8i8" else
                                     "max rel <= 1e-3 vs an fp64 numpy dot product of the decoded operands, "
                                     "denominator max(|ref|, 1e-2 rms)"),
                           "scope": "whole rows of every rank's column block"},
                "e2e": e2e, "roofline": roof,
                "gpu_launches": a.steps * G.launches_per_run(dt, ti, N, K, width),
                "clocks": clocks,
            }
            if sharded is not None:
                line["sharded"] = sharded
            if sharded_suite is not None:
                line["sharded_suite"] = sharded_suite
        # per-rank clocks of the timed region
        if dist is not None:
            rec = torch.tensor([clocks["sm_mhz"] or 0.0, clocks["sm_min_mhz"] or 0.0,
                                float(sum(REASON_BITS[r] for r in clocks["reasons"])), float(clocks["samples"])],
                               dtype=torch.float64, device=f"cuda:{local}")
            allr = [torch.zeros_like(rec) for _ in range(world)]
            dist.all_gather(allr, rec)
            if rank == 0:
                line["clocks"]["per_rank"] = [{"sm_mhz": r[0].item(), "sm_min_mhz": r[1].item(),
                                               "reasons": sorted(k for k, v in REASON_BITS.items()
                                                                 if int(r[2].item()) & v),
                                               "samples": int(r[3].item())} for r in allr]
            dist.barrier()
            dist.destroy_process_group()
        if rank != 0:
            return 0 if ok else 3

        if world == 1 and not a.no_suite:
            probe = {}
            for kname, kid in PROBE_KIND.items():
                with clk.window():
                    probe[kname] = G.peak_probe(local, kid, 4096, 5)
            line["probe"] = {k: round(v, 1) for k, v in probe.items()}
            line["probe"]["what"] = ("gemm_peak_probe: tcgen05 MMAs on operands resident in shared memory, one CTA "
                                     "per SM (pairs: one CTA pair per two SMs; *_bmn: B read MN-major; "
                                     "*_cp: with the GEMM's per-stage scale-cell copies)")
            del d, X, W, Y, WSP
            suite, windows = run_suite(G, clk, FL, probe, hbm, bf16, src)
            line["suite"] = {"rows": suite, "n": len(suite), "parity_ok": all(r["parity_ok"] for r in suite),
                             "what": ("every dtype x shape of the reference's suite (main.swift:156-160), "
                                      "default tile, L2 flushed before every timed launch, median of the "
                                      "CUDA-event times; frac = of the measured per-kind peak (thin rows: "
                                      "of the measured HBM copy bandwidth), probe_frac = of gemm_peak_probe"),
                             "clocks": clk.summary(windows=windows)}
            ok = ok and line["suite"]["parity_ok"]
    if world == 1 and not a.no_cpu_baseline:
        v, rows, thr, el = cpu_sample(dtype, ops, seconds=10.0)
        line["cpu_baseline"] = {"value": v, "unit": unit_of(dtype), "cores": thr, "kind": "port",
                                "sample": f"{rows} of {N} output rows (all {M} columns, K={K}) in {el:.1f} s: "
                                          f"the reference's host dot product (main.swift:577-583) as an OpenMP "
                                          f"host GEMM (oracle/mlp_oracle.c)"}
    print(json.dumps(line))
    sys.stdout.flush()
    return 0 if ok else 3


def gathers(a, torch, dist, world, rank, local, ops, dtype, N, K, M):
    """The collectives beside the sharded GEMM, each timed separately (median
    of 5 after a warm-up, max over ranks): the M-sharded Y all-gathered by
    NCCL and permuted to [N, M]; the N-sharded GEMM with its NCCL all-gather
    in place; the fused GEMM + all-gather over NVLink peer stores.  Every
    rank's gathered Y is checked against numpy rows (check_samples) and the
    fused Y against the NCCL-gathered Y bit for bit (mlpgemm.shard)."""
    from mlpgemm import shard
    from mlpgemm.driver import Args, ShapeCase
    sa = Args()
    sa.dtypes = [dtype]
    sa.allgather = True
    sa.data, sa.seed = "seeded", 0
    sa.warmup = 2
    sa.tile = a.tile
    sa.use_profile = False
    sa.gpus = world
    shape = ShapeCase(shape_name(N, K, M), N, K, M, 10)
    _, em = shard.run_shape(sa, shape, torch, dist, world, rank, local, {}, ops=ops)
    _, en = shard.run_shape_rows(sa, shape, torch, dist, world, rank, local, {}, ops=ops)
    _, _, _, _, ag, mblk, mgemm, mpipe, _ = em[0]
    _, _, _, _, nag, nblk, ngemm, npipe, fused = en[0]
    return {"mshard_gemm_ms": mgemm, "allgather_ms": ag, "mshard_pipeline_ms": mpipe,
            "nshard_block": nblk, "nshard_gemm_ms": ngemm, "nshard_gather_ms": nag,
            "nshard_pipeline_ms": npipe, "fused_ms": fused, "fused_equals_nccl": fused is not None,
            "what": ("allgather_ms: NCCL all-gather of the M-sharded Y blocks + permute to [N,M]; "
                     "nshard_gather_ms: rows of X per GPU, W replicated, NCCL all-gather in place into Y; "
                     "fused_ms: gemm_run_gather (N-sharded GEMM whose epilogue stores each Y tile into every "
                     "GPU's Y over NVLink) + a 1-element all-reduce; *_pipeline_ms: GEMM chunks overlapped "
                     "with NCCL all-gathers on a second stream. Medians over 5 runs, max over ranks.")}


def main():
    a = parse()
    if a.impl == "reference":
        return reference_arm(a)
    return ours(a)


if __name__ == "__main__":
    sys.exit(main())
