"""The bench driver: the reference's Swift host (main.swift) on libgemm.so.

Same flags (main.swift:162-212, including its parse quirks: boolean flags
take no value, every other key consumes one, unknown keys are skipped with
their value, a non-integer value reads as 0, any of --N/--K/--M/--iters
switches from the suite to one custom shape with 4096 defaults), same
header lines, autotune lines, profile file and table (main.swift:616-669),
same exit codes (1 bad arguments / GPU error, 2 library load failure,
3 result mismatch).

Added flags (all optional): --gpus 1|2|4|8 (sharded across GPUs; run
under torchrun), --shard m|n (split W's columns, the default, or X's rows),
--allgather (gather Y over NCCL, timed separately),
--data ref|seeded, --seed S, --rotate R (R weight copies used round-robin),
--flush (overwrite a >L2 buffer before every timed iteration),
--read-probe BYTES (time a plain streaming read of BYTES from a cold L2,
the practical ceiling of the HBM-bound thin rows, instead of the GEMM).
"""
from __future__ import annotations

import json
import os
import re
import sys
from dataclasses import dataclass, field

import numpy as np

from . import formats as F
from . import lib as G
from .data import Operands


@dataclass
class ShapeCase:
    name: str
    N: int
    K: int
    M: int
    iters: int


# suiteShapes, main.swift:156-160
SUITE = [ShapeCase("square", 4096, 4096, 4096, 100), ShapeCase("thin", 1, 4096, 11008, 200),
         ShapeCase("fat", 2048, 4096, 11008, 50)]

BOOL_FLAGS = ("--suite", "--autotune", "--no-profile", "--allgather", "--flush", "--peak")
FLUSH_BYTES = 256 << 20   # read before each timed launch with --flush: larger than the 126 MB L2


@dataclass
class Args:
    N: int = 4096
    K: int = 4096
    M: int = 4096
    iters: int = 100
    warmup: int = 5
    dtypes: list = field(default_factory=lambda: list(F.DTYPES))
    suite: bool = False
    shape_set: bool = False
    tile: str | None = None
    autotune: bool = False
    use_profile: bool = True
    gpus: int = 1
    shard: str = "m"        # "m": columns of W per GPU; "n": rows of X per GPU
    allgather: bool = False
    data: str = "seeded"
    seed: int = 0
    rotate: int = 1
    flush: bool = False
    peak: bool = False      # tensor-core peak probe instead of the GEMM (tune/peak.swift)
    read_bytes: int = 0     # > 0: streaming-read probe of that many bytes instead of the GEMM


class BenchExit(Exception):
    """Exit with the reference's status code after printing `msg` to stderr."""

    def __init__(self, code: int, msg: str = ""):
        super().__init__(msg)
        self.code = code
        self.msg = msg


def _swift_int(s: str) -> int:
    return int(s) if re.fullmatch(r"[+-]?\d+", s) else 0


def parse_args(argv, tiles=None) -> Args:
    """parseArgs, main.swift:162-212.  `tiles` is the valid --tile list."""
    a = Args()
    i = 0
    while i < len(argv):
        key = argv[i]
        if key in BOOL_FLAGS:
            if key == "--suite":
                a.suite = True
            elif key == "--autotune":
                a.autotune = True
            elif key == "--no-profile":
                a.use_profile = False
            elif key == "--allgather":
                a.allgather = True
            elif key == "--flush":
                a.flush = True
            elif key == "--peak":
                a.peak = True
            i += 1
            continue
        i += 1
        if i >= len(argv):
            break
        if key == "--tile":
            name = argv[i]
            i += 1
            if tiles is not None and name not in tiles:
                raise BenchExit(1, f"Unknown --tile {name} ({', '.join(tiles)})")
            a.tile = name
            continue
        if key == "--dtype":
            name = argv[i]
            i += 1
            if name == "all":
                a.dtypes = list(F.DTYPES)
            elif name in F.DTYPES:
                a.dtypes = [name]
            else:
                raise BenchExit(1, f"Unknown --dtype {name} ({', '.join(F.DTYPES)}, all)")
            continue
        if key == "--shard":
            a.shard = argv[i].lower()
            i += 1
            if a.shard not in ("m", "n"):
                raise BenchExit(1, f"Unknown --shard {a.shard} (m, n)")
            continue
        if key == "--data":
            a.data = argv[i]
            i += 1
            if a.data not in ("ref", "seeded"):
                raise BenchExit(1, f"Unknown --data {a.data} (ref, seeded)")
            continue
        val = _swift_int(argv[i])
        if key == "--N":
            a.N, a.shape_set = val, True
        elif key == "--K":
            a.K, a.shape_set = val, True
        elif key == "--M":
            a.M, a.shape_set = val, True
        elif key == "--iters":
            a.iters, a.shape_set = val, True
        elif key == "--warmup":
            a.warmup = val
        elif key == "--gpus":
            a.gpus = val
        elif key == "--seed":
            a.seed = val
        elif key == "--rotate":
            a.rotate = max(1, val)
        elif key == "--read-probe":
            a.read_bytes = max(0, val)
        i += 1
    return a


def shapes_for(a: Args):
    if a.suite or not a.shape_set:
        return list(SUITE)
    return [ShapeCase("custom", a.N, a.K, a.M, a.iters)]


# ---- profiles (main.swift:312-344, :639-650) ------------------------------------------
def profile_slug(device: str, arch: str) -> str:
    s = f"{device}_{arch}".lower()
    return "".join(c if c.isalnum() else "-" for c in s)


def profile_key(dtype: str, N: int, K: int, M: int) -> str:
    return f"{dtype} N={N} K={K} M={M}"


def encode_profile(device: str, arch: str, tiles: dict) -> str:
    """Pretty-printed, sorted keys, `"key" : value`, '/' escaped: the byte
    format of the reference's JSONEncoder output (profiles/*.json)."""
    obj = {"architecture": arch, "device": device, "tiles": dict(tiles)}
    text = json.dumps(obj, indent=2, sort_keys=True, separators=(",", " : "), ensure_ascii=False)
    return text.replace("/", "\\/")


def load_profile(path: str, use: bool):
    if use and os.path.exists(path):
        try:
            with open(path, encoding="utf-8") as f:
                p = json.load(f)
            if isinstance(p.get("tiles"), dict):
                return dict(p["tiles"])
        except (OSError, ValueError):
            pass
    return {}


# ---- table (main.swift:616-637) ---------------------------------------------------------
def _cell(text: str, width: int, right: bool) -> str:
    pad = " " * max(0, width - len(text))
    return pad + text if right else text + pad


def table_line(shape, n, k, m, dtype, tile, ms, tflops, vs, rel) -> str:
    return " ".join([_cell(shape, 8, False), _cell(n, 6, True), _cell(k, 6, True),
                     _cell(m, 6, True), _cell(dtype, 9, False), _cell(tile, 6, False),
                     _cell(ms, 10, True), _cell(tflops, 8, True), _cell(vs, 8, True),
                     _cell(rel, 10, True)])


def fmt_g3(x: float) -> str:
    """Swift String(format: "%.3g") of a Float (C printf semantics)."""
    return "%.3g" % x


@dataclass
class Row:
    shape: str
    N: int
    K: int
    M: int
    dtype: str
    tile: str
    median_ms: float
    tflops: float
    vs_fp16: str
    ref_rel: float
    gpus: int = 1
    allgather_ms: float | None = None

    def line(self) -> str:
        return table_line(self.shape, str(self.N), str(self.K), str(self.M), self.dtype,
                          self.tile, "%.4f" % self.median_ms, "%.3f" % self.tflops, self.vs_fp16,
                          fmt_g3(self.ref_rel))


def render_table(rows) -> list[str]:
    header = table_line("shape", "N", "K", "M", "dtype", "tile", "median_ms", "tflops",
                        "vs_fp16", "ref_rel")
    return [header, "-" * len(header)] + [r.line() for r in rows]


# ---- sample points and the result check (main.swift:452-466, :560-594) ----------------
def tile_dims(tile: str):
    m = re.fullmatch(r"(\d+)x(\d+)", tile)
    if m:
        return int(m.group(1)), int(m.group(2))
    return 16, 32   # CUDA-core thin-row kernels: the reference's N<=16 tile


def sample_points(N: int, M: int, bm: int, bn: int):
    out = []

    def add(n, m):
        if 0 <= n < N and 0 <= m < M and (n, m) not in out:
            out.append((n, m))

    add(0, 0)
    add(0, min(bn - 1, M - 1))
    add(0, min(bn, M - 1))
    add(min(bm - 1, N - 1), 0)
    add(min(bm, N - 1), min(bn, M - 1))
    add(N - 1, M - 1)
    return out


def check_samples(ops: Operands, dtype: str, Y: np.ndarray, points, shape_name: str,
                  col_offset: int = 0) -> float:
    """fp64 (int64 for i8i8) dot products at the sample points.  i8i8 must be
    bit-exact; float dtypes fail like the reference when rel > 1e-2 and
    abs > 1e-3.  Returns the max relative error (the table's ref_rel)."""
    rows = sorted({n for n, _ in points})
    cols = sorted({m for _, m in points})
    xr = ops.x_rows(dtype, rows)
    wc = ops.w_cols(dtype, [c + col_offset for c in cols])
    ref = xr @ wc                                  # float64 [rows, cols]
    ri = {n: i for i, n in enumerate(rows)}
    ci = {m: j for j, m in enumerate(cols)}
    max_rel = 0.0
    for n, m in points:
        r = ref[ri[n], ci[m]]
        got = Y[n, m]
        if dtype == "i8i8":
            if int(got) != int(round(r)):
                raise BenchExit(3, f"{shape_name} i8i8 mismatch Y[{n},{m}] gpu={int(got)} ref={int(round(r))}")
            continue
        ab = abs(float(got) - r)
        rel = ab / max(1e-6, abs(r))
        max_rel = max(max_rel, rel)
        if not np.isfinite(got) or (rel > 1e-2 and ab > 1e-3):
            raise BenchExit(3, f"{shape_name} {dtype} mismatch Y[{n},{m}] gpu={float(got):.6g} "
                               f"ref={r:.6g} abs={ab:.3g} rel={rel:.3g}")
    return float(np.float32(max_rel))


# ---- one GPU ----------------------------------------------------------------------------
class Runner:
    """Device buffers for one shape on one GPU, reused across dtypes."""

    def __init__(self, device: int, ops: Operands, M_local: int | None = None):
        self.device = device
        self.ops = ops
        self.bufs: dict = {}

    def dev(self, key, arr) -> G.DeviceBuffer:
        b = self.bufs.get(key)
        if b is None or b.nbytes < arr.nbytes:
            b = G.DeviceBuffer(self.device, arr.nbytes).upload(arr)
            self.bufs[key] = b
        return b

    def scratch(self, key, nbytes) -> G.DeviceBuffer:
        b = self.bufs.get(key)
        if b is None or b.nbytes < nbytes:
            b = G.DeviceBuffer(self.device, max(nbytes, 1)).zero()
            self.bufs[key] = b
        return b

    def close(self):
        for b in self.bufs.values():
            b.close()
        self.bufs.clear()


def run_dtype(rn: Runner, dtype: str, tile: str, N, K, M, warmup, iters, W=None, wscale=None,
              rotate=1, flush=False):
    """Time one dtype/tile; returns (per-iteration ms, Y as numpy)."""
    ops = rn.ops
    dt = F.CODE[dtype]
    ti = G.tile_index(tile)
    X = rn.dev(("X", ops.x_name(dtype)), ops.X(dtype))
    xs = ops.xscale(dtype)
    XS = rn.dev("xscale", xs) if xs is not None else None
    Warr = ops.W(dtype) if W is None else W
    wsarr = ops.wscale(dtype) if wscale is None else wscale
    Ws = [rn.dev(("W", ops.w_name(dtype), r, id(Warr)), Warr) for r in range(rotate)]
    WS = [rn.dev(("wscale", r, id(wsarr)), wsarr) for r in range(rotate)] if wsarr is not None else None
    Y = rn.scratch(("Y", N, M), N * M * 4)
    wsb = G.workspace_size(dt, ti, N, K, M)
    WSP = rn.scratch(("ws", wsb), wsb) if wsb else None
    fl = rn.scratch("flush", FLUSH_BYTES) if flush else None
    Y.zero()
    ms = G.time(rn.device, dt, ti, X, Ws, Y, N, K, M, xscale=XS, wscales=WS, workspace=WSP,
                workspace_bytes=wsb, warmup=warmup, iters=iters, flush=fl,
                flush_bytes=FLUSH_BYTES if flush else 0)
    host = np.empty((N, M), dtype=np.int32 if dtype == "i8i8" else np.float32)
    Y.download(host)
    return ms, host


def candidate_tiles(dtype: str, N: int, K: int, M: int):
    dt = F.CODE[dtype]
    return [t for i, t in enumerate(G.tile_names()) if G.tile_supported(dt, i, N, K, M)]


def choose_tile(a: Args, profile: dict, dtype: str, N: int, K: int, M: int) -> str:
    """chosenTile, main.swift:350-357: --tile, then the profile, then the default."""
    names = G.tile_names()
    dt = F.CODE[dtype]
    if a.tile is not None:
        if G.tile_supported(dt, names.index(a.tile), N, K, M):
            return a.tile
        print(f"note: tile {a.tile} cannot run {dtype} at N={N} K={K} M={M}; using the default",
              file=sys.stderr)
    if a.use_profile:
        t = profile.get(profile_key(dtype, N, K, M))
        if t in names and G.tile_supported(dt, names.index(t), N, K, M):
            return t
    return names[G.default_tile(dt, N, K, M)]


def bench_shape(a: Args, shape: ShapeCase, rn: Runner, profile: dict, out=print):
    N, K, M = shape.N, shape.K, shape.M
    flops = 2.0 * N * K * M
    medians = {}
    rows = []
    for dtype in a.dtypes:
        if not F.layout_ok(dtype, N, K, M):
            raise BenchExit(1, f"{dtype} needs even X/W counts and K a multiple of 32 "
                               f"(128 for FP8 × MXFP4)")
        tile = choose_tile(a, profile, dtype, N, K, M)
        if a.autotune:
            tune_iters = max(5, min(20, shape.iters // 5))
            results = []
            # every candidate is timed with a cold L2 (a >L2 buffer read before each
            # launch): a tile chosen on L2-resident weights would be the wrong one for
            # weights that stream from HBM, which is the thin row's whole cost
            for cand in candidate_tiles(dtype, N, K, M):
                ms, _ = run_dtype(rn, dtype, cand, N, K, M, 2, tune_iters, rotate=a.rotate,
                                  flush=True)
                results.append((cand, sorted(ms)[len(ms) // 2]))
            results.sort(key=lambda r: r[1])
            tile = results[0][0]
            profile[profile_key(dtype, N, K, M)] = tile
            top = " | ".join("%s %.4f" % (t, m) for t, m in results[:4])
            out(f"autotune {shape.name} {dtype}: {top} ms")
        bm, bn = tile_dims(tile)
        pts = sample_points(N, M, bm, bn)
        out(f"running {shape.name} {dtype} tile {tile}")
        sys.stdout.flush()
        ms, Y = run_dtype(rn, dtype, tile, N, K, M, a.warmup, shape.iters, rotate=a.rotate,
                          flush=a.flush)
        if any(t <= 0 for t in ms):
            raise BenchExit(1, "GPU timestamps unavailable")
        med = sorted(ms)[len(ms) // 2] / 1000.0
        medians[dtype] = med
        rel = check_samples(rn.ops, dtype, Y, pts, shape.name)
        if dtype == "fp16":
            vs = "1.000"
        elif "fp16" in medians:
            vs = "%.3f" % (medians["fp16"] / med)
        else:
            vs = "-"
        rows.append(Row(shape.name, N, K, M, dtype, tile, med * 1000.0, flops / med / 1e12, vs, rel))
    return rows


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    try:
        return _main(argv)
    except BenchExit as e:
        if e.msg:
            print(e.msg, file=sys.stderr)
        return e.code
    except G.GemmError as e:
        print(str(e), file=sys.stderr)
        return 2 if e.code == G.GEMM_ERR_INIT else 1


# ---- peak probe (tune/peak.swift, `./run_tune.sh peak`) ------------------------------------
PEAK_KINDS = [(0, "tcgen05 kind::f16"), (1, "tcgen05 kind::i8"), (2, "tcgen05 kind::f8f6f4"),
              (3, "tcgen05 kind::mxf8f6f4"), (4, "tcgen05 kind::mxf4"), (5, "tcgen05 kind::f16 x2"),
              (6, "tcgen05 kind::i8 x2"), (7, "tcgen05 kind::f8f6f4 x2"),
              (8, "tcgen05 kind::f16 x2 B MN-major"), (9, "tcgen05 kind::i8 x2 B MN-major"),
              (10, "tcgen05 kind::f8f6f4 x2 B MN-major"), (11, "tcgen05 kind::mxf8f6f4 x2"),
              (12, "tcgen05 kind::mxf4 x2"), (13, "kind::mxf8f6f4 x2 + SF copies"),
              (14, "kind::mxf4 x2 + SF copies")]
PEAK_REPS = 4096


def run_peak(a) -> int:
    """Dense tensor-core peak per MMA kind: MMAs on operands resident in shared
    memory, no DRAM traffic (tune/peak.metal:29-87, host tune/peak.swift:31-65).
    `x2` rows use CTA pairs (cta_group::2).  --iters sets the timed launches
    (median reported); the reference's default is 10."""
    if G.device_count() < 1:
        raise BenchExit(1, "No CUDA device")
    G.init(0)
    name, _, sms = G.device_info(0)
    iters = a.iters if a.shape_set else 10
    print(f"device: {name}  ctas={sms} R={PEAK_REPS}")
    print("%-28s %12s" % ("kernel", "TFLOPS/TOPS"))
    for kind, label in PEAK_KINDS:
        print("%-28s %12.1f" % (label, G.peak_probe(0, kind, PEAK_REPS, iters)))
    sys.stdout.flush()
    return 0


def run_read_probe(a) -> int:
    """A plain streaming read of --read-probe bytes (rounded up to 16), each
    timed launch after a 256 MiB L2 flush: the practical HBM ceiling that the
    thin rows (N <= 16, main.swift:146-150) are reported against.  --iters sets
    the timed launches (default 100), --warmup the untimed ones."""
    if G.device_count() < 1:
        raise BenchExit(1, "No CUDA device")
    G.init(0)
    nb = (a.read_bytes + 15) // 16 * 16
    iters = a.iters if a.shape_set else 100
    buf = G.DeviceBuffer(0, nb).zero()
    flush = G.DeviceBuffer(0, FLUSH_BYTES).zero()
    ms = G.read_probe(0, buf, nb, warmup=max(a.warmup, 1), iters=iters, flush=flush, flush_bytes=FLUSH_BYTES)
    med, mean = float(np.median(ms)), float(np.mean(ms))
    print(f"read probe: {nb} bytes, cold L2, {iters} launches")
    print(f"median {med * 1e3:.2f} us  mean {mean * 1e3:.2f} us  {nb / (mean * 1e-3) / 1e9:.0f} GB/s (mean)")
    sys.stdout.flush()
    return 0


def _main(argv) -> int:
    try:
        tiles = G.tile_names()
    except G.GemmError as e:
        raise BenchExit(2, f"Failed loading libgemm.so: {e}")
    a = parse_args(argv, tiles)
    if a.peak:
        return run_peak(a)
    if a.read_bytes > 0:
        return run_read_probe(a)
    shapes = shapes_for(a)
    for s in shapes:
        if s.N <= 0 or s.K <= 0 or s.M <= 0 or s.iters <= 0:
            raise BenchExit(1, "N, K, M, iters must be > 0")
    if a.gpus > 1 or int(os.environ.get("WORLD_SIZE", "1")) > 1:
        from . import shard
        return shard.main_sharded(a, shapes)
    if G.device_count() < 1:
        raise BenchExit(1, "No CUDA device")
    G.init(0)
    name, arch, _ = G.device_info(0)
    print(f"device: {name}")
    print("timing: gpu")
    print(f"dtypes: {','.join(a.dtypes)}")
    print("shapes: " + " | ".join(f"{s.name} N={s.N} K={s.K} M={s.M} iters={s.iters}" for s in shapes))
    print(f"loaded: {G.LIB_PATH}")
    slug = profile_slug(name, arch)
    ppath = os.path.join(os.getcwd(), "profiles", f"{slug}.json")
    profile = load_profile(ppath, a.use_profile)
    print(f"architecture: {arch}")
    if a.autotune:
        print(f"tiles: autotune (writes {ppath})")
    elif a.tile is not None:
        print(f"tiles: --tile {a.tile}")
    elif profile:
        print(f"tiles: profile {ppath}")
    else:
        print("tiles: built-in defaults (run --autotune to fit this device)")
    print(f"data: {a.data} seed={a.seed}" + (f" rotate={a.rotate}" if a.rotate > 1 else "")
          + (" flush" if a.flush else ""))
    rows = []
    for s in shapes:
        ops = Operands(s.N, s.K, s.M, a.data, a.seed)
        rn = Runner(0, ops)
        try:
            rows += bench_shape(a, s, rn, profile)
        finally:
            rn.close()
    if a.autotune:
        try:
            os.makedirs(os.path.dirname(ppath), exist_ok=True)
            with open(ppath, "w", encoding="utf-8") as f:
                f.write(encode_profile(name, arch, profile))
            print(f"wrote profile: {ppath}")
        except OSError as e:
            print(f"could not write profile {ppath}: {e}", file=sys.stderr)
    print("")
    for line in render_table(rows):
        print(line)
    print("ok")
    sys.stdout.flush()
    return 0
