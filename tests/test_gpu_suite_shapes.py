"""GPU parity at the suite's compute shapes, every dtype on its default tile.

The reference times three shapes (suiteShapes, main.swift:156-160): square
N=K=M=4096, thin N=1 K=4096 M=11008 and fat N=2048 K=4096 M=11008.  The
thin row is covered by tests/test_gpu_parity.py::test_suite_thin_row.  Here
the two compute shapes run through the C ABI with the tile the library
picks by default (the tile the bench times), and their outputs are checked
against the oracle (main.swift:560-594, tightened to fp64 / int64):

  * rows: 4 rows at every 128-row tile boundary (first and last row of each
    128-row tile, so every CTA-pair and 1-CTA tile row is seen from both
    sides) plus 32 seeded random rows, each over ALL M columns, so that
    every column tile, the ragged last column tile and the last wave's
    half tiles are inside the check;
  * whole outputs for i8i8 square (the integer configuration) and f8f8 fat
    (the configuration of the bench's headline).

Bar: i8i8 bit-exact; float dtypes max relative error <= 1e-3 with the
denominator max(|ref|, 1e-2 * rms(ref)).  The unfloored max relative error
(denominator |ref| alone) is printed beside it: it is large only on outputs
that cancel to near zero, where f32 accumulation of K = 4096 terms cannot
hold a relative bound.
"""
import numpy as np
import pytest

import oracle
from mlpgemm import formats as F
from mlpgemm.data import Operands

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3
SHAPES = {"square": (4096, 4096, 4096), "fat": (2048, 4096, 11008)}
WHOLE = {("i8i8", "square"), ("f8f8", "fat")}

_ops_cache = {}


def _ops(shape):
    if shape not in _ops_cache:
        _ops_cache.clear()   # one shape's operands at a time (the fat W planes are large)
        N, K, M = SHAPES[shape]
        _ops_cache[shape] = Operands(N, K, M, "seeded", 0)
    return _ops_cache[shape]


def check_rows(N, seed=0):
    edges = set()
    for t0 in range(0, N, 128):
        edges.update({t0, min(N - 1, t0 + 127)})
    rng = np.random.default_rng(seed)
    rnd = set(rng.choice(N, size=min(N, 32), replace=False).tolist())
    return np.array(sorted(edges | rnd | {N - 1}), dtype=np.int64)


def reference_rows(dtype, ops, rows):
    N, K, M = ops.N, ops.K, ops.M
    X, W = ops.X(dtype), ops.W(dtype)
    if dtype == "i8i8":
        x = np.asarray(X, np.int8).reshape(N, K)[rows].astype(np.float64)
        w = np.asarray(W, np.int8).reshape(K, M).astype(np.float64)
        return (x @ w).astype(np.int64)   # exact: integer partial sums below 2^53
    xd = oracle.decode_x(dtype, X, ops.xscale(dtype), N, K)[rows]
    wd = oracle.decode_w(dtype, W, ops.wscale(dtype), K, M)
    return xd @ wd


def rel_errors(out, ref):
    """(floored max rel, unfloored max rel, fraction of outputs whose
    unfloored rel exceeds 1e-3)."""
    o = out.astype(np.float64)
    err = np.abs(o - ref)
    rms = float(np.sqrt(np.mean(ref * ref)))
    floored = err / np.maximum(np.abs(ref), 1e-2 * rms + 1e-30)
    with np.errstate(divide="ignore", invalid="ignore"):
        unfloored = np.where(ref != 0, err / np.abs(ref), np.where(err == 0, 0.0, np.inf))
    return float(floored.max()), float(unfloored.max()), float(np.mean(unfloored > REL_TOL))


def run_default(G, dtype, ops):
    N, K, M = ops.N, ops.K, ops.M
    dt = F.CODE[dtype]
    ti = G.default_tile(dt, N, K, M)
    tile = G.tile_names()[ti]
    bufs = {}
    for name, arr in (("X", ops.X(dtype)), ("W", ops.W(dtype)), ("XS", ops.xscale(dtype)),
                      ("WS", ops.wscale(dtype))):
        bufs[name] = None if arr is None else G.DeviceBuffer(0, arr.nbytes).upload(arr)
    Y = G.DeviceBuffer(0, N * M * 4).zero()
    wsb = G.workspace_size(dt, ti, N, K, M)
    WSP = G.DeviceBuffer(0, wsb).zero() if wsb else None
    G.run(0, dt, ti, bufs["X"], bufs["W"], Y, N, K, M, bufs["XS"], bufs["WS"], WSP, wsb)
    G.sync(0)
    out = Y.download(np.empty((N, M), np.int32 if dtype == "i8i8" else np.float32))
    for b in list(bufs.values()) + [Y, WSP]:
        if b is not None:
            b.close()
    return tile, out


@pytest.mark.parametrize("shape", list(SHAPES))
@pytest.mark.parametrize("dtype", F.DTYPES)
def test_suite_shape_default_tile(gemm, dtype, shape):
    ops = _ops(shape)
    tile, out = run_default(gemm, dtype, ops)
    whole = (dtype, shape) in WHOLE
    rows = np.arange(ops.N) if whole else check_rows(ops.N)
    ref = oracle.full_reference(dtype, ops.X(dtype), ops.W(dtype), ops.xscale(dtype), ops.wscale(dtype),
                                ops.N, ops.K, ops.M) if whole else reference_rows(dtype, ops, rows)
    got = out[rows]
    what = f"{dtype} {shape} tile {tile}: {'whole output' if whole else f'{len(rows)} whole rows'}"
    if dtype == "i8i8":
        bad = np.argwhere(got.astype(np.int64) != ref)
        print(f"{what}: {bad.shape[0]} mismatches (bit-exact)")
        assert bad.size == 0, f"{what}: first mismatches {bad[:5].tolist()}"
        return
    assert np.all(np.isfinite(got)), what
    floored, unfloored, frac = rel_errors(got, ref)
    print(f"{what}: max rel {floored:.3g} (floored at 1e-2 rms), unfloored {unfloored:.3g}, "
          f"{frac:.2e} of outputs above 1e-3 unfloored")
    assert floored <= REL_TOL, what


@pytest.mark.parametrize("dtype", F.DTYPES)
def test_fat_row_shard_blocks(gemm, dtype):
    # The column blocks of the M-sharded fat row (bench.py and mlp_bench.py
    # under torchrun): the first and last GPU's block at 4 GPUs (2752 columns
    # each) and at 8 (1376), each on the tile the block picks by default, run
    # on this GPU.  Each block is a GEMM of its own: X times the block's
    # slice of W (and of its scale plane), checked on the same rows as above
    # against the oracle's decode of that slice.
    from mlpgemm.data import shard_columns
    from mlpgemm.shard import shard_plan
    G = gemm
    ops = _ops("fat")
    N, K, M = ops.N, ops.K, ops.M
    dt = F.CODE[dtype]
    rows = check_rows(N)
    xs = ops.xscale(dtype)
    xd = oracle.decode_x(dtype, ops.X(dtype), xs, N, K)[rows] if dtype != "i8i8" else \
        np.asarray(ops.X(dtype), np.int8).reshape(N, K)[rows].astype(np.float64)
    X = G.DeviceBuffer(0, ops.X(dtype).nbytes).upload(ops.X(dtype))
    XS = None if xs is None else G.DeviceBuffer(0, xs.nbytes).upload(xs)
    for world, rank in ((4, 0), (4, 3), (8, 0), (8, 7)):
        m0, width = shard_plan(M, world)[rank]
        Wsh, wsc, _, w = shard_columns(ops, dtype, rank, world)
        assert w == width
        ti = G.default_tile(dt, N, K, width)
        W = G.DeviceBuffer(0, Wsh.nbytes).upload(Wsh)
        WS = None if wsc is None else G.DeviceBuffer(0, wsc.nbytes).upload(wsc)
        Y = G.DeviceBuffer(0, N * width * 4).zero()
        wsb = G.workspace_size(dt, ti, N, K, width)
        WSP = G.DeviceBuffer(0, wsb).zero() if wsb else None
        G.run(0, dt, ti, X, W, Y, N, K, width, XS, WS, WSP, wsb)
        G.sync(0)
        out = Y.download(np.empty((N, width), np.int32 if dtype == "i8i8" else np.float32))[rows]
        what = f"{dtype} GPU {rank} of {world} (columns {m0}..{m0 + width - 1}) tile {G.tile_names()[ti]}"
        if dtype == "i8i8":
            wd = np.asarray(Wsh, np.int8).reshape(K, width).astype(np.float64)
            ref = (xd @ wd).astype(np.int64)
            assert np.array_equal(out.astype(np.int64), ref), what
        else:
            ref = xd @ oracle.decode_w(dtype, Wsh, wsc, K, width)
            assert np.all(np.isfinite(out)), what
            floored, unfloored, _ = rel_errors(out, ref)
            print(f"{what}: max rel {floored:.3g}, unfloored {unfloored:.3g}")
            assert floored <= REL_TOL, what
        for b in (W, WS, Y, WSP):
            if b is not None:
                b.close()
    X.close()
    if XS is not None:
        XS.close()
