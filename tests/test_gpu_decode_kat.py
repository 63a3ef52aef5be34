"""Bit-exact operand decodes of every kernel family, on the GPU.

Known-answer tests for the decodes of main.swift:30-48 (E4M3 with its
subnormals and NaN codes), :41-48 (E2M1), :69-78 (UE8M0) and :419-449
(refActivation / refWeight).  X is one-hot: X[n, k] = 1 exactly when k == n
(the dtype's own encoding of 1.0: half 0x3C00, int8 1, E4M3 0x38, E2M1 code
2, UE8M0 127 where X has a scale plane), so every output is ONE decoded
weight, times the X scale of its block:

    Y[n, m] = decode(W)[n, m] * xscale(n, n // 32)

with no rounding anywhere (one product, the other K-1 terms exactly zero).
The kernels must reproduce the oracle's decode bit for bit: equal f32 values
(+0 and -0 compare equal: the zero products of the other K-1 terms may turn a
-0 weight into +0) and NaN exactly where the reference decodes a NaN code.

Weights hold every code of the format in every row (E4M3: all 254 non-NaN
codes; int8: all 256 values; E2M1: all 16 codes; fp16: all 63488 finite
halves across the matrix), so the tensor-core tiles (N = K = 256: the whole
of W is read back) check every code at every position of the MMA's
operand layout, and the thin-row tiles every code of the rows they read.
UE8M0 planes run over the suite's range 124-130, over ranges outside f16's
window (the A16 path keeps E2M1 * 2^(s-127) exact with per-row exponent
offsets), and for the block-scaled kinds over codes 12-242 with X scales
117-137, the whole range whose products stay normal, finite f32 values.
"""
import numpy as np
import pytest

import oracle
from mlpgemm import formats as F
from mlpgemm.data import Operands

pytestmark = pytest.mark.gpu

E4M3_FINITE = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], dtype=np.uint8)
HALF_FINITE = np.array([c for c in range(65536) if (c & 0x7C00) != 0x7C00], dtype=np.uint16)

TC_TILES = ["256x256", "128x256", "128x128"]
SCALED_192 = {"f4f4", "mxfp4/a4", "mxfp4/a8", "mxfp4/f8"}   # 256x192 and 256x224 CTA pairs
THIN_TC = {"fp16", "int8", "i8i8", "fp8", "f8f8", "mxfp4"}
GEMV_TILES = ["gemv.k1", "gemv.k8"]

# UE8M0 ranges (W codes lo..hi; X codes where X has a plane)
MX_RANGES = {
    "mxfp4": [(124, 130), (90, 100), (150, 160)],
    "mxfp4/a4": [(124, 130), (12, 242)],
    "mxfp4/a8": [(124, 130), (12, 242)],
    "mxfp4/f8": [(124, 130), (12, 242)],
}
X_SCALE_RANGE = {(124, 130): (125, 129), (12, 242): (117, 137)}


def _shape(tile):
    if tile.startswith("gemv"):
        return 2, 256, 512
    if tile == "16x128":
        return 16, 256, 512
    return 256, 256, 512


def one_hot_ops(dtype, N, K, M, srange=None):
    """Operands with X one-hot and W holding every code of its format."""
    ops = Operands(N, K, M, "seeded", 0)
    n = np.arange(N)[:, None]
    k = np.arange(K)[None, :]
    hot = (k == n)
    if dtype in F.X_HALF:
        x = np.where(hot, np.float16(1.0), np.float16(0.0)).astype(np.float16).reshape(-1)
    elif dtype == "i8i8":
        x = hot.astype(np.int8).reshape(-1)
    elif dtype in F.X_E4M3:
        x = np.where(hot, 0x38, 0x00).astype(np.uint8).reshape(-1)
    else:
        x = F.e2m1_pack(np.where(hot, 2, 0).astype(np.uint8).reshape(-1))
    ops._cache[ops.x_name(dtype)] = x
    kk = np.arange(K)[:, None]
    mm = np.arange(M)[None, :]
    if dtype == "fp16":
        w = HALF_FINITE[(kk * M + mm) % len(HALF_FINITE)].view(np.float16).reshape(-1)
    elif dtype in ("int8", "i8i8"):
        w = ((mm + 7 * kk) % 256 - 128).astype(np.int8).reshape(-1)
    elif dtype in ("fp8", "f8f8"):
        w = E4M3_FINITE[(mm + 7 * kk) % len(E4M3_FINITE)].reshape(-1)
    elif dtype == "f4f4":
        w = F.e2m1_pack(((mm + kk) % 16).astype(np.uint8).reshape(-1))
    else:   # the mxfp4 family: W stored [M,K] packed along K, UE8M0 [M, K/32]
        wm = np.arange(M)[:, None]
        wk = np.arange(K)[None, :]
        w = F.e2m1_pack(((wm + wk) % 16).astype(np.uint8).reshape(-1))
        lo, hi = srange
        kb = np.arange(K // 32)[None, :]
        ops._cache["wscale"] = (lo + (wm * 5 + kb * 3) % (hi - lo + 1)).astype(np.uint8).reshape(-1)
        if dtype in F.X_SCALED:
            xlo, xhi = X_SCALE_RANGE[srange]
            ops._cache["xscale"] = (xlo + (np.arange(N)[:, None] + kb) % (xhi - xlo + 1)).astype(
                np.uint8).reshape(-1)
    ops._cache[ops.w_name(dtype)] = w
    return ops


def expected(dtype, ops):
    N, K, M = ops.N, ops.K, ops.M
    if dtype == "i8i8":
        return oracle.full_reference(dtype, ops.X(dtype), ops.W(dtype), None, None, N, K, M)
    xd = oracle.decode_x(dtype, ops.X(dtype), ops.xscale(dtype), N, K)
    wd = oracle.decode_w(dtype, ops.W(dtype), ops.wscale(dtype), K, M)
    # IEEE: any NaN term makes the dot product NaN (0 * NaN is NaN), whatever a
    # BLAS does with zeros; the finite part is one exact product per output
    xn, wn = np.isnan(xd), np.isnan(wd)
    ref = np.where(xn, 0.0, xd) @ np.where(wn, 0.0, wd)
    ref[xn.any(axis=1), :] = np.nan
    ref[:, wn.any(axis=0)] = np.nan
    fin = np.isfinite(ref)
    # every expected value is one f32 number (the test's premise)
    assert np.array_equal(ref[fin].astype(np.float32).astype(np.float64), ref[fin])
    return ref


def run(G, dtype, tile, ops):
    N, K, M = ops.N, ops.K, ops.M
    dt, ti = F.CODE[dtype], G.tile_index(tile)
    assert G.tile_supported(dt, ti, N, K, M), (dtype, tile, N, K, M)
    keep = []

    def up(a):
        if a is None:
            return None
        b = G.DeviceBuffer(0, a.nbytes).upload(a)
        keep.append(b)
        return b

    X, W, XS, WS = up(ops.X(dtype)), up(ops.W(dtype)), up(ops.xscale(dtype)), up(ops.wscale(dtype))
    Y = G.DeviceBuffer(0, N * M * 4).zero()
    wsb = G.workspace_size(dt, ti, N, K, M)
    WSP = G.DeviceBuffer(0, wsb).zero() if wsb else None
    G.run(0, dt, ti, X, W, Y, N, K, M, XS, WS, WSP, wsb)
    G.sync(0)
    return Y.download(np.empty((N, M), np.int32 if dtype == "i8i8" else np.float32))


def assert_bit_exact(dtype, out, ref, what):
    if dtype == "i8i8":
        bad = np.argwhere(out.astype(np.int64) != ref)
        assert bad.size == 0, f"{what}: {len(bad)} mismatches, first {bad[:4].tolist()}"
        return
    nan_ref, nan_out = np.isnan(ref), np.isnan(out)
    assert np.array_equal(nan_ref, nan_out), f"{what}: NaN positions differ"
    exp32 = ref.astype(np.float32)
    bad = np.argwhere((out != exp32) & ~nan_ref)
    assert bad.size == 0, (f"{what}: {len(bad)} decodes differ, first at {bad[0].tolist()}: "
                           f"got {out[tuple(bad[0])]!r} want {exp32[tuple(bad[0])]!r}")


def _cases():
    out = []
    for d in F.DTYPES:
        tiles = TC_TILES + (["256x192", "256x224"] if d in SCALED_192 else []) + (["16x128"] if d in THIN_TC else []) + GEMV_TILES
        for t in tiles:
            for r in MX_RANGES.get(d, [None]):
                out.append((d, t, r))
    return out


@pytest.mark.parametrize("dtype,tile,srange", _cases())
def test_one_hot_decode_is_bit_exact(gemm, dtype, tile, srange):
    N, K, M = _shape(tile)
    ops = one_hot_ops(dtype, N, K, M, srange)
    ref = expected(dtype, ops)
    out = run(gemm, dtype, tile, ops)
    assert_bit_exact(dtype, out, ref, f"{dtype} {tile} scales {srange}")


# E4M3 NaN codes (0x7F, 0xFF) decode to NaN (main.swift:33): a NaN weight makes
# its whole output column NaN (0 * NaN is NaN), a NaN activation its whole row.
NAN_CASES = [(d, t) for d in ("fp8", "f8f8") for t in TC_TILES + ["16x128"] + GEMV_TILES]
NAN_CASES += [(d, t) for d in ("mxfp4/a8", "mxfp4/f8") for t in TC_TILES + ["256x192", "256x224"] + GEMV_TILES]


@pytest.mark.parametrize("dtype,tile", NAN_CASES)
def test_e4m3_nan_codes_give_nan(gemm, dtype, tile):
    N, K, M = _shape(tile)
    srange = (124, 130) if dtype in F.W_MX else None
    ops = one_hot_ops(dtype, N, K, M, srange)
    if dtype in ("fp8", "f8f8"):   # NaN weights in columns 5 (0x7F) and 300 (0xFF)
        w = ops.W(dtype).reshape(K, M).copy()
        w[3, 5], w[N - 1, 300] = 0x7F, 0xFF
        ops._cache[ops.w_name(dtype)] = w.reshape(-1)
    if dtype in F.X_E4M3:           # a NaN activation in row 1 (off the diagonal)
        x = ops.X(dtype).reshape(N, K).copy()
        x[1, 40] = 0xFF
        ops._cache[ops.x_name(dtype)] = x.reshape(-1)
    ref = expected(dtype, ops)
    assert np.isnan(ref).any()
    out = run(gemm, dtype, tile, ops)
    assert_bit_exact(dtype, out, ref, f"{dtype} {tile} NaN codes")
