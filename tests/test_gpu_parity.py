"""GPU parity: libgemm.so kernels (through the C ABI) against the oracle.

Every case runs one GEMM on seeded operands and compares the WHOLE output
with the oracle's fp64 dot product of the decoded operands (int64 for
i8i8):
  i8i8         bit-exact
  float dtypes max relative error <= 1e-3, where the denominator is
               max(|ref|, 1e-2 * rms(ref)) so that outputs that cancel to
               near zero are judged against the scale of the output.
"""
import numpy as np
import pytest

import oracle
from mlpgemm import formats as F
from mlpgemm.data import Operands

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def run_case(G, dtype, tile, N, K, M, mode="seeded", seed=0, ops=None):
    ops = ops or Operands(N, K, M, mode, seed)
    dt = F.CODE[dtype]
    ti = G.tile_index(tile)
    assert G.tile_supported(dt, ti, N, K, M), (dtype, tile, N, K, M)
    X = G.DeviceBuffer(0, ops.X(dtype).nbytes).upload(ops.X(dtype))
    W = G.DeviceBuffer(0, ops.W(dtype).nbytes).upload(ops.W(dtype))
    xs = ops.xscale(dtype)
    ws = ops.wscale(dtype)
    XS = G.DeviceBuffer(0, xs.nbytes).upload(xs) if xs is not None else None
    WS = G.DeviceBuffer(0, ws.nbytes).upload(ws) if ws is not None else None
    Y = G.DeviceBuffer(0, N * M * 4)
    Y.zero()
    wsb = G.workspace_size(dt, ti, N, K, M)
    WSP = G.DeviceBuffer(0, wsb).zero() if wsb else None
    G.run(0, dt, ti, X, W, Y, N, K, M, XS, WS, WSP, wsb)
    G.sync(0)
    out = np.empty((N, M), dtype=np.int32 if dtype == "i8i8" else np.float32)
    Y.download(out)
    ref = oracle.full_reference(dtype, ops.X(dtype), ops.W(dtype), xs, ws, N, K, M)
    return out, ref, ops


def assert_close(dtype, out, ref):
    if dtype == "i8i8":
        bad = np.argwhere(out.astype(np.int64) != ref)
        assert bad.size == 0, f"{len(bad)} mismatches, first {bad[:5].tolist()}"
        return 0.0
    assert np.all(np.isfinite(out))
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    den = np.maximum(np.abs(ref), 1e-2 * rms + 1e-30)
    rel = np.abs(out.astype(np.float64) - ref) / den
    worst = np.unravel_index(np.argmax(rel), rel.shape)
    assert rel.max() <= REL_TOL, f"max rel {rel.max():.3g} at {worst}: got {out[worst]} ref {ref[worst]}"
    return float(rel.max())


# tensor-core tiles per dtype
TC_TILES = {d: ["256x256", "128x256", "128x128"] for d in ("fp16", "i8i8", "f8f8")}
TC_TILES.update({d: ["256x256", "128x256", "128x128"] for d in ("int8", "fp8")})   # 256x256: W widened once
TC_TILES.update({"mxfp4": ["256x256", "128x256", "128x128"]})   # 256x256: widened once to f16 [K,M]
# block-scaled kinds (and f4f4 on kind::mxf4) also run 256x192 and 256x224 CTA pairs with two
# accumulators (256x224 mxf4: two TMEM scale slots reused across the ring's stages)
TC_TILES.update({"f4f4": ["256x256", "256x192", "256x224", "128x256", "128x128"]})
TC_TILES.update({d: ["256x256", "256x192", "256x224", "128x256", "128x128"]
                 for d in ("mxfp4/a4", "mxfp4/a8", "mxfp4/f8")})
TC_CASES = [(d, t) for d in F.DTYPES for t in TC_TILES[d]]


@pytest.mark.parametrize("dtype,tile", TC_CASES)
@pytest.mark.parametrize("shape", [(256, 512, 512), (200, 384, 272), (1000, 1024, 1296)])
def test_tensor_core_tiles(gemm, dtype, tile, shape):
    N, K, M = shape
    out, ref, _ = run_case(gemm, dtype, tile, N, K, M)
    assert_close(dtype, out, ref)


@pytest.mark.parametrize("dtype", F.DTYPES)
def test_tensor_core_reference_patterns(gemm, dtype):
    # the reference's own deterministic operands (main.swift:379-390)
    tile = TC_TILES[dtype][0]
    out, ref, _ = run_case(gemm, dtype, tile, 384, 1024, 768, mode="ref")
    assert_close(dtype, out, ref)


@pytest.mark.parametrize("tile", ["256x256", "128x256"])
@pytest.mark.parametrize("lo,hi", [(124, 130), (90, 100), (150, 160), (100, 145)])
def test_mxfp4_widen_any_scale_range(gemm, lo, hi, tile):
    # E2M1 * 2^(s-127) leaves the f16 range outside s in [104, 140]; the
    # per-row exponent offsets keep the widened weights exact
    N, K, M = 256, 512, 384
    ops = Operands(N, K, M, "seeded", 4)
    rng = np.random.default_rng(9)
    ops._cache["wscale"] = rng.integers(lo, hi + 1, M * (K // 32), dtype=np.uint8)
    out, ref, _ = run_case(gemm, "mxfp4", tile, N, K, M, ops=ops)
    if hi - lo <= 36:
        assert_close("mxfp4", out, ref)
    else:
        # a row whose scales span more than f16's range loses only terms
        # below 2^-24 of its largest block
        rms = float(np.sqrt(np.mean(ref * ref)))
        assert np.all(np.abs(out - ref) <= 1e-3 * np.maximum(np.abs(ref), 1e-2 * rms))


@pytest.mark.parametrize("dtype", F.DTYPES)
@pytest.mark.parametrize("tile", ["gemv.k1", "gemv.k8", "gemv.k64"])
def test_gemv_thin_rows(gemm, dtype, tile):
    N, K, M = 1, 1024, 1504
    out, ref, _ = run_case(gemm, dtype, tile, N, K, M)
    assert_close(dtype, out, ref)


@pytest.mark.parametrize("dtype", [d for d in F.DTYPES if d in F.W_MX])
@pytest.mark.parametrize("N,K,M", [(1, 4096, 11008), (2, 4096, 11008), (1, 16384, 3001), (2, 8192, 12000)])
def test_mx_thin_rows_one_split(gemm, dtype, N, K, M):
    # gemv.k1 on [M,K] weights at N <= 2 (the kernel that keeps every lane's
    # weight blocks in flight): the suite's thin row at one and two rows of
    # X, a long K, and two rows at a ragged M
    out, ref, _ = run_case(gemm, dtype, "gemv.k1", N, K, M)
    assert_close(dtype, out, ref)


@pytest.mark.parametrize("dtype", F.DTYPES)
@pytest.mark.parametrize("N", [2, 5, 16])
def test_gemv_ragged(gemm, dtype, N):
    K = 256 if dtype in F.W_MX else 98
    M = 50
    out, ref, _ = run_case(gemm, dtype, "gemv.k4", N, K, M)
    assert_close(dtype, out, ref)


@pytest.mark.parametrize("dtype", F.DTYPES)
def test_suite_thin_row(gemm, dtype):
    # the suite's thin row (N=1, K=4096, M=11008) with the default tile
    N, K, M = 1, 4096, 11008
    tile = gemm.tile_names()[gemm.default_tile(F.CODE[dtype], N, K, M)]
    out, ref, _ = run_case(gemm, dtype, tile, N, K, M)
    assert_close(dtype, out, ref)


@pytest.mark.parametrize("dtype,N", [(d, 2) for d in ("fp16", "int8", "i8i8", "fp8", "f8f8", "f4f4")] +
                         [("f4f4", 4), ("f4f4", 8)])
def test_default_thin_tile_two_or_more_rows(gemm, dtype, N):
    # [K,M] weights at 2 <= N with the default split (two at N = 2, four for
    # f4f4 from N = 3 on): cluster-reduced K splits match the oracle
    K, M = 4096, 11008
    tile = gemm.tile_names()[gemm.default_tile(F.CODE[dtype], N, K, M)]
    assert tile == ("gemv.k2" if N == 2 else "gemv.k4")
    out, ref, _ = run_case(gemm, dtype, tile, N, K, M)
    assert_close(dtype, out, ref)


def test_gemv_deterministic_and_counters_reset(gemm):
    # two calls on one workspace: identical bits (fixed reduction order) and
    # the split-K counters are back at zero for the second call
    a, ref, ops = run_case(gemm, "fp8", "gemv.k16", 3, 2048, 777)
    b, _, _ = run_case(gemm, "fp8", "gemv.k16", 3, 2048, 777, ops=ops)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert_close("fp8", a, ref)


def test_rejects_bad_layout(gemm):
    G = gemm
    dt = F.CODE["mxfp4/a8"]
    with pytest.raises(G.GemmError) as e:
        G.run(0, dt, G.tile_index("gemv.k1"), 1, 1, 1, 4, 96, 8, 1, 1)
    assert e.value.code == G.GEMM_ERR_ARGS


@pytest.mark.parametrize("dtype", F.DTYPES)
@pytest.mark.parametrize("shape", [(1, 4096, 11008), (3, 1024, 1008), (16, 512, 640)])
def test_stream_thin_rows(gemm, dtype, shape):
    # persistent TMA-streaming kernel (stream-K split, cross-CTA reduction)
    N, K, M = shape
    if dtype in F.W_MX:
        K = max(K, 512)
    ti = gemm.tile_index("stream")
    if not gemm.tile_supported(F.CODE[dtype], ti, N, K, M):
        pytest.skip("register or shared-memory budget")
    out, ref, _ = run_case(gemm, dtype, "stream", N, K, M)
    assert_close(dtype, out, ref)


def test_stream_deterministic(gemm):
    a, ref, ops = run_case(gemm, "int8", "stream", 1, 4096, 11008)
    b, _, _ = run_case(gemm, "int8", "stream", 1, 4096, 11008, ops=ops)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


# thin rows on the tensor cores: weights as the MMA's A operand (tile 16x128)
THIN_TC = ["fp16", "int8", "i8i8", "fp8", "f8f8", "mxfp4"]


def thin_k(dtype, K):
    # the tile's TMA strides: K % 8 for half X, % 16 for byte X, % 32 for MX weights
    step = 32 if dtype in F.W_MX else (16 if dtype in ("i8i8", "f8f8") else 8)
    return max(step, K // step * step)


@pytest.mark.parametrize("dtype", THIN_TC)
@pytest.mark.parametrize("shape", [(1, 4096, 11008), (1, 1024, 1504), (3, 1000, 1296), (16, 512, 640),
                                   (5, 64, 128), (2, 8192, 256), (7, 200, 4096)])
def test_thin_tensor_core_tile(gemm, dtype, shape):
    # stream-K over (tile, K stage) units: whole tiles, tiles shared by many
    # CTAs (K=8192, two tiles), a single unit, ragged K and ragged M
    N, K, M = shape
    K = thin_k(dtype, K)
    out, ref, _ = run_case(gemm, dtype, "16x128", N, K, M)
    assert_close(dtype, out, ref)


@pytest.mark.parametrize("dtype", THIN_TC)
def test_thin_tensor_core_reference_patterns(gemm, dtype):
    out, ref, _ = run_case(gemm, dtype, "16x128", 4, 1024, 768, mode="ref")
    assert_close(dtype, out, ref)


@pytest.mark.parametrize("lo,hi", [(124, 130), (90, 100), (150, 160), (100, 145), (40, 214)])
def test_thin_mxfp4_any_scale_range(gemm, lo, hi):
    # per-(CTA, row) exponent offsets keep the widened weights exact in f16
    # (the widest range keeps the f32 results finite: 2^(214-127) * 6 * |x| * K)
    N, K, M = 3, 2048, 384
    ops = Operands(N, K, M, "seeded", 4)
    rng = np.random.default_rng(11)
    ops._cache["wscale"] = rng.integers(lo, hi + 1, M * (K // 32), dtype=np.uint8)
    out, ref, _ = run_case(gemm, "mxfp4", "16x128", N, K, M, ops=ops)
    if hi - lo <= 36:
        assert_close("mxfp4", out, ref)
    else:
        # a row whose scales span more than f16's range loses only terms
        # below 2^-24 of its largest block
        rms = float(np.sqrt(np.mean(ref * ref)))
        assert np.all(np.abs(out - ref) <= 1e-3 * np.maximum(np.abs(ref), 1e-2 * rms))


@pytest.mark.parametrize("dtype", ["fp16", "i8i8", "mxfp4"])
def test_thin_tensor_core_deterministic(gemm, dtype):
    # two calls on ONE workspace: identical bits (shared tiles are summed in
    # CTA order) and the tile counters are back at zero for the second call
    G = gemm
    N, K, M = 2, 4096, 11008
    ops = Operands(N, K, M, "seeded", 3)
    dt, ti = F.CODE[dtype], G.tile_index("16x128")
    bufs = [G.DeviceBuffer(0, a.nbytes).upload(a) for a in (ops.X(dtype), ops.W(dtype))]
    ws = ops.wscale(dtype)
    WS = G.DeviceBuffer(0, ws.nbytes).upload(ws) if ws is not None else None
    wsb = G.workspace_size(dt, ti, N, K, M)
    WSP = G.DeviceBuffer(0, wsb).zero()
    outs = []
    for _ in range(2):
        Y = G.DeviceBuffer(0, N * M * 4).zero()
        G.run(0, dt, ti, bufs[0], bufs[1], Y, N, K, M, None, WS, WSP, wsb)
        G.sync(0)
        o = np.empty((N, M), dtype=np.int32 if dtype == "i8i8" else np.float32)
        Y.download(o)
        outs.append(o)
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    ref = oracle.full_reference(dtype, ops.X(dtype), ops.W(dtype), None, ws, N, K, M)
    assert_close(dtype, outs[1], ref)


@pytest.mark.parametrize("dtype", ["fp16", "f8f8", "i8i8", "mxfp4/a8"])
def test_pair_tiles_deterministic(gemm, dtype):
    # CTA-pair tiles: identical bits on every call
    N, K, M = 1000, 1024, 1296
    a, ref, ops = run_case(gemm, dtype, "256x256", N, K, M)
    b, _, _ = run_case(gemm, dtype, "256x256", N, K, M, ops=ops)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert_close(dtype, a, ref)


@pytest.mark.parametrize("dtype", ["i8i8", "mxfp4/a8"])
def test_e2e_timing_moves_the_result(gemm, dtype):
    # both end-to-end timers copy X in and Y out on every step; the host Y they
    # leave behind is the GEMM's result, and the overlapped loop is not slower
    # per step than the serial one
    import ctypes
    G = gemm
    N, K, M = 512, 1024, 768
    ops = Operands(N, K, M, "seeded", 5)
    dt, ti = F.CODE[dtype], G.tile_index("128x256")
    xh, xs, ws = ops.X(dtype), ops.xscale(dtype), ops.wscale(dtype)
    dX = [G.DeviceBuffer(0, xh.nbytes) for _ in range(2)]
    dY = [G.DeviceBuffer(0, N * M * 4).zero() for _ in range(2)]
    dXS = [G.DeviceBuffer(0, xs.nbytes) for _ in range(2)] if xs is not None else [None, None]
    W = G.DeviceBuffer(0, ops.W(dtype).nbytes).upload(ops.W(dtype))
    WS = G.DeviceBuffer(0, ws.nbytes).upload(ws) if ws is not None else None
    wsb = G.workspace_size(dt, ti, N, K, M)
    WSP = G.DeviceBuffer(0, wsb).zero() if wsb else None
    L = G.lib()
    hX, hY = L.gemm_host_alloc(xh.nbytes), L.gemm_host_alloc(N * M * 4)
    hXS = L.gemm_host_alloc(xs.nbytes) if xs is not None else None
    try:
        ctypes.memmove(hX, xh.ctypes.data, xh.nbytes)
        if xs is not None:
            ctypes.memmove(hXS, xs.ctypes.data, xs.nbytes)
        ref = oracle.full_reference(dtype, xh, ops.W(dtype), xs, ws, N, K, M)
        out_t = np.int32 if dtype == "i8i8" else np.float32
        for run in ("serial", "pipelined"):
            ctypes.memset(hY, 0, N * M * 4)
            if run == "serial":
                ms = G.time_e2e(0, dt, ti, hX, dX[0], W, dY[0], hY, N, K, M, hXS, dXS[0], WS, WSP, wsb,
                                warmup=1, iters=4)
                per_step = sum(ms) / len(ms)
            else:
                total = G.time_e2e_pipelined(0, dt, ti, hX, dX, W, dY, hY, N, K, M, hXS, dXS, WS, WSP, wsb,
                                             warmup=1, iters=8)
                assert total > 0
                assert total / 8 <= 1.5 * per_step
            out = np.ctypeslib.as_array(ctypes.cast(hY, ctypes.POINTER(ctypes.c_uint32)), (N * M,))
            assert_close(dtype, out.view(out_t).reshape(N, M).copy(), ref)
    finally:
        L.gemm_host_free(hX)
        L.gemm_host_free(hY)
        if hXS:
            L.gemm_host_free(hXS)


@pytest.mark.parametrize("M", [512, 258])
def test_f4f4_pair_ragged_m(gemm, M):
    # W [K,M] packed along M is transposed to [M,K] (any even M) for the
    # K-major 4-bit operands of kind::mxf4 (unit scales)
    N, K = 384, 1024
    out, ref, _ = run_case(gemm, "f4f4", "256x256", N, K, M)
    assert_close("f4f4", out, ref)


# More 256x256 tiles than CTA pairs: the persistent grid takes several waves.
# When the last wave fills at most half the pairs, its tiles run as 256x128
# halves. Cases: 1 and 36 split tiles; a split last tile whose second half is
# partly (19152) or wholly (19056) past M; 160 tiles over several tile rows
# with 12 split; int8 through the widened-W pair kernel.
MANY_WAVES = [(256, 256, 19200), (512, 256, 14080), (256, 256, 19152), (256, 256, 19056), (2048, 256, 5120)]


@pytest.mark.parametrize("dtype", ["fp16", "i8i8", "f8f8", "int8"])
@pytest.mark.parametrize("shape", MANY_WAVES)
def test_pair_tiles_many_waves(gemm, dtype, shape):
    # two calls give the same bits, and the result matches the oracle
    G = gemm
    N, K, M = shape
    ops = Operands(N, K, M, "seeded", 8)
    dt, ti = F.CODE[dtype], G.tile_index("256x256")
    X = G.DeviceBuffer(0, ops.X(dtype).nbytes).upload(ops.X(dtype))
    W = G.DeviceBuffer(0, ops.W(dtype).nbytes).upload(ops.W(dtype))
    wsb = G.workspace_size(dt, ti, N, K, M)
    WSP = G.DeviceBuffer(0, wsb).zero() if wsb else None
    outs = []
    for _ in range(2):
        Y = G.DeviceBuffer(0, N * M * 4).zero()
        G.run(0, dt, ti, X, W, Y, N, K, M, None, None, WSP, wsb)
        G.sync(0)
        o = np.empty((N, M), dtype=np.int32 if dtype == "i8i8" else np.float32)
        Y.download(o)
        outs.append(o)
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    ref = oracle.full_reference(dtype, ops.X(dtype), ops.W(dtype), None, None, N, K, M)
    assert_close(dtype, outs[1], ref)


GATHER_CASES = [(d, t) for d, t in TC_CASES if not (t != "256x256" and d in ("int8", "fp8", "mxfp4"))]


@pytest.mark.parametrize("dtype,tile", GATHER_CASES)
def test_gather_epilogue_writes_every_peer(gemm, dtype, tile):
    """gemm_run_gather with seven 'peer' Y buffers on the same GPU: every
    peer gets exactly the local Y, and the local Y is the oracle's result.
    (The multi-GPU form maps other GPUs' buffers; the stores are the same.)"""
    G = gemm
    N, K, M = 200, 384, 272
    ops = Operands(N, K, M, "seeded", 3)
    dt, ti = F.CODE[dtype], G.tile_index(tile)
    assert G.gather_supported(dt, ti)
    X = G.DeviceBuffer(0, ops.X(dtype).nbytes).upload(ops.X(dtype))
    W = G.DeviceBuffer(0, ops.W(dtype).nbytes).upload(ops.W(dtype))
    xs, ws = ops.xscale(dtype), ops.wscale(dtype)
    XS = G.DeviceBuffer(0, xs.nbytes).upload(xs) if xs is not None else None
    WS = G.DeviceBuffer(0, ws.nbytes).upload(ws) if ws is not None else None
    Y = G.DeviceBuffer(0, N * M * 4).zero()
    peers = [G.DeviceBuffer(0, N * M * 4).zero() for _ in range(G.MAX_PEERS)]
    wsb = G.workspace_size(dt, ti, N, K, M)
    WSP = G.DeviceBuffer(0, wsb).zero() if wsb else None
    G.run_gather(0, dt, ti, X, W, Y, N, K, M, XS, WS, WSP, wsb, peers=peers)
    G.sync(0)
    yt = np.int32 if dtype == "i8i8" else np.float32
    out = np.empty((N, M), dtype=yt)
    Y.download(out)
    for p in peers:
        got = np.empty((N, M), dtype=yt)
        p.download(got)
        assert np.array_equal(got.view(np.uint32), out.view(np.uint32))
    ref = oracle.full_reference(dtype, ops.X(dtype), ops.W(dtype), xs, ws, N, K, M)
    assert_close(dtype, out, ref)


@pytest.mark.parametrize("dtype", ["fp16", "i8i8"])
def test_gather_epilogue_on_half_tiles(gemm, dtype):
    # 75 tiles on 74 CTA pairs: the last tile runs as two 256x128 halves, whose
    # second half is partly past M; every peer still gets exactly the local Y
    G = gemm
    N, K, M = 256, 256, 19152
    ops = Operands(N, K, M, "seeded", 5)
    dt, ti = F.CODE[dtype], G.tile_index("256x256")
    X = G.DeviceBuffer(0, ops.X(dtype).nbytes).upload(ops.X(dtype))
    W = G.DeviceBuffer(0, ops.W(dtype).nbytes).upload(ops.W(dtype))
    Y = G.DeviceBuffer(0, N * M * 4).zero()
    peers = [G.DeviceBuffer(0, N * M * 4).zero() for _ in range(3)]
    G.run_gather(0, dt, ti, X, W, Y, N, K, M, None, None, None, 0, peers=peers)
    G.sync(0)
    yt = np.int32 if dtype == "i8i8" else np.float32
    out = np.empty((N, M), dtype=yt)
    Y.download(out)
    for q in peers:
        got = np.empty((N, M), dtype=yt)
        q.download(got)
        assert np.array_equal(got.view(np.uint32), out.view(np.uint32))
    assert_close(dtype, out, oracle.full_reference(dtype, ops.X(dtype), ops.W(dtype), None, None, N, K, M))


def test_gather_rejects_unsupported_tiles(gemm):
    G = gemm
    for dtype, tile in (("int8", "128x256"), ("mxfp4", "128x128"), ("fp16", "16x128"), ("fp16", "gemv.k1")):
        assert not G.gather_supported(F.CODE[dtype], G.tile_index(tile))
    N, K, M = 8, 256, 256
    dt, ti = F.CODE["fp16"], G.tile_index("16x128")
    X = G.DeviceBuffer(0, N * K * 2).zero()
    W = G.DeviceBuffer(0, K * M * 2).zero()
    Y = G.DeviceBuffer(0, N * M * 4).zero()
    P = G.DeviceBuffer(0, N * M * 4).zero()
    wsb = G.workspace_size(dt, ti, N, K, M)
    WSP = G.DeviceBuffer(0, wsb).zero() if wsb else None
    with pytest.raises(G.GemmError) as e:
        G.run_gather(0, dt, ti, X, W, Y, N, K, M, None, None, WSP, wsb, peers=[P])
    assert e.value.code == 1 and "fused all-gather" in str(e.value)
    N = M = K = 256   # a shape the pair tile takes, with more peers than an 8-GPU node has
    X2, W2 = G.DeviceBuffer(0, N * K * 2).zero(), G.DeviceBuffer(0, K * M * 2).zero()
    Y2, P2 = G.DeviceBuffer(0, N * M * 4).zero(), G.DeviceBuffer(0, N * M * 4).zero()
    with pytest.raises(G.GemmError) as e:
        G.run_gather(0, dt, G.tile_index("256x256"), X2, W2, Y2, N, K, M, None, None, None, 0, peers=[P2] * 8)
    assert e.value.code == 1 and "npeers" in str(e.value)


# thin rows on the warp-level tensor-core MMA (tile gemv.mma): stream-K over
# weight slabs, mma.sync on weights widened to f16 in registers
MMA_DT = ["fp16", "int8", "fp8", "f8f8", "mxfp4", "mxfp4/a4", "mxfp4/a8", "mxfp4/f8"]


def mma_shape(dtype, N, K, M):
    # [K,M] weights: K % 4 and 16-byte rows; MX weights: K % 128 (steps of 4 blocks)
    if dtype in F.W_MX:
        return N, max(128, K // 128 * 128), M
    return N, max(4, K // 4 * 4), (M // 16 * 16 or 16)


@pytest.mark.parametrize("dtype", MMA_DT)
@pytest.mark.parametrize("shape", [(1, 4096, 11008), (1, 1024, 1504), (3, 1000, 1296), (8, 512, 1040),
                                   (16, 512, 640), (5, 64, 128), (2, 8192, 256), (7, 200, 4096),
                                   (1, 36, 50), (12, 4096, 300)])
def test_mma_thin_rows(gemm, dtype, shape):
    # whole slabs, slabs shared by many CTAs (K=8192, few slabs), a single
    # step, ragged K and ragged M (a part-filled last slab), N > 8 (row blocks)
    N, K, M = mma_shape(dtype, *shape)
    out, ref, _ = run_case(gemm, dtype, "gemv.mma", N, K, M)
    assert_close(dtype, out, ref)


@pytest.mark.parametrize("dtype", MMA_DT)
def test_mma_thin_reference_patterns(gemm, dtype):
    out, ref, _ = run_case(gemm, dtype, "gemv.mma", 4, 1024, 768, mode="ref")
    assert_close(dtype, out, ref)


@pytest.mark.parametrize("lo,hi", [(124, 130), (90, 100), (40, 214)])
def test_mma_mxfp4_any_scale_range(gemm, lo, hi):
    # each 32-element block is folded into f32 times its own 2^(s - 127): no
    # range limit, the whole output stays within the tolerance
    N, K, M = 3, 2048, 384
    ops = Operands(N, K, M, "seeded", 4)
    rng = np.random.default_rng(11)
    ops._cache["wscale"] = rng.integers(lo, hi + 1, M * (K // 32), dtype=np.uint8)
    out, ref, _ = run_case(gemm, "mxfp4", "gemv.mma", N, K, M, ops=ops)
    assert_close("mxfp4", out, ref)


@pytest.mark.parametrize("dtype", ["int8", "mxfp4/a8"])
def test_mma_thin_deterministic(gemm, dtype):
    # two calls on ONE workspace: identical bits (slabs summed in CTA order)
    # and the slab counters are back at zero for the second call
    a, ref, ops = run_case(gemm, dtype, "gemv.mma", 2, 4096, 11008)
    b, _, _ = run_case(gemm, dtype, "gemv.mma", 2, 4096, 11008, ops=ops)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert_close(dtype, a, ref)


def test_mma_rejects_unsupported(gemm):
    G = gemm
    ti = G.tile_index("gemv.mma")
    assert not G.tile_supported(F.CODE["i8i8"], ti, 1, 4096, 11008)
    assert not G.tile_supported(F.CODE["int8"], ti, 1, 4096, 11000)   # rows not whole 16-byte chunks
    assert not G.tile_supported(F.CODE["fp8"], ti, 17, 4096, 11008)   # N > 16


@pytest.mark.parametrize("dtype", ["mxfp4/a4", "mxfp4/a8", "mxfp4/f8"])
@pytest.mark.parametrize("N", [3, 8, 16])
def test_default_tile_mx_quantized_x(gemm, dtype, N):
    # the default tile of the MX kinds with E2M1 / E4M3 activations at
    # 3 <= N <= 16 is the warp-MMA thin tile; it matches the oracle there
    K, M = 4096, 1040
    ti = gemm.default_tile(F.CODE[dtype], N, K, M)
    assert gemm.tile_names()[ti] == "gemv.mma"
    out, ref, _ = run_case(gemm, dtype, "gemv.mma", N, K, M)
    assert_close(dtype, out, ref)


@pytest.mark.parametrize("dtype", ["mxfp4/a4", "mxfp4/a8", "f4f4"])
def test_pair_224_long_k(gemm, dtype):
    # 256x224 at K = 4096: 16 (mxf4) or 32 (mxf8f6f4) stages per tile, so the
    # mxf4 tile's two TMEM scale slots are rewritten many times per tile, over
    # two tile rows and a part-filled last column tile (2000 = 8 x 224 + 208)
    N, K, M = 512, 4096, 2000
    out, ref, _ = run_case(gemm, dtype, "256x224", N, K, M)
    assert_close(dtype, out, ref)
