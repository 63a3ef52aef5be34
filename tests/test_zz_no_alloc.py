"""gemm_run_noalloc against gemm_run, on the GPU, through the C ABI.

gemm_run_noalloc is for callers that may not allocate device memory (plugin
hosts and serving loops that own every allocation, bindings without an
allocator): it keeps the split-K scratch of the thin-row kernel in a fixed
device array inside the library instead of a caller workspace.  It must give
the same result as gemm_run with the matching "gemv.k<S>" tile and a
workspace, on two calls in a row (the array keeps the previous call's
contents).  Both entry points run the same kernel with the same split and
the same fixed reduction order, so the results must be identical bit for
bit; the output is also checked against the oracle (bit-exact for i8i8,
max relative error <= 1e-3 against fp64 for the float dtypes).  This file is
named so that pytest collects it last; it also runs alone in a fresh process
(its only fixture initialises device 0)."""
import numpy as np
import pytest

import oracle
from mlpgemm import formats as F
from mlpgemm.data import Operands

pytestmark = pytest.mark.gpu


def _upload(G, a):
    return None if a is None else G.DeviceBuffer(0, a.nbytes).upload(a)


@pytest.mark.parametrize("dtype,N,K,M,ksplit", [
    ("int8", 1, 4096, 11008, 32),      # the suite's thin row
    ("mxfp4", 1, 4096, 11008, 2),
    ("i8i8", 3, 1024, 777, 8),         # ragged M, exact int32
    ("f4f4", 16, 512, 640, 4),
])
def test_noalloc_matches_gemm_run_twice(gemm, dtype, N, K, M, ksplit):
    G = gemm
    ops = Operands(N, K, M, "seeded", 11)
    dt = F.CODE[dtype]
    X, W = _upload(G, ops.X(dtype)), _upload(G, ops.W(dtype))
    XS, WS = _upload(G, ops.xscale(dtype)), _upload(G, ops.wscale(dtype))
    host_t = np.int32 if dtype == "i8i8" else np.float32

    # the existing entry point with a caller workspace
    ti = G.tile_index(f"gemv.k{ksplit}")
    wsb = G.workspace_size(dt, ti, N, K, M)
    WSP = G.DeviceBuffer(0, wsb).zero() if wsb else None
    Y0 = G.DeviceBuffer(0, N * M * 4).zero()
    G.run(0, dt, ti, X, W, Y0, N, K, M, XS, WS, WSP, wsb)
    G.sync(0)
    want = Y0.download(np.empty((N, M), host_t))

    ref = oracle.full_reference(dtype, ops.X(dtype), ops.W(dtype), ops.xscale(dtype), ops.wscale(dtype),
                                N, K, M)
    for call in range(2):
        Y = G.DeviceBuffer(0, N * M * 4).zero()
        G.run_noalloc(0, dt, ksplit, X, W, Y, N, K, M, XS, WS)
        G.sync(0)
        got = Y.download(np.empty((N, M), host_t))
        # same kernel, same split, same reduction order: the same bits
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"call {call}"
        if dtype == "i8i8":
            assert np.array_equal(got.astype(np.int64), ref), f"call {call}"
        else:
            rms = float(np.sqrt(np.mean(ref * ref)))
            rel = np.abs(got.astype(np.float64) - ref) / np.maximum(np.abs(ref), 1e-2 * rms)
            assert rel.max() <= 1e-3, f"call {call}: max rel {rel.max():.3g} against the oracle"


def test_noalloc_rejects_oversized_scratch(gemm):
    G = gemm
    # 64 splits of a 16 x 11008 output need 64*16*11008*4 bytes > the 8 MiB array
    with pytest.raises(G.GemmError) as e:
        G.run_noalloc(0, F.CODE["fp8"], 64, 1, 1, 1, 16, 4096, 11008)
    assert e.value.code == G.GEMM_ERR_ARGS
    assert "exceeds" in G.last_error()


def test_noalloc_rejects_a_split_the_kernel_cannot_take(gemm):
    G = gemm
    # 64 splits of N = 16 rows by M = 2^20 columns need more split-K counter
    # tiles than the counter region holds: rejected with a reason before any
    # launch (the operand pointers are never used)
    with pytest.raises(G.GemmError) as e:
        G.run_noalloc(0, F.CODE["fp16"], 64, 1, 1, 1, 16, 4096, 1 << 20)
    assert e.value.code == G.GEMM_ERR_ARGS
    assert "ksplit" in G.last_error()
