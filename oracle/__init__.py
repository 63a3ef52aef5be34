"""CPU oracle for the MLP GEMM -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package.  The
product (``libgemm.so`` and the ``mlpgemm`` package) never does: it must
fail loudly without its CUDA library instead of falling back to this code.

The arithmetic lives in ``mlp_oracle.c`` (a plain-C restatement of the
reference's main.swift host semantics, cited line by line there); this
module loads ``libmlporacle.so`` through ctypes and wraps it for numpy.

Parity pinning: the reference has no golden vectors and its Swift/Metal code
cannot run here.  The decoders are pinned to constant tables read from the
reference sources (``tests/golden/reference_tables.json``); the GEMM check is
restated from main.swift:560-594 and tightened to an fp64 / int64 dot product.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmlporacle.so")

# dtype codes follow `enum DType` (main.swift:85-95)
DTYPES = ["fp16", "int8", "i8i8", "fp8", "f8f8", "f4f4", "mxfp4",
          "mxfp4/a4", "mxfp4/a8", "mxfp4/f8"]
CODE = {name: i for i, name in enumerate(DTYPES)}

_lib = None


def build() -> str:
    """Compile libmlporacle.so with oracle/Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        c_long, c_int, vp = ctypes.c_long, ctypes.c_int, ctypes.c_void_p
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        for fn in ("orc_f32_to_e4m3_ref", "orc_f32_to_e4m3_rne"):
            getattr(L, fn).restype = ctypes.c_uint8
            getattr(L, fn).argtypes = [ctypes.c_float]
        L.orc_e4m3_to_f32.restype = ctypes.c_float
        L.orc_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.orc_e2m1_to_f32.restype = ctypes.c_float
        L.orc_e2m1_to_f32.argtypes = [ctypes.c_uint8]
        L.orc_e2m1_code.restype = ctypes.c_uint8
        L.orc_e2m1_code.argtypes = [c_long]
        L.orc_ue8m0_code.restype = ctypes.c_uint8
        L.orc_ue8m0_code.argtypes = [c_long]
        L.orc_ue8m0_to_f32.restype = ctypes.c_float
        L.orc_ue8m0_to_f32.argtypes = [ctypes.c_uint8]
        L.orc_e2m1_to_e4m3_byte.restype = ctypes.c_uint8
        L.orc_e2m1_to_e4m3_byte.argtypes = [ctypes.c_uint8]
        L.orc_e2m1_at.restype = ctypes.c_float
        L.orc_e2m1_at.argtypes = [vp, c_long]
        L.orc_pack_e2m1.restype = None
        L.orc_pack_e2m1.argtypes = [vp, c_long, vp]
        L.orc_f32_to_e2m1_rne.restype = ctypes.c_uint8
        L.orc_f32_to_e2m1_rne.argtypes = [ctypes.c_float]
        L.orc_quantize_mx.restype = c_int
        L.orc_quantize_mx.argtypes = [c_int, vp, c_long, c_long, vp, vp]
        L.orc_check_layout.restype = c_int
        L.orc_check_layout.argtypes = [c_int, c_long, c_long, c_long]
        L.orc_decode_x.restype = c_int
        L.orc_decode_x.argtypes = [c_int, vp, vp, c_long, c_long, vp]
        L.orc_decode_w.restype = c_int
        L.orc_decode_w.argtypes = [c_int, vp, vp, c_long, c_long, vp]
        L.orc_dot_f64.restype = None
        L.orc_dot_f64.argtypes = [vp, vp, c_long, c_long, vp, vp, c_long, vp]
        L.orc_dot_i64.restype = None
        L.orc_dot_i64.argtypes = [vp, vp, c_long, c_long, vp, vp, c_long, vp]
        L.orc_dot_f32_korder.restype = None
        L.orc_dot_f32_korder.argtypes = [vp, vp, c_long, c_long, vp, vp, c_long, vp]
        L.orc_sample_points.restype = c_int
        L.orc_sample_points.argtypes = [c_long, c_long, c_int, c_int, vp, vp]
        L.orc_host_gemm_f32.restype = None
        L.orc_host_gemm_f32.argtypes = [vp, vp, c_long, c_long, c_long, c_long, vp, c_int]
        L.orc_host_gemm_i32.restype = None
        L.orc_host_gemm_i32.argtypes = [vp, vp, c_long, c_long, c_long, c_long, vp, c_int]
        L.orc_num_threads.restype = c_int
        L.orc_num_threads.argtypes = []
        L.orc_ref_operands.restype = None
        L.orc_ref_operands.argtypes = [c_long, c_long, c_long] + [vp] * 11
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def code(dtype) -> int:
    return CODE[dtype] if isinstance(dtype, str) else int(dtype)


# ---- scalar / vector formats -------------------------------------------------
def e4m3_to_f32(b: int) -> float:
    return lib().orc_e4m3_to_f32(b)


def e2m1_to_f32(n: int) -> float:
    return lib().orc_e2m1_to_f32(n)


def ue8m0_to_f32(c: int) -> float:
    return lib().orc_ue8m0_to_f32(c)


def f32_to_f16_bits(x: float) -> int:
    return lib().orc_f32_to_f16(x)


def f32_to_e4m3_ref(x: float) -> int:
    return lib().orc_f32_to_e4m3_ref(x)


def f32_to_e4m3_rne(x: float) -> int:
    return lib().orc_f32_to_e4m3_rne(x)


def f32_to_e2m1_rne(x: float) -> int:
    return lib().orc_f32_to_e2m1_rne(x)


def quantize_mx(elem: int, src: np.ndarray):
    """OCP MX block quantisation of a [rows, cols] f32 array (cols % 32 == 0):
    elem 0 -> (E2M1 packed [rows, cols/2], UE8M0 [rows, cols/32]); elem 1 ->
    (E4M3 [rows, cols], UE8M0 [rows, cols/32])."""
    src = np.ascontiguousarray(src, dtype=np.float32)
    rows, cols = src.shape
    vals = np.zeros((rows, cols // 2 if elem == 0 else cols), dtype=np.uint8)
    scales = np.zeros((rows, cols // 32), dtype=np.uint8)
    rc = lib().orc_quantize_mx(elem, src.ctypes.data, rows, cols, vals.ctypes.data, scales.ctypes.data)
    if rc:
        raise ValueError("quantize_mx: cols must be a multiple of 32")
    return vals, scales


def e2m1_to_e4m3_byte(n: int) -> int:
    return lib().orc_e2m1_to_e4m3_byte(n)


def check_layout(dtype, N, K, M) -> int:
    return lib().orc_check_layout(code(dtype), N, K, M)


# ---- operands ------------------------------------------------------------------
def decode_x(dtype, X: np.ndarray, xscale, N: int, K: int) -> np.ndarray:
    out = np.empty(N * K, dtype=np.float64)
    X = np.ascontiguousarray(X)
    xs = None if xscale is None else np.ascontiguousarray(xscale, dtype=np.uint8)
    rc = lib().orc_decode_x(code(dtype), _p(X), _p(xs), N, K, _p(out))
    if rc:
        raise ValueError(f"oracle: layout rejected for {dtype} N={N} K={K}")
    return out.reshape(N, K)


def decode_w(dtype, W: np.ndarray, wscale, K: int, M: int) -> np.ndarray:
    out = np.empty(K * M, dtype=np.float64)
    W = np.ascontiguousarray(W)
    ws = None if wscale is None else np.ascontiguousarray(wscale, dtype=np.uint8)
    rc = lib().orc_decode_w(code(dtype), _p(W), _p(ws), K, M, _p(out))
    if rc:
        raise ValueError(f"oracle: layout rejected for {dtype} K={K} M={M}")
    return out.reshape(K, M)


def dot_f64(xd: np.ndarray, wd: np.ndarray, rows, cols) -> np.ndarray:
    K, M = wd.shape
    r = np.ascontiguousarray(rows, dtype=np.int64)
    c = np.ascontiguousarray(cols, dtype=np.int64)
    out = np.empty(len(r), dtype=np.float64)
    lib().orc_dot_f64(_p(np.ascontiguousarray(xd)), _p(np.ascontiguousarray(wd)),
                      K, M, _p(r), _p(c), len(r), _p(out))
    return out


def dot_f32_korder(xd: np.ndarray, wd: np.ndarray, rows, cols) -> np.ndarray:
    K, M = wd.shape
    r = np.ascontiguousarray(rows, dtype=np.int64)
    c = np.ascontiguousarray(cols, dtype=np.int64)
    out = np.empty(len(r), dtype=np.float32)
    lib().orc_dot_f32_korder(_p(np.ascontiguousarray(xd)), _p(np.ascontiguousarray(wd)),
                             K, M, _p(r), _p(c), len(r), _p(out))
    return out


def dot_i64(X: np.ndarray, W: np.ndarray, K: int, M: int, rows, cols) -> np.ndarray:
    r = np.ascontiguousarray(rows, dtype=np.int64)
    c = np.ascontiguousarray(cols, dtype=np.int64)
    out = np.empty(len(r), dtype=np.int64)
    lib().orc_dot_i64(_p(np.ascontiguousarray(X, dtype=np.int8)),
                      _p(np.ascontiguousarray(W, dtype=np.int8)), K, M,
                      _p(r), _p(c), len(r), _p(out))
    return out


def sample_points(N: int, M: int, bm: int, bn: int):
    rows = np.zeros(6, dtype=np.int64)
    cols = np.zeros(6, dtype=np.int64)
    n = lib().orc_sample_points(N, M, bm, bn, _p(rows), _p(cols))
    return list(zip(rows[:n].tolist(), cols[:n].tolist()))


def ref_operands(N: int, K: int, M: int) -> dict:
    """The reference's deterministic operands (main.swift:364-390)."""
    kb = max(K // 32, 1)
    o = {
        "x_f16": np.empty(N * K, np.uint16), "x_i8": np.empty(N * K, np.int8),
        "x_e4m3": np.empty(N * K, np.uint8), "x_fp4": np.empty((N * K) // 2, np.uint8),
        "w_f16": np.empty(K * M, np.uint16), "w_i8": np.empty(K * M, np.int8),
        "w_e4m3": np.empty(K * M, np.uint8), "w_fp4": np.empty((K * M) // 2, np.uint8),
        "w_mx": np.empty((K * M) // 2, np.uint8), "wscale": np.empty(M * kb, np.uint8),
        "xscale": np.empty(N * kb, np.uint8),
    }
    lib().orc_ref_operands(N, K, M, *[_p(o[k]) for k in (
        "x_f16", "x_i8", "x_e4m3", "x_fp4", "w_f16", "w_i8", "w_e4m3", "w_fp4",
        "w_mx", "wscale", "xscale")])
    return o


# ---- host GEMM (CPU baseline) -----------------------------------------------
def num_threads() -> int:
    return lib().orc_num_threads()


def host_gemm_f32(xf: np.ndarray, wf: np.ndarray, row0: int, nrows: int,
                  nthreads: int = 0) -> np.ndarray:
    """f32 K-order GEMM over rows [row0, row0+nrows) (main.swift:577-583)."""
    K, M = wf.shape
    Y = np.empty((nrows, M), dtype=np.float32)
    lib().orc_host_gemm_f32(_p(np.ascontiguousarray(xf, np.float32)),
                            _p(np.ascontiguousarray(wf, np.float32)),
                            K, M, row0, nrows, _p(Y), nthreads)
    return Y


def host_gemm_i32(X: np.ndarray, W: np.ndarray, K: int, M: int, row0: int,
                  nrows: int, nthreads: int = 0) -> np.ndarray:
    """int32 GEMM over rows [row0, row0+nrows) (main.swift:563-568)."""
    Y = np.empty((nrows, M), dtype=np.int32)
    lib().orc_host_gemm_i32(_p(np.ascontiguousarray(X, np.int8)),
                            _p(np.ascontiguousarray(W, np.int8)),
                            K, M, row0, nrows, _p(Y), nthreads)
    return Y


def full_reference(dtype, X, W, xscale, wscale, N, K, M):
    """fp64 Y over the whole output (exact int64 for i8i8).

    i8i8 (main.swift:563-568): the product runs as an fp64 BLAS GEMM and is
    exact, whatever order the BLAS sums in: every product is an integer of
    magnitude <= 127*127 < 2^14, so every partial sum is an integer below
    K * 2^14 < 2^53 for any K < 2^39, and fp64 represents all of them.  (A
    numpy int64 matmul gives the same values without BLAS, far too slowly for
    the 4096^3 suite shape.)"""
    if code(dtype) == CODE["i8i8"]:
        x = np.asarray(X, np.int8).reshape(N, K).astype(np.float64)
        w = np.asarray(W, np.int8).reshape(K, M).astype(np.float64)
        return (x @ w).astype(np.int64)
    xd = decode_x(dtype, X, xscale, N, K)
    wd = decode_w(dtype, W, wscale, K, M)
    return xd @ wd
