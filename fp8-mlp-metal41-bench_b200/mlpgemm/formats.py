"""Number formats and dtype table of the bench (host side, numpy).

Restates the reference's host formats (main.swift:4-83) for operand
generation and for the driver's own sample-point check:
  E4M3  OCP FP8 E4M3FN: 1-4-3, bias 7, exponent 0 -> m * 2^-9, 0x7F/0xFF NaN
  E2M1  OCP FP4: 1-2-1, bias 1, magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6};
        two per byte, the low nibble holds the even element
  UE8M0 2^(code - 127), one scale per 32 elements along K
"""
from __future__ import annotations

import numpy as np

# enum DType raw values and kernel names (main.swift:85-111)
DTYPES = ["fp16", "int8", "i8i8", "fp8", "f8f8", "f4f4", "mxfp4",
          "mxfp4/a4", "mxfp4/a8", "mxfp4/f8"]
KERNELS = ["fp16_mlp_gemm", "int8_mlp_gemm", "i8i8_mlp_gemm", "fp8_mlp_gemm", "f8f8_mlp_gemm",
           "f4f4_mlp_gemm", "mxfp4_mlp_gemm", "mx4x4_mlp_gemm", "mx8x4_mlp_gemm", "f8x4_mlp_gemm"]
CODE = {n: i for i, n in enumerate(DTYPES)}

X_HALF = {"fp16", "int8", "fp8", "mxfp4"}         # half activations
X_E4M3 = {"f8f8", "mxfp4/a8", "mxfp4/f8"}
X_FP4 = {"f4f4", "mxfp4/a4"}
X_SCALED = {"mxfp4/a4", "mxfp4/a8"}
W_MX = {"mxfp4", "mxfp4/a4", "mxfp4/a8", "mxfp4/f8"}   # W stored [M,K] + UE8M0 [M,K/32]

# Dense tensor-core kind each dtype runs on (the roofline denominator).
TC_KIND = {"fp16": "f16", "int8": "f16", "fp8": "f16", "mxfp4": "f16", "i8i8": "i8",
           "f8f8": "f8f6f4", "mxfp4/a8": "f8f6f4", "mxfp4/f8": "f8f6f4",
           "mxfp4/a4": "mxf4", "f4f4": "mxf4"}


def x_bytes(dtype: str, N: int, K: int) -> int:
    if dtype in X_HALF:
        return N * K * 2
    if dtype in X_FP4:
        return N * K // 2
    return N * K


def w_bytes(dtype: str, K: int, M: int) -> int:
    if dtype == "fp16":
        return K * M * 2
    if dtype == "f4f4" or dtype in W_MX:
        return K * M // 2
    return K * M


def y_bytes(dtype: str, N: int, M: int) -> int:
    return N * M * 4


def scale_bytes(dtype: str, N: int, K: int, M: int) -> int:
    b = 0
    if dtype in W_MX:
        b += M * (K // 32)
    if dtype in X_SCALED:
        b += N * (K // 32)
    return b


def algorithmic_bytes(dtype: str, N: int, K: int, M: int) -> int:
    """X + W + Y + scale planes, each read or written once."""
    return x_bytes(dtype, N, K) + w_bytes(dtype, K, M) + y_bytes(dtype, N, M) + \
        scale_bytes(dtype, N, K, M)


def layout_ok(dtype: str, N: int, K: int, M: int) -> bool:
    """The dtype constraints of main.swift:370-376 / :473-476."""
    if N <= 0 or K <= 0 or M <= 0:
        return False
    fp4ok = (N * K) % 2 == 0 and (K * M) % 2 == 0
    mxok = fp4ok and K % 32 == 0
    if dtype == "f4f4" and not fp4ok:
        return False
    if dtype in ("mxfp4", "mxfp4/a4") and not mxok:
        return False
    if dtype in ("mxfp4/a8", "mxfp4/f8") and (not mxok or K % 128 != 0):
        return False
    return True


# ---- decoders --------------------------------------------------------------------
def _e4m3_table() -> np.ndarray:
    b = np.arange(256)
    sign = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 7
    v = np.where(e == 0, m * 2.0 ** -9, (1 + m / 8.0) * np.exp2(e - 7.0))
    v = sign * v
    v[(b & 0x7F) == 0x7F] = np.nan
    return v.astype(np.float32)


E4M3_TABLE = _e4m3_table()
E2M1_TABLE = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6],
                      dtype=np.float32)


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    return E4M3_TABLE[np.asarray(b, dtype=np.uint8)]


def e2m1_unpack(packed: np.ndarray, count: int) -> np.ndarray:
    """Nibble codes of `count` elements (low nibble = even element)."""
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty(p.size * 2, dtype=np.uint8)
    out[0::2] = p & 0xF
    out[1::2] = p >> 4
    return out[:count]


def e2m1_pack(codes: np.ndarray) -> np.ndarray:
    c = np.asarray(codes, dtype=np.uint8).reshape(-1)
    assert c.size % 2 == 0
    return (c[0::2] & 0xF) | ((c[1::2] & 0xF) << 4)


def e2m1_decode(codes: np.ndarray) -> np.ndarray:
    return E2M1_TABLE[np.asarray(codes, dtype=np.uint8) & 0xF]


def ue8m0_decode(c: np.ndarray) -> np.ndarray:
    return np.ldexp(np.float32(1.0), np.asarray(c, dtype=np.int32) - 127).astype(np.float32)


# ---- encoders --------------------------------------------------------------------
def f32_to_e4m3_ref(x: np.ndarray) -> np.ndarray:
    """The reference encoder floatToE4M3 (main.swift:6-27), vectorised.

    Keeps its quirks: round half up on the first dropped mantissa bit, flush
    of |x| < 2^-6 to a signed zero, saturation of |x| >= 256 to 0x7E."""
    x = np.asarray(x, dtype=np.float32)
    bits = np.abs(x).view(np.uint32).astype(np.int64)
    sign = np.where(x < 0, 0x80, 0).astype(np.int64)
    ex = ((bits >> 23) & 0xFF) - 127
    mant = bits & 0x7FFFFF
    e0 = ex + 7
    m3 = (mant >> 20) + ((mant >> 19) & 1)
    carry = m3 == 8
    m3 = np.where(carry, 0, m3)
    e = np.where(carry, e0 + 1, e0)
    ax = np.abs(x)
    # later rules take precedence, in the order the reference tests them
    code = sign | (np.clip(e, 0, 15) << 3) | m3
    code = np.where(e >= 15, sign | 0x7E, code)
    code = np.where(e0 >= 15, sign | 0x7E, code)
    code = np.where(e0 <= 0, sign, code)
    code = np.where(ax >= 448, sign | 0x7E, code)
    code = np.where(ax == 0, sign, code)
    code = np.where(np.isnan(x), 0x7F, code)
    return code.astype(np.uint8)


def f32_to_e4m3_rne(x: np.ndarray) -> np.ndarray:
    """OCP E4M3FN, round to nearest even, subnormals, saturating at +-448."""
    x = np.asarray(x, dtype=np.float64)
    sign = np.where(np.signbit(x), 0x80, 0).astype(np.int64)
    ax = np.minimum(np.abs(np.nan_to_num(x, nan=0.0)), 448.0)
    with np.errstate(divide="ignore"):
        E = np.floor(np.log2(np.where(ax > 0, ax, 1.0))).astype(np.int64)
    E = np.maximum(E, -6)                      # subnormal range shares 2^-6 spacing / 8
    q = np.rint(np.ldexp(ax, 3 - E))           # in [0, 16]
    up = q >= 16
    q = np.where(up, 8, q)
    E = np.where(up, E + 1, E)
    normal = q >= 8
    code = np.where(normal, ((E + 7) << 3) | (q.astype(np.int64) - 8), q.astype(np.int64))
    code = np.minimum(code, 0x7E)
    code = sign | code
    code = np.where(np.isnan(x), 0x7F, code)
    return code.astype(np.uint8)


E2M1_TO_E4M3 = f32_to_e4m3_rne(E2M1_TABLE)     # the widening of fp8_mlp.metal:305-309
E2M1_TO_E4M3[8] = 0x80                         # -0 keeps its sign bit
