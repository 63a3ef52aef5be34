"""Host operands for one shape, in two data modes.

`ref`    the reference's deterministic index patterns (main.swift:364-390):
         X = (i%97-48)*0.02, W = (i%53-26)*0.05 as half / E4M3 (the
         reference's own encoder) / int8, FP4 code cycles with offsets 0 (X),
         +3 (f4f4 W) and +5 (MX W), UE8M0 cycles 125..128 with offsets 0 (W)
         and +1 (X).
`seeded` i.i.d. values from numpy PCG64(seed): half U[-1,1] (fp16) or
         N(0,1) (A16 activations), int8 U{-127..127}, E4M3 = RNE(N(0,1)),
         E2M1 codes U{0..15}, UE8M0 U{124..130}.

Buffers are created lazily and shared across dtypes, as the reference shares
them (main.swift:391-418).  Each buffer is a flat numpy array of the exact
bytes the C ABI takes.
"""
from __future__ import annotations

import numpy as np

from . import formats as F

_BUF_IDS = {"x_half_u": 1, "x_half_n": 2, "x_i8": 3, "x_e4m3": 4, "x_fp4": 5, "xscale": 6,
            "w_half": 7, "w_i8": 8, "w_e4m3": 9, "w_fp4": 10, "w_mx": 11, "wscale": 12}


class Operands:
    def __init__(self, N: int, K: int, M: int, mode: str = "seeded", seed: int = 0):
        if mode not in ("ref", "seeded"):
            raise ValueError(f"unknown data mode {mode!r}")
        self.N, self.K, self.M = N, K, M
        self.mode, self.seed = mode, seed
        self._cache: dict[str, np.ndarray] = {}

    # ---- buffer construction ---------------------------------------------------
    def _rng(self, name: str) -> np.random.Generator:
        return np.random.Generator(np.random.PCG64([self.seed, _BUF_IDS[name]]))

    def _make(self, name: str) -> np.ndarray:
        N, K, M = self.N, self.K, self.M
        xc, wc, kb = N * K, K * M, max(K // 32, 1)
        if self.mode == "ref":
            if name.startswith("x_half"):
                i = np.arange(xc, dtype=np.int64)
                return (((i % 97) - 48).astype(np.float32) * np.float32(0.02)).astype(np.float16)
            if name == "x_i8":
                return ((np.arange(xc, dtype=np.int64) % 97) - 48).astype(np.int8)
            if name == "x_e4m3":
                i = np.arange(xc, dtype=np.int64)
                return F.f32_to_e4m3_ref(((i % 97) - 48).astype(np.float32) * np.float32(0.02))
            if name == "x_fp4":
                return F.e2m1_pack(_cycle_codes(xc, 0))
            if name == "xscale":
                return (125 + (np.arange(N * kb, dtype=np.int64) + 1) % 4).astype(np.uint8)
            if name == "w_half":
                i = np.arange(wc, dtype=np.int64)
                return (((i % 53) - 26).astype(np.float32) * np.float32(0.05)).astype(np.float16)
            if name == "w_i8":
                return ((np.arange(wc, dtype=np.int64) % 53) - 26).astype(np.int8)
            if name == "w_e4m3":
                i = np.arange(wc, dtype=np.int64)
                return F.f32_to_e4m3_ref(((i % 53) - 26).astype(np.float32) * np.float32(0.05))
            if name == "w_fp4":
                return F.e2m1_pack(_cycle_codes(wc, 3))
            if name == "w_mx":
                return F.e2m1_pack(_cycle_codes(wc, 5))
            if name == "wscale":
                return (125 + np.arange(M * kb, dtype=np.int64) % 4).astype(np.uint8)
        else:
            r = self._rng(name)
            if name == "x_half_u":
                return r.uniform(-1.0, 1.0, xc).astype(np.float16)
            if name == "x_half_n":
                return r.standard_normal(xc, dtype=np.float32).astype(np.float16)
            if name == "x_i8":
                return r.integers(-127, 128, xc, dtype=np.int8)
            if name == "x_e4m3":
                return F.f32_to_e4m3_rne(r.standard_normal(xc, dtype=np.float32))
            if name == "x_fp4":
                return F.e2m1_pack(r.integers(0, 16, xc, dtype=np.uint8))
            if name == "xscale":
                return r.integers(124, 131, N * kb, dtype=np.uint8)
            if name == "w_half":
                return r.uniform(-1.0, 1.0, wc).astype(np.float16)
            if name == "w_i8":
                return r.integers(-127, 128, wc, dtype=np.int8)
            if name == "w_e4m3":
                return F.f32_to_e4m3_rne(r.standard_normal(wc, dtype=np.float32))
            if name == "w_fp4":
                return F.e2m1_pack(r.integers(0, 16, wc, dtype=np.uint8))
            if name == "w_mx":
                return F.e2m1_pack(r.integers(0, 16, wc, dtype=np.uint8))
            if name == "wscale":
                return r.integers(124, 131, M * kb, dtype=np.uint8)
        raise KeyError(name)

    def buf(self, name: str) -> np.ndarray:
        if name not in self._cache:
            self._cache[name] = self._make(name)
        return self._cache[name]

    # ---- per-dtype views (main.swift:408-418, :477-483) -------------------------
    def x_name(self, dtype: str) -> str:
        if dtype == "fp16":
            return "x_half_u" if self.mode == "seeded" else "x_half_n"
        if dtype in F.X_HALF:
            return "x_half_n"
        if dtype == "i8i8":
            return "x_i8"
        if dtype in F.X_E4M3:
            return "x_e4m3"
        return "x_fp4"

    def w_name(self, dtype: str) -> str:
        return {"fp16": "w_half", "int8": "w_i8", "i8i8": "w_i8", "fp8": "w_e4m3",
                "f8f8": "w_e4m3", "f4f4": "w_fp4"}.get(dtype, "w_mx")

    def X(self, dtype: str) -> np.ndarray:
        return self.buf(self.x_name(dtype))

    def W(self, dtype: str) -> np.ndarray:
        return self.buf(self.w_name(dtype))

    def xscale(self, dtype: str):
        return self.buf("xscale") if dtype in F.X_SCALED else None

    def wscale(self, dtype: str):
        return self.buf("wscale") if dtype in F.W_MX else None

    # ---- decoded operands (refActivation / refWeight, main.swift:419-449) -------
    def x_rows(self, dtype: str, rows) -> np.ndarray:
        """Decoded activations of the given rows, float64 [len(rows), K]."""
        K = self.K
        rows = np.asarray(rows, dtype=np.int64)
        idx = rows[:, None] * K + np.arange(K, dtype=np.int64)[None, :]
        X = self.X(dtype)
        if dtype in F.X_HALF:
            v = X[idx].astype(np.float64)
        elif dtype == "i8i8":
            v = X[idx].astype(np.float64)
        elif dtype in F.X_E4M3:
            v = F.e4m3_decode(X[idx]).astype(np.float64)
        else:
            b = X[idx >> 1]
            v = F.e2m1_decode(np.where(idx & 1, b >> 4, b & 0xF)).astype(np.float64)
        if dtype in F.X_SCALED:
            s = self.buf("xscale")[rows[:, None] * (K // 32) + np.arange(K)[None, :] // 32]
            v = v * F.ue8m0_decode(s).astype(np.float64)
        return v

    def w_cols(self, dtype: str, cols) -> np.ndarray:
        """Decoded weights of the given output columns, float64 [K, len(cols)]."""
        K, M = self.K, self.M
        cols = np.asarray(cols, dtype=np.int64)
        W = self.W(dtype)
        k = np.arange(K, dtype=np.int64)[:, None]
        if dtype in F.W_MX:
            idx = cols[None, :] * K + k
            b = W[idx >> 1]
            v = F.e2m1_decode(np.where(idx & 1, b >> 4, b & 0xF)).astype(np.float64)
            s = self.buf("wscale")[cols[None, :] * (K // 32) + k // 32]
            return v * F.ue8m0_decode(s).astype(np.float64)
        idx = k * M + cols[None, :]
        if dtype == "fp16" or dtype in ("int8", "i8i8"):
            return W[idx].astype(np.float64)
        if dtype in ("fp8", "f8f8"):
            return F.e4m3_decode(W[idx]).astype(np.float64)
        b = W[idx >> 1]
        return F.e2m1_decode(np.where(idx & 1, b >> 4, b & 0xF)).astype(np.float64)


def _cycle_codes(count: int, offset: int) -> np.ndarray:
    """e2m1Code(i + offset) over i < count (main.swift:50-53)."""
    cyc = np.array([0x0, 0x1, 0x2, 0x3, 0x4, 0x5, 0x6, 0x9, 0xA, 0xC], dtype=np.uint8)
    return cyc[(np.arange(count, dtype=np.int64) + offset) % 10]


def shard_columns(ops: Operands, dtype: str, g: int, G: int):
    """(W shard, wscale shard, column offset, width) of GPU g of G along M.

    [K,M] weights are sliced into contiguous [K, M/G] blocks; the [M,K]
    mxfp4 weights and their [M,K/32] scales are row slices.  FP4 [K,M] slice
    widths are kept even so every shard row starts on a byte."""
    M, K = ops.M, ops.K
    align = 32 if G > 1 else 1
    base = -(-M // G)
    base = -(-base // align) * align
    m0 = min(g * base, M)
    m1 = min(m0 + base, M)
    width = m1 - m0
    W = ops.W(dtype)
    if dtype in F.W_MX:
        ws = W.reshape(M, K // 2)[m0:m1].copy().reshape(-1)
        sc = ops.buf("wscale").reshape(M, K // 32)[m0:m1].copy().reshape(-1)
        return ws, sc, m0, width
    if dtype == "f4f4":
        codes = F.e2m1_unpack(W, K * M).reshape(K, M)[:, m0:m1]
        return F.e2m1_pack(codes.reshape(-1)), None, m0, width
    return W.reshape(K, M)[:, m0:m1].copy().reshape(-1), None, m0, width
