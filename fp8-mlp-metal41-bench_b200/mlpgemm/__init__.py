"""mlpgemm -- host side of the B200 MLP GEMM (Y[N,M] = X[N,K] @ W[K,M]).

A drop-in for the Anemll/fp8-mlp-metal41-bench operator surface: the same
dtype names, operand layouts, CLI flags, tile profiles and output table,
driving the sm_100a kernels of libgemm.so through its C ABI (lib.py).
"""
from . import formats, lib
from .formats import CODE, DTYPES

__all__ = ["formats", "lib", "CODE", "DTYPES"]
