"""The C ABI library loads on a CPU-only host and exports every symbol that
include/mlpgemm.h declares; host-side tables behave like the reference's."""
import os
import re

import pytest

from conftest import ROOT, golden
from mlpgemm import formats as F
from mlpgemm import lib as G


def header_symbols():
    with open(os.path.join(ROOT, "include", "mlpgemm.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gemm_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    L = G.lib()
    syms = header_symbols()
    assert len(syms) >= 25
    for s in syms:
        assert hasattr(L, s), s
    assert sorted(G.EXPORTS) == syms


def test_init_fails_loudly_without_gpu():
    if G.device_count() > 0:
        pytest.skip("a GPU is present")
    with pytest.raises(G.GemmError) as e:
        G.init(0)
    assert e.value.code == G.GEMM_ERR_INIT


def test_dtype_and_kernel_names_match_reference():
    L = G.lib()
    ref = golden("reference_tables.json")["dtypes"]["values"]
    assert [L.gemm_dtype_name(i).decode() for i in range(10)] == ref == F.DTYPES
    assert [L.gemm_kernel_name(i).decode() for i in range(10)] == F.KERNELS


def test_tile_table():
    names = G.tile_names()
    assert "256x256" in names and "128x256" in names and "128x128" in names
    assert all(G.tile_index(n) == i for i, n in enumerate(names))
    assert G.tile_index("64x32") == -1


def test_layout_rules_and_tile_support():
    L = G.lib()
    assert L.gemm_check_layout(F.CODE["mxfp4/a8"], 4, 96, 8) == G.GEMM_ERR_ARGS
    assert L.gemm_check_layout(F.CODE["mxfp4/a8"], 4, 128, 8) == G.GEMM_OK
    t256 = G.tile_index("128x256")
    assert G.tile_supported(F.CODE["i8i8"], t256, 4096, 4096, 4096)
    assert not G.tile_supported(F.CODE["i8i8"], t256, 4096, 4100, 4096)   # TMA stride rule
    # thin rows: the CUDA-core kernel; the default tile is a gemv tile
    assert G.tile_names()[G.default_tile(F.CODE["int8"], 1, 4096, 11008)].startswith("gemv")
    assert G.tile_names()[G.default_tile(F.CODE["i8i8"], 4096, 4096, 4096)] == "256x256"
    # A16 kinds: W widened once to f16 for the CTA pair from N = 256 on
    for d in ("int8", "fp8", "mxfp4"):
        assert G.tile_names()[G.default_tile(F.CODE[d], 2048, 4096, 11008)] == "256x256"
        assert G.tile_names()[G.default_tile(F.CODE[d], 128, 4096, 11008)] == "128x256"
        assert G.workspace_size(F.CODE[d], G.tile_index("256x256"), 2048, 4096, 11008) >= 2 * 4096 * 11008
    # 3 <= N <= 16: the tensor-core thin tile where it covers the dtype
    for d in ("fp16", "int8", "i8i8", "fp8", "f8f8", "mxfp4"):
        assert G.tile_names()[G.default_tile(F.CODE[d], 8, 4096, 11008)] == "16x128"
    assert G.tile_names()[G.default_tile(F.CODE["f4f4"], 8, 4096, 11008)].startswith("gemv")
    # MX kinds with E2M1 / E4M3 activations at 3 <= N <= 16: the warp-MMA thin tile
    for d in ("mxfp4/a4", "mxfp4/a8", "mxfp4/f8"):
        assert G.tile_names()[G.default_tile(F.CODE[d], 8, 4096, 11008)] == "gemv.mma"
        assert G.tile_names()[G.default_tile(F.CODE[d], 2, 4096, 11008)].startswith("gemv.k")
    # f4f4, mxfp4/f8 (unit scale cells copied once) and mxfp4/a4: two accumulators on 256x224
    assert G.tile_names()[G.default_tile(F.CODE["f4f4"], 2048, 4096, 11008)] == "256x224"
    assert G.tile_names()[G.default_tile(F.CODE["mxfp4/f8"], 2048, 4096, 11008)] == "256x224"
    assert G.tile_names()[G.default_tile(F.CODE["mxfp4/a4"], 2048, 4096, 11008)] == "256x224"
    assert G.tile_names()[G.default_tile(F.CODE["mxfp4/a8"], 2048, 4096, 11008)] == "256x256"
    assert G.tile_names()[G.default_tile(F.CODE["f4f4"], 1, 4096, 11008)] == "gemv.k4"
    # [K,M] GEMVs with two or more rows per CTA: at most 2048 K rows per CTA,
    # at least one CTA per SM at N = 2 and three from N = 3 on (f4f4 has no
    # tensor-core thin tile)
    for d in ("fp16", "int8", "i8i8", "fp8", "f8f8", "f4f4"):
        assert G.tile_names()[G.default_tile(F.CODE[d], 2, 4096, 11008)] == "gemv.k2", d
        assert G.tile_names()[G.default_tile(F.CODE[d], 2, 11008, 4096)] == "gemv.k8", d
    for N in (3, 4, 8):
        assert G.tile_names()[G.default_tile(F.CODE["f4f4"], N, 4096, 11008)] == "gemv.k4"
        assert G.tile_names()[G.default_tile(F.CODE["f4f4"], N, 11008, 4096)] == "gemv.k8"
    assert G.tile_names()[G.default_tile(F.CODE["mxfp4"], 2, 4096, 11008)] == "gemv.k1"
    # 256x224 (two accumulators): the block-scaled kinds and f4f4 only
    t224 = G.tile_index("256x224")
    for d in ("mxfp4/a4", "f4f4"):
        assert G.tile_supported(F.CODE[d], t224, 2048, 4096, 11008)
    assert G.tile_supported(F.CODE["mxfp4/a8"], t224, 2048, 4096, 11008)
    assert not G.tile_supported(F.CODE["mxfp4/a8"], t224, 2048, 4064, 11008)   # K % 128
    for d in ("fp16", "i8i8", "f8f8", "int8", "mxfp4"):
        assert not G.tile_supported(F.CODE[d], t224, 2048, 4096, 11008), d
    # gemv.mma: N <= 16; [K,M] kinds need K % 4 and 16-byte rows, the MX kinds K % 128
    tm = G.tile_index("gemv.mma")
    assert G.tile_supported(F.CODE["int8"], tm, 1, 4096, 11008)
    assert G.tile_supported(F.CODE["fp16"], tm, 16, 4096, 11008)
    assert not G.tile_supported(F.CODE["fp16"], tm, 17, 4096, 11008)
    assert not G.tile_supported(F.CODE["int8"], tm, 1, 4094, 11008)
    assert not G.tile_supported(F.CODE["int8"], tm, 1, 4096, 11000)
    assert G.tile_supported(F.CODE["mxfp4/a4"], tm, 8, 4096, 1000)
    assert not G.tile_supported(F.CODE["mxfp4/a4"], tm, 8, 4064, 1000)
    assert not G.tile_supported(F.CODE["i8i8"], tm, 1, 4096, 11008)
    assert not G.tile_supported(F.CODE["f4f4"], tm, 1, 4096, 11008)
    assert G.workspace_size(F.CODE["int8"], tm, 1, 4096, 11008) > 65536
    t16 = G.tile_index("16x128")
    assert G.tile_supported(F.CODE["fp16"], t16, 16, 4096, 11008)
    assert not G.tile_supported(F.CODE["fp16"], t16, 17, 4096, 11008)     # N <= 16
    assert not G.tile_supported(F.CODE["i8i8"], t16, 4, 4104, 11008)      # byte X: K % 16
    assert not G.tile_supported(F.CODE["mxfp4/a8"], t16, 4, 4096, 11008)  # no thin kernel for this kind


def test_workspace_sizes():
    t = G.tile_index("gemv.k32")
    assert G.workspace_size(F.CODE["int8"], t, 1, 4096, 11008) == 65536 + 32 * 11008 * 4
    assert G.workspace_size(F.CODE["int8"], G.tile_index("gemv.k1"), 1, 4096, 11008) == 0


def test_gather_support_table():
    # the fused all-gather rides on the tensor-core epilogues: every CTA-pair
    # tile, and the 1-CTA tiles except the converter-warp A16 kernel
    pair, one = G.tile_index("256x256"), G.tile_index("128x256")
    for d in F.DTYPES:
        assert G.gather_supported(F.CODE[d], pair), d
    for d in ("fp16", "i8i8", "f8f8", "f4f4", "mxfp4/a4", "mxfp4/a8", "mxfp4/f8"):
        assert G.gather_supported(F.CODE[d], one), d
    for d in ("int8", "fp8", "mxfp4"):
        assert not G.gather_supported(F.CODE[d], one), d
    for t in ("16x128", "gemv.k1", "gemv.k4"):
        assert not G.gather_supported(F.CODE["fp16"], G.tile_index(t)), t
    assert not G.gather_supported(99, pair) and not G.gather_supported(0, 999)


def test_gather_entry_points_fail_loudly_without_gpu():
    if G.device_count() > 0:
        pytest.skip("a GPU is present")
    L = G.lib()
    with pytest.raises(G.GemmError) as e:   # no initialised device
        G.run_gather(0, F.CODE["fp16"], G.tile_index("256x256"), 1 << 20, 1 << 20, 1 << 20, 256, 256, 256,
                     peers=[1 << 20])
    assert e.value.code == G.GEMM_ERR_INIT
    with pytest.raises(G.GemmError):
        G.peer_alloc(0, 4096)
    with pytest.raises(G.GemmError):
        G.peer_open(0, bytes(G.PEER_HANDLE_BYTES))
    import ctypes
    assert L.gemm_peer_alloc(0, 16, None, None) == G.GEMM_ERR_ARGS
    assert L.gemm_peer_open(0, None, ctypes.byref(ctypes.c_void_p())) == G.GEMM_ERR_ARGS
