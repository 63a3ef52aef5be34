"""The oracle pinned against the reference's own tables and semantics (CPU).

The reference ships no golden vectors; these checks pin the oracle to the
constant tables read out of its sources (tests/golden/reference_tables.json,
made by tests/golden/make_golden.py) and to independent implementations
(numpy float16, torch float8_e4m3fn)."""
import math

import numpy as np
import pytest

import oracle
from conftest import golden

T = golden("reference_tables.json")


def test_e2m1_magnitudes_match_reference_table():
    mags = T["e2m1_magnitudes"]["values"]          # main.swift:45
    for n in range(16):
        v = oracle.e2m1_to_f32(n)
        assert abs(v) == mags[n & 7]
        assert math.copysign(1.0, v) == (-1.0 if n & 8 else 1.0)


def test_e2m1_to_e4m3_lut_matches_reference():
    lut = T["e2m1_to_e4m3_lut"]["values"]           # fp8_mlp.metal:306-309
    for n in range(16):
        assert oracle.e2m1_to_e4m3_byte(n) == lut[n]
        # and the widening is exact: E4M3 decode of the LUT byte == E2M1 value
        assert oracle.e4m3_to_f32(lut[n]) == oracle.e2m1_to_f32(n)


def test_code_cycles_match_reference():
    assert [oracle.lib().orc_e2m1_code(i) for i in range(10)] == T["e2m1_code_cycle"]["values"]
    assert [oracle.lib().orc_ue8m0_code(i) for i in range(4)] == T["ue8m0_code_cycle"]["values"]


def test_e4m3_decode_all_256_against_torch():
    torch = pytest.importorskip("torch")
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8)
    ref = codes.view(torch.float8_e4m3fn).to(torch.float32).numpy()
    for b in range(256):
        v = oracle.e4m3_to_f32(b)
        if (b & 0x7F) == 0x7F:
            assert math.isnan(v) and math.isnan(ref[b])
        else:
            assert v == ref[b], b


def test_ue8m0_decode_all_256():
    for c in range(256):
        with np.errstate(over="ignore"):
            want = np.float32(np.ldexp(1.0, c - 127))
        assert oracle.ue8m0_to_f32(c) == want, c


def test_f16_conversion_matches_numpy():
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.standard_normal(20000) * 10.0 ** rng.integers(-8, 6, 20000),
                         [0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e-8, 2.0 ** -24, 2.0 ** -25,
                          3 * 2.0 ** -26]]).astype(np.float32)
    got = np.array([oracle.f32_to_f16_bits(float(x)) for x in xs], dtype=np.uint16)
    with np.errstate(over="ignore"):
        want = xs.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)


def test_rne_encoder_against_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(2)
    xs = np.concatenate([rng.standard_normal(50000) * 8, rng.standard_normal(5000) * 0.01,
                         np.linspace(-448, 448, 4001)]).astype(np.float32)
    want = torch.from_numpy(xs).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    got = np.array([oracle.f32_to_e4m3_rne(float(x)) for x in xs], dtype=np.uint8)
    assert np.array_equal(got, want)


def test_reference_encoder_quirks():
    # main.swift:6-27: half-up rounding on the first dropped bit, flush below
    # 2^-6, saturation of everything from 256 up to 0x7E.
    assert oracle.f32_to_e4m3_ref(0.0) == 0x00
    assert oracle.f32_to_e4m3_ref(-0.0) == 0x00          # `x < 0` is false for -0
    assert oracle.f32_to_e4m3_ref(2.0 ** -7) == 0x00     # flushed (RNE gives a subnormal)
    assert oracle.f32_to_e4m3_rne(2.0 ** -7) == 0x04
    assert oracle.f32_to_e4m3_ref(300.0) == 0x7E
    assert oracle.f32_to_e4m3_rne(300.0) == 0x79        # 288 = 1.125 * 2^8 (grid of 32)
    assert oracle.f32_to_e4m3_ref(1.0625) == 0x39        # tie rounds up
    assert oracle.f32_to_e4m3_rne(1.0625) == 0x38        # tie rounds to even
    assert oracle.f32_to_e4m3_ref(float("nan")) == 0x7F


def test_layout_rules():
    # main.swift:473-476
    assert oracle.check_layout("f4f4", 1, 3, 3) == 1      # odd counts
    assert oracle.check_layout("f4f4", 2, 3, 2) == 0
    assert oracle.check_layout("mxfp4", 4, 48, 8) == 1   # K % 32
    assert oracle.check_layout("mxfp4/a4", 4, 64, 8) == 0
    assert oracle.check_layout("mxfp4/a8", 4, 64, 8) == 1  # K % 128
    assert oracle.check_layout("mxfp4/f8", 4, 128, 8) == 0
    assert oracle.check_layout("i8i8", 0, 4, 4) == 1


def test_sample_points():
    # main.swift:452-466
    assert oracle.sample_points(4096, 4096, 128, 64) == [
        (0, 0), (0, 63), (0, 64), (127, 0), (128, 64), (4095, 4095)]
    assert oracle.sample_points(1, 11008, 16, 32) == [(0, 0), (0, 31), (0, 32), (0, 11007)]
    assert oracle.sample_points(1, 1, 16, 32) == [(0, 0)]


def test_decode_semantics_mx_weight_transposed():
    # refWeight for the MX family reads W[m*K+k] and wscale[m*(K/32)+k/32]
    K, M = 64, 3
    codes = np.arange(K * M, dtype=np.uint8) % 16
    W = ((codes[0::2] & 0xF) | (codes[1::2] << 4)).astype(np.uint8)
    ws = np.array([125, 126, 127, 128, 129, 130], dtype=np.uint8)
    wd = oracle.decode_w("mxfp4", W, ws, K, M)
    for k in (0, 1, 31, 32, 63):
        for m in range(M):
            want = oracle.e2m1_to_f32(int(codes[m * K + k])) * 2.0 ** (int(ws[m * 2 + k // 32]) - 127)
            assert wd[k, m] == want


def test_dot_products_agree():
    ops = oracle.ref_operands(8, 256, 40)
    xd = oracle.decode_x("f8f8", ops["x_e4m3"], None, 8, 256)
    wd = oracle.decode_w("f8f8", ops["w_e4m3"], None, 256, 40)
    pts = [(0, 0), (7, 39), (3, 17)]
    r = [p[0] for p in pts]
    c = [p[1] for p in pts]
    f64 = oracle.dot_f64(xd, wd, r, c)
    f32 = oracle.dot_f32_korder(xd, wd, r, c)
    assert np.allclose(f64, (xd @ wd)[r, c])
    assert np.allclose(f32, f64, rtol=1e-5, atol=1e-5)
    i64 = oracle.dot_i64(ops["x_i8"], ops["w_i8"], 256, 40, r, c)
    x = ops["x_i8"].reshape(8, 256).astype(np.int64)
    w = ops["w_i8"].reshape(256, 40).astype(np.int64)
    assert np.array_equal(i64, (x @ w)[r, c])


def test_host_gemm_matches_korder_dot():
    ops = oracle.ref_operands(9, 128, 300)
    xd = oracle.decode_x("fp16", ops["x_f16"], None, 9, 128).astype(np.float32)
    wd = oracle.decode_w("fp16", ops["w_f16"], None, 128, 300).astype(np.float32)
    Y = oracle.host_gemm_f32(xd, wd, 2, 5)
    r = [2 + i for i in range(5) for _ in range(300)]
    c = [j for _ in range(5) for j in range(300)]
    want = oracle.dot_f32_korder(xd.astype(np.float64), wd.astype(np.float64), r, c)
    assert np.array_equal(Y.reshape(-1), want)       # bit-identical: same K order in f32
    Yi = oracle.host_gemm_i32(ops["x_i8"], ops["w_i8"], 128, 300, 0, 9)
    x = ops["x_i8"].reshape(9, 128).astype(np.int64)
    w = ops["w_i8"].reshape(128, 300).astype(np.int64)
    assert np.array_equal(Yi, x @ w)
