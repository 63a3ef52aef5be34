"""Host logic of the driver against the reference (CPU only).

The table, header and profile formats are compared byte for byte with the
reference's published output (tests/golden/reference_outputs.json); the
operand generators and the driver's own sample-point check with the oracle."""
import json

import numpy as np
import pytest

import oracle
from conftest import golden
from mlpgemm import driver as D
from mlpgemm import formats as F
from mlpgemm.data import Operands

OUT = golden("reference_outputs.json")
TAB = golden("reference_tables.json")


def _parse_row(line):
    p = line.split()
    return D.Row(p[0], int(p[1]), int(p[2]), int(p[3]), p[4], p[5], float(p[6]), float(p[7]),
                 p[8], float(p[9]))


@pytest.mark.parametrize("t", OUT["tables"], ids=[t["where"] for t in OUT["tables"]])
def test_table_reproduces_published_bytes(t):
    rows = [_parse_row(line) for line in t["rows"]]
    lines = D.render_table(rows)
    assert lines[0] == t["header"]
    assert lines[1] == t["rule"]
    assert lines[2:] == t["rows"]


@pytest.mark.parametrize("name", sorted(OUT["profiles"]))
def test_profile_writer_reproduces_published_file(name):
    text = OUT["profiles"][name]
    p = json.loads(text)
    assert D.encode_profile(p["device"], p["architecture"], p["tiles"]) == text


def test_profile_slug_rule():
    # main.swift:321-326: lowercase "<device>_<arch>", non-alphanumerics -> '-'
    assert D.profile_slug("Apple M5 Max", "applegpu_g17s") == "apple-m5-max-applegpu-g17s"
    assert D.profile_slug("NVIDIA B200", "sm_100") == "nvidia-b200-sm-100"
    assert "apple-m5-max-applegpu-g17s.json" in OUT["profiles"]


def test_header_and_log_line_formats():
    lines = OUT["log_lines"]
    assert lines[1] == "timing: gpu"
    assert lines[2] == "dtypes: " + ",".join(F.DTYPES)
    shapes = " | ".join(f"{s.name} N={s.N} K={s.K} M={s.M} iters={s.iters}" for s in D.SUITE)
    assert lines[3] == "shapes: " + shapes
    assert "running square fp16 tile 128x64" in lines
    auto = [l for l in lines if l.startswith("autotune square fp16:")][0]
    # "autotune <shape> <dtype>: <tile> <ms %.4f> | ... ms"
    body = auto.split(": ", 1)[1]
    assert body.endswith(" ms")
    for part in body[:-3].split(" | "):
        tile, ms = part.split()
        assert "%.4f" % float(ms) == ms


def test_suite_shapes_match_reference():
    assert [(s.name, s.N, s.K, s.M, s.iters) for s in D.SUITE] == [
        (s["name"], s["N"], s["K"], s["M"], s["iters"]) for s in TAB["suite_shapes"]["values"]]


def test_parse_args_quirks():
    tiles = ["128x256", "128x128"]
    a = D.parse_args([], tiles)
    assert D.shapes_for(a) == D.SUITE and a.warmup == 5 and a.dtypes == F.DTYPES
    a = D.parse_args(["--N", "1"], tiles)                  # any shape flag -> custom, 4096 defaults
    s = D.shapes_for(a)
    assert len(s) == 1 and (s[0].name, s[0].N, s[0].K, s[0].M, s[0].iters) == ("custom", 1, 4096, 4096, 100)
    a = D.parse_args(["--iters", "7", "--suite"], tiles)   # --suite wins
    assert D.shapes_for(a) == D.SUITE
    a = D.parse_args(["--bogus", "--N", "--M", "8"], tiles)  # unknown key eats the next token
    assert a.M == 8 and a.N == 4096
    a = D.parse_args(["--K", "abc"], tiles)                # non-integer reads as 0
    assert a.K == 0 and a.shape_set
    a = D.parse_args(["--warmup", "2", "--autotune", "--no-profile", "--dtype", "mxfp4/a8"], tiles)
    assert a.warmup == 2 and a.autotune and not a.use_profile and a.dtypes == ["mxfp4/a8"]
    a = D.parse_args(["--dtype", "all", "--N"], tiles)      # trailing key without value is ignored
    assert a.dtypes == F.DTYPES and not a.shape_set
    with pytest.raises(D.BenchExit) as e:
        D.parse_args(["--dtype", "bf16"], tiles)
    assert e.value.code == 1
    with pytest.raises(D.BenchExit) as e:
        D.parse_args(["--tile", "64x32"], tiles)
    assert e.value.code == 1 and "Unknown --tile 64x32" in e.value.msg
    a = D.parse_args(["--peak", "--iters", "3"], tiles)     # peak probe mode (tune/peak.swift)
    assert a.peak and a.iters == 3 and not a.suite
    a = D.parse_args(["--read-probe", "45133824"], tiles)   # streaming-read ceiling instead of the GEMM
    assert a.read_bytes == 45133824 and not a.shape_set
    assert D.parse_args(["--read-probe", "-5"], tiles).read_bytes == 0 == D.parse_args([], tiles).read_bytes
    a = D.parse_args(["--gpus", "2", "--shard", "N", "--allgather"], tiles)
    assert a.gpus == 2 and a.shard == "n" and a.allgather
    assert D.parse_args([], tiles).shard == "m"
    with pytest.raises(D.BenchExit) as e:
        D.parse_args(["--shard", "k"], tiles)
    assert e.value.code == 1


def test_sample_points_match_oracle():
    for N, M, bm, bn in [(4096, 4096, 128, 256), (1, 11008, 16, 32), (200, 272, 128, 128), (1, 1, 8, 8)]:
        assert D.sample_points(N, M, bm, bn) == oracle.sample_points(N, M, bm, bn)


def test_ref_mode_operands_match_oracle():
    N, K, M = 6, 64, 40
    ops = Operands(N, K, M, "ref")
    o = oracle.ref_operands(N, K, M)
    assert np.array_equal(ops.buf("x_half_n").view(np.uint16), o["x_f16"])
    assert np.array_equal(ops.buf("x_i8"), o["x_i8"])
    assert np.array_equal(ops.buf("x_e4m3"), o["x_e4m3"])
    assert np.array_equal(ops.buf("x_fp4"), o["x_fp4"])
    assert np.array_equal(ops.buf("w_half").view(np.uint16), o["w_f16"])
    assert np.array_equal(ops.buf("w_i8"), o["w_i8"])
    assert np.array_equal(ops.buf("w_e4m3"), o["w_e4m3"])
    assert np.array_equal(ops.buf("w_fp4"), o["w_fp4"])
    assert np.array_equal(ops.buf("w_mx"), o["w_mx"])
    assert np.array_equal(ops.buf("wscale"), o["wscale"])
    assert np.array_equal(ops.buf("xscale"), o["xscale"])


@pytest.mark.parametrize("dtype", F.DTYPES)
@pytest.mark.parametrize("mode", ["ref", "seeded"])
def test_driver_decode_matches_oracle(dtype, mode):
    N, K, M = 3, 256, 20
    ops = Operands(N, K, M, mode, 5)
    xd = oracle.decode_x(dtype, ops.X(dtype), ops.xscale(dtype), N, K)
    wd = oracle.decode_w(dtype, ops.W(dtype), ops.wscale(dtype), K, M)
    assert np.array_equal(ops.x_rows(dtype, range(N)), xd)
    assert np.array_equal(ops.w_cols(dtype, range(M)), wd)


def test_seeded_distributions():
    ops = Operands(64, 4096, 64, "seeded", 0)
    assert ops.buf("x_i8").min() >= -127 and ops.buf("x_i8").max() <= 127
    s = ops.buf("wscale")
    assert s.min() == 124 and s.max() == 130
    codes = F.e2m1_unpack(ops.buf("w_mx"), 4096 * 64)
    assert set(np.unique(codes)) == set(range(16))
    e = ops.buf("x_e4m3")
    assert not np.any((e & 0x7F) == 0x7F)                # no NaN codes
    xd = F.e4m3_decode(e)
    assert abs(float(np.std(xd)) - 1.0) < 0.05


def test_check_samples_flags_mismatch():
    N, K, M = 4, 64, 8
    ops = Operands(N, K, M, "seeded", 1)
    ref = ops.x_rows("i8i8", range(N)) @ ops.w_cols("i8i8", range(M))
    Y = ref.astype(np.int32)
    pts = D.sample_points(N, M, 2, 2)
    assert D.check_samples(ops, "i8i8", Y, pts, "custom") == 0.0
    Y[N - 1, M - 1] += 1
    with pytest.raises(D.BenchExit) as e:
        D.check_samples(ops, "i8i8", Y, pts, "custom")
    assert e.value.code == 3
    refd = ops.x_rows("fp8", range(N)) @ ops.w_cols("fp8", range(M))
    Yf = refd.astype(np.float32)
    assert D.check_samples(ops, "fp8", Yf, pts, "custom") < 1e-6
    Yf[0, 0] += 1.0 + abs(refd[0, 0])
    with pytest.raises(D.BenchExit):
        D.check_samples(ops, "fp8", Yf, pts, "custom")


def test_shard_columns_cover_the_matrix():
    from mlpgemm.data import shard_columns
    N, K, M = 2, 64, 11008
    for dtype in ("i8i8", "f4f4", "mxfp4"):
        ops = Operands(N, K, M, "seeded", 3)
        full = ops.w_cols(dtype, range(M))
        got = 0
        for g in range(8):
            W, sc, m0, w = shard_columns(ops, dtype, g, 8)
            sub = Operands(N, K, w, "seeded", 3)
            sub._cache[ops.w_name(dtype)] = W
            if sc is not None:
                sub._cache["wscale"] = sc
            assert np.array_equal(sub.w_cols(dtype, range(w)), full[:, m0:m0 + w])
            got += w
        assert got == M
