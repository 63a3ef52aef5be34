"""The peak probe and the autotune sweep on the GPU.

gemm_peak_probe restates tune/peak.metal:29-87 with tune/peak.swift:42-63 as
host: MMAs of each tcgen05 kind on operands resident in shared memory.  Each
kind's rate must be a finite, positive number, and its ratio to the f16
probe must match the B200's dense-rate ratios (int8 and the 8-bit float
kinds twice the f16 rate, kind::mxf4 four times) within 25 %.

--autotune (main.swift:523-539, profile writer :639-650) sweeps every tile
that can run a dtype and shape, keeps the fastest, writes it into
profiles/<device slug>.json under the working directory and then runs the
shape with that tile; the run's own sample check (main.swift:560-594) must
pass (exit status 0), the profile must name a supported tile, and that tile
must match the oracle over the whole output.
"""
import json
import math
import os

import numpy as np
import pytest

import oracle
from mlpgemm import driver as D
from mlpgemm import formats as F
from mlpgemm.data import Operands

pytestmark = pytest.mark.gpu

# probe kind -> dense rate relative to kind::f16 on the same number of SMs
RATIO = {0: 1.0, 1: 2.0, 2: 2.0, 3: 2.0, 4: 4.0, 5: 1.0, 6: 2.0, 7: 2.0}
# pair kinds with B MN-major, and the block-scaled pairs without and with the
# GEMM's per-stage scale-cell copies: finite and positive (their rate is what
# they measure)
MN_KINDS = (8, 9, 10, 11, 12, 13, 14)


def test_peak_probe_every_kind(gemm):
    rates = {k: gemm.peak_probe(0, k, 4096, 5) for k in RATIO}
    print("peak probe TFLOP/s (TOP/s for i8):", {k: round(v, 1) for k, v in rates.items()})
    for k, v in rates.items():
        assert math.isfinite(v) and v > 0, (k, v)
    f16 = rates[0]
    # f16 on one SM per tile reaches at least a fifth of B200's nominal dense rate
    assert f16 > 0.2 * 2250.0
    for k, v in rates.items():
        r = v / f16
        assert 0.75 * RATIO[k] <= r <= 1.25 * RATIO[k], f"kind {k}: {v:.1f} is {r:.2f}x f16, want ~{RATIO[k]}x"
    mn = {k: gemm.peak_probe(0, k, 4096, 5) for k in MN_KINDS}
    print("pair probes (B MN-major; block-scaled):", {k: round(v, 1) for k, v in mn.items()})
    for k, v in mn.items():
        assert math.isfinite(v) and v > 0, (k, v)
    # the per-stage scale copies cost MMA time, never add to it
    assert mn[13] <= 1.05 * mn[11] and mn[14] <= 1.05 * mn[12]


def test_peak_probe_rejects_unknown_kind(gemm):
    with pytest.raises(gemm.GemmError) as e:
        gemm.peak_probe(0, 99, 16, 1)
    assert e.value.code == gemm.GEMM_ERR_ARGS


def test_read_probe_rate_and_arguments(gemm):
    """The streaming-read ceiling of the thin rows: a 64 MiB read from a cold L2
    must land between a fifth of B200's nominal 7.7 TB/s and just above it, and
    a misaligned or ragged request is an argument error."""
    import torch
    nb = 64 << 20
    buf = torch.zeros(nb, dtype=torch.uint8, device="cuda:0")
    fl = torch.zeros(256 << 20, dtype=torch.uint8, device="cuda:0")
    ms = gemm.read_probe(0, buf, nb, warmup=2, iters=5, flush=fl, flush_bytes=fl.numel())
    gbs = nb / (sorted(ms)[len(ms) // 2] / 1e3) / 1e9
    print(f"read probe: {gbs:.0f} GB/s")
    assert math.isfinite(gbs) and 0.2 * 7700 < gbs < 1.1 * 7700
    for args in ((buf, nb - 8), (buf[1:], 1 << 20), (buf, 0)):
        with pytest.raises(gemm.GemmError) as e:
            gemm.read_probe(0, args[0], args[1], warmup=0, iters=1)
        assert e.value.code == gemm.GEMM_ERR_ARGS


@pytest.mark.parametrize("dtype,N,K,M", [("i8i8", 256, 512, 768), ("mxfp4", 1, 1024, 1536),
                                         ("mxfp4/a8", 384, 512, 640)])
def test_autotune_writes_a_profile_and_picks_a_parity_green_tile(gemm, tmp_path, monkeypatch, capsys, dtype,
                                                                 N, K, M):
    G = gemm
    monkeypatch.chdir(tmp_path)
    rc = D.main(["--N", str(N), "--K", str(K), "--M", str(M), "--dtype", dtype, "--iters", "5",
                 "--warmup", "1", "--autotune"])
    text = capsys.readouterr().out
    assert rc == 0, text
    assert f"autotune custom {dtype}:" in text and text.rstrip().endswith("ok")
    name, arch, _ = G.device_info(0)
    path = os.path.join("profiles", D.profile_slug(name, arch) + ".json")
    with open(path, encoding="utf-8") as f:
        raw = f.read()
    prof = json.loads(raw)
    assert prof["device"] == name and prof["architecture"] == arch
    assert raw == D.encode_profile(name, arch, prof["tiles"])   # the reference's byte format
    tile = prof["tiles"][D.profile_key(dtype, N, K, M)]
    dt, ti = F.CODE[dtype], G.tile_index(tile)
    assert ti >= 0 and G.tile_supported(dt, ti, N, K, M), tile
    assert f"running custom {dtype} tile {tile}" in text

    # the chosen tile against the oracle, whole output
    ops = Operands(N, K, M, "seeded", 0)
    keep = [G.DeviceBuffer(0, a.nbytes).upload(a) if a is not None else None
            for a in (ops.X(dtype), ops.W(dtype), ops.xscale(dtype), ops.wscale(dtype))]
    Y = G.DeviceBuffer(0, N * M * 4).zero()
    wsb = G.workspace_size(dt, ti, N, K, M)
    WSP = G.DeviceBuffer(0, wsb).zero() if wsb else None
    G.run(0, dt, ti, keep[0], keep[1], Y, N, K, M, keep[2], keep[3], WSP, wsb)
    G.sync(0)
    out = Y.download(np.empty((N, M), np.int32 if dtype == "i8i8" else np.float32))
    ref = oracle.full_reference(dtype, ops.X(dtype), ops.W(dtype), ops.xscale(dtype), ops.wscale(dtype), N, K, M)
    if dtype == "i8i8":
        assert np.array_equal(out.astype(np.int64), ref)
    else:
        rms = float(np.sqrt(np.mean(ref * ref)))
        rel = np.abs(out - ref) / np.maximum(np.abs(ref), 1e-2 * rms)
        assert rel.max() <= 1e-3, rel.max()
