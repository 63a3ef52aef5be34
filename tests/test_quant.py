"""Quantisers: f32 -> the bench's operand formats (E4M3, E2M1, OCP MX).

CPU tests pin the oracle's new encoders against independent numpy
restatements; GPU tests check gemm_quantize bit for bit against the oracle and
feed its output straight into the GEMM.
"""
import numpy as np
import pytest

import oracle
from mlpgemm import formats as F

E2M1_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def e2m1_rne_numpy(x: np.ndarray) -> np.ndarray:
    """Nearest point of the E2M1 grid, ties to the even code, saturating at 6;
    sign kept; NaN -> 0x7 (independent of the oracle's branch structure)."""
    x = np.asarray(x, dtype=np.float64)
    ax = np.abs(np.nan_to_num(x, nan=6.0, posinf=6.0, neginf=6.0))
    d = np.abs(ax[..., None] - E2M1_GRID)                 # distance to each code 0..7
    best = d.min(axis=-1, keepdims=True)
    tie = d == best
    # among the nearest codes prefer the even one (RNE on the mantissa bit)
    score = np.where(tie, (np.arange(8) % 2) * 10 + np.arange(8) * 0, 100)
    code = np.argmin(score + np.where(tie, 0, 1000), axis=-1)
    code = np.where(ax >= 6.0, 7, code)
    sign = np.where(np.signbit(x) & ~np.isnan(x), 8, 0)
    return (code | sign).astype(np.uint8)


def specials():
    v = [0.0, -0.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, 6.0, 448.0, 464.0, 1e30, -1e-30,
         2.0 ** -6, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -11, 1e-45, np.inf, -np.inf, np.nan]
    return np.array(v + [-t for t in v[:-1]], dtype=np.float32)


def random_f32(n, seed=0):
    rng = np.random.default_rng(seed)
    mag = np.exp2(rng.uniform(-20, 12, n)) * rng.uniform(0.5, 1.0, n)
    x = np.where(rng.random(n) < 0.5, -mag, mag).astype(np.float32)
    x[::97] = 0.0
    return x


def test_e2m1_oracle_matches_grid_rounding():
    x = np.concatenate([specials(), random_f32(4000),
                        (np.arange(-56, 57) / 8.0).astype(np.float32)])   # every half- and quarter-step tie
    got = np.array([oracle.f32_to_e2m1_rne(float(v)) for v in x], dtype=np.uint8)
    assert np.array_equal(got, e2m1_rne_numpy(x))


def mx_numpy(elem, src):
    """OCP MX restated in numpy (independent of the C oracle)."""
    rows, cols = src.shape
    blocks = src.reshape(rows, cols // 32, 32).astype(np.float64)
    bad = ~np.isfinite(blocks).all(axis=-1)
    amax = np.where(np.isfinite(blocks), np.abs(blocks), 0).max(axis=-1)
    with np.errstate(divide="ignore"):
        fl = np.floor(np.log2(np.where(amax > 0, amax, 1.0)))
    X = np.clip(fl - (2 if elem == 0 else 8), -127, 127).astype(np.int64)
    X = np.where(amax == 0, -127, X)
    code = np.where(bad, 0xFF, X + 127).astype(np.uint8)
    scaled = np.ldexp(np.where(np.isfinite(blocks), blocks, 0), -np.where(bad, 0, X)[..., None])
    q = e2m1_rne_numpy(scaled) if elem == 0 else F.f32_to_e4m3_rne(scaled)
    q = np.where(bad[..., None], 0, q).reshape(rows, cols)
    if elem == 0:
        q = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    return q, code


@pytest.mark.parametrize("elem", [0, 1])
def test_mx_oracle_matches_numpy(elem):
    rows, cols = 24, 256
    src = random_f32(rows * cols, seed=elem + 3).reshape(rows, cols)
    src[0, :32] = 0.0                                      # zero block -> code 0
    src[1, 40] = np.nan                                    # NaN block -> 0xFF
    src[2, 70] = np.inf
    src[3, :32] = np.float32(2.0 ** -140)                  # subnormal amax -> X clamped to -127
    src[4, :32] = np.float32(3e38)                         # huge amax
    vals, scales = oracle.quantize_mx(elem, src)
    nv, ns = mx_numpy(elem, src)
    assert np.array_equal(scales, ns)
    assert np.array_equal(vals, nv)
    assert scales[0, 0] == 0 and scales[1, 1] == 0xFF and scales[2, 2] == 0xFF and scales[3, 0] == 0


def test_mx_representable_values_round_trip():
    # values already on the E2M1 grid times a block power of two come back exactly
    rng = np.random.default_rng(5)
    codes = rng.integers(0, 16, (8, 128)).astype(np.uint8)
    codes[:, ::32] = 7                                     # every block holds 6.0 -> X = k exactly
    k = rng.integers(-20, 20, (8, 4))
    vals = F.e2m1_decode(codes).reshape(8, 4, 32) * np.exp2(k)[..., None]
    q, s = oracle.quantize_mx(0, vals.reshape(8, 128).astype(np.float32))
    assert np.array_equal(s, (k + 127).astype(np.uint8))
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    # -0 (code 8) and +0 both decode to 0: compare decoded values
    dec = F.e2m1_decode(F.e2m1_unpack(q.reshape(-1), 8 * 128)).reshape(8, 128)
    assert np.array_equal(dec, F.e2m1_decode(F.e2m1_unpack(packed.reshape(-1), 8 * 128)).reshape(8, 128))


# ---- GPU ------------------------------------------------------------------------------
def _quantize_gpu(G, fmt, src):
    rows, cols = src.shape
    d_src = G.DeviceBuffer(0, src.nbytes).upload(np.ascontiguousarray(src, dtype=np.float32))
    nbytes = {G.Q_E4M3_REF: rows * cols, G.Q_E4M3: rows * cols, G.Q_E2M1: rows * cols // 2,
              G.Q_MXFP4: rows * cols // 2, G.Q_MXFP8: rows * cols}[fmt]
    d_dst = G.DeviceBuffer(0, nbytes)
    mx = fmt in (G.Q_MXFP4, G.Q_MXFP8)
    d_sc = G.DeviceBuffer(0, rows * cols // 32) if mx else None
    G.quantize(0, fmt, d_src, d_dst, d_sc, rows, cols)
    G.sync(0)
    out = np.empty(nbytes, dtype=np.uint8)
    d_dst.download(out)
    sc = None
    if mx:
        sc = np.empty(rows * cols // 32, dtype=np.uint8)
        d_sc.download(sc)
    return out, sc


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["e4m3_ref", "e4m3", "e2m1"])
def test_quantize_elementwise_matches_oracle(gemm, fmt):
    G = gemm
    x = np.concatenate([specials(), random_f32(64 * 512 - len(specials()) - 1, seed=11)]).astype(np.float32)
    x = np.concatenate([x, np.float32([1.5])])             # even count
    src = x.reshape(64, 512)
    code = {"e4m3_ref": G.Q_E4M3_REF, "e4m3": G.Q_E4M3, "e2m1": G.Q_E2M1}[fmt]
    out, _ = _quantize_gpu(G, code, src)
    if fmt == "e4m3_ref":
        ref = np.array([oracle.f32_to_e4m3_ref(float(v)) for v in x], dtype=np.uint8)
    elif fmt == "e4m3":
        ref = np.array([oracle.f32_to_e4m3_rne(float(v)) for v in x], dtype=np.uint8)
    else:
        q = np.array([oracle.f32_to_e2m1_rne(float(v)) for v in x], dtype=np.uint8)
        ref = (q[0::2] | (q[1::2] << 4)).astype(np.uint8)
    bad = np.flatnonzero(out != ref)
    assert bad.size == 0, [(float(x[i if fmt != 'e2m1' else 2 * i]), hex(out[i]), hex(ref[i])) for i in bad[:6]]


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["mxfp4", "mxfp8"])
def test_quantize_mx_matches_oracle(gemm, fmt):
    G = gemm
    rows, cols = 48, 1024
    src = random_f32(rows * cols, seed=21).reshape(rows, cols)
    src[0, :32] = 0.0
    src[1, 33] = np.nan
    src[2, 64] = -np.inf
    src[3, :32] = np.float32(2.0 ** -140)
    elem = 0 if fmt == "mxfp4" else 1
    out, sc = _quantize_gpu(G, G.Q_MXFP4 if elem == 0 else G.Q_MXFP8, src)
    vals, scales = oracle.quantize_mx(elem, src)
    assert np.array_equal(sc, scales.reshape(-1))
    assert np.array_equal(out, vals.reshape(-1))


@pytest.mark.gpu
def test_quantised_operands_feed_the_gemm(gemm):
    # mxfp4/a8 with X and W produced on the device: E4M3 X + UE8M0 [N,K/32],
    # E2M1 W [M,K] + UE8M0 [M,K/32]; the GEMM result matches the oracle on them
    G = gemm
    N, K, M = 128, 512, 256
    rng = np.random.default_rng(2)
    xf = rng.standard_normal((N, K)).astype(np.float32)
    wf = (rng.standard_normal((M, K)) * 0.05).astype(np.float32)
    xq, xs = _quantize_gpu(G, G.Q_MXFP8, xf)
    wq, ws = _quantize_gpu(G, G.Q_MXFP4, wf)
    dt = F.CODE["mxfp4/a8"]
    ti = G.tile_index("128x128")
    bufs = [G.DeviceBuffer(0, a.nbytes).upload(a) for a in (xq, wq, xs, ws)]
    Y = G.DeviceBuffer(0, N * M * 4)
    wsb = G.workspace_size(dt, ti, N, K, M)
    WSP = G.DeviceBuffer(0, wsb).zero() if wsb else None
    G.run(0, dt, ti, bufs[0], bufs[1], Y, N, K, M, bufs[2], bufs[3], WSP, wsb)
    G.sync(0)
    out = np.empty((N, M), dtype=np.float32)
    Y.download(out)
    ref = oracle.full_reference("mxfp4/a8", xq, wq, xs, ws, N, K, M)
    rms = float(np.sqrt(np.mean(ref * ref)))
    assert np.max(np.abs(out - ref) / np.maximum(np.abs(ref), 1e-2 * rms)) <= 1e-3
    # and the quantised product is close to the f32 product it came from
    exact = xf.astype(np.float64) @ wf.astype(np.float64).T
    assert np.sqrt(np.mean((out - exact) ** 2)) / np.sqrt(np.mean(exact ** 2)) < 0.2
