"""CPU tests of the scaled FP8 conversions (te_ref ptx.cuh:923-1693): the
oracle's E4M3 / E5M2 codecs against ml_dtypes' independent float8 casts on
every bf16 and f16 value, the known answers the reference's PTX implies
(saturation, signed zeros, the +0 addend of the 4x forms), and the C ABI's
argument checks (no GPU needed)."""
import numpy as np
import pytest

ml_dtypes = pytest.importorskip("ml_dtypes")

E4M3_MAX, E5M2_MAX = 448.0, 57344.0


def _all_f32_from_16bit():
    from oracle import oracle
    bf = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    f_bf = (bf.astype(np.uint32) << 16).view(np.float32)
    f_h = bf.view(np.float16).astype(np.float32)
    return np.concatenate([f_bf, f_h])


def _midpoints(dec, codes):
    """Values on, between and just beside consecutive FP8 grid points."""
    v = np.array([dec(c) for c in codes], np.float64)
    mid = (v[:-1] + v[1:]) / 2
    pts = np.concatenate([v, mid]).astype(np.float32)
    up = np.nextafter(pts, np.float32(np.inf))
    dn = np.nextafter(pts, np.float32(-np.inf))
    allp = np.concatenate([pts, up, dn])
    return np.concatenate([allp, -allp])


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_codec_matches_ml_dtypes(orc, fmt):
    enc = orc.e4m3 if fmt == "e4m3" else orc.e5m2
    dec = orc.e4m3_decode if fmt == "e4m3" else orc.e5m2_decode
    mx = E4M3_MAX if fmt == "e4m3" else E5M2_MAX
    ml = ml_dtypes.float8_e4m3fn if fmt == "e4m3" else ml_dtypes.float8_e5m2
    top = 0x7E if fmt == "e4m3" else 0x7B
    x = np.concatenate([_all_f32_from_16bit(), _midpoints(dec, range(top + 1))])
    x = x[np.isfinite(x) & (np.abs(x) < mx)]
    ours = np.array([enc(float(v)) for v in x], np.uint8)
    theirs = x.astype(ml).view(np.uint8)
    bad = np.nonzero(ours != theirs)[0]
    assert bad.size == 0, [(float(x[i]), hex(ours[i]), hex(theirs[i])) for i in bad[:8]]


@pytest.mark.parametrize("fmt,maxcode", [("e4m3", 0x7E), ("e5m2", 0x7B)])
def test_codec_saturates(orc, fmt, maxcode):
    enc = orc.e4m3 if fmt == "e4m3" else orc.e5m2
    mx = E4M3_MAX if fmt == "e4m3" else E5M2_MAX
    for v in (mx, mx * 1.01, mx * 2, 1e38, np.inf):
        assert enc(v) == maxcode and enc(-v) == 0x80 | maxcode
    assert enc(0.0) == 0x00 and enc(-0.0) == 0x80


def test_decode_roundtrip(orc):
    for c in range(256):
        for enc, dec, top in ((orc.e4m3, orc.e4m3_decode, 0x7E), (orc.e5m2, orc.e5m2_decode, 0x7B)):
            if (c & 0x7F) <= top:
                assert enc(dec(c)) == c


def test_mul_cvt_signed_zero_rules(orc):
    """mul_cvt_2x multiplies by mul.f32x2 (ptx.cuh:923-1062): -0 * 1 stays -0.
    mul_cvt_4x uses fma.rn.f32x2(x, s, +0) (ptx.cuh:1172-1693): an exact zero
    product becomes +0, an underflowing negative product stays -0."""
    s = np.array([1.0, 1.0, 1.0, 1.0], np.float32)
    x2 = np.array([-0.0, 0.0], np.float32)
    assert list(orc.mul_cvt_fp8(x2, "f32", s, 0, 2, 2, "e4m3")) == [0x80, 0x00]
    x4 = np.array([-0.0, 0.0, -0.0, -2.0**-100], np.float32)
    s4 = np.array([1.0, 1.0, 1.0, 2.0**-100], np.float32)
    assert list(orc.mul_cvt_fp8(x4, "f32", s4, 0, 4, 4, "e4m3")) == [0x00, 0x00, 0x00, 0x80]
    assert list(orc.mul_cvt_fp8(x4, "f32", s4, 0, 4, 4, "e5m2")) == [0x00, 0x00, 0x00, 0x80]


def test_mul_cvt_scale_layouts(orc):
    """floatx2 scales repeat over a group of 4 (elements 0, 2 take .x); floatx4
    scales are per element; scale_stride 0 shares one vector."""
    x = np.ones(8, np.float32)
    s = np.array([1.0, 2.0, 4.0, 8.0, 16.0, 32.0, 64.0, 128.0], np.float32)
    dec = np.vectorize(orc.e4m3_decode)
    assert list(dec(orc.mul_cvt_fp8(x, "f32", s, 0, 4, 2, "e4m3"))) == [1, 2, 1, 2, 1, 2, 1, 2]
    assert list(dec(orc.mul_cvt_fp8(x, "f32", s, 4, 4, 4, "e4m3"))) == [1, 2, 4, 8, 16, 32, 64,
                                                                        128]
    assert list(dec(orc.mul_cvt_fp8(x, "f32", s, 2, 4, 2, "e4m3"))) == [1, 2, 1, 2, 4, 8, 4, 8]
    assert list(dec(orc.mul_cvt_fp8(x, "f32", s, 2, 2, 2, "e4m3"))) == [1, 2, 4, 8, 16, 32, 64,
                                                                        128]


def test_mul_cvt_input_widening(orc):
    """bf16 and f16 inputs widen exactly before the product."""
    bf = np.array([0x3F80, 0xBFC0, 0x0001, 0x7F80], np.uint16)   # 1, -1.5, tiny, +inf
    h = np.array([0x3C00, 0xBE00, 0x0001, 0x7C00], np.uint16)    # 1, -1.5, 2^-24, +inf
    one = np.ones(4, np.float32)
    for arr, dt in ((bf, "bf16"), (h, "f16")):
        got = orc.mul_cvt_fp8(arr, dt, one, 0, 4, 4, "e4m3")
        assert list(got[[0, 1, 3]]) == [0x38, 0xBC, 0x7E]
        assert got[2] == 0x00


def test_abi_rejects_bad_arguments(nvlib):
    lib = nvlib.load()
    # bad format, bad dtype, bad scale width
    assert lib.nvfp4_mul_cvt_fp8_2x(16, 0, 16, 0, 16, 7, 4, None) == 2
    assert lib.nvfp4_mul_cvt_fp8_2x(16, 9, 16, 0, 16, 0, 4, None) == 2
    assert lib.nvfp4_mul_cvt_fp8_4x(16, 0, 16, 3, 0, 16, 0, 4, None) == 2
    # null pointers, misaligned input / output / scale
    assert lib.nvfp4_mul_cvt_fp8_4x(None, 0, 16, 2, 0, 16, 0, 4, None) == 2
    assert lib.nvfp4_mul_cvt_fp8_4x(0x1002, 0, 16, 2, 0, 16, 0, 4, None) == 3
    assert lib.nvfp4_mul_cvt_fp8_2x(16, 1, 16, 0, 0x1001, 0, 4, None) == 3
    assert lib.nvfp4_mul_cvt_fp8_4x_loose(16, 1, 0x1002, 0, 16, 1, 4, None) == 3
    # zero groups is a no-op
    assert lib.nvfp4_mul_cvt_fp8_4x(None, 0, None, 4, 0, None, 1, 0, None) == 0


GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def _fixture():
    p = GOLDEN / "teref_fp8.npz"
    if not p.exists():
        pytest.skip("teref_fp8.npz not generated")
    return np.load(p)


def _widen(x, dt):
    if dt == "f32":
        return x.astype(np.float32)
    if dt == "bf16":
        return (x.astype(np.uint32) << 16).view(np.float32)
    return x.view(np.float16).astype(np.float32)


@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
def test_oracle_vs_reference_fixture(orc, dt):
    """The oracle against the reference's own mul_cvt_2x / mul_cvt_4x run on a
    B200 (tests/golden/gen_teref_fp8_fixtures.py), every form and format."""
    g = _fixture()
    x = g[f"in_{dt}"]
    for fmt in ("e4m3", "e5m2"):
        for width, sw in ((2, 2), (4, 2), (4, 4)):
            fn = "2x" if width == 2 else "4x"
            s = np.resize(g["scales"], (x.size // width) * sw).astype(np.float32)
            want = g[f"{dt}_{fn}_s{sw}_{fmt}"]
            got = orc.mul_cvt_fp8(x, dt, s, sw, width, sw, fmt)
            bad = np.nonzero(got != want)[0]
            assert bad.size == 0, (fmt, width, sw, [(int(i), hex(got[i]), hex(want[i]))
                                                    for i in bad[:6]])


@pytest.mark.parametrize("dt", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_loose_precision_fixture_properties(orc, dt, fmt):
    """The reference's _LOOSE_PRECISION build (cvt.rs with the constant word
    0x80008000): every finite in-range product lands on one of its two
    bracketing FP8 values, and elements 0 and 2 of each group round half up in
    magnitude (their random value is one half)."""
    g = _fixture()
    x = g[f"in_{dt}"]
    ng = x.size // 4
    s = np.resize(g["scales"], ng * 2).astype(np.float32)
    xf = _widen(x, dt).astype(np.float64)
    sf = np.tile(s.reshape(ng, 2), (1, 2)).reshape(-1).astype(np.float64)
    with np.errstate(all="ignore"):
        p = np.abs((xf * sf).astype(np.float32).astype(np.float64))
    dec = np.vectorize(orc.e4m3_decode if fmt == "e4m3" else orc.e5m2_decode)
    top = 0x7E if fmt == "e4m3" else 0x7B
    grid = dec(np.arange(top + 1)).astype(np.float64)
    loose = g[f"{dt}_4x_loose_{fmt}"] & 0x7F
    ok = np.isfinite(p) & (p < grid[-1])
    lo = np.searchsorted(grid, p, side="right") - 1
    idx = np.nonzero(ok)[0]
    assert idx.size > 1000
    lo_i = lo[idx]
    assert np.all((loose[idx] == lo_i) | (loose[idx] == lo_i + 1))
    even = idx[(idx % 2) == 0]
    l_e = lo[even]
    frac = (p[even] - grid[l_e]) / (grid[np.minimum(l_e + 1, top)] - grid[l_e])
    expect = np.where(frac >= 0.5, l_e + 1, l_e)
    assert np.all(loose[even] == expect)
