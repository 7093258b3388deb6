"""GPU parity of the scaled FP8 conversions (include/nvfp4_fp8.cuh through the
nvfp4_mul_cvt_fp8_* batch entry points) against the oracle (bit-exact) and
against the reference's own mul_cvt_2x / mul_cvt_4x (te_ref ptx.cuh:923-1693)
compiled from the reference tree and run on the same GPU (bit-exact),
including its _LOOSE_PRECISION build."""
import numpy as np
import pytest
import torch

from tests.gpu_helpers import dev, host

pytestmark = pytest.mark.gpu

DTYPES = ["f32", "bf16", "f16"]
FORMS = [(2, 2), (4, 2), (4, 4)]   # (group width, scale width)


def _values(dtype, n, seed):
    """n input elements: every 16-bit pattern (bf16 / f16, so NaN, Inf,
    subnormals and both zeros) or, for f32, specials, FP8 grid points and
    their midpoints, and N(0, 1) spread over many binades."""
    rng = np.random.default_rng(seed)
    if dtype != "f32":
        v = np.arange(65536, dtype=np.uint32).astype(np.uint16)
        return np.resize(rng.permutation(v), n)
    from oracle import oracle
    grid = []
    for dec, top in ((oracle.e4m3_decode, 0x7E), (oracle.e5m2_decode, 0x7B)):
        g = np.array([dec(c) for c in range(top + 1)], np.float64)
        grid += [g, (g[:-1] + g[1:]) / 2]
    grid = np.concatenate(grid).astype(np.float32)
    grid = np.concatenate([grid, np.nextafter(grid, np.float32(np.inf)),
                           np.nextafter(grid, np.float32(-np.inf))])
    specials = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 1e-40, 3e38,
                         -3e38, 448.0, 464.0, 57344.0, 61440.0], np.float32)
    body = (rng.standard_normal(n) * np.exp2(rng.integers(-20, 20, n))).astype(np.float32)
    v = np.concatenate([specials, grid, -grid, body])[:n]
    return rng.permutation(v).astype(np.float32)


def _scales(n, seed):
    rng = np.random.default_rng(seed)
    s = np.exp2(rng.integers(-12, 12, n)).astype(np.float32) * \
        rng.choice(np.array([1.0, -1.0, 0.75, 1.3], np.float32), n)
    special = np.array([1.0, 0.0, -0.0, np.inf, np.nan, 2.0**-100, 2.0**100, -1.0], np.float32)
    k = min(n, special.size)
    s[:k] = special[:k]
    return rng.permutation(s).astype(np.float32)


def _run_ours(nvlib, x, dtype, scale, stride, width, sw, fmt, loose=False, offset=0):
    """Runs one batch; `offset` shifts input and output by whole groups from a
    16-byte boundary (the unaligned path)."""
    ng = x.size // width
    xb = dev(np.concatenate([np.zeros(offset * width, x.dtype), x]))
    ob = torch.zeros(ng * width + offset * width, dtype=torch.uint8, device="cuda")
    esz = x.dtype.itemsize
    xin = xb.data_ptr() + offset * width * esz
    o = ob.data_ptr() + offset * width
    ds = dev(scale)
    if width == 2:
        nvlib.mul_cvt_fp8_2x(xin, dtype, ds, stride, o, fmt, ng)
    else:
        nvlib.mul_cvt_fp8_4x(xin, dtype, ds, sw, stride, o, fmt, ng, loose=loose)
    return host(ob, np.uint8)[offset * width:]


def _diff(a, b, x, width):
    bad = np.nonzero(a != b)[0]
    return [(int(i), float(np.asarray(x).reshape(-1)[i]) if np.asarray(x).dtype == np.float32
             else hex(int(np.asarray(x).reshape(-1)[i])), hex(a[i]), hex(b[i])) for i in bad[:6]]


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("width,sw", FORMS)
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("per_group", [False, True])
def test_vs_oracle(nvlib, orc, dtype, width, sw, fmt, per_group):
    ng = 40001 if width == 2 else 20001          # odd: the vector body plus a tail
    x = _values(dtype, ng * width, seed=width * 7 + sw)
    stride = sw if per_group else 0
    s = _scales(max(ng * sw, 4), seed=3) if per_group else np.array([0.75, -2.0, 1.0, 0.5],
                                                                   np.float32)
    got = _run_ours(nvlib, x, dtype, s, stride, width, sw, fmt)
    want = orc.mul_cvt_fp8(x, dtype, s, stride, width, sw, fmt)
    assert (got == want).all(), _diff(got, want, x, width)


@pytest.mark.parametrize("width,sw", FORMS)
@pytest.mark.parametrize("dtype", DTYPES)
def test_unaligned_and_small(nvlib, orc, dtype, width, sw):
    for ng, off in ((1, 0), (3, 1), (17, 1), (1000, 3)):
        x = _values(dtype, ng * width, seed=ng)
        s = _scales(ng * sw + 4, seed=ng)
        got = _run_ours(nvlib, x, dtype, s, sw, width, sw, "e4m3", offset=off)
        want = orc.mul_cvt_fp8(x, dtype, s, sw, width, sw, "e4m3")
        assert (got == want).all(), (ng, off, _diff(got, want, x, width))


def _ref_or_skip():
    from oracle import ref
    if not ref.fp8_available():
        pytest.skip("reference FP8 library not built")
    return ref.fp8()


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("width,sw", FORMS)
@pytest.mark.parametrize("dtype", DTYPES)
def test_vs_reference_functions(nvlib, dtype, width, sw, fmt):
    """Bit-exact against TE's own mul_cvt_2x / mul_cvt_4x run on this GPU."""
    L = _ref_or_skip()
    ng = 1 << 16
    x = _values(dtype, ng * width, seed=99 + width + sw)
    s = _scales(ng * sw, seed=5)
    got = _run_ours(nvlib, x, dtype, s, sw, width, sw, fmt)
    dx, ds = dev(x), dev(s)
    ref_out = torch.zeros(ng * width, dtype=torch.uint8, device="cuda")
    code = {"f32": 0, "bf16": 1, "f16": 2}[dtype]
    f = {"e4m3": 0, "e5m2": 1}[fmt]
    if width == 2:
        rc = L.teref_mul_cvt_fp8_2x(dx.data_ptr(), code, ds.data_ptr(), sw, ref_out.data_ptr(), f,
                                    ng, None)
    else:
        rc = L.teref_mul_cvt_fp8_4x(dx.data_ptr(), code, ds.data_ptr(), sw, sw,
                                    ref_out.data_ptr(), f, ng, None)
    assert rc == 0
    want = host(ref_out, np.uint8)
    assert (got == want).all(), _diff(got, want, x, width)


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("dtype", DTYPES)
def test_loose_precision_vs_reference(nvlib, dtype, fmt):
    """The _LOOSE_PRECISION build (cvt.rs with the constant 0x80008000) against
    the reference's build with the same macro."""
    L = _ref_or_skip()
    ng = 1 << 16
    x = _values(dtype, ng * 4, seed=123)
    s = _scales(ng * 2, seed=6)
    got = _run_ours(nvlib, x, dtype, s, 2, 4, 2, fmt, loose=True)
    dx, ds = dev(x), dev(s)
    ref_out = torch.zeros(ng * 4, dtype=torch.uint8, device="cuda")
    rc = L.teref_mul_cvt_fp8_4x_loose(dx.data_ptr(), {"f32": 0, "bf16": 1, "f16": 2}[dtype],
                                      ds.data_ptr(), 2, ref_out.data_ptr(),
                                      {"e4m3": 0, "e5m2": 1}[fmt], ng, None)
    assert rc == 0
    want = host(ref_out, np.uint8)
    assert (got == want).all(), _diff(got, want, x, 4)


def test_large_batch_matches_oracle_sample(nvlib, orc):
    """2^26 groups of bf16 x4 (the throughput case): sampled groups checked."""
    ng = 1 << 26
    rng = np.random.default_rng(7)
    x = torch.randn(ng * 4, device="cuda").to(torch.bfloat16)
    s = torch.tensor([0.5, 2.0], device="cuda")
    out = torch.empty(ng * 4, dtype=torch.uint8, device="cuda")
    nvlib.mul_cvt_fp8_4x(x, "bf16", s, 2, 0, out, "e4m3", ng)
    idx = rng.integers(0, ng, 4096)
    xs = x.view(torch.int16).view(ng, 4)[torch.from_numpy(idx).cuda()].cpu().numpy()
    got = out.view(ng, 4)[torch.from_numpy(idx).cuda()].cpu().numpy()
    want = orc.mul_cvt_fp8(xs.view(np.uint16).reshape(-1), "bf16", np.array([0.5, 2.0],
                           np.float32), 0, 4, 2, "e4m3")
    assert (got.reshape(-1) == want).all()
