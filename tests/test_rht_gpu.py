"""GPU parity of the tcgen05 RHT GEMM + NVFP4 cast (C-ABI
nvfp4_rht_gemm_ntt_w_sfc) against the oracle (bit-exact for RN and SR, one FP4
step for fast math, whose device reciprocal is rcp.approx) and against the
reference's own TE SM100 kernel on the same GPU (bit-exact in every mode)."""
import numpy as np
import pytest
import torch

from tests.gpu_helpers import activations, dev, fp4_step_diff, h16, host

pytestmark = pytest.mark.gpu


def run_ours(nvlib, m, n, A, B, amax, rng_state=None, sr=False, fm=False, k_tile=2048,
             sm_count=0):
    C = torch.full((m, n // 2), 0xAA, dtype=torch.uint8, device="cuda")
    S = torch.full((m, n // 16), 0xAA, dtype=torch.uint8, device="cuda")
    dr = None if rng_state is None else torch.tensor([int(v) for v in rng_state],
                                                      dtype=torch.int64, device="cuda")
    nvlib.rht_gemm_ntt_w_sfc(m, n, dev(A) if isinstance(A, np.ndarray) else A, dev(B), C, S,
                             torch.tensor([amax], dtype=torch.float32, device="cuda"), dr,
                             sm_count, None, k_tile, stochastic_rounding=sr, use_fast_math=fm)
    assert nvlib.device_error() == 0
    return C, S


def check_vs_oracle(orc, nvlib, m, n, A, B, amax, rng_state, sr, fm, k_tile=2048):
    C, S = run_ours(nvlib, m, n, A, B, amax, rng_state, sr, fm, k_tile)
    wc, ws = orc.rht_gemm_ntt_w_sfc(m, n, A, B, amax, rng_state, k_tile, sr, fm)
    gc, gs = host(C, np.uint8), host(S, np.uint8)
    if fm:
        assert (gs == ws).mean() > 0.999
        d = fp4_step_diff(orc, gc, wc)
        assert (d[np.isfinite(d)] <= 2.0).all()
    else:
        assert (gs == ws).all(), f"SFC mismatches: {(gs != ws).sum()}"
        mism = (orc.unpack_nibbles(gc) != orc.unpack_nibbles(wc))
        assert not mism.any(), f"FP4 mismatches: {mism.sum()} of {mism.size}, first at " \
            f"{np.nonzero(mism)[0][:5]}"


SHAPES = [(128, 64), (256, 128), (128, 256), (384, 320), (256, 1024), (640, 768)]


@pytest.mark.parametrize("m,n", SHAPES)
@pytest.mark.parametrize("mode", ["rn", "sr", "fm"])
def test_rht_vs_oracle(nvlib, orc, m, n, mode):
    rng = np.random.default_rng(m * 7919 + n)
    A = activations(rng, m * n)
    signs = np.where(rng.integers(0, 2, 16) == 0, -1.0, 1.0)
    B = h16(signs)
    amax = orc.amax_bf16(A)
    check_vs_oracle(orc, nvlib, m, n, A, B, amax, (20260101, 5), mode == "sr", mode == "fm")


@pytest.mark.parametrize("k_tile", [64, 128, 192, 1024])
def test_rht_k_tile_mapping(nvlib, orc, k_tile):
    rng = np.random.default_rng(k_tile)
    m, n = 256, 1280
    A = activations(rng, m * n)
    check_vs_oracle(orc, nvlib, m, n, A, h16(), 4.0, (777, 2**32 - 2), True, False, k_tile)


EXTREMES = {
    "all_zeros": (lambda g, k: np.zeros(k), 1.0),
    "all_zeros_amax0": (lambda g, k: np.zeros(k), 0.0),
    "very_small": (lambda g, k: np.where(g.integers(0, 2, k) == 0, -1, 1) * 1e-6 *
                   (1 + g.integers(0, 100, k) / 100.0), 1e-4),
    "very_large": (lambda g, k: np.where(g.integers(0, 2, k) == 0, -1, 1) *
                   (500.0 + g.integers(0, 1000, k)), 1000.0),
    "very_large_small_amax": (lambda g, k: np.where(g.integers(0, 2, k) == 0, -1, 1) *
                              (500.0 + g.integers(0, 1000, k)), 1.0),
    "sparse_outliers": (lambda g, k: np.where(g.integers(0, 256, k) == 0,
                                              np.where(g.integers(0, 2, k) == 0, -100.0, 100.0),
                                              0.0), 100.0),
    "uniform_one": (lambda g, k: np.ones(k), 4.0),
    "uniform_one_tiny_amax": (lambda g, k: np.ones(k), 0.001),
    "contains_inf": (lambda g, k: np.where(g.integers(0, 256, k) == 0,
                                           np.where(g.integers(0, 2, k) == 0, np.inf, -np.inf),
                                           g.standard_normal(k)), 4.0),
    "contains_nan": (lambda g, k: np.where(g.integers(0, 256, k) == 0, np.nan,
                                           g.standard_normal(k)), 4.0),
    "amax_nan": (lambda g, k: g.standard_normal(k), float("nan")),
    "amax_inf": (lambda g, k: g.standard_normal(k), float("inf")),
}


@pytest.mark.parametrize("name", sorted(EXTREMES))
@pytest.mark.parametrize("sr", [False, True])
def test_rht_extreme_patterns(nvlib, orc, name, sr):
    """The reference's extreme-data cases (rht_gemm/test_compare.cu:334-388)."""
    from oracle import oracle
    fill, amax = EXTREMES[name]
    g = np.random.default_rng(42)
    m, n = 128, 256   # API view of a 256 x 128 activation
    A = oracle.f32_to_bf16(fill(g, m * n).astype(np.float32))
    check_vs_oracle(orc, nvlib, m, n, A, h16(), amax, (12345, 0), sr, False)


def test_rht_null_rng_state_is_seed_zero(nvlib):
    rng = np.random.default_rng(1)
    m, n = 128, 512
    A = activations(rng, m * n)
    a = run_ours(nvlib, m, n, A, h16(), 4.0, None, sr=True)
    b = run_ours(nvlib, m, n, A, h16(), 4.0, (0, 0), sr=True)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


@pytest.mark.parametrize("sm_count", [1, 3, 7, 1000])
def test_rht_sm_count_cap_does_not_change_results(nvlib, sm_count):
    rng = np.random.default_rng(2)
    m, n = 512, 2048
    A = dev(activations(rng, m * n))
    ref = run_ours(nvlib, m, n, A, h16(), 7.0, (5, 6), sr=True)
    got = run_ours(nvlib, m, n, A, h16(), 7.0, (5, 6), sr=True, sm_count=sm_count)
    assert torch.equal(ref[0], got[0]) and torch.equal(ref[1], got[1])


@pytest.mark.parametrize("parts", [2, 4])
def test_rht_sharded_concatenates_to_full(nvlib, parts):
    """Column shards with global RNG coordinates reproduce the unsharded call."""
    rng = np.random.default_rng(3)
    m, n, kt = 256, 8192, 2048
    A = dev(activations(rng, m * n))
    amax = torch.tensor([9.0], device="cuda")
    rs = torch.tensor([31337, 11], dtype=torch.int64, device="cuda")
    B = dev(h16())
    Cf = torch.empty((m, n // 2), dtype=torch.uint8, device="cuda")
    Sf = torch.empty((m, n // 16), dtype=torch.uint8, device="cuda")
    nvlib.rht_gemm_ntt_w_sfc(m, n, A, B, Cf, Sf, amax, rs, 0, None, kt, stochastic_rounding=True)
    w = n // parts
    Cs, Ss = [], []
    for r in range(parts):
        Ash = A[r * w * m:(r + 1) * w * m]          # column block of a column-major matrix
        C = torch.empty((m, w // 2), dtype=torch.uint8, device="cuda")
        S = torch.empty((m, w // 16), dtype=torch.uint8, device="cuda")
        nvlib.rht_gemm_ntt_w_sfc_sharded(m, w, Ash, B, C, S, amax, rs, r * w, n, 0, None, kt,
                                         stochastic_rounding=True)
        Cs.append(C)
        Ss.append(S)
    assert torch.equal(torch.cat(Cs, 1), Cf)
    assert torch.equal(torch.cat(Ss, 1), Sf)


def test_ttt_wrapper_swaps_dims(nvlib):
    rng = np.random.default_rng(4)
    rows, cols = 256, 384        # row-major activation = column-major (cols x rows)
    X = dev(activations(rng, rows * cols))
    amax = torch.tensor([5.0], device="cuda")
    B = dev(h16())
    C1 = torch.empty((rows, cols // 2), dtype=torch.uint8, device="cuda")
    S1 = torch.empty((rows, cols // 16), dtype=torch.uint8, device="cuda")
    nvlib.rht_gemm_ttt_wrapper(cols, rows, X, B, C1, S1, amax, None, 0, None, 1024)
    C2 = torch.empty_like(C1)
    S2 = torch.empty_like(S1)
    nvlib.rht_gemm_ntt_w_sfc(rows, cols, X, B, C2, S2, amax, None, 0, None, 1024)
    assert torch.equal(C1, C2) and torch.equal(S1, S2)


def _teref():
    from oracle import ref
    if not ref.gpu_available():
        pytest.skip("reference GPU library not built")
    return ref.gpu()


@pytest.mark.parametrize("m,n", [(128, 256), (256, 128), (1024, 1024), (8192, 5120),
                                 (5120, 8192)])
@pytest.mark.parametrize("mode", ["rn", "fm", "sr"])
def test_rht_vs_reference_te_kernel(nvlib, m, n, mode):
    """Bit-exact against TE's SM100 kernel (rht_gemm/test_compare.cu:296-321
    shapes plus BASELINE config 4), every mode including fast math."""
    L = _teref()
    rng = np.random.default_rng(m + n)
    A = dev(activations(rng, m * n))
    B = dev(h16(np.where(rng.integers(0, 2, 16) == 0, -1.0, 1.0)))
    amax = torch.empty(1, dtype=torch.float32, device="cuda")
    nvlib.amax_bf16(A, m * n, amax)
    rs = torch.tensor([12345, 0], dtype=torch.int64, device="cuda")
    sr, fm = mode == "sr", mode == "fm"
    C, S = run_ours(nvlib, m, n, A, host(B, np.uint16), float(host(amax, np.float32)[0]),
                    (12345, 0), sr, fm)
    Cr = torch.zeros_like(C)
    Sr = torch.zeros_like(S)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    rc = L.teref_rht_gemm_ntt_w_sfc(m, n, A.data_ptr(), B.data_ptr(), Cr.data_ptr(),
                                    Sr.data_ptr(), amax.data_ptr(), rs.data_ptr(), sms, None,
                                    int(sr), int(fm))
    torch.cuda.synchronize()
    assert rc == 0
    assert torch.equal(S, Sr), f"SFC mismatches: {(S != Sr).sum().item()}"
    assert torch.equal(C, Cr), f"FP4 byte mismatches: {(C != Cr).sum().item()}"


def test_rht_full_size_sharded_vs_reference(nvlib):
    """BASELINE config 5 at full size (A 65536 x 14336 activation -> API
    m = 14336, n = 65536): our 8-way column-sharded computation, concatenated,
    is bit-exact with TE's kernel on the whole matrix."""
    L = _teref()
    m, n, parts = 14336, 65536, 8
    g = torch.Generator(device="cuda").manual_seed(0)
    A = torch.randn(m * n, device="cuda", dtype=torch.float32, generator=g)
    A[torch.rand(m * n, device="cuda", generator=g) < 0.001] *= 50.0
    A = A.to(torch.bfloat16)
    amax = torch.empty(1, dtype=torch.float32, device="cuda")
    nvlib.amax_bf16(A, m * n, amax)
    rs = torch.tensor([2024, 0], dtype=torch.int64, device="cuda")
    B = dev(h16())
    Cr = torch.empty((m, n // 2), dtype=torch.uint8, device="cuda")
    Sr = torch.empty((m, n // 16), dtype=torch.uint8, device="cuda")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert L.teref_rht_gemm_ntt_w_sfc(m, n, A.data_ptr(), B.data_ptr(), Cr.data_ptr(),
                                      Sr.data_ptr(), amax.data_ptr(), rs.data_ptr(), sms, None,
                                      1, 0) == 0
    w = n // parts
    for r in range(parts):
        C = torch.empty((m, w // 2), dtype=torch.uint8, device="cuda")
        S = torch.empty((m, w // 16), dtype=torch.uint8, device="cuda")
        nvlib.rht_gemm_ntt_w_sfc_sharded(m, w, A[r * w * m:(r + 1) * w * m], B, C, S, amax, rs,
                                         r * w, n, 0, None, 2048, stochastic_rounding=True)
        assert torch.equal(C, Cr[:, r * w // 2:(r + 1) * w // 2]), r
        assert torch.equal(S, Sr[:, r * w // 16:(r + 1) * w // 16]), r
    assert nvlib.device_error() == 0
