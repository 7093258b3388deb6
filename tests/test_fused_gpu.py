"""GPU parity of the fused amax + cast kernel (nvfp4_quantize_rht_fused):
identical amax, FP4 codes and scale factors to nvfp4_amax_bf16 followed by
nvfp4_rht_gemm_ntt_w_sfc, on repeated launches that reuse the workspace, with
capped grids, ragged shapes and NaN inputs."""
import numpy as np
import pytest
import torch

from tests.gpu_helpers import activations, dev, h16

pytestmark = pytest.mark.gpu


def _two_paths(nv, m, n, A, sr, fm, k_tile=2048, sm_count=0, ws=None, repeats=2):
    B = dev(h16(np.array([1, -1] * 8)))
    rs = torch.tensor([4242, 17], dtype=torch.int64, device="cuda")
    am = torch.empty(1, device="cuda")
    nv.amax_bf16(A, m * n, am)
    C = torch.empty((m, n // 2), dtype=torch.uint8, device="cuda")
    S = torch.empty((m, n // 16), dtype=torch.uint8, device="cuda")
    nv.rht_gemm_ntt_w_sfc(m, n, A, B, C, S, am, rs, 0, None, k_tile,
                          stochastic_rounding=sr, use_fast_math=fm)
    ws = nv.fused_workspace() if ws is None else ws
    for _ in range(repeats):
        C2 = torch.full_like(C, 0xAA)
        S2 = torch.full_like(S, 0xAA)
        am2 = torch.full((1,), -1.0, device="cuda")
        nv.quantize_rht_fused(m, n, A, B, C2, S2, am2, rs, ws, sm_count, None, k_tile,
                              stochastic_rounding=sr, use_fast_math=fm)
        torch.cuda.synchronize()
        assert nv.device_error() == 0
        assert torch.equal(am2.view(torch.int32), am.view(torch.int32)), (am2, am)
        assert torch.equal(S2, S), f"SFC mismatches {(S2 != S).sum().item()}"
        assert torch.equal(C2, C), f"FP4 mismatches {(C2 != C).sum().item()}"


@pytest.mark.parametrize("m,n", [(128, 64), (384, 320), (1024, 1024), (5120, 8192),
                                 (14336, 8192)])
@pytest.mark.parametrize("mode", ["rn", "sr", "fm"])
def test_fused_equals_amax_then_cast(nvlib, m, n, mode):
    rng = np.random.default_rng(m + n)
    A = dev(activations(rng, m * n))
    _two_paths(nvlib, m, n, A, mode == "sr", mode == "fm")


@pytest.mark.parametrize("sm_count", [1, 5, 64])
def test_fused_with_capped_grid(nvlib, sm_count):
    rng = np.random.default_rng(sm_count)
    m, n = 512, 2048
    A = dev(activations(rng, m * n))
    _two_paths(nvlib, m, n, A, True, False, sm_count=sm_count, repeats=3)


def test_fused_k_tile_and_nan(nvlib):
    from oracle import oracle
    rng = np.random.default_rng(3)
    m, n = 256, 1280
    x = rng.standard_normal(m * n).astype(np.float32)
    A = dev(oracle.f32_to_bf16(x))
    _two_paths(nvlib, m, n, A, True, False, k_tile=192)
    x[12345] = np.nan
    A = dev(oracle.f32_to_bf16(x))
    _two_paths(nvlib, m, n, A, True, False)


def test_fused_full_size_cfg5(nvlib):
    """BASELINE config 5 in one launch, twice."""
    m, n = 14336, 65536
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(m * n, device="cuda", generator=g)
    A[torch.rand(m * n, device="cuda", generator=g) < 0.001] *= 50.0
    A = A.to(torch.bfloat16)
    _two_paths(nvlib, m, n, A, True, False)


def _cfg_input(m, n, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(m * n, device="cuda", generator=g)
    A[torch.rand(m * n, device="cuda", generator=g) < 0.001] *= 50.0
    return A.to(torch.bfloat16)


@pytest.mark.parametrize("m,n", [(5120, 8192), (14336, 65536)])
def test_fused_vs_reference_te_kernel(nvlib, m, n):
    """BASELINE configs 4 and 5, SR: the fused amax + cast is bit-exact with
    the reference's own TE SM100 kernel (hadamard_transform_cast_fusion_core.inc
    :513-644, compiled in place) given the amax, and its amax equals torch's
    max of |A| (an amax computed independently of this library)."""
    from oracle import ref
    if not ref.gpu_available():
        pytest.skip("reference GPU library not built")
    L = ref.gpu()
    A = _cfg_input(m, n, m + n)
    B = dev(h16(np.array([1, -1, -1, 1] * 4)))
    rs = torch.tensor([777, 5], dtype=torch.int64, device="cuda")
    want_amax = A.float().abs().max().view(1)
    C = torch.full((m, n // 2), 0xAA, dtype=torch.uint8, device="cuda")
    S = torch.full((m, n // 16), 0xAA, dtype=torch.uint8, device="cuda")
    am = torch.full((1,), -1.0, device="cuda")
    nvlib.quantize_rht_fused(m, n, A, B, C, S, am, rs, nvlib.fused_workspace(), 0, None, 2048,
                             stochastic_rounding=True)
    Cr, Sr = torch.zeros_like(C), torch.zeros_like(S)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    rc = L.teref_rht_gemm_ntt_w_sfc(m, n, A.data_ptr(), B.data_ptr(), Cr.data_ptr(),
                                    Sr.data_ptr(), want_amax.data_ptr(), rs.data_ptr(), sms,
                                    None, 1, 0)
    torch.cuda.synchronize()
    assert rc == 0 and nvlib.device_error() == 0
    assert torch.equal(am.view(torch.int32), want_amax.view(torch.int32)), (am, want_amax)
    assert torch.equal(S, Sr), f"SFC mismatches: {(S != Sr).sum().item()}"
    assert torch.equal(C, Cr), f"FP4 byte mismatches: {(C != Cr).sum().item()}"
