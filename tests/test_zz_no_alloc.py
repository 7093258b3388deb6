"""The fused amax + cast entry point that allocates nothing.

Callers that cannot allocate device memory -- hosts that hand out every byte
through their own pool and do not allow a library to call cudaMalloc -- use
nvfp4_quantize_rht_fused_noalloc, whose grid-barrier scratch is built into the
library.  This test calls it through the C ABI twice in a row (the built-in
scratch is reused) and checks every output against the existing entry point
that takes a caller-provided workspace, bit for bit (the same tolerance as the
other parity tests of this kernel).  It is collected last so that a run that
stops at the first failure has run every other test first; it also passes
alone in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_noalloc_matches_workspace_entry_twice():
    from fp4_sm120a_b200 import _native, ops
    from tests.gpu_helpers import activations, dev, h16
    lib = _native.load()
    rng = np.random.default_rng(99)
    for m, n, sr, fm in [(1024, 2048, 1, 0), (384, 320, 0, 0), (5120, 8192, 1, 0)]:
        A = dev(activations(rng, m * n))
        B = dev(h16())
        rs = torch.tensor([7, 3], dtype=torch.int64, device="cuda")
        C0 = torch.empty((m, n // 2), dtype=torch.uint8, device="cuda")
        S0 = torch.empty((m, n // 16), dtype=torch.uint8, device="cuda")
        am0 = torch.empty(1, device="cuda")
        ops.quantize_rht_fused(m, n, A, B, C0, S0, am0, rs, ops.fused_workspace(), 0, None,
                               2048, stochastic_rounding=bool(sr), use_fast_math=bool(fm))
        stream = torch.cuda.current_stream().cuda_stream
        for _ in range(2):
            C = torch.full_like(C0, 0xAA)
            S = torch.full_like(S0, 0xAA)
            am = torch.full((1,), -1.0, device="cuda")
            rc = lib.nvfp4_quantize_rht_fused_noalloc(
                m, n, A.data_ptr(), B.data_ptr(), C.data_ptr(), S.data_ptr(), am.data_ptr(),
                rs.data_ptr(), 0, ctypes.c_void_p(stream), 2048, sr, fm)
            assert rc == 0, lib.nvfp4_status_string(rc)
            torch.cuda.synchronize()
            assert ops.device_error() == 0
            assert torch.equal(am.view(torch.int32), am0.view(torch.int32))
            assert torch.equal(S, S0)
            assert torch.equal(C, C0)


def test_noalloc_refused_call_enqueues_nothing():
    """A call refused for a misaligned A returns NVFP4_ERR_MISALIGNED and puts
    nothing on the stream: captured on a side stream, it leaves an empty graph."""
    from cuda.bindings import runtime as rt
    from fp4_sm120a_b200 import _native
    from tests.gpu_helpers import activations, dev, h16
    lib = _native.load()
    m, n = 256, 512
    rng = np.random.default_rng(5)
    A = dev(activations(rng, m * n + 8))
    B = dev(h16())
    C = torch.empty((m, n // 2), dtype=torch.uint8, device="cuda")
    S = torch.empty((m, n // 16), dtype=torch.uint8, device="cuda")
    am = torch.empty(1, device="cuda")
    s = torch.cuda.Stream()
    # a first, accepted call does the per-device set-up outside the capture
    rc = lib.nvfp4_quantize_rht_fused_noalloc(m, n, A.data_ptr(), B.data_ptr(), C.data_ptr(),
                                              S.data_ptr(), am.data_ptr(), None, 0,
                                              ctypes.c_void_p(s.cuda_stream), 2048, 0, 0)
    assert rc == 0, lib.nvfp4_status_string(rc)
    s.synchronize()
    (err,) = rt.cudaStreamBeginCapture(
        s.cuda_stream, rt.cudaStreamCaptureMode.cudaStreamCaptureModeRelaxed)
    assert err == rt.cudaError_t.cudaSuccess
    rc = lib.nvfp4_quantize_rht_fused_noalloc(m, n, A.data_ptr() + 2, B.data_ptr(),
                                              C.data_ptr(), S.data_ptr(), am.data_ptr(), None,
                                              0, ctypes.c_void_p(s.cuda_stream), 2048, 0, 0)
    err, graph = rt.cudaStreamEndCapture(s.cuda_stream)
    assert err == rt.cudaError_t.cudaSuccess
    err, _, num = rt.cudaGraphGetNodes(graph)
    rt.cudaGraphDestroy(graph)
    assert rc == 3, lib.nvfp4_status_string(rc)      # NVFP4_ERR_MISALIGNED
    assert num == 0


@pytest.mark.parametrize("m,n", [(5120, 8192), (14336, 65536)])
def test_noalloc_vs_reference_te_kernel(m, n):
    """BASELINE configs 4 and 5, SR: the no-allocation entry point, called
    twice through the C ABI, is bit-exact with the reference's own TE SM100
    kernel given torch's max of |A| as the amax."""
    from oracle import ref
    from fp4_sm120a_b200 import _native, ops
    from tests.gpu_helpers import h16, dev
    if not ref.gpu_available():
        pytest.skip("reference GPU library not built")
    L = ref.gpu()
    lib = _native.load()
    g = torch.Generator(device="cuda").manual_seed(m * 3 + n)
    x = torch.randn(m * n, device="cuda", generator=g)
    x[torch.rand(m * n, device="cuda", generator=g) < 0.001] *= 50.0
    A = x.to(torch.bfloat16)
    del x
    B = dev(h16(np.array([-1, 1] * 8)))
    rs = torch.tensor([31337, 2], dtype=torch.int64, device="cuda")
    want_amax = A.float().abs().max().view(1)
    Cr = torch.zeros((m, n // 2), dtype=torch.uint8, device="cuda")
    Sr = torch.zeros((m, n // 16), dtype=torch.uint8, device="cuda")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert L.teref_rht_gemm_ntt_w_sfc(m, n, A.data_ptr(), B.data_ptr(), Cr.data_ptr(),
                                      Sr.data_ptr(), want_amax.data_ptr(), rs.data_ptr(), sms,
                                      None, 1, 0) == 0
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        C = torch.full_like(Cr, 0xAA)
        S = torch.full_like(Sr, 0xAA)
        am = torch.full((1,), -1.0, device="cuda")
        rc = lib.nvfp4_quantize_rht_fused_noalloc(
            m, n, A.data_ptr(), B.data_ptr(), C.data_ptr(), S.data_ptr(), am.data_ptr(),
            rs.data_ptr(), 0, ctypes.c_void_p(stream), 2048, 1, 0)
        assert rc == 0, lib.nvfp4_status_string(rc)
        torch.cuda.synchronize()
        assert ops.device_error() == 0
        assert torch.equal(am.view(torch.int32), want_amax.view(torch.int32))
        assert torch.equal(S, Sr), f"SFC mismatches: {(S != Sr).sum().item()}"
        assert torch.equal(C, Cr), f"FP4 byte mismatches: {(C != Cr).sum().item()}"
