"""Speed against the reference's own SM100 kernel (TE's rht_gemm_ntt_w_sfc,
compiled in place into oracle/_ref/libref_gpu.so), same inputs, same
protocol: L2 flushed before each launch, CUDA events, median of 10.  The
cast must be faster than TE's at BASELINE cfg4 and cfg5 with stochastic
rounding; the timings are printed (pytest -s) for the record."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _median_ms(fn, reps=10):
    flush = torch.empty(128 << 20, dtype=torch.float32, device="cuda")
    ts = []
    for i in range(reps + 3):
        flush.add_(1.0)
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        if i >= 3:
            ts.append(a.elapsed_time(b))
    ts.sort()
    return ts[len(ts) // 2]


@pytest.mark.parametrize("m,n", [(5120, 8192), (14336, 65536)])
def test_faster_than_te_kernel(nvlib, m, n):
    from oracle import ref
    if not ref.gpu_available():
        pytest.skip("reference GPU library not built")
    L = ref.gpu()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    g = torch.Generator(device="cuda").manual_seed(1)
    A = torch.randn(m * n, device="cuda", generator=g).to(torch.bfloat16)
    B = nvlib.hadamard16(device="cuda")
    C = torch.empty(m * n // 2, dtype=torch.uint8, device="cuda")
    S = torch.empty(m * n // 16, dtype=torch.uint8, device="cuda")
    C2, S2 = torch.empty_like(C), torch.empty_like(S)
    am = torch.tensor([4.0], device="cuda")
    rs = torch.tensor([12345, 0], dtype=torch.int64, device="cuda")

    def ours():
        nvlib.rht_gemm_ntt_w_sfc(m, n, A, B, C, S, am, rs, 0, None, 2048,
                                 stochastic_rounding=True)

    def te():
        rc = L.teref_rht_gemm_ntt_w_sfc(m, n, A.data_ptr(), B.data_ptr(), C2.data_ptr(),
                                        S2.data_ptr(), am.data_ptr(), rs.data_ptr(), sms, None,
                                        1, 0)
        assert rc == 0

    t_ours, t_te = _median_ms(ours), _median_ms(te)
    assert torch.equal(C, C2) and torch.equal(S, S2)       # same bits
    gbs = lambda t: m * n * 2.5625 / t / 1e6
    print(f"\nm={m} n={n} SR: ours {t_ours * 1e3:.1f} us ({gbs(t_ours):.0f} GB/s), "
          f"TE SM100 kernel {t_te * 1e3:.1f} us ({gbs(t_te):.0f} GB/s), "
          f"speed-up {t_te / t_ours:.2f}x")
    assert t_ours < t_te
