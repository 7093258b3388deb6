"""HostPipeline: host-resident shards through double-buffered device memory
and overlapped PCIe transfers give, step for step, the same FP4 codes and SFC
bytes as the device-resident path."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("sr", [True, False])
def test_pipeline_matches_device_path(nvlib, sr):
    from fp4_sm120a_b200.host_pipeline import HostPipeline
    from fp4_sm120a_b200.sharded import ShardedRhtQuantizer
    m, n = 1024, 4096
    rs = torch.tensor([7, 3], dtype=torch.int64, device="cuda")
    qz = ShardedRhtQuantizer(m, n, stochastic_rounding=sr, rng_state=rs)
    B = nvlib.hadamard16(torch.where(torch.arange(16) % 2 == 0, 1.0, -1.0), device="cuda")
    g = torch.Generator(device="cuda").manual_seed(5)
    steps = 5
    inputs = [(torch.randn(m * n, device="cuda", generator=g) * (1 + i)).to(torch.bfloat16)
              for i in range(steps)]
    hA = [x.cpu().pin_memory() for x in inputs]
    hC = [torch.empty((m, n // 2), dtype=torch.uint8).pin_memory() for _ in range(steps)]
    hS = [torch.empty((m, n // 16), dtype=torch.uint8).pin_memory() for _ in range(steps)]
    pipe = HostPipeline(qz, B)
    for i in range(steps):
        pipe.submit(hA[i], hC[i], hS[i])
    pipe.synchronize()
    for i in range(steps):
        C, S = qz.outputs()
        qz(inputs[i], B, C, S)
        torch.cuda.synchronize()
        assert torch.equal(hC[i], C.cpu()), i
        assert torch.equal(hS[i], S.cpu()), i
    assert nvlib.device_error() == 0
