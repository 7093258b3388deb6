"""Small reproducible launches for profiling (ncu) and quick timing.

    python -m fp4_sm120a_b200.profile_case rht  --m 14336 --n 8192 --sr 1 --fm 0
    python -m fp4_sm120a_b200.profile_case amax --n 117440512
    python -m fp4_sm120a_b200.profile_case sr   --groups 67108864

Each runs three launches of one kernel on seeded inputs (larger than L2 at the
defaults) and exits 0; the inputs hold a few hundred MB of device memory.
"""
from __future__ import annotations

import argparse

import torch

from . import ops


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["rht", "amax", "sr"])
    ap.add_argument("--m", type=int, default=14336)
    ap.add_argument("--n", type=int, default=8192)
    ap.add_argument("--sr", type=int, default=1)
    ap.add_argument("--fm", type=int, default=0)
    ap.add_argument("--groups", type=int, default=1 << 26)
    ap.add_argument("--launches", type=int, default=3)
    a = ap.parse_args(argv)
    g = torch.Generator(device="cuda").manual_seed(0)
    if a.kernel == "rht":
        A = torch.randn(a.m * a.n, device="cuda", generator=g).to(torch.bfloat16)
        B = ops.hadamard16(device="cuda")
        C = torch.empty(a.m * a.n // 2, dtype=torch.uint8, device="cuda")
        S = torch.empty(a.m * a.n // 16, dtype=torch.uint8, device="cuda")
        am = torch.tensor([4.0], device="cuda")
        rs = torch.tensor([1, 0], dtype=torch.int64, device="cuda")
        for _ in range(a.launches):
            ops.rht_gemm_ntt_w_sfc(a.m, a.n, A, B, C, S, am, rs, 0, None, 2048,
                                   stochastic_rounding=bool(a.sr), use_fast_math=bool(a.fm))
    elif a.kernel == "amax":
        n = a.m * a.n
        A = torch.randn(n, device="cuda", generator=g).to(torch.bfloat16)
        am = torch.empty(1, device="cuda")
        for _ in range(a.launches):
            ops.amax_bf16(A, n, am)
    else:
        x = torch.randn(4 * a.groups, device="cuda", generator=g) * 3
        rb = torch.randint(-2**31, 2**31 - 1, (a.groups,), device="cuda", dtype=torch.int32,
                           generator=g)
        out = torch.empty(a.groups, dtype=torch.int16, device="cuda")
        for _ in range(a.launches):
            ops.cvt_fp32_to_fp4_4x_sr(x, rb, out, a.groups)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    print("ok")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
