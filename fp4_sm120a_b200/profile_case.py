"""Small reproducible launches for profiling (ncu) and quick timing.

    python -m fp4_sm120a_b200.profile_case rht  --m 14336 --n 8192 --sr 1 --fm 0
    python -m fp4_sm120a_b200.profile_case amax --m 14336 --n 8192
    python -m fp4_sm120a_b200.profile_case sr   --groups 67108864
    python -m fp4_sm120a_b200.profile_case rowwise --m 16384 --n 8192
    python -m fp4_sm120a_b200.profile_case fp8  --groups 67108864
    ... --time 20      # time 20 launches instead (L2 flushed before each)
    ... --evict-after  # after each launch, read a 512 MB buffer with the amax
                       # kernel (reads only), so that the dirty lines the launch
                       # left in L2 are written back inside that kernel, where a
                       # per-kernel DRAM capture counts them

Each case runs `--launches` launches of one kernel on seeded inputs and exits
0.  With --time N it prints one JSON line per case with the median launch time
(CUDA events on the launching stream, a 512 MB buffer written between
launches so no input is served from L2) and the algorithmic GB/s.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import ops


def _case(a, g):
    """Returns (launch function, algorithmic bytes per launch, elements)."""
    if a.kernel == "rht":
        A = torch.randn(a.m * a.n, device="cuda", generator=g).to(torch.bfloat16)
        B = ops.hadamard16(device="cuda")
        C = torch.empty(a.m * a.n // 2, dtype=torch.uint8, device="cuda")
        S = torch.empty(a.m * a.n // 16, dtype=torch.uint8, device="cuda")
        am = torch.tensor([4.0], device="cuda")
        rs = torch.tensor([1, 0], dtype=torch.int64, device="cuda")

        def f():
            ops.rht_gemm_ntt_w_sfc(a.m, a.n, A, B, C, S, am, rs, 0, None, 2048,
                                   stochastic_rounding=bool(a.sr), use_fast_math=bool(a.fm))
        return f, a.m * a.n * 2.5625 + 516, a.m * a.n
    if a.kernel in ("fused", "twostep"):
        # amax + cast: one fused launch, or the amax pre-pass then the cast
        A = torch.randn(a.m * a.n, device="cuda", generator=g).to(torch.bfloat16)
        B = ops.hadamard16(device="cuda")
        C = torch.empty(a.m * a.n // 2, dtype=torch.uint8, device="cuda")
        S = torch.empty(a.m * a.n // 16, dtype=torch.uint8, device="cuda")
        am = torch.empty(1, device="cuda")
        rs = torch.tensor([1, 0], dtype=torch.int64, device="cuda")
        ws = ops.fused_workspace()

        def f():
            if a.kernel == "fused":
                ops.quantize_rht_fused(a.m, a.n, A, B, C, S, am, rs, ws, 0, None, 2048,
                                       stochastic_rounding=bool(a.sr), use_fast_math=bool(a.fm))
            else:
                ops.amax_bf16(A, a.m * a.n, am)
                ops.rht_gemm_ntt_w_sfc(a.m, a.n, A, B, C, S, am, rs, 0, None, 2048,
                                       stochastic_rounding=bool(a.sr), use_fast_math=bool(a.fm))
        return f, a.m * a.n * 2.5625 + 516, a.m * a.n
    if a.kernel == "amax":
        n = a.m * a.n
        A = torch.randn(n, device="cuda", generator=g).to(torch.bfloat16)
        am = torch.empty(1, device="cuda")
        return (lambda: ops.amax_bf16(A, n, am)), 2 * n, n
    if a.kernel == "rowwise":
        rows, cols = a.m, a.n
        X = torch.randn(rows * cols, device="cuda", generator=g)
        X[torch.rand(rows * cols, device="cuda", generator=g) < 0.001] *= 50.0
        X = X.to(torch.bfloat16)
        rb = torch.randint(-2**31, 2**31 - 1, (rows * cols // 4,), device="cuda",
                           dtype=torch.int32, generator=g)
        am = torch.empty(1, device="cuda")
        ops.amax_bf16(X, rows * cols, am)
        C = torch.empty(rows * cols // 2, dtype=torch.uint8, device="cuda")
        S = torch.empty(rows * cols // 16, dtype=torch.uint8, device="cuda")
        return ((lambda: ops.quantize_rowwise_bf16_sr(rows, cols, X, am, rb, C, S)),
                rows * cols * 3.5625, rows * cols)
    if a.kernel == "fp8":
        # mul_cvt_4x, bf16 in, E4M3 out, one floatx2 scale: 8 + 4 B per group
        x = torch.randn(4 * a.groups, device="cuda", generator=g).to(torch.bfloat16)
        s = torch.tensor([0.5, 2.0], device="cuda")
        out = torch.empty(4 * a.groups, dtype=torch.uint8, device="cuda")
        return ((lambda: ops.mul_cvt_fp8_4x(x, "bf16", s, 2, 0, out, "e4m3", a.groups)),
                a.groups * 12, 4 * a.groups)
    x = torch.randn(4 * a.groups, device="cuda", generator=g) * 3
    rb = torch.randint(-2**31, 2**31 - 1, (a.groups,), device="cuda", dtype=torch.int32,
                       generator=g)
    out = torch.empty(a.groups, dtype=torch.int16, device="cuda")
    return ((lambda: ops.cvt_fp32_to_fp4_4x_sr(x, rb, out, a.groups)), a.groups * 22,
            4 * a.groups)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["rht", "amax", "sr", "rowwise", "fused", "twostep", "fp8"])
    ap.add_argument("--m", type=int, default=14336)
    ap.add_argument("--n", type=int, default=8192)
    ap.add_argument("--sr", type=int, default=1)
    ap.add_argument("--fm", type=int, default=0)
    ap.add_argument("--groups", type=int, default=1 << 26)
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--time", type=int, default=0)
    ap.add_argument("--evict-after", action="store_true")
    a = ap.parse_args(argv)
    g = torch.Generator(device="cuda").manual_seed(0)
    f, nbytes, elems = _case(a, g)
    if a.evict_after:
        ev = torch.zeros(256 << 20, dtype=torch.bfloat16, device="cuda")
        ev_out = torch.empty(1, device="cuda")
        f0 = f

        def f():
            f0()
            ops.amax_bf16(ev, ev.numel(), ev_out)
    if a.time:
        flush = torch.empty(128 * 1024 * 1024, dtype=torch.float32, device="cuda")
        ts = []
        for i in range(a.time + 3):
            flush.add_(1.0)
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            f()
            e1.record()
            torch.cuda.synchronize()
            if i >= 3:
                ts.append(e0.elapsed_time(e1))
        ts.sort()
        ms = ts[len(ts) // 2]
        print(json.dumps({"kernel": a.kernel, "m": a.m, "n": a.n, "sr": a.sr, "fm": a.fm,
                          "groups": a.groups if a.kernel in ("sr", "fp8") else None, "ms": ms,
                          "gbs": nbytes / ms / 1e6, "elem_per_s": elems / ms * 1e3}))
    else:
        for _ in range(a.launches):
            f()
        torch.cuda.synchronize()
        print("ok")
    assert ops.device_error() == 0
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
