#!/usr/bin/env python
"""Benchmark of the NVFP4 quantization hot path on B200.

One step = the row-sharded quantization of BASELINE config 5: an activation
X (65536 x 14336 bf16, N(0,1) with 0.1% x50 outliers) is split by row blocks
across the ranks (API view: m = 14336, n = 65536 / N columns per rank), and
each rank runs
    global-amax pre-pass (nvfp4_amax_bf16)
    -> RHT GEMM + NVFP4 cast with stochastic rounding in the full problem's
       RNG coordinates; for N > 1 the cast kernel itself combines the ranks'
       amax over NVLink peer memory before its first quantization
       (nvfp4_rht_gemm_ntt_w_sfc_sharded_exchange; --exchange nccl uses an
       NCCL int32-MAX all-reduce of the scalar between the two kernels instead).
Per-rank problems of >= 14336 x 32768 elements (N <= 2) run the step as the
fused single kernel instead (nvfp4_quantize_rht_fused[_sharded_exchange]:
amax pass, grid barrier, cast), which is faster there (--path chooses).
`value` is GB/s in the reference's byte convention for the cast
(2.5625 B per element: 2 read + 0.5 FP4 + 0.0625 SFC, rht_gemm/test_compare.cu:256)
over all ranks' elements divided by the max-over-ranks step time; the amax
pass is inside the step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's own CPU implementation of the path
(NaiveReference from rht_gemm/test_correctness.cu, compiled in place into
oracle/_ref/libref_cpu.so) on the host cores, on a bounded sample of the same
workload; beside it the reference's scalar sr.software quantizer
(stochastic_rounding/sr.software.cuh) at BASELINE configs 1 and 3.

Besides `value` (exactly K timed steps) the line carries:
  parity     the step's outputs compared bit for bit with an independent path
             (N = 1: the fused single-kernel quantizer; N > 1: every rank's
             shard against the NCCL-exchange path, and rank 0 regenerates the
             whole input and compares the gathered shards with a single-GPU run)
  sustained  the same step timed over 200 (N = 1) or 1000 (N > 1) steps
  cfg4       the cast alone at BASELINE config 4 (5120 x 8192 and the reference
             test's 8192 x 5120), SR, L2 flushed before every launch
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

ROWS, COLS = 65536, 14336          # activation X (tokens x features)
BYTES_PER_ELEM = 2 + 0.5 + 1.0 / 16
RHT_FIXED_BYTES = 512 + 4          # B matrix + amax
SEED = 20260101
NOMINAL_HBM_GBS = 8000.0


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class NvmlClockSampler:
    """SM clock and throttle-reason sampling during the timed region, read
    from NVML every ~0.5 ms in a thread (read-only queries), so that timed
    regions of a few milliseconds still get samples."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, cuda_indices):
        import threading
        import pynvml
        import torch
        self.nv = pynvml
        pynvml.nvmlInit()
        self.handles = []
        for i in cuda_indices:
            pr = torch.cuda.get_device_properties(i)
            try:
                bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
                self.handles.append(pynvml.nvmlDeviceGetHandleByPciBusId(bus))
            except Exception:
                self.handles.append(pynvml.nvmlDeviceGetHandleByIndex(i))
        self.samples, self.reasons = [], set()
        self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handles[0], pynvml.NVML_CLOCK_SM)
        self.stop = threading.Event()
        self.active = threading.Event()   # sample only while set (GPU busy windows)
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self.nv
        while not self.stop.is_set():
            if not self.active.wait(timeout=0.01):
                continue
            for h in self.handles:
                try:
                    self.samples.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                    bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    for name, mask in self.REASONS.items():
                        if bits & mask:
                            self.reasons.add(name)
                except Exception:
                    pass
            time.sleep(0.0005)

    def __enter__(self):
        self.thread.start()
        return self

    def window(self, on: bool):
        (self.active.set if on else self.active.clear)()

    def __exit__(self, *a):
        self.active.clear()
        self.stop.set()
        self.thread.join(timeout=5)

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples), "source": "NVML"}


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region (used when
    NVML cannot be loaded)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.proc = None
        self.idx = ",".join(str(i) for i in gpu_indices)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.idx, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_shard(torch, rank, n_cols):
    """This rank's shard of X: rows [rank*n_cols, (rank+1)*n_cols), which in the
    API's column-major view is an m x n_cols matrix (contiguous)."""
    g = torch.Generator(device="cuda").manual_seed(SEED + rank)
    x = torch.randn(n_cols * COLS, device="cuda", dtype=torch.float32, generator=g)
    mask = torch.rand(n_cols * COLS, device="cuda", generator=g) < 0.001
    x[mask] *= 50.0
    out = x.to(torch.bfloat16)
    del x, mask
    return out


class CpuReference:
    """The reference's own CPU implementation of the path (NaiveReference,
    rht_gemm/test_correctness.cu:110-198, compiled in place into
    oracle/_ref/libref_cpu.so; kind "reference"), or the oracle port when that
    library is absent (kind "port"), on a bounded column slice of the
    workload: API m = 14336 rows x `ncols` columns, sized so one call takes
    about `target_s` seconds."""

    def __init__(self, target_s: float, threads: int | None = None):
        from oracle import oracle, ref
        self.oracle, self.ref = oracle, ref
        self.threads = threads or os.cpu_count() or 1
        self.kind = "reference" if ref.cpu_available() else "port"
        i = np.arange(16)
        par = np.array([[bin(a & b).count("1") & 1 for b in i] for a in i])
        self.B = oracle.f32_to_bf16(np.where(par == 0, 0.25, -0.25).astype(np.float32))
        self.m = COLS
        self.rng = np.random.default_rng(SEED)
        ncols = 64 * self.threads
        dt = self._size(ncols)
        while dt < target_s / 8 and ncols < ROWS:
            ncols = min(ROWS, ncols * 4)
            dt = self._size(ncols)
        ncols = int(min(ROWS, max(64, ncols * target_s / max(dt, 1e-3))) // 64 * 64)
        self._size(ncols)

    def _size(self, ncols):
        self.ncols = ncols
        self.A = self.oracle.f32_to_bf16(self.rng.standard_normal(self.m * ncols)
                                         .astype(np.float32))
        self.C = np.zeros((self.m, ncols // 2), np.uint8)
        self.S = np.zeros((self.m, ncols // 16), np.uint8)
        return self.step()

    def step(self) -> float:
        t0 = time.perf_counter()
        if self.kind == "reference":
            self.ref.cpu().ref_naive_rht(self.m, self.ncols, self.A.ctypes.data,
                                         self.B.ctypes.data, self.C.ctypes.data,
                                         self.S.ctypes.data, 4.0, 0, 64, self.threads)
        else:
            self.oracle.rht_gemm_ntt_w_sfc(self.m, self.ncols, self.A, self.B, 4.0, (SEED, 0),
                                           2048, True, False)
        return time.perf_counter() - t0

    @property
    def elems(self):
        return self.m * self.ncols

    def describe(self, dt):
        if self.kind == "reference":
            return (f"NaiveReference::compute (rht_gemm/test_correctness.cu:110-198; "
                    f"round-to-nearest, the reference has no CPU stochastic-rounding RHT) on "
                    f"API m={self.m} x n={self.ncols} columns of the workload, "
                    f"{self.threads} threads, {dt:.2f} s per step")
        return f"oracle port (SR) on m={self.m} x n={self.ncols}, 1 thread, {dt:.2f} s"

    def baseline(self, steps=1):
        ts = sorted(self.step() for _ in range(steps))
        dt = ts[len(ts) // 2]
        return {"value": self.elems * BYTES_PER_ELEM / dt / 1e9, "unit": "GB/s",
                "elem_per_s": self.elems / dt,
                "cores": self.threads if self.kind == "reference" else 1,
                "kind": self.kind, "sample": self.describe(dt)}


def sr_software_baseline(reps: int = 3):
    """The reference's scalar software SR quantizer (stochastic_rounding/
    sr.software.cuh:100-323, compiled in place into oracle/_ref/libref_cpu.so)
    on the host cores: cvt_fp32_to_fp4_4x at BASELINE config 1 (2^20 fp32
    values ~N(0,1)x3) and mul_cvt_bf16_to_fp4_8x at config 3 (16384 x 8192
    bf16 with 0.1% x50 outliers, scale 1), each on 1 thread and on all
    threads (median of `reps`).  Bytes counted: input + rbits + FP4 output."""
    from oracle import oracle, ref
    if not ref.cpu_available():
        return {"unavailable": "oracle/_ref/libref_cpu.so not built"}
    L = ref.cpu()
    rng = np.random.default_rng(SEED)
    threads = os.cpu_count() or 1
    out = {"cores_all": threads}
    n1 = 1 << 20
    x1 = (rng.standard_normal(n1) * 3).astype(np.float32)
    r1 = rng.integers(0, 2**32, n1 // 4, dtype=np.uint32)
    o1 = np.zeros(n1 // 4, np.uint16)
    n3 = 16384 * 8192
    x3 = rng.standard_normal(n3).astype(np.float32)
    x3[rng.random(n3) < 0.001] *= 50.0
    x3 = oracle.f32_to_bf16(x3)
    r3 = rng.integers(0, 2**32, n3 // 4, dtype=np.uint32)
    o3 = np.zeros(n3 // 8, np.uint32)

    def timed(fn):
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return sorted(ts)[len(ts) // 2]

    for name, n, bpe, call in (
            ("cfg1_cvt_fp32_to_fp4_4x", n1, 4 + 1 + 0.5,
             lambda th: L.ref_sw_cvt_fp32_to_fp4_4x_sr(x1.ctypes.data, r1.ctypes.data,
                                                      o1.ctypes.data, n1 // 4, th)),
            ("cfg3_mul_cvt_bf16_to_fp4_8x", n3, 2 + 1 + 0.5,
             lambda th: L.ref_sw_mul_cvt_bf16_to_fp4_8x_sr(x3.ctypes.data, 1.0, r3.ctypes.data,
                                                          o3.ctypes.data, n3 // 8, th))):
        res = {"elements": n, "bytes_per_elem": bpe}
        for th in (1, threads):
            dt = timed(lambda: call(th))
            res[f"threads_{th}"] = {"s": round(dt, 5), "elem_per_s": n / dt,
                                    "GB/s": round(n * bpe / dt / 1e9, 4)}
        out[name] = res
    out["kind"] = "reference"
    out["note"] = ("scalar software SR of the reference (not bit-exact to cvt.rs by design: "
                   "sr.software.cuh:67-75 hashes the random bits)")
    return out


def bench_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    cpu = CpuReference(target_s=float(os.environ.get("NVFP4_CPU_STEP_S", "1.5")))
    for _ in range(args.warmup):
        cpu.step()
    base = cpu.baseline(args.steps)
    line = {
        "metric": "RHT+NVFP4 quant HBM GB/s (frac of 8 TB/s) and elem/s at 1/2/4/8 B200",
        "impl": "reference",
        "value": round(base["value"], 3),
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": None,
        "higher_is_better": True,
        "scaling": "strong",
        "dtype": "bf16",
        "data": "synthetic",
        "config": workload_config(args.gpus, args.exchange,
                                  step_path(args, COLS, ROWS // args.gpus)),
        "elem_per_s": base["elem_per_s"],
        "sr_software": sr_software_baseline(),
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": round(base["value"], 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "vs_baseline": None,
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config(n, exchange="peer", path="two"):
    ex = "none" if n == 1 else exchange
    if path == "fused":
        how = {"none": "global amax and RHT GEMM + NVFP4 cast in one kernel "
                       "(nvfp4_quantize_rht_fused)",
               "peer": "global amax and RHT GEMM + NVFP4 cast in one kernel, the ranks' amax "
                       "combined inside it over NVLink peer memory",
               "nccl": "global amax and RHT GEMM + NVFP4 cast in one kernel"}[ex]
    else:
        how = {"none": "amax pre-pass + RHT GEMM + NVFP4 cast",
               "peer": "amax pre-pass + RHT GEMM + NVFP4 cast with the ranks' amax combined "
                       "inside the cast kernel over NVLink peer memory",
               "nccl": "amax pre-pass + NCCL int32-MAX all-reduce of the amax + RHT GEMM + "
                       "NVFP4 cast"}[ex]
    return {"workload": "BASELINE cfg5: X 65536x14336 bf16 N(0,1)+0.1% x50 outliers, "
                        f"row-sharded (API m=14336, n=65536/N per rank), {how}, "
                        "stochastic rounding",
            "m": COLS, "n_total": ROWS, "n_per_rank": ROWS // n, "k_tile_size": 2048,
            "stochastic_rounding": True, "parallelism": f"row-shard x{n}",
            "amax_exchange": ex, "path": path,
            "l2": "inputs larger than L2 (per-rank shard >= 235 MB > 126 MB)"}


# Per-rank problems of at least this many elements run the step as the fused
# single kernel (--path auto): there its second pass re-reads part of A from
# L2 and it saves a launch; below it the amax kernel + cast kernel are faster
# (measured on one B200, m = 14336: fused 638-644 vs 659-664 us at n = 65536,
# 331 vs 336 us at n = 32768, 177 vs 174 us at n = 16384, 101 vs 96 us at
# n = 8192).
FUSED_MIN_ELEMS = 14336 * 32768


def step_path(args, m, n_per_rank):
    if args.path != "auto":
        return args.path
    return "fused" if m * n_per_rank >= FUSED_MIN_ELEMS else "two"


def check_parity(torch, dist, nv, qz, A, B, C, S, amax, rng_state, ws, rank, fused=False):
    """Bit-for-bit check of the step's outputs (C, S and the amax of the
    last step) against independent paths.  N = 1: the fused single-kernel
    quantizer.  N > 1: (a) on every rank, the NCCL path -- amax kernel,
    int32-MAX all-reduce, sharded cast -- on the same shard; (b) rank 0
    regenerates the whole input from the ranks' seeds, runs the single-GPU
    amax + cast on it and compares the shards gathered from all ranks."""
    from fp4_sm120a_b200.sharded import combine_amax
    m, n, n_total = qz.m, qz.n, qz.n_total
    C2, S2 = torch.empty_like(C), torch.empty_like(S)
    am2 = torch.empty(1, dtype=torch.float32, device="cuda")
    if ws == 1:
        if fused:
            # the step ran the fused kernel: check it against amax + cast
            nv.amax_bf16(A, m * n, am2)
            nv.rht_gemm_ntt_w_sfc(m, n, A, B, C2, S2, am2, rng_state, 0, None, 2048,
                                  stochastic_rounding=True)
            vs = "amax kernel + cast kernel (nvfp4_amax_bf16, nvfp4_rht_gemm_ntt_w_sfc), same input"
        else:
            wsp = nv.fused_workspace()
            nv.quantize_rht_fused(m, n, A, B, C2, S2, am2, rng_state, wsp, 0, None, 2048,
                                  stochastic_rounding=True)
            vs = "fused single-kernel quantizer (nvfp4_quantize_rht_fused), same input"
        torch.cuda.synchronize()
        cnt = torch.tensor([int((C2 != C).sum()), int((S2 != S).sum()),
                            int(not torch.equal(am2.view(torch.int32), amax.view(torch.int32)))],
                           dtype=torch.int64)
        return {"checked": True, "fp4_mismatch": int(cnt[0]), "sfc_mismatch": int(cnt[1]),
                "amax_mismatch": int(cnt[2]), "vs": vs}
    # (a) this rank's shard through the NCCL exchange path
    nv.amax_bf16(A, m * n, am2)
    combine_amax(am2)
    nv.rht_gemm_ntt_w_sfc_sharded(m, n, A, B, C2, S2, am2, rng_state, qz.n_offset, n_total, 0,
                                  None, 2048, stochastic_rounding=True)
    torch.cuda.synchronize()
    cnt = torch.tensor([int((C2 != C).sum()), int((S2 != S).sum()),
                        int(not torch.equal(am2.view(torch.int32), amax.view(torch.int32))),
                        0, 0, 0], dtype=torch.int64, device="cuda")
    del C2, S2
    # (b) the gathered shards against one GPU running the whole problem
    sizes = qz.plan.sizes
    Cs = [torch.empty((m, sz // 2), dtype=torch.uint8, device="cuda") for sz in sizes]
    Ss = [torch.empty((m, sz // 16), dtype=torch.uint8, device="cuda") for sz in sizes]
    dist.all_gather(Cs, C)
    dist.all_gather(Ss, S)
    if rank == 0:
        Af = torch.cat([make_shard(torch, r, sizes[r]) for r in range(ws)])
        Cf = torch.empty((m, n_total // 2), dtype=torch.uint8, device="cuda")
        Sf = torch.empty((m, n_total // 16), dtype=torch.uint8, device="cuda")
        amf = torch.empty(1, dtype=torch.float32, device="cuda")
        nv.amax_bf16(Af, m * n_total, amf)
        nv.rht_gemm_ntt_w_sfc(m, n_total, Af, B, Cf, Sf, amf, rng_state, 0, None, 2048,
                              stochastic_rounding=True)
        torch.cuda.synchronize()
        cnt[3] = int((torch.cat(Cs, 1) != Cf).sum())
        cnt[4] = int((torch.cat(Ss, 1) != Sf).sum())
        cnt[5] = int(not torch.equal(amf.view(torch.int32), amax.view(torch.int32)))
        del Af, Cf, Sf
    del Cs, Ss
    dist.all_reduce(cnt)
    c = cnt.tolist()
    return {"checked": True, "fp4_mismatch": c[0] + c[3], "sfc_mismatch": c[1] + c[4],
            "amax_mismatch": c[2] + c[5],
            "detail": {"vs_nccl_path": {"fp4": c[0], "sfc": c[1], "amax": c[2]},
                       "vs_single_gpu": {"fp4": c[3], "sfc": c[4], "amax": c[5]}},
            "vs": "single-GPU run of the whole input + NCCL-exchange path on every shard"}


def bench_cfg4(torch, nv, peak, reps=50):
    """The cast alone at BASELINE config 4: m=5120, n=8192 (and the reference
    test's 8192 x 5120), SR, bf16 N(0,1) with 0.1% x50 outliers.  Two
    protocols:
      cold    one launch between CUDA events, after a read-only pass over
              512 MB (the amax kernel) that evicts the previous launch's data
              from L2 and leaves no dirty lines behind; median of `reps`.
              Includes the launch latency of a lone kernel.
      stream  `reps` back-to-back launches cycling through enough input /
              output sets that their total exceeds L2 (126 MB), so every
              launch reads its input from HBM, timed as a whole; the average
              per launch (what the cast costs inside a longer stream of work,
              as in rht_gemm/test_compare.cu:62-92, which times back-to-back
              launches)."""
    out = {}
    ev = torch.zeros(256 << 20, dtype=torch.bfloat16, device="cuda")
    ev_out = torch.empty(1, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    B = nv.hadamard16(device="cuda")
    rs = torch.tensor([SEED, 0], dtype=torch.int64, device="cuda")
    for m, n in ((5120, 8192), (8192, 5120)):
        nbytes = m * n * BYTES_PER_ELEM + RHT_FIXED_BYTES
        sets = []
        for k in range(max(2, -(-(300 << 20) // int(nbytes)))):
            g = torch.Generator(device="cuda").manual_seed(SEED + k)
            x = torch.randn(m * n, device="cuda", generator=g)
            x[torch.rand(m * n, device="cuda", generator=g) < 0.001] *= 50.0
            A = x.to(torch.bfloat16)
            del x
            C = torch.empty((m, n // 2), dtype=torch.uint8, device="cuda")
            S = torch.empty((m, n // 16), dtype=torch.uint8, device="cuda")
            am = torch.empty(1, dtype=torch.float32, device="cuda")
            nv.amax_bf16(A, m * n, am)
            sets.append((A, C, S, am))

        def launch(k):
            A, C, S, am = sets[k % len(sets)]
            nv.rht_gemm_ntt_w_sfc(m, n, A, B, C, S, am, rs, 0, stream, 2048,
                                  stochastic_rounding=True)
        ts = []
        for i in range(reps + 5):
            nv.amax_bf16(ev, ev.numel(), ev_out, stream)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            launch(i)
            e1.record(stream)
            ts.append((e0, e1))
        torch.cuda.synchronize()
        cold_us = sorted(a.elapsed_time(b) * 1e3 for a, b in ts[5:])[reps // 2]
        for i in range(5):
            launch(i)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(reps):
            launch(i)
        e1.record(stream)
        torch.cuda.synchronize()
        stream_us = e0.elapsed_time(e1) * 1e3 / reps
        res = {}
        for name, us in (("cold", cold_us), ("stream", stream_us)):
            gbs = nbytes / (us * 1e-6) / 1e9
            res[name] = {"us": round(us, 2), "GB/s": round(gbs, 1),
                         "frac_of_8TBs": round(gbs / NOMINAL_HBM_GBS, 4),
                         "frac_of_measured": round(gbs / peak, 4)}
        res["buffer_sets"] = len(sets)
        out[f"m{m}_n{n}"] = res
        del sets
    out["method"] = ("cast only (rht_nvfp4_kernel<SR=1>); cold: one launch between CUDA events "
                     "after a read-only 512 MB pass, median of %d; stream: %d back-to-back "
                     "launches over rotating input sets totalling > L2, average" % (reps, reps))
    return out


def bench_ours(args):
    import torch
    import torch.distributed as dist

    ws, rank, local = dist_env()
    if ws != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={ws}")
    torch.cuda.set_device(local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))

    import fp4_sm120a_b200 as nv
    from fp4_sm120a_b200.sharded import ShardedRhtQuantizer, combine_amax
    nv.load()
    m = COLS
    n_total = ROWS
    rng_state = torch.tensor([SEED, 0], dtype=torch.int64, device="cuda")
    fused = step_path(args, m, n_total // ws) == "fused"
    qz = ShardedRhtQuantizer(m, n_total, k_tile_size=2048, stochastic_rounding=True,
                             rng_state=rng_state, exchange=args.exchange, fused=fused)
    n = qz.n
    A = make_shard(torch, rank, n)
    B = nv.hadamard16(torch.where(torch.arange(16) % 3 == 0, -1.0, 1.0), device="cuda")
    C = torch.empty((m, n // 2), dtype=torch.uint8, device="cuda")
    S = torch.empty((m, n // 16), dtype=torch.uint8, device="cuda")
    amax = torch.empty(1, dtype=torch.float32, device="cuda")
    # the two-kernel step's amax words, alternating between steps (the chained
    # amax kernel clears the other one for the next step: no memset)
    words = torch.zeros(2, dtype=torch.float32, device="cuda")
    nstep = [0]
    stream = torch.cuda.current_stream()

    def step(ev=None):
        if fused:
            # one kernel: amax pass, (peer exchange,) cast
            if ev is not None:
                ev[0].record(stream)
            qz(A, B, C, S, amax, stream)
            if ev is not None:
                ev[1].record(stream)
            return
        # amax pre-pass -> exchange of the scalar -> RHT + NVFP4 cast.  With the
        # peer exchange the cast kernel itself combines the ranks' amax.  The
        # amax kernel runs chained: it starts while the previous step's cast
        # drains (A is not written by it) and needs no memset.
        i = nstep[0]
        nstep[0] += 1
        am = words[i % 2:i % 2 + 1]
        nv.amax_bf16_chained(A, m * n, am, words[(i + 1) % 2:(i + 1) % 2 + 1], stream)
        if qz.peer is None:
            combine_amax(am)
        if ev is not None:
            ev[0].record(stream)
        if qz.peer is None:
            nv.rht_gemm_ntt_w_sfc_sharded(m, n, A, B, C, S, am, rng_state, qz.n_offset,
                                          n_total, 0, stream, 2048, stochastic_rounding=True)
        else:
            nv.rht_gemm_ntt_w_sfc_sharded_exchange(m, n, A, B, C, S, am, am, rng_state,
                                                   qz.n_offset, n_total, qz.peer, 0, stream,
                                                   2048, stochastic_rounding=True)
        if ev is not None:
            ev[1].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if nv.device_error() != 0:
        raise SystemExit("kernel reported a device timeout")

    gpu_list = [local] if ws == 1 else list(range(ws))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = None
    if rank == 0:
        try:
            sampler = NvmlClockSampler(gpu_list)
        except Exception:
            sampler = ClockSampler(gpu_list)
    if sampler:
        sampler.__enter__()
    window = getattr(sampler, "window", lambda on: None)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    window(True)
    t0.record(stream)
    for i in range(args.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize()
    window(False)
    # The cast's per-launch duration for the roofline: the same K steps again,
    # now with CUDA events around each cast.  They are kept out of the timed
    # steps above because an event recorded between the amax kernel and the
    # cast ends the cast's programmatic-dependent overlap with the amax.
    if ws > 1:
        dist.barrier()
    window(True)
    for i in range(args.steps):
        step(evs[i])
    torch.cuda.synchronize()
    window(False)
    # A longer run of the same step, for a steadier figure than K steps give.
    sus_steps = 200 if ws == 1 else 1000
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    window(True)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for i in range(sus_steps):
        step()
    s1.record(stream)
    torch.cuda.synchronize()
    window(False)
    if ws > 1:
        dist.barrier()
    if sampler:
        sampler.__exit__()
    if nv.device_error() != 0:
        raise SystemExit("kernel reported a device timeout")
    ms_total = t0.elapsed_time(t1)
    rht_ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    tt = torch.tensor([ms_total, rht_ms, s0.elapsed_time(s1)], dtype=torch.float64,
                      device="cuda")
    if ws > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms_total, rht_ms, sus_ms = tt.tolist()
    if not fused:
        amax = words[(nstep[0] - 1) % 2:(nstep[0] - 1) % 2 + 1]   # the last step's amax
    parity = check_parity(torch, dist, nv, qz, A, B, C, S, amax, rng_state, ws, rank, fused)
    ms_step = ms_total / args.steps
    elems_total = m * n_total
    value = elems_total * BYTES_PER_ELEM / (ms_step * 1e-3) / 1e9

    # ---------------- end to end through the public API, host buffers -------
    # HostPipeline: each step copies the host shard in, runs the step and
    # copies FP4 + SFC out; consecutive steps overlap their two transfers on
    # PCIe (full duplex) through double-buffered device memory.
    from fp4_sm120a_b200.host_pipeline import HostPipeline
    e2e_steps = max(4, min(args.steps, 8))
    hA = torch.empty(A.numel(), dtype=torch.bfloat16, pin_memory=True)
    hA.copy_(A)
    hC = torch.empty(C.shape, dtype=torch.uint8, pin_memory=True)
    hS = torch.empty(S.shape, dtype=torch.uint8, pin_memory=True)
    pipe = HostPipeline(qz, B)
    pipe.submit(hA, hC, hS)
    pipe.synchronize()
    if ws > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(pipe.s_in)
    for _ in range(e2e_steps):
        last = pipe.submit(hA, hC, hS)
    pipe.s_out.wait_event(last)
    e1.record(pipe.s_out)
    pipe.synchronize()
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1) / e2e_steps], dtype=torch.float64, device="cuda")
    if ws > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = te.item()
    # output check of the e2e path against the device-resident path
    same = bool(torch.equal(hC.cuda(), C) and torch.equal(hS.cuda(), S))

    if rank == 0:
        peak, peak_kind = measured_peaks()
        # the timed kernel: the cast (2.5625 B/elem), or the fused kernel, which
        # also reads A for the amax (4.5625 B/elem)
        kbpe = BYTES_PER_ELEM + (2.0 if fused else 0.0)
        rht_bytes = m * n * kbpe + RHT_FIXED_BYTES
        achieved = rht_bytes / (rht_ms * 1e-3) / 1e9
        traffic = None
        tp = ROOT / "profiles" / "rht_nvfp4_traffic.txt"
        if tp.exists():
            for line in tp.read_text().splitlines():
                key = "fused_dram_bytes_per_element" if fused else "dram_bytes_per_element"
                if line.startswith(key + " "):
                    traffic = round(float(line.split("=")[1]) * m * n)
        clocks = sampler.summary() if sampler else {}
        line = {
            "metric": "RHT+NVFP4 quant HBM GB/s (frac of 8 TB/s) and elem/s at 1/2/4/8 B200",
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 5),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16 with 0.1% x50 outliers; BASELINE cfg5 shape)",
            "config": workload_config(ws, args.exchange, "fused" if fused else "two"),
            "elem_per_s": elems_total / (ms_step * 1e-3),
            "frac_of_8TBs": round(value / NOMINAL_HBM_GBS, 4),
            "step_hbm_gbs": round(elems_total * (BYTES_PER_ELEM + 2.0) / (ms_step * 1e-3) / 1e9,
                                  2),
            "roofline": {"bound": "hbm",
                         "kernel": ("rht_fused_kernel<SR=1,FM=0>" if fused
                                    else "rht_nvfp4_kernel<SR=1,FM=0>"),
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                         "algorithmic_bytes_per_launch": rht_bytes,
                         "avg_launch_ms": round(rht_ms, 5),
                         "launch_timing": "CUDA events around each "
                                          + ("fused launch" if fused else "cast")
                                          + " over a second pass of the K steps, right after "
                                            "the timed region"},
            "clocks": {"sm_mhz": clocks.get("sm_mhz"), "sm_max_mhz": clocks.get("sm_max_mhz"),
                       "reasons": clocks.get("reasons", []), "samples": clocks.get("samples")},
            "e2e": {"value": round(elems_total * BYTES_PER_ELEM / (e2e_ms * 1e-3) / 1e9, 3),
                    "unit": "GB/s", "h2d_bytes_per_step": A.numel() * 2,
                    "d2h_bytes_per_step": C.numel() + S.numel(), "ms_per_step": round(e2e_ms, 3),
                    "matches_device_path": same,
                    "pipeline": f"HostPipeline, 2 device buffer sets, {e2e_steps} steps timed"},
            # in the timed region: the fused kernel, or amax + cast, per step
            "gpu_launches": (1 if fused else 2) * args.steps,
            "parity": parity,
            "sustained": {"steps": sus_steps, "ms_per_step": round(sus_ms / sus_steps, 5),
                          "value": round(elems_total * BYTES_PER_ELEM /
                                         (sus_ms / sus_steps * 1e-3) / 1e9, 2),
                          "unit": "GB/s"},
        }
        if ws == 1:
            line["cfg4"] = bench_cfg4(torch, nv, peak)
        if ws == 1 and not args.no_cpu_baseline:
            base = CpuReference(float(os.environ.get("NVFP4_CPU_STEP_S", "3"))).baseline(3)
            line["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind",
                                                         "sample")}
            line["cpu_baseline"]["sr_software"] = sr_software_baseline()
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--path", choices=["auto", "two", "fused"], default="auto",
                    help="fused: one kernel per step; two: amax kernel + cast kernel; "
                         "auto: fused for per-rank problems of >= 14336 x 32768 elements")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="how ranks combine the amax when --gpus > 1")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return bench_reference(args)
    return bench_ours(args)


if __name__ == "__main__":
    sys.exit(main())
