"""Build recipe for the test oracle (TEST INFRASTRUCTURE, not product code).

Two outputs:
  oracle/build/liboracle.so  -- the C restatement (nvfp4_oracle.c), gcc.
  oracle/_ref/*.so           -- the reference's own code compiled in place from
                                its source tree (only when that tree exists):
      libref_cpu.so  sr.software.cuh quantizer (g++) + NaiveReference from
                     rht_gemm/test_correctness.cu (nvcc host code)
      libref_gpu.so  TE's SM100 rht_gemm_ntt_w_sfc (rht_gemm/test_compare_ref.cu)
                     and TE's native cvt.rs functions (ptx.cuh), sm_100a.
      libref_fp8.so  TE's scaled FP8 conversions mul_cvt_2x / mul_cvt_4x
                     (ptx.cuh:923-1693), default and _LOOSE_PRECISION builds.

The reference tree is located by $NVFP4_REFERENCE_ROOT (default: a directory
named "reference" beside this repository).  On the GPU box the tree is absent and
the prebuilt oracle/_ref/*.so files are used as they are.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / "build"
REF_OUT = HERE / "_ref"
SHIMS = HERE / "ref_shims"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _ref_root() -> Path:
    # default: a "reference" directory beside this repository
    return Path(os.environ.get("NVFP4_REFERENCE_ROOT", str(HERE.parents[1] / "reference")))


def _cutlass_root() -> Path | None:
    env = os.environ.get("CUTLASS_HOME")
    if env:
        return Path(env)
    try:
        import flashinfer  # noqa: F401  (header tree only; never imported at run time)
        p = Path(flashinfer.__file__).resolve().parent / "data" / "cutlass"
    except Exception:
        import site
        p = None
        for sp in site.getsitepackages():
            cand = Path(sp) / "flashinfer" / "data" / "cutlass"
            if cand.exists():
                p = cand
    return p if p is not None and (p / "include" / "cute").exists() else None


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"oracle build step failed: {cmd[0]} ... {cmd[-1]}")


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.exists() and d.stat().st_mtime > t for d in deps)


def build_oracle(force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    out = BUILD / "liboracle.so"
    src = HERE / "nvfp4_oracle.c"
    if force or _stale(out, [src]):
        _run(["gcc", "-O2", "-std=c99", "-fPIC", "-shared", "-ffp-contract=off",
              "-fno-fast-math", "-fvisibility=hidden", str(src), "-o", str(out), "-lm"])
    return out


def build_ref(force: bool = False) -> dict[str, Path]:
    """Compile the reference's own code from its tree; no-op when it is absent."""
    root = _ref_root()
    outs: dict[str, Path] = {}
    if not (root / "rht_gemm").exists():
        return outs
    REF_OUT.mkdir(exist_ok=True)
    sr_dir, rht_dir = root / "stochastic_rounding", root / "rht_gemm"

    cpu = REF_OUT / "libref_cpu.so"
    cpu_deps = [SHIMS / "ref_cpu_srsw.cpp", SHIMS / "ref_cpu_naive.cu",
                sr_dir / "sr.software.cuh", rht_dir / "test_correctness.cu"]
    if force or _stale(cpu, cpu_deps):
        o1 = REF_OUT / "ref_cpu_srsw.o"
        o2 = REF_OUT / "ref_cpu_naive.o"
        _run(["g++", "-O3", "-march=x86-64-v2", "-std=c++17", "-fPIC", "-fopenmp",
              "-fvisibility=hidden", f"-I{sr_dir}", "-c", str(SHIMS / "ref_cpu_srsw.cpp"),
              "-o", str(o1)])
        _run([NVCC, *ARCH, "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-fopenmp",
              f"-I{rht_dir}", "-c", str(SHIMS / "ref_cpu_naive.cu"), "-o", str(o2)])
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fopenmp", str(o1), str(o2),
              "-o", str(cpu), "-lgomp"])
        o1.unlink(); o2.unlink()
    outs["cpu"] = cpu

    cut = _cutlass_root()
    gpu = REF_OUT / "libref_gpu.so"
    if cut is not None:
        gpu_deps = [SHIMS / "ref_gpu_teref.cu", rht_dir / "test_compare_ref.cu",
                    rht_dir / "te_ref" / "hadamard_transform_cast_fusion_core.inc"]
        if force or _stale(gpu, gpu_deps):
            _run([NVCC, *ARCH, "-O3", "-std=c++20", "--expt-relaxed-constexpr",
                  "-Xcompiler", "-fPIC", "-shared",
                  f"-I{cut / 'include'}", f"-I{cut / 'tools' / 'util' / 'include'}",
                  f"-I{rht_dir}", f"-I{rht_dir / 'te_ref' / 'stubs'}",
                  str(SHIMS / "ref_gpu_teref.cu"), "-o", str(gpu)])
        outs["gpu"] = gpu

        # The reference's scaled FP8 conversions (ptx.cuh:923-1693), default
        # and _LOOSE_PRECISION builds linked into one library.
        fp8 = REF_OUT / "libref_fp8.so"
        stubs = rht_dir / "te_ref" / "stubs"
        fp8_deps = [SHIMS / "ref_gpu_fp8.cu", stubs / "common" / "util" / "ptx.cuh"]
        if force or _stale(fp8, fp8_deps):
            objs = []
            for tag, defs in (("rn", []), ("loose", ["-D_LOOSE_PRECISION", "-DREF_FP8_LOOSE"])):
                o = REF_OUT / f"ref_gpu_fp8_{tag}.o"
                _run([NVCC, *ARCH, "-O3", "-std=c++20", "--expt-relaxed-constexpr",
                      "-Xcompiler", "-fPIC", *defs, f"-I{cut / 'include'}", f"-I{stubs}",
                      "-c", str(SHIMS / "ref_gpu_fp8.cu"), "-o", str(o)])
                objs.append(o)
            _run([NVCC, *ARCH, "-shared", *map(str, objs), "-o", str(fp8)])
            for o in objs:
                o.unlink()
        outs["fp8"] = fp8
    return outs


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
    print(build_ref(force="--force" in sys.argv))
