"""Generate tests/golden/ref_naive_rht.npz by running the reference's own CPU
RHT + NVFP4 code (NaiveReference, rht_gemm/test_correctness.cu:110-198,
compiled from the reference tree into oracle/_ref/libref_cpu.so by
oracle/build.py).  Inputs are seeded N(0, 1) bf16 with the reference tests'
H16 / 4 matrix and amax = 4 (rht_gemm/test_compare.cu:95-127).

Run from the repository root:  python tests/golden/gen_ref_cpu_fixtures.py
"""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import oracle, ref  # noqa: E402


def h16_over_4() -> np.ndarray:
    i = np.arange(16)
    par = np.array([[bin(a & b).count("1") & 1 for b in i] for a in i])
    return oracle.f32_to_bf16(np.where(par == 0, 0.25, -0.25).astype(np.float32))


def main() -> None:
    from oracle import build
    build.build_ref()
    L = ref.cpu()
    B = h16_over_4()
    out = {"B": B}
    rng = np.random.default_rng(20240601)
    for tag, (m, n, fm) in {"256x128": (256, 128, 0), "128x256": (128, 256, 0),
                            "128x256_fm": (128, 256, 1), "384x320": (384, 320, 0)}.items():
        A = oracle.f32_to_bf16(rng.standard_normal(m * n).astype(np.float32))
        C = np.zeros((m, n // 2), np.uint8)
        S = np.zeros((m, n // 16), np.uint8)
        L.ref_naive_rht(m, n, A.ctypes.data, B.ctypes.data, C.ctypes.data, S.ctypes.data, 4.0,
                        fm, n, 1)
        out["A_" + tag] = A
        out["C_" + tag] = C
        out["SFC_" + tag] = S
        out["shape_" + tag] = np.array([m, n, fm])
        out["amax_" + tag] = np.float32(4.0)
    np.savez_compressed(Path(__file__).resolve().parent / "ref_naive_rht.npz", **out)
    print("wrote ref_naive_rht.npz:", sorted(out))


if __name__ == "__main__":
    main()
