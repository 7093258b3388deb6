"""Generate tests/golden/teref_rht.npz and tests/golden/teref_sr.npz by running
the reference's own SM100 code on a B200: TE's rht_gemm_ntt_w_sfc and TE's
native cvt.rs conversion functions, compiled from the reference tree into
oracle/_ref/libref_gpu.so (oracle/build.py).  The inputs follow the reference
tests: rht_gemm/test_compare.cu:95-127 (N(0,1) bf16, H16/4, amax 4,
rng_state {12345, 0}) and its 11 extreme patterns (:334-388), plus
BASELINE config 2 (X 256x128 -> API m=128, n=256 with a random-sign H16/4 and
amax = max|A|), k_tile variants, and stochastic_rounding/compare.cu:258-325
style inputs for the SR functions.

Run on a GPU box from the repository root:
    python tests/golden/gen_teref_fixtures.py --out <dir>
then copy the two .npz files into tests/golden/.
"""
import argparse
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import oracle, ref  # noqa: E402


def h16(signs=None) -> np.ndarray:
    i = np.arange(16)
    par = np.array([[bin(a & b).count("1") & 1 for b in i] for a in i])
    h = np.where(par == 0, 0.25, -0.25).astype(np.float32)
    if signs is not None:
        h = h * signs[None, :].astype(np.float32)
    return oracle.f32_to_bf16(h)


def run_teref(m, n, A, B, amax, rng_state, sr, fm):
    L = ref.gpu()
    dA = torch.from_numpy(A.view(np.int16)).cuda()
    dB = torch.from_numpy(B.view(np.int16)).cuda()
    dC = torch.zeros(m * n // 2, dtype=torch.uint8, device="cuda")
    dS = torch.zeros(m * n // 16, dtype=torch.uint8, device="cuda")
    dAm = torch.tensor([amax], dtype=torch.float32, device="cuda")
    dR = torch.tensor([int(rng_state[0]), int(rng_state[1])], dtype=torch.int64, device="cuda")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    rc = L.teref_rht_gemm_ntt_w_sfc(m, n, dA.data_ptr(), dB.data_ptr(), dC.data_ptr(),
                                    dS.data_ptr(), dAm.data_ptr(), dR.data_ptr(), sms, None,
                                    int(sr), int(fm))
    torch.cuda.synchronize()
    assert rc == 0, rc
    return dC.cpu().numpy().reshape(m, n // 2), dS.cpu().numpy().reshape(m, n // 16)


def rht_cases():
    rng = np.random.default_rng(42)
    cases = {}
    H = h16()

    def normal(k):
        return oracle.f32_to_bf16(rng.standard_normal(k).astype(np.float32))

    # reference test shapes (test_compare.cu:297-321), reduced to the small ones
    A = normal(256 * 128)
    for mode, (sr, fm) in {"rn": (0, 0), "fm": (0, 1), "sr": (1, 0)}.items():
        cases[f"ref256x128_{mode}"] = (256, 128, A, H, 4.0, (12345, 0), sr, fm, 2048)
    # X 256 x 128 -> API m = 128, n = 256, random-sign H16
    X = normal(256 * 128)
    signs = np.where(rng.integers(0, 2, 16) == 0, -1.0, 1.0)
    Hs = h16(signs)
    amax = float(np.abs(oracle.bf16_to_f32(X)).max())
    for mode, (sr, fm) in {"rn": (0, 0), "sr": (1, 0)}.items():
        cases[f"cfg2_{mode}"] = (128, 256, X, Hs, amax, (20260101, 0), sr, fm, 2048)
    # k-tile mapping: several chunks, a ragged last chunk, a non-zero offset
    A2 = normal(256 * 512)
    cases["ktile128_sr"] = (256, 512, A2, Hs, 4.0, (777, 3), 1, 0, 128)
    cases["ktile192_sr"] = (256, 512, A2, Hs, 4.0, (777, 2**32 - 2), 1, 0, 192)
    A3 = normal(128 * 320)
    cases["n320_sr"] = (128, 320, A3, H, 4.0, (99, 0), 1, 0, 128)
    cases["n320_rn"] = (128, 320, A3, H, 4.0, (99, 0), 0, 0, 2048)
    # extreme patterns (test_compare.cu:334-388), 256 x 128
    EM, EN = 256, 128
    g = np.random.default_rng(7)

    def sign(k):
        return np.where(g.integers(0, 2, k) == 0, -1.0, 1.0)

    k = EM * EN
    ext = {
        "all_zeros": (np.zeros(k), 1.0),
        "all_zeros_amax0": (np.zeros(k), 0.0),
        "very_small": (sign(k) * 1e-6 * (1 + g.integers(0, 100, k) / 100.0), 1e-4),
        "very_large": (sign(k) * (500.0 + g.integers(0, 1000, k)), 1000.0),
        "very_large_small_amax": (sign(k) * (500.0 + g.integers(0, 1000, k)), 1.0),
        "sparse_outliers": (np.where(g.integers(0, 256, k) == 0, sign(k) * 100.0, 0.0), 100.0),
        "uniform_one": (np.ones(k), 4.0),
        "uniform_one_tiny_amax": (np.ones(k), 0.001),
    }
    for name, (vals, am) in ext.items():
        Ab = oracle.f32_to_bf16(vals.astype(np.float32))
        cases[f"ext_{name}_rn"] = (EM, EN, Ab, H, am, (12345, 0), 0, 0, 2048)
        cases[f"ext_{name}_sr"] = (EM, EN, Ab, H, am, (12345, 0), 1, 0, 2048)
    inf_mask = g.integers(0, 256, k) == 0
    Ainf = oracle.f32_to_bf16(g.standard_normal(k).astype(np.float32))
    Ainf[inf_mask] = np.where(g.integers(0, 2, inf_mask.sum()) == 0, 0x7F80, 0xFF80)
    cases["ext_contains_inf_rn"] = (EM, EN, Ainf, H, 4.0, (12345, 0), 0, 0, 2048)
    cases["ext_contains_inf_sr"] = (EM, EN, Ainf, H, 4.0, (12345, 0), 1, 0, 2048)
    Anan = oracle.f32_to_bf16(g.standard_normal(k).astype(np.float32))
    Anan[g.integers(0, 256, k) == 0] = 0x7FC0
    cases["ext_contains_nan_rn"] = (EM, EN, Anan, H, 4.0, (12345, 0), 0, 0, 2048)
    cases["ext_contains_nan_sr"] = (EM, EN, Anan, H, 4.0, (12345, 0), 1, 0, 2048)
    return cases


def gen_rht(out_dir: Path) -> None:
    out = {}
    for tag, (m, n, A, B, amax, rng_state, sr, fm, ktile) in rht_cases().items():
        if ktile != 2048:
            # the reference wrappers fix k_tile_size = 2048; k-tile cases are
            # produced through the oracle only after it matched every 2048 case
            continue
        C, S = run_teref(m, n, A, B, amax, rng_state, sr, fm)
        out[tag + "__A"] = A
        out[tag + "__B"] = B
        out[tag + "__amax"] = np.array([amax], np.float32)
        out[tag + "__rng"] = np.array(rng_state, np.uint64)
        out[tag + "__cfg"] = np.array([m, n, sr, fm, ktile])
        out[tag + "__C"] = C
        out[tag + "__SFC"] = S
    np.savez_compressed(out_dir / "teref_rht.npz", **out)


def gen_sr(out_dir: Path) -> None:
    L = ref.gpu()
    rng = np.random.default_rng(123)
    ng = 1 << 14
    f = (rng.uniform(-6.5, 6.5, 4 * ng)).astype(np.float32)
    specials = np.array([0.0, -0.0, 0.25, -0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -6.0,
                         7.0, 1e30, -1e30, np.inf, -np.inf, np.nan, 1e-40, -1e-40, 0.5, 3.0,
                         5.999, 0.2499, 0.2501, 4.0, 2.0, 1.0], np.float32)
    f[:specials.size] = specials
    f[specials.size:2 * specials.size] = -specials
    bf = oracle.f32_to_bf16(rng.uniform(-8, 8, 4 * ng).astype(np.float32))
    bf[:65536 // 16] = np.arange(0, 65536, 16, dtype=np.uint16)   # every 16th bf16 pattern
    rb = rng.integers(0, 2**32, 4 * ng, dtype=np.uint32)
    scale = (0.75, 1.25)
    d_f = torch.from_numpy(f).cuda()
    d_b = torch.from_numpy(bf.view(np.int16)).cuda()
    d_r = torch.from_numpy(rb.view(np.int32)).cuda()
    o16 = torch.zeros(ng, dtype=torch.int16, device="cuda")
    o32 = torch.zeros(ng // 2, dtype=torch.int32, device="cuda")
    res = {"f32": f, "bf16": bf, "rb": rb, "scale": np.array(scale, np.float32)}

    def grab16():
        torch.cuda.synchronize()
        return o16.cpu().numpy().view(np.uint16).copy()

    L.teref_cvt_fp32_to_fp4_4x_sr(d_f.data_ptr(), d_r.data_ptr(), o16.data_ptr(), ng, None)
    res["cvt_fp32_4x"] = grab16()
    L.teref_mul_cvt_fp32_to_fp4_4x_sr(d_f.data_ptr(), scale[0], scale[1], d_r.data_ptr(),
                                      o16.data_ptr(), ng, None)
    res["mul_fp32_4x"] = grab16()
    L.teref_mul_cvt_bf16_to_fp4_4x_sr(d_b.data_ptr(), scale[0], scale[1], d_r.data_ptr(),
                                      o16.data_ptr(), ng, None)
    res["mul_bf16_4x"] = grab16()
    for key, bfs in (("bf16_8x", 0), ("bf16_8x_bfscale", 1)):
        L.teref_mul_cvt_bf16_to_fp4_8x_sr(d_b.data_ptr(), scale[0], bfs, d_r.data_ptr(),
                                          o32.data_ptr(), ng // 2, None)
        torch.cuda.synchronize()
        res[key] = o32.cpu().numpy().view(np.uint32).copy()
    # single-value codecs on specials, neighbours of every E4M3 / E2M1 grid
    # point, and random values
    grid = [oracle.e4m3_decode(c) for c in range(0x7F)] + [0, .5, 1, 1.5, 2, 3, 4, 6]
    near = []
    for v in grid:
        v = np.float32(v)
        near += [v, np.nextafter(v, np.float32(np.inf)), np.nextafter(v, np.float32(-np.inf)),
                 v * np.float32(1.0625), v * np.float32(0.9375)]
    mids = [np.float32(a + b) / np.float32(2) for a, b in zip(sorted(set(map(float, grid))),
                                                              sorted(set(map(float, grid)))[1:])]
    cin = np.concatenate([specials, -specials, np.array(near, np.float32),
                          np.array(mids, np.float32), -np.array(mids, np.float32),
                          rng.uniform(-500, 500, 2048).astype(np.float32),
                          (2.0 ** rng.uniform(-12, 10, 2048)).astype(np.float32)])
    d_c = torch.from_numpy(cin).cuda()
    e2 = torch.zeros(cin.size, dtype=torch.uint8, device="cuda")
    e4 = torch.zeros(cin.size, dtype=torch.uint8, device="cuda")
    L.teref_codecs(d_c.data_ptr(), e2.data_ptr(), e4.data_ptr(), cin.size, None)
    torch.cuda.synchronize()
    res["codec_in"] = cin
    res["codec_e2m1"] = e2.cpu().numpy()
    res["codec_e4m3"] = e4.cpu().numpy()
    np.savez_compressed(out_dir / "teref_sr.npz", **res)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(Path(__file__).resolve().parent))
    a = ap.parse_args()
    out = Path(a.out)
    out.mkdir(parents=True, exist_ok=True)
    assert ref.gpu_available(), "oracle/_ref/libref_gpu.so missing (python oracle/build.py)"
    gen_sr(out)
    gen_rht(out)
    print("wrote", sorted(p.name for p in out.glob("teref_*.npz")))


if __name__ == "__main__":
    main()
