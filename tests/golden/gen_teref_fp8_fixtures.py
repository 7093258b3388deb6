"""Generate tests/golden/teref_fp8.npz by running the reference's own scaled
FP8 conversions (mul_cvt_2x / mul_cvt_4x of
rht_gemm/te_ref/stubs/common/util/ptx.cuh:923-1693, compiled from the
reference tree into oracle/_ref/libref_fp8.so by oracle/build.py) on a B200.

Inputs: every fourth bf16 and f16 bit pattern plus all their NaN / Inf /
subnormal / zero patterns, and f32 values on, between and beside the E4M3 and
E5M2 grids; scales from a fixed list (one floatx2 / floatx4 per group, cycled).
Outputs for every (input type, form, format), and the _LOOSE_PRECISION build's
floatx2 4x form.

Run on a GPU box from the repository root:
    python tests/golden/gen_teref_fp8_fixtures.py --out <dir>
then copy teref_fp8.npz into tests/golden/.
"""
import argparse
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import oracle, ref  # noqa: E402

SCALES = np.array([1.0, 0.75, -2.0, 0.5, 3.0, -0.0, 2.0**-100, 1.25, 448.0, 1.0 / 448.0,
                   np.inf, 0.0, 65536.0, -1.0, 1e-3, 7.0], np.float32)
FORMS = [(2, 2), (4, 2), (4, 4)]


def inputs():
    pats = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    out = {}
    for dt, expo_mask, mant_mask in (("bf16", 0x7F80, 0x007F), ("f16", 0x7C00, 0x03FF)):
        e = pats & expo_mask
        special = (e == expo_mask) | (e == 0)
        keep = special | (np.arange(65536) % 4 == 0)
        v = pats[keep]
        out[dt] = v[: v.size - v.size % 4]
    grid = []
    for dec, top in ((oracle.e4m3_decode, 0x7E), (oracle.e5m2_decode, 0x7B)):
        g = np.array([dec(c) for c in range(top + 1)], np.float64)
        grid += [g, (g[:-1] + g[1:]) / 2]
    g = np.concatenate(grid).astype(np.float32)
    g = np.concatenate([g, np.nextafter(g, np.float32(np.inf)), np.nextafter(g, np.float32(-np.inf))])
    g = np.concatenate([g, -g, np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-45, 3e38,
                                         -3e38], np.float32)])
    out["f32"] = g[: g.size - g.size % 4]
    return out


def scales_for(ngroups, sw):
    return np.resize(SCALES, ngroups * sw).astype(np.float32)


def run(L, fn, x, dt, width, sw, fmt):
    code = {"f32": 0, "bf16": 1, "f16": 2}[dt]
    f = {"e4m3": 0, "e5m2": 1}[fmt]
    ng = x.size // width
    s = scales_for(ng, sw)
    dx = torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).cuda()
    ds = torch.from_numpy(s).cuda()
    o = torch.zeros(ng * width, dtype=torch.uint8, device="cuda")
    if fn == "2x":
        rc = L.teref_mul_cvt_fp8_2x(dx.data_ptr(), code, ds.data_ptr(), sw, o.data_ptr(), f, ng,
                                    None)
    elif fn == "4x":
        rc = L.teref_mul_cvt_fp8_4x(dx.data_ptr(), code, ds.data_ptr(), sw, sw, o.data_ptr(), f,
                                    ng, None)
    else:
        rc = L.teref_mul_cvt_fp8_4x_loose(dx.data_ptr(), code, ds.data_ptr(), sw, o.data_ptr(),
                                          f, ng, None)
    torch.cuda.synchronize()
    assert rc == 0, rc
    return o.cpu().numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=".")
    a = ap.parse_args()
    L = ref.fp8()
    res = {"scales": SCALES}
    for dt, x in inputs().items():
        res[f"in_{dt}"] = x
        for fmt in ("e4m3", "e5m2"):
            for width, sw in FORMS:
                fn = "2x" if width == 2 else "4x"
                res[f"{dt}_{fn}_s{sw}_{fmt}"] = run(L, fn, x, dt, width, sw, fmt)
            res[f"{dt}_4x_loose_{fmt}"] = run(L, "loose", x, dt, 4, 2, fmt)
    out = Path(a.out) / "teref_fp8.npz"
    np.savez_compressed(out, **res)
    print(out, sum(v.nbytes for v in res.values()))


if __name__ == "__main__":
    main()
