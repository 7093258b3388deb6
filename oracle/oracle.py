"""numpy/ctypes front end of the C restatement (oracle/nvfp4_oracle.c).

TEST INFRASTRUCTURE.  Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline leg use this module, always as the checker.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_size_t, c_uint8, c_uint32, c_uint64, c_void_p
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        from . import build as _b
        path = _b.build_oracle()     # no-op unless the C source is newer
        L = ctypes.CDLL(str(path))
        sig = {
            "orc_bf16_to_f32": ([ctypes.c_uint16], c_float),
            "orc_f32_to_bf16": ([c_float], ctypes.c_uint16),
            "orc_philox_te": ([c_uint64, c_uint64, c_uint64, c_uint32, c_void_p], None),
            "orc_f32_to_e4m3": ([c_float], c_uint8),
            "orc_e4m3_to_f32": ([c_uint8], c_float),
            "orc_f32_to_e2m1_rn": ([c_float], c_uint8),
            "orc_f32_to_e2m1_rs": ([c_float, c_uint32], c_uint8),
            "orc_f32_to_e2m1_sr_polyfill": ([c_float, c_uint32], c_uint8),
            "orc_rs_random16": ([c_uint32, c_int], c_uint32),
            "orc_cvt_x4_polyfill": ([c_float, c_float, c_float, c_float, c_uint32],
                                    ctypes.c_uint16),
            "orc_e2m1_to_f32": ([c_uint8], c_float),
            "orc_set_e2m1_nan_code": ([c_uint8], None),
            "orc_get_e2m1_nan_code": ([], c_uint8),
            "orc_cvt_fp32_to_fp4_4x_sr": ([c_void_p, c_void_p, c_void_p, c_size_t], None),
            "orc_mul_cvt_fp32_to_fp4_4x_sr": ([c_void_p, c_float, c_float, c_void_p, c_void_p,
                                               c_size_t], None),
            "orc_mul_cvt_bf16_to_fp4_4x_sr": ([c_void_p, c_float, c_float, c_void_p, c_void_p,
                                               c_size_t], None),
            "orc_mul_cvt_bf16_to_fp4_8x_sr": ([c_void_p, c_float, c_int, c_void_p, c_void_p,
                                               c_size_t], None),
            "orc_f16_to_f32": ([ctypes.c_uint16], c_float),
            "orc_f32_to_e5m2": ([c_float], c_uint8),
            "orc_e5m2_to_f32": ([c_uint8], c_float),
            "orc_set_e5m2_nan_code": ([c_uint8], None),
            "orc_mul_cvt_fp8": ([c_void_p, c_int, c_void_p, c_size_t, c_int, c_int, c_int,
                                 c_void_p, c_size_t], None),
            "orc_global_encode_scale": ([c_float], c_float),
            "orc_amax_bf16": ([c_void_p, c_size_t], c_float),
            "orc_rht_gemm_ntt_w_sfc": ([c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_float, c_int, c_uint64, c_uint64, c_int, c_int, c_int,
                                        c_int, c_int], c_int),
            "orc_quantize_rowwise_8x_sr": ([c_int, c_int, c_void_p, c_float, c_void_p, c_void_p,
                                            c_void_p], c_int),
        }
        for name, (a, r) in sig.items():
            f = getattr(L, name)
            f.argtypes = a
            f.restype = r
        _LIB = L
    return _LIB


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ---------------------------------------------------------------- conversions

def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


def philox(seed: int, subseq: int, offset: int, skip: int = 0) -> np.ndarray:
    out = np.zeros(4, np.uint32)
    lib().orc_philox_te(seed, subseq, offset, skip, _p(out))
    return out


def e4m3(x: float) -> int:
    return int(lib().orc_f32_to_e4m3(float(x)))


def e4m3_decode(b: int) -> float:
    return float(lib().orc_e4m3_to_f32(b))


def e2m1_rn(x: float) -> int:
    return int(lib().orc_f32_to_e2m1_rn(float(x)))


def e2m1_rs(x: float, r16: int) -> int:
    """cvt.rs E2M1 of one value with its 16-bit random number (B200 rule)."""
    return int(lib().orc_f32_to_e2m1_rs(float(x), r16))


def rs_random16(word: int, k: int) -> int:
    """The 16-bit random number cvt.rs.satfinite.e2m1x4.f32 uses for nibble k."""
    return int(lib().orc_rs_random16(word, k))


def e2m1_sr_polyfill(x: float, rand_byte: int) -> int:
    """The reference SM120 polyfill's noise model (sr.sm120.cuh:27-106)."""
    return int(lib().orc_f32_to_e2m1_sr_polyfill(float(x), rand_byte))


def cvt_x4_polyfill(x4, word: int) -> int:
    return int(lib().orc_cvt_x4_polyfill(*(float(v) for v in x4), word))


def e5m2(x: float) -> int:
    return int(lib().orc_f32_to_e5m2(float(x)))


def e5m2_decode(b: int) -> float:
    return float(lib().orc_e5m2_to_f32(b))


_DT = {"f32": (0, np.float32), "bf16": (1, np.uint16), "f16": (2, np.uint16)}


def mul_cvt_fp8(x: np.ndarray, in_dtype: str, scale: np.ndarray, scale_stride: int, width: int,
                scale_width: int, fmt: str) -> np.ndarray:
    """mul_cvt_2x / mul_cvt_4x (te_ref ptx.cuh:923-1693) over a batch; x holds
    f32 values or bf16 / f16 bit patterns (uint16), width * ngroups of them."""
    code, dt = _DT[in_dtype]
    x = np.ascontiguousarray(x, dt)
    scale = np.ascontiguousarray(scale, np.float32)
    ngroups = x.size // width
    out = np.zeros(ngroups * width, np.uint8)
    lib().orc_mul_cvt_fp8(_p(x), code, _p(scale), scale_stride, width, scale_width,
                          {"e4m3": 0, "e5m2": 1}[fmt], _p(out), ngroups)
    return out


def e2m1_decode(nib) -> np.ndarray:
    t = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], np.float32)
    nib = np.asarray(nib, np.uint8)
    v = t[nib & 7]
    return np.where(nib & 8, -v, v).astype(np.float32)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    """Bytes -> nibbles, low nibble first (element 2k in the low nibble of byte k)."""
    p = np.asarray(packed, np.uint8).reshape(-1)
    out = np.empty(p.size * 2, np.uint8)
    out[0::2] = p & 0xF
    out[1::2] = p >> 4
    return out


# ---------------------------------------------------------------- batch SR forms

def cvt_fp32_to_fp4_4x_sr(x: np.ndarray, rbits: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    rbits = np.ascontiguousarray(rbits, np.uint32)
    n = x.size // 4
    out = np.zeros(n, np.uint16)
    lib().orc_cvt_fp32_to_fp4_4x_sr(_p(x), _p(rbits), _p(out), n)
    return out


def mul_cvt_fp32_to_fp4_4x_sr(x, scale, rbits) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    rbits = np.ascontiguousarray(rbits, np.uint32)
    n = x.size // 4
    out = np.zeros(n, np.uint16)
    lib().orc_mul_cvt_fp32_to_fp4_4x_sr(_p(x), scale[0], scale[1], _p(rbits), _p(out), n)
    return out


def mul_cvt_bf16_to_fp4_4x_sr(xb, scale, rbits) -> np.ndarray:
    xb = np.ascontiguousarray(xb, np.uint16).reshape(-1)
    rbits = np.ascontiguousarray(rbits, np.uint32)
    n = xb.size // 4
    out = np.zeros(n, np.uint16)
    lib().orc_mul_cvt_bf16_to_fp4_4x_sr(_p(xb), scale[0], scale[1], _p(rbits), _p(out), n)
    return out


def mul_cvt_bf16_to_fp4_8x_sr(xb, scale: float, rbits, scale_is_bf16: bool = False):
    xb = np.ascontiguousarray(xb, np.uint16).reshape(-1)
    rbits = np.ascontiguousarray(rbits, np.uint32)
    n = xb.size // 8
    out = np.zeros(n, np.uint32)
    if scale_is_bf16:
        scale = float(bf16_to_f32(f32_to_bf16(np.array([scale], np.float32)))[0])
    lib().orc_mul_cvt_bf16_to_fp4_8x_sr(_p(xb), scale, int(scale_is_bf16), _p(rbits), _p(out), n)
    return out


# ---------------------------------------------------------------- tensor forms

def amax_bf16(xb: np.ndarray) -> float:
    xb = np.ascontiguousarray(xb, np.uint16).reshape(-1)
    return float(lib().orc_amax_bf16(_p(xb), xb.size))


def rht_gemm_ntt_w_sfc(m: int, n: int, A_colmajor_bf16: np.ndarray, B_bf16: np.ndarray,
                       global_amax: float, rng_state=None, k_tile_size: int = 2048,
                       sr: bool = False, fast_math: bool = False, n_offset: int = 0,
                       n_total: int = 0):
    """Returns (C [m, n/2] uint8, SFC [m, n/16] uint8).  A is passed as the flat
    column-major buffer (A[i + m*j]) of bf16 bit patterns."""
    A = np.ascontiguousarray(A_colmajor_bf16, np.uint16).reshape(-1)
    B = np.ascontiguousarray(B_bf16, np.uint16).reshape(-1)
    assert A.size == m * n and B.size == 256
    C = np.zeros((m, n // 2), np.uint8)
    S = np.zeros((m, n // 16), np.uint8)
    has = rng_state is not None
    seed, off = (int(rng_state[0]), int(rng_state[1])) if has else (0, 0)
    rc = lib().orc_rht_gemm_ntt_w_sfc(m, n, _p(A), _p(B), _p(C), _p(S), float(global_amax),
                                      int(has), seed, off, k_tile_size, int(sr), int(fast_math),
                                      n_offset, n_total)
    if rc != 0:
        raise ValueError(f"oracle rejected shape m={m} n={n} k_tile={k_tile_size}")
    return C, S


def quantize_rowwise_8x_sr(X_bf16: np.ndarray, global_amax: float, rbits: np.ndarray):
    rows, cols = X_bf16.shape
    X = np.ascontiguousarray(X_bf16, np.uint16)
    rb = np.ascontiguousarray(rbits, np.uint32)
    C = np.zeros((rows, cols // 2), np.uint8)
    S = np.zeros((rows, cols // 16), np.uint8)
    rc = lib().orc_quantize_rowwise_8x_sr(rows, cols, _p(X), float(global_amax), _p(rb), _p(C),
                                          _p(S))
    if rc != 0:
        raise ValueError("bad shape")
    return C, S
