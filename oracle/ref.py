"""ctypes front end of the reference's own code compiled in place
(oracle/_ref/libref_cpu.so, oracle/_ref/libref_gpu.so).  TEST / BASELINE
INFRASTRUCTURE: checker and timed CPU baseline only."""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_size_t, c_uint32, c_void_p
from pathlib import Path

_HERE = Path(__file__).resolve().parent
REF_DIR = _HERE / "_ref"
_cpu = None
_gpu = None


def cpu_available() -> bool:
    return (REF_DIR / "libref_cpu.so").exists()


def gpu_available() -> bool:
    return (REF_DIR / "libref_gpu.so").exists()


def cpu() -> ctypes.CDLL:
    global _cpu
    if _cpu is None:
        L = ctypes.CDLL(str(REF_DIR / "libref_cpu.so"))
        L.ref_sw_cvt_fp32_to_fp4_4x_sr.argtypes = [c_void_p, c_void_p, c_void_p, c_size_t, c_int]
        L.ref_sw_mul_cvt_fp32_to_fp4_4x_sr.argtypes = [c_void_p, c_float, c_float, c_void_p,
                                                       c_void_p, c_size_t, c_int]
        L.ref_sw_mul_cvt_bf16_to_fp4_4x_sr.argtypes = [c_void_p, c_float, c_float, c_void_p,
                                                       c_void_p, c_size_t, c_int]
        L.ref_sw_mul_cvt_bf16_to_fp4_8x_sr.argtypes = [c_void_p, c_float, c_void_p, c_void_p,
                                                       c_size_t, c_int]
        L.ref_naive_rht.argtypes = [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_float,
                                    c_int, c_int, c_int]
        for f in ("ref_sw_cvt_fp32_to_fp4_4x_sr", "ref_sw_mul_cvt_fp32_to_fp4_4x_sr",
                  "ref_sw_mul_cvt_bf16_to_fp4_4x_sr", "ref_sw_mul_cvt_bf16_to_fp4_8x_sr",
                  "ref_naive_rht"):
            getattr(L, f).restype = None
        _cpu = L
    return _cpu


def gpu() -> ctypes.CDLL:
    global _gpu
    if _gpu is None:
        L = ctypes.CDLL(str(REF_DIR / "libref_gpu.so"))
        L.teref_rht_gemm_ntt_w_sfc.argtypes = [c_int, c_int, c_void_p, c_void_p, c_void_p,
                                               c_void_p, c_void_p, c_void_p, c_uint32, c_void_p,
                                               c_int, c_int]
        L.teref_mul_cvt_bf16_to_fp4_4x_sr.argtypes = [c_void_p, c_float, c_float, c_void_p,
                                                      c_void_p, c_size_t, c_void_p]
        L.teref_mul_cvt_fp32_to_fp4_4x_sr.argtypes = [c_void_p, c_float, c_float, c_void_p,
                                                      c_void_p, c_size_t, c_void_p]
        L.teref_mul_cvt_bf16_to_fp4_8x_sr.argtypes = [c_void_p, c_float, c_int, c_void_p,
                                                      c_void_p, c_size_t, c_void_p]
        L.teref_cvt_fp32_to_fp4_4x_sr.argtypes = [c_void_p, c_void_p, c_void_p, c_size_t,
                                                  c_void_p]
        L.teref_codecs.argtypes = [c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]
        for f in ("teref_rht_gemm_ntt_w_sfc", "teref_mul_cvt_bf16_to_fp4_4x_sr",
                  "teref_mul_cvt_fp32_to_fp4_4x_sr", "teref_mul_cvt_bf16_to_fp4_8x_sr",
                  "teref_cvt_fp32_to_fp4_4x_sr", "teref_codecs"):
            getattr(L, f).restype = c_int
        _gpu = L
    return _gpu


_fp8 = None


def fp8_available() -> bool:
    return (REF_DIR / "libref_fp8.so").exists()


def fp8() -> ctypes.CDLL:
    """The reference's own mul_cvt_2x / mul_cvt_4x (te_ref ptx.cuh:923-1693),
    default and _LOOSE_PRECISION builds, one group per thread."""
    global _fp8
    if _fp8 is None:
        L = ctypes.CDLL(str(REF_DIR / "libref_fp8.so"))
        L.teref_mul_cvt_fp8_2x.argtypes = [c_void_p, c_int, c_void_p, c_size_t, c_void_p, c_int,
                                           c_size_t, c_void_p]
        L.teref_mul_cvt_fp8_4x.argtypes = [c_void_p, c_int, c_void_p, c_int, c_size_t, c_void_p,
                                           c_int, c_size_t, c_void_p]
        L.teref_mul_cvt_fp8_4x_loose.argtypes = [c_void_p, c_int, c_void_p, c_size_t, c_void_p,
                                                 c_int, c_size_t, c_void_p]
        for f in ("teref_mul_cvt_fp8_2x", "teref_mul_cvt_fp8_4x", "teref_mul_cvt_fp8_4x_loose"):
            getattr(L, f).restype = c_int
        _fp8 = L
    return _fp8
