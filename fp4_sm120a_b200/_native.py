"""ctypes binding of libnvfp4_b200.so (the C ABI declared in include/nvfp4_b200.h).

The library is loaded from this package directory.  There is no fallback:
if the library is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_size_t, c_uint32, c_void_p, POINTER
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libnvfp4_b200.so"

# Every symbol declared in include/nvfp4_b200.h with its argument types.
SIGNATURES: dict[str, tuple[list, object]] = {
    "nvfp4_status_string": ([c_int], ctypes.c_char_p),
    "nvfp4_last_cuda_error": ([], c_int),
    "nvfp4_rht_gemm_ntt_w_sfc": ([c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_uint32, c_void_p, c_int, c_int, c_int], c_int),
    "nvfp4_rht_gemm_ntt_w_sfc_sharded": ([c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                          c_void_p, c_void_p, c_uint32, c_void_p, c_int, c_int,
                                          c_int, c_int, c_int], c_int),
    "nvfp4_run_rht": ([c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                       c_uint32, c_void_p], c_int),
    "nvfp4_run_rht_fast": ([c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                            c_void_p, c_uint32, c_void_p], c_int),
    "nvfp4_run_rht_sr": ([c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                          c_void_p, c_uint32, c_void_p], c_int),
    "nvfp4_rht_gemm_ttt": ([c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                            c_void_p, c_uint32, c_void_p, c_int, c_int, c_int], c_int),
    "nvfp4_cvt_fp32_to_fp4_4x_sr": ([c_void_p, c_void_p, c_void_p, c_size_t, c_void_p], c_int),
    "nvfp4_mul_cvt_fp32_to_fp4_4x_sr": ([c_void_p, c_float, c_float, c_void_p, c_void_p,
                                         c_size_t, c_void_p], c_int),
    "nvfp4_mul_cvt_bf16_to_fp4_4x_sr": ([c_void_p, c_float, c_float, c_void_p, c_void_p,
                                         c_size_t, c_void_p], c_int),
    "nvfp4_mul_cvt_bf16_to_fp4_8x_sr": ([c_void_p, c_float, c_int, c_void_p, c_void_p, c_size_t,
                                         c_void_p], c_int),
    "nvfp4_quantize_rowwise_bf16_sr": ([c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_void_p], c_int),
    "nvfp4_amax_bf16": ([c_void_p, c_size_t, c_void_p, c_void_p], c_int),
    "nvfp4_amax_bf16_chained": ([c_void_p, c_size_t, c_void_p, c_void_p, c_void_p], c_int),
    "nvfp4_mul_cvt_fp8_2x": ([c_void_p, c_int, c_void_p, c_size_t, c_void_p, c_int, c_size_t,
                              c_void_p], c_int),
    "nvfp4_mul_cvt_fp8_4x": ([c_void_p, c_int, c_void_p, c_int, c_size_t, c_void_p, c_int,
                              c_size_t, c_void_p], c_int),
    "nvfp4_mul_cvt_fp8_4x_loose": ([c_void_p, c_int, c_void_p, c_size_t, c_void_p, c_int,
                                    c_size_t, c_void_p], c_int),
    "nvfp4_device_error": ([POINTER(c_uint32), c_int], c_int),
    "nvfp4_fused_workspace_bytes": ([], c_size_t),
    "nvfp4_quantize_rht_fused": ([c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_uint32, c_void_p, c_int, c_int, c_int, c_void_p],
                                 c_int),
    "nvfp4_quantize_rht_fused_noalloc": ([c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                          c_void_p, c_void_p, c_uint32, c_void_p, c_int, c_int,
                                          c_int], c_int),
    "nvfp4_quantize_rht_fused_sharded_exchange": ([c_int, c_int, c_void_p, c_void_p, c_void_p,
                                                   c_void_p, c_void_p, c_void_p, c_uint32,
                                                   c_void_p, c_int, c_int, c_int, c_int, c_int,
                                                   c_void_p, c_void_p], c_int),
    "nvfp4_exchange_create": ([c_int, c_int, POINTER(c_void_p), c_void_p], c_int),
    "nvfp4_exchange_connect": ([c_void_p, c_void_p], c_int),
    "nvfp4_exchange_destroy": ([c_void_p], c_int),
    "nvfp4_rht_gemm_ntt_w_sfc_sharded_exchange": ([c_int, c_int, c_void_p, c_void_p, c_void_p,
                                                   c_void_p, c_void_p, c_void_p, c_void_p,
                                                   c_uint32, c_void_p, c_int, c_int, c_int,
                                                   c_int, c_int, c_void_p], c_int),
}

_lib = None


class NVFP4Error(RuntimeError):
    """A C-ABI call returned a non-zero nvfp4_status."""

    def __init__(self, fn: str, status: int, detail: str = ""):
        self.status = status
        super().__init__(f"{fn} failed with status {status}: {detail}")


def library_path() -> Path:
    return LIB_PATH


def load() -> ctypes.CDLL:
    """Load the CUDA library (build it first with fp4_sm120a_b200.build)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH.name} is not built; run `python -m fp4_sm120a_b200.build` "
            "(nvcc, sm_100a). There is no CPU fallback.")
    lib = ctypes.CDLL(os.fspath(LIB_PATH))
    for name, (argtypes, restype) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    _lib = lib
    return lib


def check(fn: str, status: int) -> None:
    if status != 0:
        lib = load()
        detail = lib.nvfp4_status_string(status).decode()
        if status == 4:
            detail += f" (cudaError {lib.nvfp4_last_cuda_error()})"
        raise NVFP4Error(fn, status, detail)


def call(fn: str, *args) -> None:
    lib = load()
    check(fn, getattr(lib, fn)(*args))
