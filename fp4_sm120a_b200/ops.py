"""Host-side mirror of the reference's NVFP4 operator interface.

Functions take CUDA tensors (torch is used only for device memory and
streams) or raw device pointers, keep the reference's argument order and
meaning, and raise NVFP4Error where the reference would abort
(NVTE_CHECK in rht_gemm/te_ref/stubs/common/common.h:17-33).
"""
from __future__ import annotations

from typing import Optional, Union

import torch

from ._native import call

Ptr = Union[int, torch.Tensor, None]


def _ptr(x: Ptr) -> Optional[int]:
    if x is None:
        return None
    if isinstance(x, torch.Tensor):
        if not x.is_cuda:
            raise ValueError("expected a CUDA tensor")
        return x.data_ptr()
    return int(x)


def _stream(stream) -> Optional[int]:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def rht_gemm_ntt_w_sfc(m: int, n: int, A: Ptr, B: Ptr, C: Ptr, SFC: Ptr, global_amax: Ptr,
                       rng_state: Ptr, sm_count: int = 0, stream=None, k_tile_size: int = 2048,
                       *, stochastic_rounding: bool = False, use_fast_math: bool = False) -> None:
    """rht_gemm_ntt_w_sfc<bf16, bf16, e2m1, ue4m3, SR, FM>
    (rht_gemm/te_ref/hadamard_transform_cast_fusion_core.inc:513-644).

    A: m x n column-major bf16 (a row-major n x m tensor), B: 16 x 16 row-major bf16,
    C: m x n/2 bytes (FP4, row-major), SFC: m x n/16 bytes (E4M3), global_amax:
    device float, rng_state: device int64[2] {seed, offset} or None."""
    call("nvfp4_rht_gemm_ntt_w_sfc", m, n, _ptr(A), _ptr(B), _ptr(C), _ptr(SFC),
         _ptr(global_amax), _ptr(rng_state), sm_count, _stream(stream), k_tile_size,
         int(stochastic_rounding), int(use_fast_math))


def rht_gemm_ntt_w_sfc_sharded(m: int, n: int, A: Ptr, B: Ptr, C: Ptr, SFC: Ptr,
                               global_amax: Ptr, rng_state: Ptr, n_offset: int, n_total: int,
                               sm_count: int = 0, stream=None, k_tile_size: int = 2048, *,
                               stochastic_rounding: bool = False,
                               use_fast_math: bool = False) -> None:
    """Columns [n_offset, n_offset + n) of an m x n_total problem (RNG in global
    coordinates, so shard outputs concatenate to the unsharded result)."""
    call("nvfp4_rht_gemm_ntt_w_sfc_sharded", m, n, _ptr(A), _ptr(B), _ptr(C), _ptr(SFC),
         _ptr(global_amax), _ptr(rng_state), sm_count, _stream(stream), k_tile_size,
         int(stochastic_rounding), int(use_fast_math), n_offset, n_total)


class PeerExchange:
    """Handle of the cross-GPU amax exchange over peer memory (one per rank).

    create() allocates this rank's slots and returns its 64-byte CUDA IPC
    handle; connect() takes every rank's handle in rank order."""

    def __init__(self, rank: int, world: int):
        import ctypes
        from ._native import load
        self._lib = load()
        self.rank, self.world = rank, world
        self.ptr = ctypes.c_void_p()
        self.handle = ctypes.create_string_buffer(64)
        call("nvfp4_exchange_create", rank, world, ctypes.byref(self.ptr), self.handle)

    def connect(self, handles: list) -> None:
        import ctypes
        blob = ctypes.create_string_buffer(b"".join(bytes(h) for h in handles), 64 * self.world)
        call("nvfp4_exchange_connect", self.ptr, blob)

    def close(self) -> None:
        if self.ptr:
            call("nvfp4_exchange_destroy", self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def rht_gemm_ntt_w_sfc_sharded_exchange(m: int, n: int, A: Ptr, B: Ptr, C: Ptr, SFC: Ptr,
                                        local_amax: Ptr, global_amax_out: Ptr, rng_state: Ptr,
                                        n_offset: int, n_total: int, exchange: PeerExchange,
                                        sm_count: int = 0, stream=None, k_tile_size: int = 2048,
                                        *, stochastic_rounding: bool = False,
                                        use_fast_math: bool = False) -> None:
    """Sharded cast whose kernel also combines every rank's amax over peer
    memory (no separate collective)."""
    call("nvfp4_rht_gemm_ntt_w_sfc_sharded_exchange", m, n, _ptr(A), _ptr(B), _ptr(C),
         _ptr(SFC), _ptr(local_amax), _ptr(global_amax_out), _ptr(rng_state), sm_count,
         _stream(stream), k_tile_size, int(stochastic_rounding), int(use_fast_math), n_offset,
         n_total, exchange.ptr)


def fused_workspace(device="cuda") -> torch.Tensor:
    """Zeroed workspace for the fused amax + cast kernel (one per concurrent
    stream of fused launches)."""
    from ._native import load
    return torch.zeros(load().nvfp4_fused_workspace_bytes(), dtype=torch.uint8, device=device)


def quantize_rht_fused(m: int, n: int, A: Ptr, B: Ptr, C: Ptr, SFC: Ptr, amax_out: Ptr,
                       rng_state: Ptr, workspace: Ptr, sm_count: int = 0, stream=None,
                       k_tile_size: int = 2048, *, stochastic_rounding: bool = False,
                       use_fast_math: bool = False) -> None:
    """Global amax of A and the RHT + NVFP4 cast in one kernel (results equal
    amax_bf16 followed by rht_gemm_ntt_w_sfc)."""
    call("nvfp4_quantize_rht_fused", m, n, _ptr(A), _ptr(B), _ptr(C), _ptr(SFC), _ptr(amax_out),
         _ptr(rng_state), sm_count, _stream(stream), k_tile_size, int(stochastic_rounding),
         int(use_fast_math), _ptr(workspace))


def quantize_rht_fused_sharded_exchange(m: int, n: int, A: Ptr, B: Ptr, C: Ptr, SFC: Ptr,
                                        amax_out: Ptr, rng_state: Ptr, n_offset: int,
                                        n_total: int, exchange: "PeerExchange", workspace: Ptr,
                                        sm_count: int = 0, stream=None, k_tile_size: int = 2048,
                                        *, stochastic_rounding: bool = False,
                                        use_fast_math: bool = False) -> None:
    call("nvfp4_quantize_rht_fused_sharded_exchange", m, n, _ptr(A), _ptr(B), _ptr(C),
         _ptr(SFC), _ptr(amax_out), _ptr(rng_state), sm_count, _stream(stream), k_tile_size,
         int(stochastic_rounding), int(use_fast_math), n_offset, n_total, exchange.ptr,
         _ptr(workspace))


def rht_gemm_ttt_wrapper(m: int, n: int, A: Ptr, B: Ptr, C: Ptr, SFC: Ptr, global_amax: Ptr,
                         rng_state: Ptr, sm_count: int = 0, stream=None, k_tile_size: int = 1024,
                         *, stochastic_rounding: bool = False,
                         use_fast_math: bool = False) -> None:
    """rht_gemm_ttt_wrapper (core.inc:648-678): m and n swapped, k_tile 1024."""
    call("nvfp4_rht_gemm_ttt", m, n, _ptr(A), _ptr(B), _ptr(C), _ptr(SFC), _ptr(global_amax),
         _ptr(rng_state), sm_count, _stream(stream), k_tile_size, int(stochastic_rounding),
         int(use_fast_math))


def cvt_fp32_to_fp4_4x_sr(inp: Ptr, rbits: Ptr, out: Ptr, ngroups: int, stream=None) -> None:
    """Batch cvt_fp32_to_fp4_4x_with_stochastic_rounding: 4 floats + 1 word -> 16 bits."""
    call("nvfp4_cvt_fp32_to_fp4_4x_sr", _ptr(inp), _ptr(rbits), _ptr(out), ngroups,
         _stream(stream))


def mul_cvt_fp32_to_fp4_4x_sr(inp: Ptr, scale: tuple[float, float], rbits: Ptr, out: Ptr,
                              ngroups: int, stream=None) -> None:
    call("nvfp4_mul_cvt_fp32_to_fp4_4x_sr", _ptr(inp), float(scale[0]), float(scale[1]),
         _ptr(rbits), _ptr(out), ngroups, _stream(stream))


def mul_cvt_bf16_to_fp4_4x_sr(inp: Ptr, scale: tuple[float, float], rbits: Ptr, out: Ptr,
                              ngroups: int, stream=None) -> None:
    call("nvfp4_mul_cvt_bf16_to_fp4_4x_sr", _ptr(inp), float(scale[0]), float(scale[1]),
         _ptr(rbits), _ptr(out), ngroups, _stream(stream))


def mul_cvt_bf16_to_fp4_8x_sr(inp: Ptr, scale: float, rbits: Ptr, out: Ptr, ngroups: int,
                              scale_is_bf16: bool = False, stream=None) -> None:
    call("nvfp4_mul_cvt_bf16_to_fp4_8x_sr", _ptr(inp), float(scale), int(scale_is_bf16),
         _ptr(rbits), _ptr(out), ngroups, _stream(stream))


def quantize_rowwise_bf16_sr(rows: int, cols: int, X: Ptr, global_amax: Ptr, rbits: Ptr, C: Ptr,
                             SFC: Ptr, stream=None) -> None:
    call("nvfp4_quantize_rowwise_bf16_sr", rows, cols, _ptr(X), _ptr(global_amax), _ptr(rbits),
         _ptr(C), _ptr(SFC), _stream(stream))


def amax_bf16(x: Ptr, n: int, out: Ptr, stream=None) -> None:
    call("nvfp4_amax_bf16", _ptr(x), n, _ptr(out), _stream(stream))


def amax_bf16_chained(x: Ptr, n: int, out: Ptr, clear: Ptr, stream=None) -> None:
    """amax into *out (which must hold +0) and clear *clear for the next step,
    without a memset, overlapping the previous kernel's tail (see
    nvfp4_amax_bf16_chained)."""
    call("nvfp4_amax_bf16_chained", _ptr(x), n, _ptr(out), _ptr(clear), _stream(stream))


DTYPE_CODES = {"f32": 0, "bf16": 1, "f16": 2}
FP8_FORMATS = {"e4m3": 0, "e5m2": 1}


def _dtype_code(dtype) -> int:
    if isinstance(dtype, str):
        return DTYPE_CODES[dtype]
    return {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[dtype]


def mul_cvt_fp8_2x(inp: Ptr, in_dtype, scale: Ptr, scale_stride: int, out: Ptr, fmt: str,
                   ngroups: int, stream=None) -> None:
    """mul_cvt_2x over `ngroups` element pairs (te_ref ptx.cuh:923-1062)."""
    call("nvfp4_mul_cvt_fp8_2x", _ptr(inp), _dtype_code(in_dtype), _ptr(scale), scale_stride,
         _ptr(out), FP8_FORMATS[fmt], ngroups, _stream(stream))


def mul_cvt_fp8_4x(inp: Ptr, in_dtype, scale: Ptr, scale_width: int, scale_stride: int,
                   out: Ptr, fmt: str, ngroups: int, loose: bool = False, stream=None) -> None:
    """mul_cvt_4x over `ngroups` groups of 4 (ptx.cuh:1172-1693); `loose` is the
    _LOOSE_PRECISION build (floatx2 scale only)."""
    if loose:
        if scale_width != 2:
            raise ValueError("the _LOOSE_PRECISION form takes a floatx2 scale")
        call("nvfp4_mul_cvt_fp8_4x_loose", _ptr(inp), _dtype_code(in_dtype), _ptr(scale),
             scale_stride, _ptr(out), FP8_FORMATS[fmt], ngroups, _stream(stream))
    else:
        call("nvfp4_mul_cvt_fp8_4x", _ptr(inp), _dtype_code(in_dtype), _ptr(scale), scale_width,
             scale_stride, _ptr(out), FP8_FORMATS[fmt], ngroups, _stream(stream))


def device_error(clear: bool = True) -> int:
    import ctypes
    code = ctypes.c_uint32(0)
    call("nvfp4_device_error", ctypes.byref(code), int(clear))
    return code.value


# ----------------------------------------------------------------------------
# Tensor-level convenience wrappers (allocate outputs with torch)
# ----------------------------------------------------------------------------

def hadamard16(signs: Optional[torch.Tensor] = None, device="cuda") -> torch.Tensor:
    """B = H16 * diag(signs) / 4 as 16 x 16 row-major bf16 (entries are +-0.25,
    exact in bf16); signs=None gives the reference tests' plain H16 / 4
    (rht_gemm/test_compare.cu:95-102)."""
    idx = torch.arange(16)
    par = torch.zeros(16, 16, dtype=torch.int64)
    x = idx[:, None] & idx[None, :]
    for b in range(4):
        par += (x >> b) & 1
    h = torch.where(par % 2 == 0, 1.0, -1.0) * 0.25
    if signs is not None:
        h = h * signs.to(h.dtype).cpu()[None, :]
    return h.to(torch.bfloat16).to(device)


def quantize_rht(x: torch.Tensor, B: torch.Tensor, global_amax: torch.Tensor,
                 rng_state: Optional[torch.Tensor] = None, *, stochastic_rounding: bool = True,
                 use_fast_math: bool = False, k_tile_size: int = 2048, stream=None):
    """Transposed RHT + NVFP4 cast of a row-major (rows x cols) bf16 activation:
    the API sees m = cols, n = rows.  Returns (C [cols, rows/2] uint8,
    SFC [cols, rows/16] uint8)."""
    rows, cols = x.shape
    C = torch.empty((cols, rows // 2), dtype=torch.uint8, device=x.device)
    S = torch.empty((cols, rows // 16), dtype=torch.uint8, device=x.device)
    rht_gemm_ntt_w_sfc(cols, rows, x, B, C, S, global_amax, rng_state, 0, stream, k_tile_size,
                       stochastic_rounding=stochastic_rounding, use_fast_math=use_fast_math)
    return C, S
