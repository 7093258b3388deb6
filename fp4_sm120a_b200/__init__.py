"""B200-native (sm_100a) NVFP4 quantization: the RHT GEMM + NVFP4 cast
(rht_gemm_ntt_w_sfc), the four FP4 stochastic-rounding conversions and the
scaled FP8 conversions of Harry-Chen/fp4_sm120a, behind a C ABI
(include/nvfp4_b200.h)."""
from ._native import NVFP4Error, library_path, load  # noqa: F401
from .ops import (  # noqa: F401
    amax_bf16,
    amax_bf16_chained,
    cvt_fp32_to_fp4_4x_sr,
    device_error,
    hadamard16,
    mul_cvt_bf16_to_fp4_4x_sr,
    mul_cvt_bf16_to_fp4_8x_sr,
    mul_cvt_fp32_to_fp4_4x_sr,
    mul_cvt_fp8_2x,
    mul_cvt_fp8_4x,
    quantize_rht,
    quantize_rht_fused,
    quantize_rht_fused_sharded_exchange,
    fused_workspace,
    quantize_rowwise_bf16_sr,
    rht_gemm_ntt_w_sfc,
    rht_gemm_ntt_w_sfc_sharded,
    rht_gemm_ntt_w_sfc_sharded_exchange,
    PeerExchange,
    rht_gemm_ttt_wrapper,
)

__version__ = "0.1.0"
