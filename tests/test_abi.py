"""CPU tests of the C ABI: the library loads, exports every symbol that
include/nvfp4_b200.h declares, and rejects bad arguments with the documented
status codes before touching a GPU (argument checks run first)."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    text = (ROOT / "include" / "nvfp4_b200.h").read_text()
    return re.findall(r"NVFP4_API\s+[\w\s\*]+?\b(nvfp4_\w+)\s*\(", text)


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "nvfp4_rht_gemm_ntt_w_sfc" in syms and "nvfp4_cvt_fp32_to_fp4_4x_sr" in syms
    assert len(syms) == len(set(syms))


def test_library_exports_every_declared_symbol(nvlib):
    lib = nvlib.load()
    from fp4_sm120a_b200._native import SIGNATURES
    for s in declared_symbols():
        assert hasattr(lib, s), s
        assert s in SIGNATURES, f"{s} has no ctypes signature"


def test_status_strings(nvlib):
    lib = nvlib.load()
    assert lib.nvfp4_status_string(0) == b"ok"
    assert b"shape" in lib.nvfp4_status_string(1)
    assert lib.nvfp4_status_string(99) == b"unknown status"


@pytest.mark.parametrize("m,n,k_tile", [(100, 64, 2048), (128, 96, 2048), (-128, 64, 2048),
                                        (128, 64, 32)])
def test_rht_rejects_bad_shapes(nvlib, m, n, k_tile):
    lib = nvlib.load()
    rc = lib.nvfp4_rht_gemm_ntt_w_sfc(m, n, 16, 16, 16, 16, 16, None, 0, None, k_tile, 0, 0)
    assert rc == 1


def test_rht_zero_size_is_noop(nvlib):
    lib = nvlib.load()
    assert lib.nvfp4_rht_gemm_ntt_w_sfc(0, 64, None, None, None, None, None, None, 0, None,
                                        2048, 0, 0) == 0
    assert lib.nvfp4_rht_gemm_ntt_w_sfc(128, 0, None, None, None, None, None, None, 0, None,
                                        2048, 1, 0) == 0


def test_rht_rejects_null_and_misaligned(nvlib):
    lib = nvlib.load()
    assert lib.nvfp4_rht_gemm_ntt_w_sfc(128, 64, None, 16, 16, 16, 16, None, 0, None, 2048, 0,
                                        0) == 2
    assert lib.nvfp4_rht_gemm_ntt_w_sfc(128, 64, 0x1008, 16, 16, 16, 16, None, 0, None, 2048,
                                        0, 0) == 3


def test_sharded_offset_must_align_to_k_tile_chunks(nvlib):
    lib = nvlib.load()
    # n_offset = 1024 is not a multiple of the 2048-column chunk
    assert lib.nvfp4_rht_gemm_ntt_w_sfc_sharded(128, 1024, 16, 16, 16, 16, 16, None, 0, None,
                                                2048, 1, 0, 1024, 4096) == 1
    # shard past the end of the problem
    assert lib.nvfp4_rht_gemm_ntt_w_sfc_sharded(128, 2048, 16, 16, 16, 16, 16, None, 0, None,
                                                2048, 1, 0, 4096, 4096) == 1


def test_batch_entry_points_validate_arguments(nvlib):
    lib = nvlib.load()
    assert lib.nvfp4_cvt_fp32_to_fp4_4x_sr(None, None, None, 0, None) == 0
    assert lib.nvfp4_cvt_fp32_to_fp4_4x_sr(None, 16, 16, 4, None) == 2
    assert lib.nvfp4_quantize_rowwise_bf16_sr(4, 24, 16, 16, 16, 16, 16, None) == 1
    assert lib.nvfp4_quantize_rowwise_bf16_sr(4, 32, 0x1008, 16, 16, 16, 16, None) == 3
    assert lib.nvfp4_amax_bf16(16, 8, None, None) == 2


def test_product_path_has_no_oracle_dependency():
    """The shipped package never imports the oracle (checker only)."""
    pkg = ROOT / "fp4_sm120a_b200"
    for p in pkg.rglob("*.py"):
        t = p.read_text()
        assert "oracle" not in t.replace("no oracle", ""), p


def test_exchange_and_fused_entry_points_validate_arguments(nvlib):
    """Argument checks that run before any CUDA call (no GPU needed)."""
    import ctypes
    lib = nvlib.load()
    ex = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    # world must be 2..64 and 0 <= rank < world
    assert lib.nvfp4_exchange_create(0, 1, ctypes.byref(ex), handle) == 2
    assert lib.nvfp4_exchange_create(2, 2, ctypes.byref(ex), handle) == 2
    assert lib.nvfp4_exchange_create(0, 65, ctypes.byref(ex), handle) == 2
    assert lib.nvfp4_exchange_create(0, 2, None, handle) == 2
    # the exchange cast needs an exchange handle
    assert lib.nvfp4_rht_gemm_ntt_w_sfc_sharded_exchange(128, 64, 16, 16, 16, 16, 16, None,
                                                         None, 0, None, 2048, 1, 0, 0, 64,
                                                         None) == 2
    # the fused cast needs a workspace, aligned to 4 bytes
    assert lib.nvfp4_quantize_rht_fused(128, 64, 16, 16, 16, 16, None, None, 0, None, 2048, 1,
                                        0, None) == 2
    assert lib.nvfp4_quantize_rht_fused(128, 64, 16, 16, 16, 16, None, None, 0, None, 2048, 1,
                                        0, 0x1002) == 3
    # bad shapes are refused before anything is launched
    assert lib.nvfp4_quantize_rht_fused_noalloc(100, 64, 16, 16, 16, 16, None, None, 0, None,
                                                2048, 1, 0) == 1


def test_ttt_wrapper_swaps_m_and_n(nvlib):
    """rht_gemm_ttt_wrapper (core.inc:648-678) calls the ntt form with m and n
    swapped: a shape valid only after the swap passes the checks (and is a
    no-op when one side is zero)."""
    lib = nvlib.load()
    # ntt(m=64, n=128) is invalid (m % 128); the ttt form swaps it to ntt(128, 64)
    assert lib.nvfp4_rht_gemm_ntt_w_sfc(64, 128, None, 16, 16, 16, 16, None, 0, None, 2048, 0,
                                        0) == 1
    assert lib.nvfp4_rht_gemm_ttt(64, 128, None, 16, 16, 16, 16, None, 0, None, 2048, 0,
                                  0) == 2     # passes the shape check, then refuses NULL A
    assert lib.nvfp4_rht_gemm_ttt(0, 128, None, None, None, None, None, None, 0, None, 2048, 0,
                                  0) == 0


def test_noalloc_rejects_more_units_than_its_scratch_counts(nvlib):
    """nvfp4_quantize_rht_fused_noalloc's built-in scratch counts work units
    (128 x 256 tiles) in 32 bits: a problem with more than 2^31 - 1 of them is
    refused with NVFP4_ERR_SCRATCH_CAPACITY by the argument checks, before
    any CUDA call (so this runs without a GPU; the pointers are placeholders
    that are never used)."""
    from fp4_sm120a_b200 import _native
    lib = _native.load()
    m, n = 2**31 - 128, 2**31 - 64          # 16777215 x 8388608 units
    rc = lib.nvfp4_quantize_rht_fused_noalloc(m, n, 256, 256, 256, 256, None, None, 0, None,
                                              2048, 1, 0)
    assert rc == 7, lib.nvfp4_status_string(rc)
    assert b"scratch" in lib.nvfp4_status_string(7)


def test_amax_chained_validates_arguments(nvlib):
    """The chained amax needs two distinct words (the one it accumulates into
    and the one it clears for the next step) and refuses anything else before
    any CUDA call."""
    from fp4_sm120a_b200 import _native
    lib = _native.load()
    assert lib.nvfp4_amax_bf16_chained(16, 8, 64, 64, None) == 2     # out == clear
    assert lib.nvfp4_amax_bf16_chained(16, 8, None, 64, None) == 2
    assert lib.nvfp4_amax_bf16_chained(16, 8, 64, None, None) == 2
    assert lib.nvfp4_amax_bf16_chained(None, 8, 64, 128, None) == 2   # no input
    assert lib.nvfp4_amax_bf16_chained(18, 8, 64, 128, None) == 3     # misaligned input
