"""The drop-in headers compile standalone, the way a reference caller would
use them (no GPU needed):
- include/nvfp4_b200.h as plain C (gcc), and a C program linked against the
  library that makes a no-op call;
- include/nvfp4_b200.hpp's launcher templates instantiated from C++ (g++);
- include/nvfp4_sr.cuh and include/nvfp4_fp8.cuh from device code (nvcc,
  sm_100a), the FP8 header both as is and with _LOOSE_PRECISION, called the
  way TE code calls transformer_engine::ptx."""
import os
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
INC = ROOT / "include"
CUDA_INC = "/usr/local/cuda/include"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def _run(cmd, cwd):
    r = subprocess.run(cmd, cwd=cwd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return r


def test_c_header_compiles_and_links(nvlib, tmp_path):
    lib = nvlib.library_path()
    (tmp_path / "t.c").write_text(r'''
#include "nvfp4_b200.h"
#include <stdio.h>
int main(void) {
  /* m == 0 is a no-op that touches no device */
  int rc = nvfp4_rht_gemm_ntt_w_sfc(0, 64, 0, 0, 0, 0, 0, 0, 0, 0, 2048, 0, 0);
  printf("%d %s\n", rc, nvfp4_status_string(rc));
  return rc;
}
''')
    _run(["gcc", "-std=c99", "-Wall", "-Werror", f"-I{INC}", "t.c", "-o", "t",
          str(lib), f"-Wl,-rpath,{Path(lib).parent}"], tmp_path)
    r = _run(["./t"], tmp_path)
    assert r.stdout.startswith("0 ok")


def test_cpp_launcher_templates_compile(tmp_path):
    (tmp_path / "t.cpp").write_text(r'''
#include "nvfp4_b200.hpp"
#include <cstdint>
void f(const uint16_t* A, const uint16_t* B, uint8_t* C, uint8_t* S, const float* am,
       const size_t* rs, cudaStream_t st) {
  nvfp4_b200::rht_gemm_ntt_w_sfc<uint16_t, uint16_t, uint8_t, uint8_t, true, false>(
      128, 64, A, B, C, S, am, rs, 0, st);
  nvfp4_b200::rht_gemm_ttt_wrapper<uint16_t, uint16_t, uint8_t, uint8_t>(
      64, 128, A, B, C, S, am, rs, 0, st);
}
''')
    _run(["g++", "-std=c++17", "-Wall", "-Werror", "-c", f"-I{INC}", f"-I{CUDA_INC}", "t.cpp",
          "-o", "t.o"], tmp_path)


DEVICE_SRC = r'''
#include "nvfp4_sr.cuh"
#include "nvfp4_fp8.cuh"
namespace ptx = nvfp4_b200::ptx;
__global__ void k(const uint64_t* in, const float4* f, uint32_t* out, ptx::fp8e4m3x4* o8,
                  ptx::fp8e5m2x2* o2, const ptx::bf16x4* b4, const ptx::floatx2* f2) {
  const int i = threadIdx.x;
  fp4e2m1x4 a = mul_cvt_bf16_to_fp4_4x_with_stochastic_rounding(in[i], make_float2(1.f, 2.f), 7u);
  fp4e2m1x4 b = cvt_fp32_to_fp4_4x_with_stochastic_rounding(make_float2(f[i].x, f[i].y),
                                                            make_float2(f[i].z, f[i].w), 9u);
  out[i] = mul_cvt_bf16_to_fp4_8x_stochastic_rounding<float>(in[i], in[i], 0.5f, 1u, 2u) ^
           *reinterpret_cast<uint16_t*>(&a) ^ *reinterpret_cast<uint16_t*>(&b);
  ptx::mul_cvt_4x(o8[i], b4[i], ptx::floatx2{1.f, 2.f});
  ptx::mul_cvt_2x(o2[i], f2[i], ptx::floatx2{0.5f, 4.f});
#if !defined(_LOOSE_PRECISION)
  ptx::mul_cvt_4x(o8[i], b4[i], ptx::floatx4{1.f, 2.f, 3.f, 4.f});
#endif
  ptx::floatx4 w = ptx::up_cast(b4[i]);
  out[i] += __float_as_uint(w.x1);
}
'''


@pytest.mark.parametrize("loose", [False, True])
def test_device_headers_compile_for_sm100a(tmp_path, loose):
    (tmp_path / "t.cu").write_text(DEVICE_SRC)
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-c",
           f"-I{INC}", "t.cu", "-o", "t.o"]
    if loose:
        cmd.insert(1, "-D_LOOSE_PRECISION")
    _run(cmd, tmp_path)
