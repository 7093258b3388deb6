// Host build (nvcc, host code only runs) of the reference's scalar RHT +
// NVFP4 CPU reference, NaiveReference in rht_gemm/test_correctness.cu:110-198,
// compiled in place from the reference tree (-I <reference>/rht_gemm) with its
// main() renamed.  TEST / BASELINE INFRASTRUCTURE: the timed CPU baseline of
// the RHT path and a cross-check of the oracle's round-to-nearest path.
#define main ref_test_correctness_main
#include "test_correctness.cu"
#undef main
#include <omp.h>

#define REF_API extern "C" __attribute__((visibility("default")))

// Runs NaiveReference::compute on column blocks of width `block` (a multiple
// of 16) in parallel and scatters the per-block outputs into C (M x N/2) and
// SFC (M x N/16).  A is M x N column-major bf16, B is 16x16 row-major bf16.
REF_API void ref_naive_rht(int M, int N, const uint16_t* A, const uint16_t* B, uint8_t* C,
                           uint8_t* SFC, float global_amax, int use_fast_math, int block,
                           int nthreads) {
  if (block <= 0 || block > N) block = N;
  const int nblk = (N + block - 1) / block;
#pragma omp parallel for num_threads(nthreads) schedule(dynamic, 1)
  for (int b = 0; b < nblk; b++) {
    const int j0 = b * block;
    const int w = (N - j0) < block ? (N - j0) : block;
    NaiveReference ref;
    ref.M = M;
    ref.N = w;
    ref.compute(reinterpret_cast<const __nv_bfloat16*>(A) + (size_t)M * j0,
                reinterpret_cast<const __nv_bfloat16*>(B), global_amax, use_fast_math != 0);
    for (int i = 0; i < M; i++) {
      std::memcpy(C + (size_t)i * (N / 2) + j0 / 2, ref.C_fp4.data() + (size_t)i * (w / 2), w / 2);
      std::memcpy(SFC + (size_t)i * (N / 16) + j0 / 16, ref.SFC.data() + (size_t)i * (w / 16), w / 16);
    }
  }
}
