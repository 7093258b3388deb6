// Host (g++) build of the reference's scalar software SR quantizer,
// stochastic_rounding/sr.software.cuh, compiled in place from the reference
// tree (-I <reference>/stochastic_rounding).  TEST / BASELINE INFRASTRUCTURE:
// used as the timed CPU baseline and as a statistical cross-check; it is not
// bit-exact to cvt.rs by design (sr.software.cuh:67-75 hashes the random bits).
#include <cstddef>
#include <cstdint>
#include <cstring>
#define __host__
#define __device__
#define __forceinline__ inline
struct float2 { float x, y; };
static inline float2 make_float2(float x, float y) { return float2{x, y}; }
#include "sr.software.cuh"

#define REF_API extern "C" __attribute__((visibility("default")))

// cvt_fp32_to_fp4_4x_with_stochastic_rounding over ngroups groups of 4 floats.
REF_API void ref_sw_cvt_fp32_to_fp4_4x_sr(const float* in, const uint32_t* rbits,
                                          uint16_t* out, size_t ngroups, int nthreads) {
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (long long g = 0; g < (long long)ngroups; g++) {
    float2 a{in[4 * g], in[4 * g + 1]}, b{in[4 * g + 2], in[4 * g + 3]};
    out[g] = raw_bits(cvt_fp32_to_fp4_4x_with_stochastic_rounding(a, b, rbits[g]));
  }
}

REF_API void ref_sw_mul_cvt_fp32_to_fp4_4x_sr(const float* in, float sx, float sy,
                                              const uint32_t* rbits, uint16_t* out,
                                              size_t ngroups, int nthreads) {
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (long long g = 0; g < (long long)ngroups; g++) {
    float2 a{in[4 * g], in[4 * g + 1]}, b{in[4 * g + 2], in[4 * g + 3]};
    out[g] = raw_bits(mul_cvt_fp32_to_fp4_4x_with_stochastic_rounding(a, b, float2{sx, sy}, rbits[g]));
  }
}

REF_API void ref_sw_mul_cvt_bf16_to_fp4_4x_sr(const uint64_t* in, float sx, float sy,
                                              const uint32_t* rbits, uint16_t* out,
                                              size_t ngroups, int nthreads) {
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (long long g = 0; g < (long long)ngroups; g++)
    out[g] = raw_bits(mul_cvt_bf16_to_fp4_4x_with_stochastic_rounding(in[g], float2{sx, sy}, rbits[g]));
}

REF_API void ref_sw_mul_cvt_bf16_to_fp4_8x_sr(const uint64_t* in, float s,
                                              const uint32_t* rbits, uint32_t* out,
                                              size_t ngroups, int nthreads) {
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (long long g = 0; g < (long long)ngroups; g++)
    out[g] = mul_cvt_bf16_to_fp4_8x_stochastic_rounding<float>(in[2 * g], in[2 * g + 1], s,
                                                               rbits[2 * g], rbits[2 * g + 1]);
}
