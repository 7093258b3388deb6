// GPU build of the reference's own scaled FP8 conversions, compiled in place
// from the reference tree: mul_cvt_2x / mul_cvt_4x of
// rht_gemm/te_ref/stubs/common/util/ptx.cuh:923-1693.  Built twice: as is,
// and with -D_LOOSE_PRECISION (-DREF_FP8_LOOSE), where only the floatx2-scale
// 4x forms assemble.  TEST INFRASTRUCTURE: the bit-exact GPU oracle for the
// FP8 parity tests.  Nothing in the product links it.
#include <cstring>
#include "common/util/ptx.cuh"

#define REF_API extern "C" __attribute__((visibility("default")))

// The two builds are linked into one library: give each its own namespace so
// their kernel templates do not merge.
#if defined(REF_FP8_LOOSE)
#define teref_fp8 teref_fp8_loose
#endif

namespace teref_fp8 {
namespace tp = transformer_engine::ptx;
using transformer_engine::bf16;
using transformer_engine::fp16;
using transformer_engine::fp8e4m3;
using transformer_engine::fp8e5m2;

// One group per thread; the scale vector is copied from scale + g * stride.
template <int W, typename In, typename F8, typename Sc>
__global__ void k_group(const void* in, const float* scale, size_t stride, void* out, size_t n) {
  using InG = std::conditional_t<W == 2, tp::FPx2<In>, tp::FPx4<In>>;
  using OutG = std::conditional_t<W == 2, tp::FPx2<F8>, tp::FPx4<F8>>;
  const size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (g >= n) return;
  Sc s;
  memcpy(&s, scale + g * stride, sizeof(Sc));
  InG x = reinterpret_cast<const InG*>(in)[g];
  OutG o;
  if constexpr (W == 2) tp::mul_cvt_2x(o, x, s);
  else tp::mul_cvt_4x(o, x, s);
  reinterpret_cast<OutG*>(out)[g] = o;
}

template <int W, typename Sc>
int launch(const void* in, int dtype, const float* scale, size_t stride, void* out, int fmt,
           size_t n, cudaStream_t st) {
  if (n == 0) return 0;
  const unsigned b = (unsigned)((n + 255) / 256);
#define REF_FP8_CASE(IN, F8) k_group<W, IN, F8, Sc><<<b, 256, 0, st>>>(in, scale, stride, out, n)
  if (dtype == 0) { if (fmt == 0) REF_FP8_CASE(float, fp8e4m3); else REF_FP8_CASE(float, fp8e5m2); }
  else if (dtype == 1) { if (fmt == 0) REF_FP8_CASE(bf16, fp8e4m3); else REF_FP8_CASE(bf16, fp8e5m2); }
  else { if (fmt == 0) REF_FP8_CASE(fp16, fp8e4m3); else REF_FP8_CASE(fp16, fp8e5m2); }
#undef REF_FP8_CASE
  return (int)cudaGetLastError();
}
}  // namespace teref_fp8

#if defined(REF_FP8_LOOSE)
REF_API int teref_mul_cvt_fp8_4x_loose(const void* in, int dtype, const float* scale,
                                       size_t stride, void* out, int fmt, size_t n,
                                       cudaStream_t st) {
  return teref_fp8::launch<4, teref_fp8::tp::floatx2>(in, dtype, scale, stride, out, fmt, n, st);
}
#else
REF_API int teref_mul_cvt_fp8_2x(const void* in, int dtype, const float* scale, size_t stride,
                                 void* out, int fmt, size_t n, cudaStream_t st) {
  return teref_fp8::launch<2, teref_fp8::tp::floatx2>(in, dtype, scale, stride, out, fmt, n, st);
}
REF_API int teref_mul_cvt_fp8_4x(const void* in, int dtype, const float* scale, int scale_width,
                                 size_t stride, void* out, int fmt, size_t n, cudaStream_t st) {
  if (scale_width == 2)
    return teref_fp8::launch<4, teref_fp8::tp::floatx2>(in, dtype, scale, stride, out, fmt, n, st);
  return teref_fp8::launch<4, teref_fp8::tp::floatx4>(in, dtype, scale, stride, out, fmt, n, st);
}
#endif
