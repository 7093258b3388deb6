// The same batch conversions built with _LOOSE_PRECISION: mul_cvt_4x with a
// floatx2 scale then rounds by cvt.rs.satfinite.{e4m3,e5m2}x4.f32 with the
// constant random word 0x80008000, as the reference does under that macro.
#define _LOOSE_PRECISION 1
#include "fp8_batch.cuh"

using namespace nvfp4;

extern "C" {

NVFP4_API int nvfp4_mul_cvt_fp8_4x_loose(const void* in, int in_dtype, const float* scale,
                                         size_t scale_stride, void* out, int fp8_format,
                                         size_t ngroups, nvfp4_stream_t stream) {
  return launch_fp8<4, 2>(in, in_dtype, scale, scale_stride, out, fp8_format, ngroups,
                          (cudaStream_t)stream);
}

}  // extern "C"
