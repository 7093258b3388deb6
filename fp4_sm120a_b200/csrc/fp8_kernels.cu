// C ABI of the scaled FP8 conversions (mul_cvt_2x / mul_cvt_4x of
// nvfp4_fp8.cuh, round-to-nearest) over batches of groups.
#include "fp8_batch.cuh"

using namespace nvfp4;

extern "C" {

NVFP4_API int nvfp4_mul_cvt_fp8_2x(const void* in, int in_dtype, const float* scale,
                                   size_t scale_stride, void* out, int fp8_format,
                                   size_t ngroups, nvfp4_stream_t stream) {
  return launch_fp8<2, 2>(in, in_dtype, scale, scale_stride, out, fp8_format, ngroups,
                          (cudaStream_t)stream);
}

NVFP4_API int nvfp4_mul_cvt_fp8_4x(const void* in, int in_dtype, const float* scale,
                                   int scale_width, size_t scale_stride, void* out,
                                   int fp8_format, size_t ngroups, nvfp4_stream_t stream) {
  if (scale_width == 2)
    return launch_fp8<4, 2>(in, in_dtype, scale, scale_stride, out, fp8_format, ngroups,
                            (cudaStream_t)stream);
  if (scale_width == 4)
    return launch_fp8<4, 4>(in, in_dtype, scale, scale_stride, out, fp8_format, ngroups,
                            (cudaStream_t)stream);
  return NVFP4_ERR_INVALID_ARGUMENT;
}

}  // extern "C"
