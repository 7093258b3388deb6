// Batch kernels over the scaled FP8 conversions of nvfp4_fp8.cuh
// (mul_cvt_2x / mul_cvt_4x).  Included by fp8_kernels.cu and, with
// _LOOSE_PRECISION defined, by fp8_kernels_loose.cu; everything here has
// internal linkage so the two builds stay apart.
//
// Layout: group g reads W consecutive input elements starting at element W*g
// and writes W consecutive FP8 bytes starting at byte W*g.  Its scale vector
// (SW floats) starts at scale + g * scale_stride; scale_stride 0 gives every
// group the same scale vector.
#pragma once

#include <cstdint>
#include <type_traits>
#include <cuda_runtime.h>

#include "launch_common.h"
#include "nvfp4_b200.h"
#include "nvfp4_fp8.cuh"

namespace nvfp4 {
namespace {
namespace px = nvfp4_b200::ptx;

template <typename In, typename F8, int W, int SW>
struct Fp8Io {
  static_assert(W == 2 || W == 4, "group width");
  static_assert(SW == 2 || (W == 4 && SW == 4), "scale width");
  using InG = std::conditional_t<W == 2, px::FPx2<In>, px::FPx4<In>>;
  using OutG = std::conditional_t<W == 2, px::FPx2<F8>, px::FPx4<F8>>;
  using Scale = std::conditional_t<SW == 2, px::floatx2, px::floatx4>;
  // groups per thread in the vector kernel: one 16-byte output vector
  static constexpr int kG = 16 / (int)sizeof(OutG);
  static constexpr int kInVec = kG * (int)sizeof(InG) / 16;
  static_assert(kInVec * 16 == kG * (int)sizeof(InG), "whole 16-byte input vectors");
};

template <int SW>
__device__ __forceinline__ std::conditional_t<SW == 2, px::floatx2, px::floatx4> load_scale(
    const float* p) {
  if constexpr (SW == 2) return px::floatx2{p[0], p[1]};
  else return px::floatx4{p[0], p[1], p[2], p[3]};
}

template <typename In, typename F8, int W, int SW>
__device__ __forceinline__ void convert_group(typename Fp8Io<In, F8, W, SW>::OutG& o,
                                              const typename Fp8Io<In, F8, W, SW>::InG& g,
                                              const typename Fp8Io<In, F8, W, SW>::Scale& s) {
  if constexpr (W == 2) px::mul_cvt_2x(o, g, s);
  else px::mul_cvt_4x(o, g, s);
}

// Aligned bulk: each thread converts kG groups per 16-byte output vector,
// streaming loads and stores, grid-stride over nvec vectors.
template <typename In, typename F8, int W, int SW>
__global__ void __launch_bounds__(256) k_fp8_batch(const uint4* __restrict__ in,
                                                   const float* __restrict__ scale,
                                                   size_t scale_stride, uint4* __restrict__ out,
                                                   size_t nvec) {
  using IO = Fp8Io<In, F8, W, SW>;
  const auto s0 = load_scale<SW>(scale);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < nvec; v += stride) {
    uint4 raw[IO::kInVec];
#pragma unroll
    for (int i = 0; i < IO::kInVec; ++i) raw[i] = __ldcs(in + v * IO::kInVec + i);
    typename IO::InG g[IO::kG];
    __builtin_memcpy(g, raw, sizeof(g));
    typename IO::OutG o[IO::kG];
#pragma unroll
    for (int j = 0; j < IO::kG; ++j) {
      const auto s = scale_stride ? load_scale<SW>(scale + (v * IO::kG + j) * scale_stride) : s0;
      convert_group<In, F8, W, SW>(o[j], g[j], s);
    }
    uint4 ov;
    __builtin_memcpy(&ov, o, sizeof(ov));
    __stcs(out + v, ov);
  }
}

// Remainder and unaligned buffers: one group per thread, groups [g0, ngroups).
template <typename In, typename F8, int W, int SW>
__global__ void __launch_bounds__(256) k_fp8_scalar(
    const typename Fp8Io<In, F8, W, SW>::InG* __restrict__ in, const float* __restrict__ scale,
    size_t scale_stride, typename Fp8Io<In, F8, W, SW>::OutG* __restrict__ out, size_t g0,
    size_t ngroups) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t g = g0 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < ngroups; g += stride) {
    const auto s = load_scale<SW>(scale + g * scale_stride);
    convert_group<In, F8, W, SW>(out[g], in[g], s);
  }
}

template <typename In, typename F8, int W, int SW>
int launch_fp8_typed(const void* in, const float* scale, size_t scale_stride, void* out,
                     size_t ngroups, cudaStream_t st) {
  using IO = Fp8Io<In, F8, W, SW>;
  if (ngroups == 0) return NVFP4_OK;
  if (!in || !scale || !out) return NVFP4_ERR_INVALID_ARGUMENT;
  if ((uintptr_t)scale % alignof(float) || (uintptr_t)in % alignof(typename IO::InG) ||
      (uintptr_t)out % alignof(typename IO::OutG))
    return NVFP4_ERR_MISALIGNED;
  int sms = 0;
  if (int e = device_sm_count(&sms)) return e;
  const bool vec = (uintptr_t)in % 16 == 0 && (uintptr_t)out % 16 == 0;
  const size_t nvec = vec ? ngroups / IO::kG : 0;
  if (nvec) {
    size_t blocks = (nvec + 255) / 256;
    const size_t cap = (size_t)sms * 16;
    if (blocks > cap) blocks = cap;
    k_fp8_batch<In, F8, W, SW><<<(unsigned)blocks, 256, 0, st>>>(
        reinterpret_cast<const uint4*>(in), scale, scale_stride, reinterpret_cast<uint4*>(out),
        nvec);
  }
  const size_t g0 = nvec * IO::kG;
  if (g0 < ngroups) {
    size_t blocks = (ngroups - g0 + 255) / 256;
    const size_t cap = (size_t)sms * 8;
    if (blocks > cap) blocks = cap;
    k_fp8_scalar<In, F8, W, SW><<<(unsigned)blocks, 256, 0, st>>>(
        reinterpret_cast<const typename IO::InG*>(in), scale, scale_stride,
        reinterpret_cast<typename IO::OutG*>(out), g0, ngroups);
  }
  return cuda_status(cudaGetLastError());
}

// Run-time dispatch over (input type, FP8 format) for one (W, SW).
template <int W, int SW>
int launch_fp8(const void* in, int in_dtype, const float* scale, size_t scale_stride, void* out,
               int fp8_format, size_t ngroups, cudaStream_t st) {
  if (fp8_format != NVFP4_FP8_E4M3 && fp8_format != NVFP4_FP8_E5M2)
    return NVFP4_ERR_INVALID_ARGUMENT;
  const bool e4 = fp8_format == NVFP4_FP8_E4M3;
  switch (in_dtype) {
    case NVFP4_DTYPE_F32:
      return e4 ? launch_fp8_typed<float, px::fp8e4m3, W, SW>(in, scale, scale_stride, out, ngroups, st)
                : launch_fp8_typed<float, px::fp8e5m2, W, SW>(in, scale, scale_stride, out, ngroups, st);
    case NVFP4_DTYPE_BF16:
      return e4 ? launch_fp8_typed<px::bf16, px::fp8e4m3, W, SW>(in, scale, scale_stride, out, ngroups, st)
                : launch_fp8_typed<px::bf16, px::fp8e5m2, W, SW>(in, scale, scale_stride, out, ngroups, st);
    case NVFP4_DTYPE_F16:
      return e4 ? launch_fp8_typed<px::fp16, px::fp8e4m3, W, SW>(in, scale, scale_stride, out, ngroups, st)
                : launch_fp8_typed<px::fp16, px::fp8e5m2, W, SW>(in, scale, scale_stride, out, ngroups, st);
    default:
      return NVFP4_ERR_INVALID_ARGUMENT;
  }
}

}  // namespace
}  // namespace nvfp4
