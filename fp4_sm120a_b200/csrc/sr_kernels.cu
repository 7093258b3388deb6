// Batch stochastic-rounding kernels over the four drop-in device functions,
// the row-wise NVFP4 quantizer built on the 8x function, and the global-amax
// pre-pass.  All memory-bound: 128-bit streaming loads/stores, grid sized in
// multiples of the SM count.
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "nvfp4_device.cuh"
#include "nvfp4_sr.cuh"
#include "nvfp4_b200.h"
#include "launch_common.h"

namespace nvfp4 {
namespace {

enum SrKind : int {
  kCvtFp32x4 = 0,     // cvt_fp32_to_fp4_4x_with_stochastic_rounding
  kMulCvtFp32x4 = 1,  // mul_cvt_fp32_to_fp4_4x_with_stochastic_rounding
  kMulCvtBf16x4 = 2,  // mul_cvt_bf16_to_fp4_4x_with_stochastic_rounding
  kMulCvtBf16x8 = 3,  // mul_cvt_bf16_to_fp4_8x_stochastic_rounding<float>
  kMulCvtBf16x8BfScale = 4,  // ... <bf16>
};

// One group: the unit a single call of the device function converts.
template <int KIND>
struct GroupIO;
template <>
struct GroupIO<kCvtFp32x4> {
  using In = float4; using Out = uint16_t; static constexpr int kWords = 1;
};
template <>
struct GroupIO<kMulCvtFp32x4> : GroupIO<kCvtFp32x4> {};
template <>
struct GroupIO<kMulCvtBf16x4> {
  using In = uint2; using Out = uint16_t; static constexpr int kWords = 1;
};
template <>
struct GroupIO<kMulCvtBf16x8> {
  using In = uint4; using Out = uint32_t; static constexpr int kWords = 2;
};
template <>
struct GroupIO<kMulCvtBf16x8BfScale> : GroupIO<kMulCvtBf16x8> {};

template <int KIND>
__device__ __forceinline__ typename GroupIO<KIND>::Out convert_group(
    const typename GroupIO<KIND>::In& x, const uint32_t* r, float sx, float sy) {
  if constexpr (KIND == kCvtFp32x4) {
    fp4e2m1x4 o = cvt_fp32_to_fp4_4x_with_stochastic_rounding(make_float2(x.x, x.y),
                                                               make_float2(x.z, x.w), r[0]);
    return *reinterpret_cast<uint16_t*>(&o);
  } else if constexpr (KIND == kMulCvtFp32x4) {
    fp4e2m1x4 o = mul_cvt_fp32_to_fp4_4x_with_stochastic_rounding(
        make_float2(x.x, x.y), make_float2(x.z, x.w), make_float2(sx, sy), r[0]);
    return *reinterpret_cast<uint16_t*>(&o);
  } else if constexpr (KIND == kMulCvtBf16x4) {
    const uint64_t v = (uint64_t)x.x | ((uint64_t)x.y << 32);
    fp4e2m1x4 o = mul_cvt_bf16_to_fp4_4x_with_stochastic_rounding(v, make_float2(sx, sy), r[0]);
    return *reinterpret_cast<uint16_t*>(&o);
  } else if constexpr (KIND == kMulCvtBf16x8) {
    return mul_cvt_bf16_to_fp4_8x_stochastic_rounding<float>(
        (uint64_t)x.x | ((uint64_t)x.y << 32), (uint64_t)x.z | ((uint64_t)x.w << 32), sx, r[0],
        r[1]);
  } else {
    return mul_cvt_bf16_to_fp4_8x_stochastic_rounding<__nv_bfloat16>(
        (uint64_t)x.x | ((uint64_t)x.y << 32), (uint64_t)x.z | ((uint64_t)x.w << 32),
        __float2bfloat16_rn(sx), r[0], r[1]);
  }
}

constexpr int kGroupsPerThread = 8;
static_assert(kGroupsPerThread * sizeof(uint16_t) % 16 == 0,
              "each thread must write whole 16-byte output vectors");

// Small batches: one group per thread with typed (naturally aligned) loads,
// so that a few hundred thousand groups still spread over every SM.
template <int KIND>
__global__ void __launch_bounds__(256) k_sr_batch1(const typename GroupIO<KIND>::In* __restrict__ in,
                                                   const uint32_t* __restrict__ rbits,
                                                   typename GroupIO<KIND>::Out* __restrict__ out,
                                                   size_t ngroups, float sx, float sy) {
  using IO = GroupIO<KIND>;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < ngroups; g += stride) {
    uint32_t r[IO::kWords];
#pragma unroll
    for (int w = 0; w < IO::kWords; ++w) r[w] = __ldcs(rbits + g * IO::kWords + w);
    out[g] = convert_group<KIND>(__ldcs(in + g), r, sx, sy);
  }
}

// Below this many groups the one-group-per-thread kernel has more parallelism
// than the vector kernel can use.
constexpr size_t kSmallBatch = (size_t)1 << 22;

// Each thread converts 8 consecutive groups: inputs, random words and outputs
// move as 16-byte vectors (the host only launches this when every base
// pointer is 16-byte aligned); the tail is handled group by group.
template <int KIND>
__global__ void __launch_bounds__(256) k_sr_batch(const typename GroupIO<KIND>::In* __restrict__ in,
                                                  const uint32_t* __restrict__ rbits,
                                                  typename GroupIO<KIND>::Out* __restrict__ out,
                                                  size_t ngroups, float sx, float sy) {
  using IO = GroupIO<KIND>;
  using In = typename IO::In;
  using Out = typename IO::Out;
  constexpr int G = kGroupsPerThread;
  constexpr int W = IO::kWords;
  const size_t nvec = ngroups / G;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t v = blockIdx.x * (size_t)blockDim.x + threadIdx.x; v < nvec; v += stride) {
    const size_t g0 = v * G;
    In x[G];
#pragma unroll
    for (int k = 0; k < G; ++k) x[k] = __ldcs(in + g0 + k);
    uint32_t r[G * W];
#pragma unroll
    for (int k = 0; k < G * W / 4; ++k) {
      uint4 q = __ldcs(reinterpret_cast<const uint4*>(rbits + g0 * W) + k);
      r[4 * k] = q.x; r[4 * k + 1] = q.y; r[4 * k + 2] = q.z; r[4 * k + 3] = q.w;
    }
    Out o[G];
#pragma unroll
    for (int k = 0; k < G; ++k) o[k] = convert_group<KIND>(x[k], r + k * W, sx, sy);
#pragma unroll
    for (int k = 0; k < (int)(G * sizeof(Out) / 16); ++k)
      __stcs(reinterpret_cast<uint4*>(out + g0) + k, reinterpret_cast<const uint4*>(o)[k]);
  }
  // tail (fewer than G groups), one thread per group
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (tid < ngroups - nvec * G) {
    const size_t t = nvec * G + tid;
    uint32_t r[W];
#pragma unroll
    for (int w = 0; w < W; ++w) r[w] = rbits[t * W + w];
    out[t] = convert_group<KIND>(in[t], r, sx, sy);
  }
}

// Unaligned fallback: one group per thread, element-wise loads.
template <int KIND>
__global__ void __launch_bounds__(256) k_sr_batch_scalar(const unsigned char* __restrict__ in,
                                                         const uint32_t* __restrict__ rbits,
                                                         unsigned char* __restrict__ out,
                                                         size_t ngroups, float sx, float sy) {
  using IO = GroupIO<KIND>;
  using In = typename IO::In;
  using Out = typename IO::Out;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < ngroups; g += stride) {
    In x;
    __builtin_memcpy(&x, in + g * sizeof(In), sizeof(In));
    uint32_t r[IO::kWords];
    __builtin_memcpy(r, reinterpret_cast<const unsigned char*>(rbits) + g * sizeof(r), sizeof(r));
    Out o = convert_group<KIND>(x, r, sx, sy);
    __builtin_memcpy(out + g * sizeof(Out), &o, sizeof(Out));
  }
}

template <int KIND>
int launch_sr_batch(const void* in, const uint32_t* rbits, void* out, size_t ngroups, float sx,
                    float sy, cudaStream_t stream) {
  using IO = GroupIO<KIND>;
  if (ngroups == 0) return NVFP4_OK;
  if (!in || !rbits || !out) return NVFP4_ERR_INVALID_ARGUMENT;
  int sms = 0;
  if (int e = device_sm_count(&sms)) return e;
  const bool aligned = ((uintptr_t)in % 16 == 0) && ((uintptr_t)rbits % 16 == 0) &&
                       ((uintptr_t)out % 16 == 0);
  if (aligned && ngroups < kSmallBatch) {
    size_t blocks = (ngroups + 255) / 256;
    const size_t cap = (size_t)sms * 32;
    if (blocks > cap) blocks = cap;
    k_sr_batch1<KIND><<<(unsigned)blocks, 256, 0, stream>>>(
        reinterpret_cast<const typename IO::In*>(in), rbits,
        reinterpret_cast<typename IO::Out*>(out), ngroups, sx, sy);
  } else if (aligned) {
    const size_t nvec = ngroups / kGroupsPerThread;
    size_t blocks = (nvec + 255) / 256;
    const size_t cap = (size_t)sms * 32;  // enough 256-thread blocks to fill every SM
    if (blocks > cap) blocks = cap;
    if (blocks == 0) blocks = 1;
    k_sr_batch<KIND><<<(unsigned)blocks, 256, 0, stream>>>(
        reinterpret_cast<const typename IO::In*>(in), rbits,
        reinterpret_cast<typename IO::Out*>(out), ngroups, sx, sy);
  } else {
    size_t blocks = (ngroups + 255) / 256;
    const size_t cap = (size_t)sms * 8;
    if (blocks > cap) blocks = cap;
    k_sr_batch_scalar<KIND><<<(unsigned)blocks, 256, 0, stream>>>(
        reinterpret_cast<const unsigned char*>(in), rbits, reinterpret_cast<unsigned char*>(out),
        ngroups, sx, sy);
  }
  return cuda_status(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Row-wise NVFP4 quantization (16-element blocks along the contiguous
// dimension) with the 8x stochastic-rounding function.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_quantize_rowwise_8x_sr(
    const uint4* __restrict__ x, size_t nblocks, const float* __restrict__ global_amax,
    const uint4* __restrict__ rbits, uint2* __restrict__ c, uint8_t* __restrict__ sfc) {
  const float enc = global_encode_scale(*global_amax);
  const float dec = __fdiv_rn(1.0f, enc);
  const float enc_mult = enc * (1.0f / 6.0f);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nblocks; b += stride) {
    const uint4 lo = __ldcs(x + 2 * b);
    const uint4 hi = __ldcs(x + 2 * b + 1);
    const uint4 r = __ldcs(rbits + b);
    const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    // NaN-propagating amax on |bf16| bit patterns: for non-NaN values the
    // unsigned order of (bits & 0x7FFF) is the order of magnitudes, and every
    // NaN pattern is above +Inf.
    uint32_t m2 = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) m2 = __vmaxu2(m2, w[k] & 0x7FFF7FFFu);
    const uint32_t mbits = max(m2 & 0xFFFFu, m2 >> 16);
    const float amax = __uint_as_float(mbits << 16);
    const uint32_t code = e4m3_encode(amax * enc_mult);
    const float acc = fmin_nan(__fdiv_rn(1.0f, e4m3_decode(code) * dec), 3.402823466e38f);
    uint2 o;
    o.x = mul_cvt_bf16_to_fp4_8x_stochastic_rounding<float>(
        (uint64_t)lo.x | ((uint64_t)lo.y << 32), (uint64_t)lo.z | ((uint64_t)lo.w << 32), acc, r.x,
        r.y);
    o.y = mul_cvt_bf16_to_fp4_8x_stochastic_rounding<float>(
        (uint64_t)hi.x | ((uint64_t)hi.y << 32), (uint64_t)hi.z | ((uint64_t)hi.w << 32), acc, r.z,
        r.w);
    __stcs(c + b, o);
    sfc[b] = (uint8_t)code;
  }
}

// ---------------------------------------------------------------------------
// Global amax of a bf16 tensor, NaN-propagating, as an fp32 bit pattern
// accumulated with atomicMax (valid because the value is never negative).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(512) k_amax_bf16(const uint4* __restrict__ x, size_t nvec,
                                                   const uint16_t* __restrict__ tail, int ntail,
                                                   uint32_t* __restrict__ out_bits,
                                                   uint32_t* __restrict__ clear_bits) {
  // The next kernel (the cast) may launch now; it waits for this one to
  // complete before it reads the amax.
  asm volatile("griddepcontrol.launch_dependents;");
  if (clear_bits != nullptr && blockIdx.x == 0 && threadIdx.x == 0) {
    // Chained form: this launch may overlap the previous kernel of the stream,
    // which can still be reading *clear_bits; only this thread waits for it
    // to complete before clearing the word for the next launch.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    *clear_bits = 0u;
  }
  uint32_t m2 = 0;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  // 4 independent 16-byte loads in flight per iteration
  for (; i + 3 * stride < nvec; i += 4 * stride) {
    uint4 a = __ldcs(x + i), b = __ldcs(x + i + stride), c = __ldcs(x + i + 2 * stride),
          d = __ldcs(x + i + 3 * stride);
    m2 = __vmaxu2(m2, a.x & 0x7FFF7FFFu); m2 = __vmaxu2(m2, a.y & 0x7FFF7FFFu);
    m2 = __vmaxu2(m2, a.z & 0x7FFF7FFFu); m2 = __vmaxu2(m2, a.w & 0x7FFF7FFFu);
    m2 = __vmaxu2(m2, b.x & 0x7FFF7FFFu); m2 = __vmaxu2(m2, b.y & 0x7FFF7FFFu);
    m2 = __vmaxu2(m2, b.z & 0x7FFF7FFFu); m2 = __vmaxu2(m2, b.w & 0x7FFF7FFFu);
    m2 = __vmaxu2(m2, c.x & 0x7FFF7FFFu); m2 = __vmaxu2(m2, c.y & 0x7FFF7FFFu);
    m2 = __vmaxu2(m2, c.z & 0x7FFF7FFFu); m2 = __vmaxu2(m2, c.w & 0x7FFF7FFFu);
    m2 = __vmaxu2(m2, d.x & 0x7FFF7FFFu); m2 = __vmaxu2(m2, d.y & 0x7FFF7FFFu);
    m2 = __vmaxu2(m2, d.z & 0x7FFF7FFFu); m2 = __vmaxu2(m2, d.w & 0x7FFF7FFFu);
  }
  for (; i < nvec; i += stride) {
    uint4 a = __ldcs(x + i);
    m2 = __vmaxu2(m2, a.x & 0x7FFF7FFFu); m2 = __vmaxu2(m2, a.y & 0x7FFF7FFFu);
    m2 = __vmaxu2(m2, a.z & 0x7FFF7FFFu); m2 = __vmaxu2(m2, a.w & 0x7FFF7FFFu);
  }
  if (blockIdx.x == 0 && threadIdx.x < (unsigned)ntail)
    m2 = __vmaxu2(m2, (uint32_t)(tail[threadIdx.x] & 0x7FFFu));
  uint32_t m = max(m2 & 0xFFFFu, m2 >> 16);
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  __shared__ uint32_t warp_max[16];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) warp_max[wid] = m;
  __syncthreads();
  if (wid == 0) {
    m = lane < (int)(blockDim.x >> 5) ? warp_max[lane] : 0u;
    m = __reduce_max_sync(0xFFFFFFFFu, m);
    if (lane == 0 && m != 0u) atomicMax(out_bits, m << 16);
  }
}

}  // namespace
}  // namespace nvfp4

using namespace nvfp4;

extern "C" {

NVFP4_API int nvfp4_cvt_fp32_to_fp4_4x_sr(const float* in, const uint32_t* rbits, uint16_t* out,
                                          size_t ngroups, nvfp4_stream_t stream) {
  return launch_sr_batch<kCvtFp32x4>(in, rbits, out, ngroups, 1.0f, 1.0f, (cudaStream_t)stream);
}

NVFP4_API int nvfp4_mul_cvt_fp32_to_fp4_4x_sr(const float* in, float scale_x, float scale_y,
                                              const uint32_t* rbits, uint16_t* out, size_t ngroups,
                                              nvfp4_stream_t stream) {
  return launch_sr_batch<kMulCvtFp32x4>(in, rbits, out, ngroups, scale_x, scale_y,
                                        (cudaStream_t)stream);
}

NVFP4_API int nvfp4_mul_cvt_bf16_to_fp4_4x_sr(const void* in_bf16, float scale_x, float scale_y,
                                              const uint32_t* rbits, uint16_t* out, size_t ngroups,
                                              nvfp4_stream_t stream) {
  return launch_sr_batch<kMulCvtBf16x4>(in_bf16, rbits, out, ngroups, scale_x, scale_y,
                                        (cudaStream_t)stream);
}

NVFP4_API int nvfp4_mul_cvt_bf16_to_fp4_8x_sr(const void* in_bf16, float scale, int scale_is_bf16,
                                              const uint32_t* rbits, uint32_t* out, size_t ngroups,
                                              nvfp4_stream_t stream) {
  if (scale_is_bf16)
    return launch_sr_batch<kMulCvtBf16x8BfScale>(in_bf16, rbits, out, ngroups, scale, scale,
                                                 (cudaStream_t)stream);
  return launch_sr_batch<kMulCvtBf16x8>(in_bf16, rbits, out, ngroups, scale, scale,
                                        (cudaStream_t)stream);
}

NVFP4_API int nvfp4_quantize_rowwise_bf16_sr(int rows, int cols, const void* X,
                                             const float* global_amax, const uint32_t* rbits,
                                             void* C, void* SFC, nvfp4_stream_t stream) {
  if (rows < 0 || cols < 0) return NVFP4_ERR_INVALID_SHAPE;
  if (cols % 16 != 0) return NVFP4_ERR_INVALID_SHAPE;
  const size_t nblocks = (size_t)rows * (size_t)(cols / 16);
  if (nblocks == 0) return NVFP4_OK;
  if (!X || !global_amax || !rbits || !C || !SFC) return NVFP4_ERR_INVALID_ARGUMENT;
  if ((uintptr_t)X % 16 || (uintptr_t)rbits % 16 || (uintptr_t)C % 8)
    return NVFP4_ERR_MISALIGNED;
  int sms = 0;
  if (int e = device_sm_count(&sms)) return e;
  size_t blocks = (nblocks + 255) / 256;
  if (blocks > (size_t)sms * 8) blocks = (size_t)sms * 8;
  k_quantize_rowwise_8x_sr<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint4*>(X), nblocks, global_amax,
      reinterpret_cast<const uint4*>(rbits), reinterpret_cast<uint2*>(C),
      reinterpret_cast<uint8_t*>(SFC));
  return cuda_status(cudaGetLastError());
}

NVFP4_API int nvfp4_amax_bf16(const void* x, size_t n, float* out, nvfp4_stream_t stream) {
  if (!out) return NVFP4_ERR_INVALID_ARGUMENT;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float), st)) return cuda_status(e);
  if (n == 0) return NVFP4_OK;
  if (!x) return NVFP4_ERR_INVALID_ARGUMENT;
  if ((uintptr_t)x % 16) return NVFP4_ERR_MISALIGNED;
  int sms = 0;
  if (int e = device_sm_count(&sms)) return e;
  const size_t nvec = n / 8;
  const int ntail = (int)(n % 8);
  size_t blocks = (nvec + 511) / 512;
  if (blocks > (size_t)sms * 4) blocks = (size_t)sms * 4;
  if (blocks == 0) blocks = 1;
  k_amax_bf16<<<(unsigned)blocks, 512, 0, st>>>(
      reinterpret_cast<const uint4*>(x), nvec,
      reinterpret_cast<const uint16_t*>(x) + nvec * 8, ntail, reinterpret_cast<uint32_t*>(out),
      nullptr);
  return cuda_status(cudaGetLastError());
}

NVFP4_API int nvfp4_amax_bf16_chained(const void* x, size_t n, float* out, float* clear,
                                      nvfp4_stream_t stream) {
  if (!out || !clear || out == clear) return NVFP4_ERR_INVALID_ARGUMENT;
  if (n > 0 && !x) return NVFP4_ERR_INVALID_ARGUMENT;
  if ((uintptr_t)x % 16) return NVFP4_ERR_MISALIGNED;
  int sms = 0;
  if (int e = device_sm_count(&sms)) return e;
  const size_t nvec = n / 8;
  const int ntail = (int)(n % 8);
  size_t blocks = (nvec + 511) / 512;
  if (blocks > (size_t)sms * 4) blocks = (size_t)sms * 4;
  if (blocks == 0) blocks = 1;
  // A programmatic dependent of the previous kernel of the stream: its blocks
  // start while that kernel drains.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(512);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaError_t e = cudaLaunchKernelEx(
          &cfg, k_amax_bf16, reinterpret_cast<const uint4*>(x), nvec,
          reinterpret_cast<const uint16_t*>(x) + nvec * 8, ntail,
          reinterpret_cast<uint32_t*>(out), reinterpret_cast<uint32_t*>(clear)))
    return cuda_status(e);
  return cuda_status(cudaGetLastError());
}

}  // extern "C"
