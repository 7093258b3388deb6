// GPU build of the reference's own SM100 kernels, compiled in place from the
// reference tree: TE's rht_gemm_ntt_w_sfc (rht_gemm/test_compare_ref.cu:70-88,
// which includes te_ref/hadamard_transform_cast_fusion_core.inc) and TE's
// native cvt.rs conversion functions (te_ref/stubs/common/util/ptx.cuh:563-918).
// TEST INFRASTRUCTURE: the bit-exact GPU oracle for parity tests and the
// reference kernel timed beside ours.  Nothing in the product links it.
#include "test_compare_ref.cu"

#define REF_API extern "C" __attribute__((visibility("default")))

// run_ref / run_ref_fast / run_ref_sr under C linkage.
REF_API int teref_rht_gemm_ntt_w_sfc(int m, int n, const void* A, const void* B, void* C,
                                     void* SFC, const float* global_amax,
                                     const size_t* rng_state, uint32_t sm_count,
                                     cudaStream_t stream, int sr, int fast_math) {
  auto a = reinterpret_cast<const __nv_bfloat16*>(A);
  auto b = reinterpret_cast<const __nv_bfloat16*>(B);
  auto c = reinterpret_cast<uint8_t*>(C);
  auto s = reinterpret_cast<uint8_t*>(SFC);
  if (sr && !fast_math) run_ref_sr(m, n, a, b, c, s, global_amax, rng_state, sm_count, stream);
  else if (!sr && fast_math) run_ref_fast(m, n, a, b, c, s, global_amax, rng_state, sm_count, stream);
  else if (!sr && !fast_math) run_ref(m, n, a, b, c, s, global_amax, rng_state, sm_count, stream);
  else return 2;
  return (int)cudaGetLastError();
}

namespace teref_native {
using namespace transformer_engine::ptx;

__global__ void k_bf16_4x(const uint64_t* in, float2 scale, const uint32_t* rb, uint16_t* out,
                          size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) {
    fp4e2m1x4 r = mul_cvt_bf16_to_fp4_4x_with_stochastic_rounding(in[i], scale, rb[i]);
    out[i] = *reinterpret_cast<uint16_t*>(&r);
  }
}
__global__ void k_fp32_4x(const float4* in, float2 scale, const uint32_t* rb, uint16_t* out,
                          size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) {
    float4 v = in[i];
    fp4e2m1x4 r = mul_cvt_fp32_to_fp4_4x_with_stochastic_rounding(
        make_float2(v.x, v.y), make_float2(v.z, v.w), scale, rb[i]);
    out[i] = *reinterpret_cast<uint16_t*>(&r);
  }
}
__global__ void k_bf16_8x(const uint64_t* in, float s, int use_bf16_scale, const uint32_t* rb,
                          uint32_t* out, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) {
    if (use_bf16_scale)
      out[i] = mul_cvt_bf16_to_fp4_8x_stochastic_rounding<transformer_engine::bf16>(
          in[2 * i], in[2 * i + 1], __float2bfloat16(s), rb[2 * i], rb[2 * i + 1]);
    else
      out[i] = mul_cvt_bf16_to_fp4_8x_stochastic_rounding<float>(in[2 * i], in[2 * i + 1], s,
                                                                 rb[2 * i], rb[2 * i + 1]);
  }
}
// The scale-free fp32 4x form, with the operand order of
// stochastic_rounding/compare.cuh:51-62 (not present in TE's ptx.cuh).
__global__ void k_cvt_fp32_4x(const float4* in, const uint32_t* rb, uint16_t* out, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) {
    float4 v = in[i];
    uint16_t o;
    asm volatile("cvt.rs.satfinite.e2m1x4.f32 %0, {%1, %2, %3, %4}, %5;"
                 : "=h"(o) : "f"(v.w), "f"(v.z), "f"(v.y), "f"(v.x), "r"(rb[i]));
    out[i] = o;
  }
}
// cvt.rn.satfinite.e2m1x2.f32 and cvt.rn.satfinite.e4m3x2.f32 on single
// values, for pinning the oracle's codecs.
__global__ void k_codecs(const float* in, uint8_t* e2m1, uint8_t* e4m3, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) {
    uint16_t b;
    asm volatile("{\n.reg .b8 t;\ncvt.rn.satfinite.e2m1x2.f32 t, %1, %1;\ncvt.u16.u8 %0, t;\n}"
                 : "=h"(b) : "f"(in[i]));
    e2m1[i] = (uint8_t)(b & 0xF);
    uint16_t h;
    asm volatile("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %1;" : "=h"(h) : "f"(in[i]));
    e4m3[i] = (uint8_t)(h & 0xFF);
  }
}
}  // namespace teref_native

static inline unsigned nblocks(size_t n) { return (unsigned)((n + 255) / 256); }

REF_API int teref_mul_cvt_bf16_to_fp4_4x_sr(const void* in, float sx, float sy,
                                            const uint32_t* rb, uint16_t* out, size_t n,
                                            cudaStream_t st) {
  if (n) teref_native::k_bf16_4x<<<nblocks(n), 256, 0, st>>>((const uint64_t*)in, make_float2(sx, sy), rb, out, n);
  return (int)cudaGetLastError();
}
REF_API int teref_mul_cvt_fp32_to_fp4_4x_sr(const float* in, float sx, float sy,
                                            const uint32_t* rb, uint16_t* out, size_t n,
                                            cudaStream_t st) {
  if (n) teref_native::k_fp32_4x<<<nblocks(n), 256, 0, st>>>((const float4*)in, make_float2(sx, sy), rb, out, n);
  return (int)cudaGetLastError();
}
REF_API int teref_mul_cvt_bf16_to_fp4_8x_sr(const void* in, float s, int use_bf16_scale,
                                            const uint32_t* rb, uint32_t* out, size_t n,
                                            cudaStream_t st) {
  if (n) teref_native::k_bf16_8x<<<nblocks(n), 256, 0, st>>>((const uint64_t*)in, s, use_bf16_scale, rb, out, n);
  return (int)cudaGetLastError();
}
REF_API int teref_cvt_fp32_to_fp4_4x_sr(const float* in, const uint32_t* rb, uint16_t* out,
                                        size_t n, cudaStream_t st) {
  if (n) teref_native::k_cvt_fp32_4x<<<nblocks(n), 256, 0, st>>>((const float4*)in, rb, out, n);
  return (int)cudaGetLastError();
}
REF_API int teref_codecs(const float* in, uint8_t* e2m1, uint8_t* e4m3, size_t n, cudaStream_t st) {
  if (n) teref_native::k_codecs<<<nblocks(n), 256, 0, st>>>(in, e2m1, e4m3, n);
  return (int)cudaGetLastError();
}
