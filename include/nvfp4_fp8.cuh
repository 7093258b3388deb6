// nvfp4_fp8.cuh -- drop-in device functions for the scaled FP8 conversions
// of TE's vendored ptx helpers, for sm_100a:
//
//   mul_cvt_2x(fp8{e4m3,e5m2}x2 &out, const {float,bf16,fp16}x2 &in, const floatx2 &scale)
//       replaces te_ref/stubs/common/util/ptx.cuh:923-1062 (6 overloads)
//   mul_cvt_4x(fp8{e4m3,e5m2}x4 &out, const {bf16,fp16,float}x4 &in, const floatx2 &scale)
//   mul_cvt_4x(fp8{e4m3,e5m2}x4 &out, const {bf16,fp16,float}x4 &in, const floatx4 &scale)
//       replace ptx.cuh:1172-1693 (12 overloads)
//   up_cast({bf16,fp16}x2 / x4) -> floatx2 / floatx4
//       replaces ptx.cuh:1709-1770
//
// The types (FPx2, FPx4 and the floatx2 ... fp8e5m2x4 aliases) have the
// layout and alignment of TE's (ptx.cuh:488-536).  Code written against
// transformer_engine::ptx compiles against this header after
// `namespace ptx = nvfp4_b200::ptx;`.
//
// Semantics:
//   - inputs widen to fp32 exactly (bf16, fp16 -> f32);
//   - mul_cvt_2x multiplies element i by scale component i with mul.rn.f32x2;
//   - mul_cvt_4x multiplies with fma.rn.f32x2(x, s, +0): one rounding of the
//     exact product, and an exact zero product becomes +0.  With a floatx2
//     scale, elements 0 and 2 take scale.x and elements 1 and 3 scale.y; with
//     a floatx4 scale, element i takes component i;
//   - each product converts by cvt.rn.satfinite.{e4m3,e5m2}x2.f32: round to
//     nearest even, finite overflow and +-Inf saturate to the largest finite
//     value; element 0 lands in byte 0.
//   - With _LOOSE_PRECISION defined (as in the reference) the 4x forms with a
//     floatx2 scale convert by cvt.rs.satfinite.{e4m3,e5m2}x4.f32 with the
//     constant random word 0x80008000 instead.  The floatx4-scale 4x forms are
//     unavailable in that mode: the reference's versions do not assemble
//     there (they pass the 64-bit scale as the random-bits operand).
//
// Include from CUDA code compiled for sm_100a (or sm_103a).
#pragma once

#include <cstdint>
#include <type_traits>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

namespace nvfp4_b200 {
namespace ptx {

using bf16 = __nv_bfloat16;
using fp16 = __half;
using fp8e4m3 = __nv_fp8_e4m3;
using fp8e5m2 = __nv_fp8_e5m2;

template <typename T>
struct alignas(2 * sizeof(T)) FPx2 {
  T x;
  T y;
};

template <typename T>
struct FPx4 {
  T x1;
  T x2;
  T x3;
  T x4;
};

using floatx2 = FPx2<float>;
using bf16x2 = FPx2<bf16>;
using fp16x2 = FPx2<fp16>;
using fp8e4m3x2 = FPx2<fp8e4m3>;
using fp8e5m2x2 = FPx2<fp8e5m2>;

using floatx4 = FPx4<float>;
using bf16x4 = FPx4<bf16>;
using fp16x4 = FPx4<fp16>;
using fp8e4m3x4 = FPx4<fp8e4m3>;
using fp8e5m2x4 = FPx4<fp8e5m2>;

static_assert(sizeof(floatx2) == 8 && sizeof(bf16x2) == 4 && sizeof(fp16x2) == 4, "layout");
static_assert(sizeof(fp8e4m3x2) == 2 && sizeof(fp8e5m2x2) == 2, "layout");
static_assert(sizeof(floatx4) == 16 && sizeof(bf16x4) == 8 && sizeof(fp8e4m3x4) == 4, "layout");

// The conversions live in an inline namespace named for the rounding mode, so
// translation units built with and without _LOOSE_PRECISION can be linked
// together without two definitions of one function.
#if defined(_LOOSE_PRECISION)
inline namespace loose_precision {
#else
inline namespace round_nearest {
#endif

namespace fp8_detail {

template <typename T>
struct is_fp8 : std::integral_constant<bool, std::is_same<T, fp8e4m3>::value ||
                                                 std::is_same<T, fp8e5m2>::value> {};
template <typename T>
struct is_wide_in : std::integral_constant<bool, std::is_same<T, float>::value ||
                                                     std::is_same<T, bf16>::value ||
                                                     std::is_same<T, fp16>::value> {};

template <typename To, typename From>
__device__ __forceinline__ To bitcast(const From& v) {
  static_assert(sizeof(To) == sizeof(From), "bitcast size");
  To r;
  __builtin_memcpy(&r, &v, sizeof(To));
  return r;
}

// One element widened to fp32, exactly.
__device__ __forceinline__ float widen(float v) { return v; }
__device__ __forceinline__ float widen(bf16 v) {
  return __uint_as_float((uint32_t)bitcast<uint16_t>(v) << 16);
}
__device__ __forceinline__ float widen(fp16 v) { return __half2float(v); }

// Two fp32 values as one 64-bit operand, element `lo` in the low word.
__device__ __forceinline__ uint64_t pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t mul_x2(uint64_t a, uint64_t s) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(s));
  return r;
}
__device__ __forceinline__ uint64_t mul_x2_plus_zero(uint64_t a, uint64_t s) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(s), "l"(0ull));
  return r;
}

// cvt.rn.satfinite.{e4m3,e5m2}x2.f32: `lo` in the low byte.
template <typename F8>
__device__ __forceinline__ uint16_t cvt_x2(float lo, float hi) {
  uint16_t r;
  if constexpr (std::is_same<F8, fp8e4m3>::value)
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

#if defined(_LOOSE_PRECISION)
// cvt.rs.satfinite.{e4m3,e5m2}x4.f32 with the reference's constant random
// word; e0 lands in byte 0.
template <typename F8>
__device__ __forceinline__ uint32_t cvt_x4_loose(float e0, float e1, float e2, float e3) {
  uint32_t r;
  if constexpr (std::is_same<F8, fp8e4m3>::value)
    asm("cvt.rs.satfinite.e4m3x4.f32 %0, {%1, %2, %3, %4}, %5;"
        : "=r"(r) : "f"(e3), "f"(e2), "f"(e1), "f"(e0), "r"(0x80008000u));
  else
    asm("cvt.rs.satfinite.e5m2x4.f32 %0, {%1, %2, %3, %4}, %5;"
        : "=r"(r) : "f"(e3), "f"(e2), "f"(e1), "f"(e0), "r"(0x80008000u));
  return r;
}
#endif

template <typename T>
struct dependent_false : std::false_type {};

}  // namespace fp8_detail

// out = fp8x2(in * scale), elementwise; mul.rn.f32x2 then RN satfinite.
template <typename F8, typename In>
__device__ __forceinline__ void mul_cvt_2x(FPx2<F8>& out, const FPx2<In>& in,
                                           const floatx2& scale) {
  using namespace fp8_detail;
  static_assert(is_fp8<F8>::value && is_wide_in<In>::value, "mul_cvt_2x: unsupported types");
  float a, b;
  unpack(mul_x2(pack(widen(in.x), widen(in.y)), bitcast<uint64_t>(scale)), a, b);
  out = bitcast<FPx2<F8>>(cvt_x2<F8>(a, b));
}

// out = fp8x4(in * (scale.x, scale.y, scale.x, scale.y)).
template <typename F8, typename In>
__device__ __forceinline__ void mul_cvt_4x(FPx4<F8>& out, const FPx4<In>& in,
                                           const floatx2& scale) {
  using namespace fp8_detail;
  static_assert(is_fp8<F8>::value && is_wide_in<In>::value, "mul_cvt_4x: unsupported types");
  const uint64_t s = bitcast<uint64_t>(scale);
  float e0, e1, e2, e3;
  unpack(mul_x2_plus_zero(pack(widen(in.x1), widen(in.x2)), s), e0, e1);
  unpack(mul_x2_plus_zero(pack(widen(in.x3), widen(in.x4)), s), e2, e3);
#if defined(_LOOSE_PRECISION)
  out = bitcast<FPx4<F8>>(cvt_x4_loose<F8>(e0, e1, e2, e3));
#else
  out = bitcast<FPx4<F8>>((uint32_t)cvt_x2<F8>(e0, e1) | ((uint32_t)cvt_x2<F8>(e2, e3) << 16));
#endif
}

// out = fp8x4(in * scale), elementwise.
template <typename F8, typename In>
__device__ __forceinline__ void mul_cvt_4x(FPx4<F8>& out, const FPx4<In>& in,
                                           const floatx4& scale) {
  using namespace fp8_detail;
  static_assert(is_fp8<F8>::value && is_wide_in<In>::value, "mul_cvt_4x: unsupported types");
#if defined(_LOOSE_PRECISION)
  static_assert(dependent_false<F8>::value,
                "mul_cvt_4x with a floatx4 scale is unavailable under _LOOSE_PRECISION");
#else
  const floatx2 s01{scale.x1, scale.x2}, s23{scale.x3, scale.x4};
  float e0, e1, e2, e3;
  unpack(mul_x2_plus_zero(pack(widen(in.x1), widen(in.x2)), bitcast<uint64_t>(s01)), e0, e1);
  unpack(mul_x2_plus_zero(pack(widen(in.x3), widen(in.x4)), bitcast<uint64_t>(s23)), e2, e3);
  out = bitcast<FPx4<F8>>((uint32_t)cvt_x2<F8>(e0, e1) | ((uint32_t)cvt_x2<F8>(e2, e3) << 16));
#endif
}

// Exact widening to fp32.
__device__ __forceinline__ floatx2 up_cast(const bf16x2& in) {
  return floatx2{fp8_detail::widen(in.x), fp8_detail::widen(in.y)};
}
__device__ __forceinline__ floatx2 up_cast(const fp16x2& in) {
  return floatx2{fp8_detail::widen(in.x), fp8_detail::widen(in.y)};
}
__device__ __forceinline__ floatx4 up_cast(const bf16x4& in) {
  using fp8_detail::widen;
  return floatx4{widen(in.x1), widen(in.x2), widen(in.x3), widen(in.x4)};
}
__device__ __forceinline__ floatx4 up_cast(const fp16x4& in) {
  using fp8_detail::widen;
  return floatx4{widen(in.x1), widen(in.x2), widen(in.x3), widen(in.x4)};
}

}  // inline namespace
}  // namespace ptx
}  // namespace nvfp4_b200
