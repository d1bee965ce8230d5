// f32 multiply / divide with the NaN results of x86-64 SSE arithmetic.
//
// The reference computes on x86-64, where an operation with a NaN operand
// returns that operand (quieted), and an invalid operation (0/0, inf/inf,
// 0*inf) returns the "default NaN" 0xFFC00000, whose sign bit is set. The
// GPU returns the canonical NaN 0x7FFFFFFF in all these cases. The sign of
// a NaN decides its E4M3 code (sign|0x7F) and its f32 bits, so kernels whose
// outputs must equal the reference bit for bit use these helpers. Results
// for non-NaN outcomes are the plain IEEE round-to-nearest ones.
#pragma once

#include <cstdint>

namespace rb200 {

__device__ __forceinline__ float x86_quiet(float a) {
  return __uint_as_float(__float_as_uint(a) | 0x00400000u);
}

__device__ __forceinline__ float x86_div(float x, float s) {
  if (isnan(x)) return x86_quiet(x);
  if (isnan(s)) return x86_quiet(s);
  const float q = __fdiv_rn(x, s);
  return isnan(q) ? __uint_as_float(0xFFC00000u) : q;
}

__device__ __forceinline__ float x86_mul(float a, float b) {
  if (isnan(a)) return x86_quiet(a);
  if (isnan(b)) return x86_quiet(b);
  const float p = __fmul_rn(a, b);
  return isnan(p) ? __uint_as_float(0xFFC00000u) : p;
}

// Two f32 values to packed bf16 (lo in bits 0-15) with the hardware RNE
// conversion. For every non-NaN input this equals the reference's
// (bits + 0x7fff + lsb) >> 16 (fp16.cpp:101-112), including subnormals and
// overflow to infinity; NaN inputs must be mapped to 0x7fc0 by the caller.
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Two f32 values to packed IEEE half (lo in bits 0-15), hardware round to
// nearest even with overflow to infinity.
__device__ __forceinline__ uint32_t f16x2_rn(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// x86_mul with the NaN handling moved off the common path: one multiply
// and one NaN test, the full rule only when the product is NaN.
__device__ __forceinline__ float x86_mul_fast(float a, float b) {
  const float p = __fmul_rn(a, b);
  return isnan(p) ? x86_mul(a, b) : p;
}

}  // namespace rb200
