// Narrow floating-point codecs shared by host and device code.
//
// Semantics follow the rouge-numerics reference bit for bit, including its
// corner cases, so that GPU codes equal the reference CPU codes:
//   f16  encode/decode  fp16.cpp:31-92   (RNE, overflow -> Inf, NaN -> 0x7e00;
//                                         a subnormal that rounds up to 2^-14
//                                         keeps only its low 10 bits, i.e.
//                                         becomes signed zero, fp16.cpp:83)
//   bf16 encode/decode  fp16.cpp:95-112  (RNE by bias add, NaN -> 0x7fc0)
//   e4m3 encode/decode  fp8.cpp:42-106   (OCP E4M3: RNE, satfinite to 0x7e,
//                                         NaN -> sign|0x7f, |x| < 2^-10 -> +0)
#pragma once

#include <cstdint>
#include <cstring>

#if defined(__CUDACC__)
#define RB_HD __host__ __device__ __forceinline__
#else
#define RB_HD inline
#endif

namespace rb200 {

RB_HD uint32_t f32_bits(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
#endif
}

RB_HD float bits_f32(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f;
  std::memcpy(&f, &u, 4);
  return f;
#endif
}

// Shift the 24-bit significand right by `sh` (1..31) with round to nearest
// even on the dropped bits.
RB_HD uint32_t shr_rne(uint32_t sig, int sh) {
  const uint32_t kept = sig >> sh;
  const uint32_t dropped = sig & ((1u << sh) - 1u);
  const uint32_t half = 1u << (sh - 1);
  return kept + ((dropped > half || (dropped == half && (kept & 1u))) ? 1u : 0u);
}

// Number of leading zeros of a value known to be < 2^bits, relative to bit
// (bits - 1); used to normalise subnormal significands.
RB_HD int lead_zeros_small(uint32_t v, int bits) {
  int n = 0;
  while (!(v & (1u << (bits - 1)))) {
    v <<= 1;
    ++n;
  }
  return n;
}

// ------------------------------------------------------------------- f16

RB_HD uint16_t encode_f16(float f) {
  const uint32_t x = f32_bits(f);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t bexp = (x >> 23) & 0xFFu;
  const uint32_t frac = x & 0x7FFFFFu;
  if (bexp == 0xFFu) return static_cast<uint16_t>(sign | (frac ? 0x7E00u : 0x7C00u));
  if ((x & 0x7FFFFFFFu) == 0) return static_cast<uint16_t>(sign);
  const int e = static_cast<int>(bexp) - 112;  // half biased exponent
  if (e >= 31) return static_cast<uint16_t>(sign | 0x7C00u);
  if (e <= 0) {
    if (e < -10) return static_cast<uint16_t>(sign);
    const uint32_t q = shr_rne(frac | 0x800000u, 14 - e);
    return static_cast<uint16_t>(sign | (q & 0x3FFu));
  }
  // Normal: keep 10 fraction bits; a carry may ripple into the exponent.
  const uint32_t q = shr_rne((static_cast<uint32_t>(e) << 23) | frac, 13);
  return static_cast<uint16_t>(sign | (q >= 0x7C00u ? 0x7C00u : q));
}

RB_HD float decode_f16(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu;
  const uint32_t m = h & 0x3FFu;
  if (e == 0x1Fu) return bits_f32(sign | 0x7F800000u | (m << 13));
  if (e != 0) return bits_f32(sign | ((e + 112u) << 23) | (m << 13));
  if (m == 0) return bits_f32(sign);
  const int lz = lead_zeros_small(m, 11);  // bring the leading one to bit 10
  return bits_f32(sign | (static_cast<uint32_t>(113 - lz) << 23) | (((m << lz) & 0x3FFu) << 13));
}

// ------------------------------------------------------------------- bf16

RB_HD uint16_t encode_bf16(float f) {
  const uint32_t x = f32_bits(f);
  if ((x & 0x7F800000u) == 0x7F800000u) {
    return (x & 0x7FFFFFu) ? static_cast<uint16_t>(0x7FC0u) : static_cast<uint16_t>(x >> 16);
  }
  return static_cast<uint16_t>((x + 0x7FFFu + ((x >> 16) & 1u)) >> 16);
}

RB_HD float decode_bf16(uint16_t b) { return bits_f32(static_cast<uint32_t>(b) << 16); }

// ------------------------------------------------------------------- e4m3

RB_HD uint8_t encode_e4m3(float f) {
  const uint32_t x = f32_bits(f);
  const uint32_t sign = (x >> 24) & 0x80u;
  const uint32_t bexp = (x >> 23) & 0xFFu;
  const uint32_t frac = x & 0x7FFFFFu;
  if (bexp == 0xFFu) return static_cast<uint8_t>(sign | (frac ? 0x7Fu : 0x7Eu));
  if ((x & 0x7FFFFFFFu) == 0) return static_cast<uint8_t>(sign);
  const int e = static_cast<int>(bexp) - 120;  // e4m3 biased exponent
  if (e > 15) return static_cast<uint8_t>(sign | 0x7Eu);
  if (e <= 0) {
    if (e < -3) return 0;  // below half the smallest subnormal: +0, sign dropped
    return static_cast<uint8_t>(sign | shr_rne(frac | 0x800000u, 21 - e));
  }
  const uint32_t q = shr_rne((static_cast<uint32_t>(e) << 23) | frac, 20);
  // 0x7F is NaN in E4M3; anything at or past it saturates to MAX (0x7E).
  return static_cast<uint8_t>(sign | (q >= 0x7Fu ? 0x7Eu : q));
}

RB_HD float decode_e4m3(uint8_t c) {
  const uint32_t sign = static_cast<uint32_t>(c & 0x80u) << 24;
  const uint32_t e = (c >> 3) & 0xFu;
  const uint32_t m = c & 0x7u;
  if (e == 0xFu && m == 0x7u) return bits_f32(sign | 0x7FC00000u);
  if (e != 0) return bits_f32(sign | ((e + 120u) << 23) | (m << 20));
  if (m == 0) return bits_f32(sign);
  const int lz = lead_zeros_small(m, 4);
  return bits_f32(sign | (static_cast<uint32_t>(121 - lz) << 23) | (((m << lz) & 0x7u) << 20));
}

}  // namespace rb200
