// Base-2 exponential on the FMA pipe, used for a fixed fraction of the
// softmax exponentials so that the MUFU unit (16 ex2/clk/SM) is not the only
// source of exponentials. The reference kernel offloads 1/8 of its exp2s the
// same way (ex2_poly_pair, llm_fa.cu:268-307); the method and coefficients
// here are this project's own:
//
//   2^x = 2^j * p(f),  j = round-to-nearest(x), f = x - j in [-0.5, 0.5]
//
// j is obtained with the 1.5*2^23 add/subtract rounding trick (exact for
// |x| < 2^22), p is a degree-3 polynomial fitted by Remez exchange for
// minimum relative error on [-0.5, 0.5] (fit_exp2_poly.py, max relative error
// 7.5e-5 in float32 Horner arithmetic, far below bf16's 2^-9 half-ulp), and
// the final 2^j scaling adds j to the exponent field with an integer add.
// Inputs are clamped at -125 so that the exponent field never underflows.
#pragma once
#include <cstdint>

#include "ptx.cuh"

namespace llmfa {

// Remez degree-3 fit of 2^f on [-0.5, 0.5] (relative error), float32.
constexpr float kExp2C0 = 0x1.fff692p-1f;
constexpr float kExp2C1 = 0x1.62f31ap-1f;
constexpr float kExp2C2 = 0x1.f0de1ap-3f;
constexpr float kExp2C3 = 0x1.c3f76p-5f;
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23
constexpr float kExp2MinArg = -125.0f;

// Two exponentials at once with packed f32x2 arithmetic.
__device__ __forceinline__ uint64_t exp2_poly_x2(uint64_t x2) {
  float x0, x1;
  ptx::f2_unpack(x2, x0, x1);
  x0 = fmaxf(x0, kExp2MinArg);
  x1 = fmaxf(x1, kExp2MinArg);
  const uint64_t xc = ptx::f2_pack(x0, x1);
  const uint64_t magic = ptx::f2_pack(kRoundMagic, kRoundMagic);
  const uint64_t t = ptx::f2_add(xc, magic);      // round(x) in the low mantissa bits
  const uint64_t jf = ptx::f2_sub(t, magic);      // round(x) as a float
  const uint64_t f = ptx::f2_sub(xc, jf);         // in [-0.5, 0.5]
  uint64_t p = ptx::f2_fma(ptx::f2_pack(kExp2C3, kExp2C3), f, ptx::f2_pack(kExp2C2, kExp2C2));
  p = ptx::f2_fma(p, f, ptx::f2_pack(kExp2C1, kExp2C1));
  p = ptx::f2_fma(p, f, ptx::f2_pack(kExp2C0, kExp2C0));
  const uint32_t t0 = static_cast<uint32_t>(t), t1 = static_cast<uint32_t>(t >> 32);
  const uint32_t p0 = static_cast<uint32_t>(p), p1 = static_cast<uint32_t>(p >> 32);
  // (t_bits << 23) == (round(x) << 23) mod 2^32: the 0x4B40_0000 bias shifts out.
  const uint32_t r0 = p0 + (t0 << 23);
  const uint32_t r1 = p1 + (t1 << 23);
  return (static_cast<uint64_t>(r1) << 32) | r0;
}

__device__ __forceinline__ uint64_t exp2_mufu_x2(uint64_t x2) {
  float x0, x1;
  ptx::f2_unpack(x2, x0, x1);
  return ptx::f2_pack(ptx::ex2_mufu(x0), ptx::ex2_mufu(x1));
}

}  // namespace llmfa
