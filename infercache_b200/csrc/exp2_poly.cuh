// 2^x on the FP32 pipe, two lanes at a time (PTX f32x2 arithmetic, sm_100).
//
// The exponential-bound loops of kernel C route part of their 2^x work here
// so the multi-function unit (16 results per clock per SM) and the FP32 pipe
// share it.
//
// Method: Cody-Waite style range reduction x = j + f with j = rint(x) and
// f = x - j in [-1/2, 1/2] (j found with the 1.5 * 2^23 shifter: adding it
// leaves rint(x) in the low mantissa bits, subtracting it back gives j as a
// float, and f = x - j is exact), 2^f by a degree-4 polynomial in Horner
// form, and 2^j applied by adding j to the exponent field.  The coefficients
// are this repository's own minimax (Remez exchange) fit of 2^f for
// relative error on [-1/2, 1/2], rounded to fp32; `exp2_poly_fit.py` beside
// this file recomputes them.  Maximum relative error of the fp32 evaluation,
// checked on a dense grid: 2.7e-6.
//
// Domain: x <= 127.  Inputs below -126 (including -inf) are clamped to -126
// and return a value in (0, 2^-125]; callers that need an exact 0 there use
// the multi-function unit instead.
#pragma once
#include <stdint.h>

namespace ic {
namespace poly {

typedef unsigned long long f2;  // two fp32 lanes in one 64-bit register pair

__device__ __forceinline__ f2 pack(float a, float b) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void unpack(f2 v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  f2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  f2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
  f2 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 splat(float a) { return pack(a, a); }

// fp32 bit patterns of the coefficients c0 .. c4 (2^f ~ sum c_k f^k).
constexpr uint32_t EXP2_C0 = 0x3F7FFFF4u;  // 0.99999928
constexpr uint32_t EXP2_C1 = 0x3F31706Eu;  // 0.69312179
constexpr uint32_t EXP2_C2 = 0x3E76036Du;  // 0.24024744
constexpr uint32_t EXP2_C3 = 0x3D650A20u;  // 0.05591786
constexpr uint32_t EXP2_C4 = 0x3C1CCBEBu;  // 0.00957010
constexpr float EXP2_SHIFTER = 12582912.0f;  // 1.5 * 2^23
constexpr float EXP2_MIN_ARG = -126.0f;

// (2^x0, 2^x1) with the FP32 pipe.
__device__ __forceinline__ f2 exp2x2(f2 x) {
  float x0, x1;
  unpack(x, x0, x1);
  x = pack(fmaxf(x0, EXP2_MIN_ARG), fmaxf(x1, EXP2_MIN_ARG));
  const f2 sh = splat(EXP2_SHIFTER);
  const f2 t = add2(x, sh);   // rint(x) in the low mantissa bits of t
  const f2 f = sub2(x, sub2(t, sh));
  f2 p = fma2(splat(__uint_as_float(EXP2_C4)), f, splat(__uint_as_float(EXP2_C3)));
  p = fma2(p, f, splat(__uint_as_float(EXP2_C2)));
  p = fma2(p, f, splat(__uint_as_float(EXP2_C1)));
  p = fma2(p, f, splat(__uint_as_float(EXP2_C0)));
  float p0, p1, t0, t1;
  unpack(p, p0, p1);
  unpack(t, t0, t1);
  // bits(t) << 23 == rint(x) << 23 (mod 2^32): the shifter's own bits shift out
  return pack(__uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23)),
              __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23)));
}

}  // namespace poly
}  // namespace ic
