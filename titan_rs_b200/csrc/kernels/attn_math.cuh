// Softmax arithmetic for the attention kernels on sm_100a: packed fp32 pairs on the
// FMA pipe (FFMA2 / FADD2 / FMUL2), a three-input max, and base-2 exponentials either
// on the MUFU (ex2.approx) or on the FMA/ALU pipes only.
//
// Why two exponentials: the MUFU retires 16 results per SM per clock, so a softmax
// that sends every score through ex2 is bounded by it long before the issue slots
// are; evaluating a share of the scores with FMA/ALU instructions spreads the work
// over both. That share must use no XU-pipe instruction at all: floorf (FRND) and
// float->int conversions (F2I) issue on the same XU pipe as ex2, so a polynomial
// built on them costs more XU time than the ex2 it replaces.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace tb {

__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x on the MUFU; 2^-inf = 0.
__device__ __forceinline__ float exp2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for a pair, x <= 64, with FMA/ALU instructions only.
//   x is clamped at -127 (2^-127 comes out as exactly 0, so 2^-inf = 0);
//   t = x + 1.5*2^23 rounded toward -inf puts floor(x) in t's low mantissa bits
//       (t stays in [2^23, 2^24), where the fp32 spacing is 1);
//   f = x - floor(x) in [0, 1) is exact;
//   2^f from a degree-3 polynomial fitted for these kernels by least squares on
//       relative error with p(0) = 1 (max relative error 8.6e-5 on [0, 1), below the
//       2^-9 rounding of the bf16 probabilities it feeds);
//   2^floor(x) by adding t's bits shifted left 23 places (floor(x) mod 2^9 lands in
//       the exponent field; t's other mantissa bits shift out) to the bits of p.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -127.0f);
  x.y = fmaxf(x.y, -127.0f);
  const float2 t = __fadd2_rd(x, make_float2(kShift, kShift));
  const float2 neg_n = __ffma2_rn(t, make_float2(-1.0f, -1.0f), make_float2(kShift, kShift));  // -floor(x), exact
  const float2 f = __fadd2_rn(x, neg_n);
  float2 p = __ffma2_rn(make_float2(0.0770670622587204f, 0.0770670622587204f), f,
                        make_float2(0.22764495015144348f, 0.22764495015144348f));
  p = __ffma2_rn(p, f, make_float2(0.6951168179512024f, 0.6951168179512024f));
  p = __ffma2_rn(p, f, make_float2(1.0f, 1.0f));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

}  // namespace tb
