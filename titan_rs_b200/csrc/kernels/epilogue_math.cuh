// Activations fused into tensor-core epilogues, computed in fp32 on the accumulator
// (after the bias, before the bf16 rounding of the output).
//
//   GELU as the titan.rs CPU reference defines it (titan-runtime/src/lib.rs:625-640):
//     0.5 x (1 + erf(x / sqrt 2)), with erf from the published Abramowitz & Stegun
//     formula 7.1.26: for z >= 0, erf(z) ~ 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5)
//     e^{-z^2}, t = 1 / (1 + p z), p = 0.3275911, a1..a5 = 0.254829592, -0.284496736,
//     1.421413741, -1.453152027, 1.061405429 (|error| <= 1.5e-7); erf is odd.
//   SiLU as the reference defines it (titan-runtime/src/lib.rs:3064): x / (1 + e^{-x}).
#pragma once

#include <cuda_runtime.h>

#include "kernel_configs.h"

namespace tb {

enum Activation : int { kActNone = TB_ACT_NONE, kActGelu = TB_ACT_GELU, kActSilu = TB_ACT_SILU };

__device__ __forceinline__ float gelu_erf(float x) {
  const float z = fabsf(x) * 0.70710678118654752f;
  const float t = 1.0f / (1.0f + 0.3275911f * z);
  float p = fmaf(1.061405429f, t, -1.453152027f);
  p = fmaf(p, t, 1.421413741f);
  p = fmaf(p, t, -0.284496736f);
  p = fmaf(p, t, 0.254829592f);
  const float erf_abs = 1.0f - p * t * expf(-z * z);
  return 0.5f * x * (1.0f + copysignf(erf_abs, x));
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

__device__ __forceinline__ float activate(float x, int act) {
  return act == kActGelu ? gelu_erf(x) : act == kActSilu ? silu(x) : x;
}

}  // namespace tb
