// b2q_q8.cuh -- device arithmetic shared by every producer of Q8_0 activations
// (the stand-alone quantize kernel and the GEMM's fused GELU + quantize
// epilogue), so both produce the same bytes from the same fp32 values.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "b2q_internal.h"

namespace b2q {

// ggml from_float for GGML_TYPE_Q8_0, one block: amax -> fp32 scale d and the
// inverse used for the codes.  VARIANT 0 (x86 SIMD): inverse = 127 / amax,
// VARIANT 1 (scalar reference): inverse = 1 / d.  Each step is one IEEE op.
template <int VARIANT>
__device__ __forceinline__ void q8_scale(float amax, float& d, float& inv) {
  d = __fdiv_rn(amax, 127.0f);
  if (VARIANT == 0)
    inv = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
  else
    inv = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
}

// One code: VARIANT 0 rounds to nearest-even and clamps to int8, VARIANT 1
// rounds half away from zero (|x * inv| <= 127 there by construction).
template <int VARIANT>
__device__ __forceinline__ uint32_t quantize_code(float v, float inv) {
  const float s = __fmul_rn(v, inv);
  if (VARIANT == 0) {
    const int q = __float2int_rn(s);
    return static_cast<uint32_t>(max(-128, min(127, q))) & 0xffu;
  }
  return static_cast<uint32_t>(static_cast<int>(roundf(s))) & 0xffu;
}

// Split-layout activation scale: fp16-rounded d, pre-multiplied by 2^49 (exact).
__device__ __forceinline__ float q8_split_scale(float d) {
  return __half2float(__float2half_rn(d)) * kActScaleMul;
}

// ggml_gelu as the ggml CPU backend computes it (ggml-cpu/vec.h, the default
// GGML_GELU_FP16 build): 0 for x <= -10, x for x >= 10; otherwise x rounded to
// fp16, then 0.5f*f*(1.0f + tanhf(SQRT_2_OVER_PI*f*(1.0f + GELU_COEF_A*f*f)))
// evaluated left to right in fp32 with every product and sum rounded
// separately (no contraction), then rounded to fp16 -- the value of ggml's
// 65536-entry fp16 table, computed instead of looked up.  Only 65536 inputs
// reach the formula, so a test can compare all of them with the table.
//
// Branch-free (the range cases are selects after the formula), so that a warp
// evaluating many independent values interleaves them instead of running one
// dependent chain at a time.
__device__ __forceinline__ float gelu_ggml(float x) {
  const float f = __half2float(__float2half_rn(x));
  const float inner = __fadd_rn(1.0f, __fmul_rn(__fmul_rn(0.044715f, f), f));
  const float t = tanhf(__fmul_rn(__fmul_rn(0.79788456080286535587989211986876f, f), inner));
  const float g = __half2float(__float2half_rn(__fmul_rn(__fmul_rn(0.5f, f), __fadd_rn(1.0f, t))));
  return x >= 10.0f ? x : (x <= -10.0f ? 0.0f : g);
}

}  // namespace b2q
