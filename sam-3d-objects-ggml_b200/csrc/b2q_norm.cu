// b2q_norm.cu -- the pre-norm of the DiT blocks: ggml_norm (LayerNorm without
// affine, eps 1e-6) followed by the adaLN modulate h*(1+scale) + shift, with
// the Q8_0 quantize of the next mul_mat fused in (cpp_ggml/src/ss_flow_graph.cpp:
// 45-53 modulate, :200-204 and :378-379 its uses; graph_builder.cpp:62-68
// gb_layer_norm).  HBM-bound: one fp32 read of the row, one Q8_0 (or fp32)
// write.
//
// Arithmetic per row of c values (each step one IEEE fp32 operation unless
// marked double):
//   sum   = sum of x                       (double; cast to float)
//   mean  = sum / c                        (float)
//   v     = x - mean                       (float)
//   var   = (sum of v*v) / c               (v*v in float, the sum and the division in double; cast to float)
//   scale = 1 / sqrtf(var + eps)
//   h     = v * scale
//   h     = (h * mod_scale + h) + mod_shift        (ggml_add(ggml_mul(h, s), h), then ggml_add(., shift))
// The double sums are exact for ordinary data (their terms span far fewer than
// 53 bits), so the warp's tree order gives the same value as a sequential loop.
//
// Mapping: one warp per row; lane l holds blocks l, l+32, ... of the row (32
// consecutive values each) in registers, so the quantize of a block needs no
// cross-lane work, and the codes of a row leave as contiguous 16-byte stores.
#include "b2q_internal.h"
#include "b2q_q8.cuh"

#include <cuda_fp16.h>

namespace b2q {

namespace {

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// KB: blocks per lane (c <= 1024 * KB).  Q8: write the split-layout Q8_0
// activations (VARIANT = quantizer variant), else fp32 y.
template <int KB, bool Q8, int VARIANT>
__global__ void __launch_bounds__(256) norm_modulate_kernel(const float* __restrict__ x, int64_t m, int c,
                                                            int64_t ldx, float eps,
                                                            const float* __restrict__ mscale,
                                                            const float* __restrict__ mshift,
                                                            float* __restrict__ y, int64_t ldy,
                                                            int8_t* __restrict__ codes,
                                                            float* __restrict__ qscales, int64_t qld) {
  const int lane = threadIdx.x & 31;
  const int nb = c / kQK;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; row < m; row += warps) {
    const float* xr = x + row * ldx;
    float v[KB][kQK];
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < KB; ++i) {
      const int b = lane + 32 * i;
      if (b < nb) {
        const float4* p = reinterpret_cast<const float4*>(xr + b * kQK);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 q = __ldg(p + j);
          v[i][4 * j] = q.x;
          v[i][4 * j + 1] = q.y;
          v[i][4 * j + 2] = q.z;
          v[i][4 * j + 3] = q.w;
        }
#pragma unroll
        for (int j = 0; j < kQK; ++j) s += static_cast<double>(v[i][j]);
      }
    }
    s = warp_sum(s);
    const float mean = __fdiv_rn(__double2float_rn(s), static_cast<float>(c));
    double s2 = 0.0;
#pragma unroll
    for (int i = 0; i < KB; ++i) {
      if (lane + 32 * i < nb) {
#pragma unroll
        for (int j = 0; j < kQK; ++j) {
          const float d = __fsub_rn(v[i][j], mean);
          v[i][j] = d;
          s2 += static_cast<double>(__fmul_rn(d, d));
        }
      }
    }
    s2 = warp_sum(s2);
    const float var = __double2float_rn(__ddiv_rn(s2, static_cast<double>(c)));
    const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
    for (int i = 0; i < KB; ++i) {
      const int b = lane + 32 * i;
      if (b >= nb) continue;
#pragma unroll
      for (int j = 0; j < kQK; ++j) {
        float h = __fmul_rn(v[i][j], rs);
        if (mscale) h = __fadd_rn(__fmul_rn(h, __ldg(mscale + b * kQK + j)), h);
        if (mshift) h = __fadd_rn(h, __ldg(mshift + b * kQK + j));
        v[i][j] = h;
      }
      if (Q8) {
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < kQK; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
        float d, inv;
        q8_scale<VARIANT>(amax, d, inv);
        uint32_t q[8];
#pragma unroll
        for (int t = 0; t < 8; ++t)
          q[t] = quantize_code<VARIANT>(v[i][4 * t], inv) | (quantize_code<VARIANT>(v[i][4 * t + 1], inv) << 8) |
                 (quantize_code<VARIANT>(v[i][4 * t + 2], inv) << 16) |
                 (quantize_code<VARIANT>(v[i][4 * t + 3], inv) << 24);
        uint4* dst = reinterpret_cast<uint4*>(codes + row * static_cast<int64_t>(c) + b * kQK);
        dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
        dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
        qscales[b * qld + row] = q8_split_scale(d);
      } else {
        float4* dst = reinterpret_cast<float4*>(y + row * ldy + b * kQK);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          dst[j] = make_float4(v[i][4 * j], v[i][4 * j + 1], v[i][4 * j + 2], v[i][4 * j + 3]);
      }
    }
  }
}

template <int KB, bool Q8, int VARIANT>
cudaError_t launch_kb(const float* x, int64_t m, int c, int64_t ldx, float eps, const float* ms, const float* sh,
                      float* y, int64_t ldy, int8_t* codes, float* qs, int64_t qld, cudaStream_t s) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = (m + 7) / 8;  // 8 rows (warps) per block
  const int cap = sms * (KB == 1 ? 8 : KB == 2 ? 4 : 2);
  const int grid = static_cast<int>(blocks < cap ? blocks : cap);
  norm_modulate_kernel<KB, Q8, VARIANT><<<grid, 256, 0, s>>>(x, m, c, ldx, eps, ms, sh, y, ldy, codes, qs, qld);
  return cudaGetLastError();
}

template <bool Q8, int VARIANT>
cudaError_t launch_q(const float* x, int64_t m, int c, int64_t ldx, float eps, const float* ms, const float* sh,
                     float* y, int64_t ldy, int8_t* codes, float* qs, int64_t qld, cudaStream_t s) {
  if (c <= 1024) return launch_kb<1, Q8, VARIANT>(x, m, c, ldx, eps, ms, sh, y, ldy, codes, qs, qld, s);
  if (c <= 2048) return launch_kb<2, Q8, VARIANT>(x, m, c, ldx, eps, ms, sh, y, ldy, codes, qs, qld, s);
  return launch_kb<4, Q8, VARIANT>(x, m, c, ldx, eps, ms, sh, y, ldy, codes, qs, qld, s);
}

}  // namespace

cudaError_t launch_norm_modulate(const float* x, int64_t m, int64_t c, int64_t ldx_floats, float eps,
                                 const float* mscale, const float* mshift, float* y, int64_t ldy_floats,
                                 int8_t* codes, float* qscales, int64_t qld, int variant, cudaStream_t s) {
  if (m == 0) return cudaSuccess;
  if (c <= 0 || c % kQK != 0 || c > kNormMaxC) return cudaErrorInvalidValue;
  const int ci = static_cast<int>(c);
  if (!codes) return launch_q<false, 0>(x, m, ci, ldx_floats, eps, mscale, mshift, y, ldy_floats, nullptr, nullptr, 0, s);
  if (variant == 0)
    return launch_q<true, 0>(x, m, ci, ldx_floats, eps, mscale, mshift, nullptr, 0, codes, qscales, qld, s);
  return launch_q<true, 1>(x, m, ci, ldx_floats, eps, mscale, mshift, nullptr, 0, codes, qscales, qld, s);
}

}  // namespace b2q
