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
//   or, as gb_layer_norm with affine weight and bias (the cross-attention's norm2),
//   h     = (h * weight) + bias                    (ggml_mul, then ggml_add)
// The double sums are exact for ordinary data (their terms span far fewer than
// 53 bits), so the warp's tree order gives the same value as a sequential loop.
//
// Mapping: one warp per row.  Lane l holds the float4 groups 32*j + l of the
// row (j = 0 .. c/128 - 1): every load, modulation read and store of a warp is
// one contiguous 512-byte run.  A Q8_0 block is then 8 consecutive lanes, whose
// absmax takes three xor-shuffles within the group.  For c <= 1024 the warps
// are persistent and each copies its next row into shared memory (cp.async,
// two buffers per warp) while it works on the current one, so the row's load
// latency is off the per-row chain.  When c is a power of two the two
// divisions by c are multiplications by its exact reciprocal (the same
// correctly rounded value).
#include "b2q_internal.h"
#include "b2q_q8.cuh"

#include <cuda_fp16.h>

namespace b2q {

namespace {

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// This lane's float4 groups of row `row` into buf (one commit group, empty
// past the last row).
template <int NJ>
__device__ __forceinline__ void norm_prefetch(const float* __restrict__ x, int64_t row, int64_t m, int64_t ldx,
                                              int ng, int lane, float4* buf) {
  if (row < m) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * ldx);
#pragma unroll
    for (int j = 0; j < NJ; ++j)
      if (32 * j + lane < ng) cp_async16(buf + 32 * j + lane, xr + 32 * j + lane);
  }
  cp_async_commit();
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// NJ: float4 groups per lane (c <= 128 * NJ).  Q8: write the split-layout Q8_0
// activations (VARIANT = quantizer variant), else fp32 y.  PIPE: persistent
// warps, next row prefetched into shared memory (2 * 32 * NJ float4 per warp).
// pow2: c is a power of two.
template <int NJ, bool Q8, int VARIANT, bool PIPE>
__global__ void __launch_bounds__(256, PIPE ? 2 : 1) norm_modulate_kernel(const float* __restrict__ x, int64_t m, int c,
                                                            int64_t ldx, float eps,
                                                            const float* __restrict__ mscale,
                                                            const float* __restrict__ mshift,
                                                            float* __restrict__ y, int64_t ldy,
                                                            int8_t* __restrict__ codes,
                                                            float* __restrict__ qscales, int64_t qld,
                                                            bool affine, bool pow2) {
  extern __shared__ float4 norm_rows[];  // PIPE: [warp][2][32 * NJ]
  const int lane = threadIdx.x & 31;
  const int ng = c / 4;  // float4 groups per row
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  const float rcf = __frcp_rn(static_cast<float>(c));   // exact when pow2
  const double rcd = __drcp_rn(static_cast<double>(c));
  float4* rows = PIPE ? norm_rows + (threadIdx.x >> 5) * 2 * 32 * NJ : nullptr;
  int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  if (PIPE) norm_prefetch<NJ>(x, row, m, ldx, ng, lane, rows);
  for (int b = 0; row < m; row += warps, b ^= 1) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * ldx);
    if (PIPE) {
      // Next row into the other buffer, then wait for this row's copies (each
      // lane reads back only what it copied).
      norm_prefetch<NJ>(x, row + warps, m, ldx, ng, lane, rows + (b ^ 1) * 32 * NJ);
      cp_async_wait<1>();
    }
    float4 v[NJ];
    double s[4] = {0.0, 0.0, 0.0, 0.0};  // four chains; the sums are exact, so their order is free
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int g = 32 * j + lane;
      v[j] = g < ng ? (PIPE ? rows[b * 32 * NJ + g] : __ldg(xr + g)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      s[0] += static_cast<double>(v[j].x);
      s[1] += static_cast<double>(v[j].y);
      s[2] += static_cast<double>(v[j].z);
      s[3] += static_cast<double>(v[j].w);
    }
    const double st = warp_sum((s[0] + s[1]) + (s[2] + s[3]));
    const float mean =
        pow2 ? __fmul_rn(__double2float_rn(st), rcf) : __fdiv_rn(__double2float_rn(st), static_cast<float>(c));
    double q[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      if (32 * j + lane < ng) {
        v[j] = make_float4(__fsub_rn(v[j].x, mean), __fsub_rn(v[j].y, mean), __fsub_rn(v[j].z, mean),
                           __fsub_rn(v[j].w, mean));
        q[0] += static_cast<double>(__fmul_rn(v[j].x, v[j].x));
        q[1] += static_cast<double>(__fmul_rn(v[j].y, v[j].y));
        q[2] += static_cast<double>(__fmul_rn(v[j].z, v[j].z));
        q[3] += static_cast<double>(__fmul_rn(v[j].w, v[j].w));
      }
    }
    const double qt = warp_sum((q[0] + q[1]) + (q[2] + q[3]));
    const float var = __double2float_rn(pow2 ? __dmul_rn(qt, rcd) : __ddiv_rn(qt, static_cast<double>(c)));
    const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    // Each phase runs over all of the lane's groups before the next, so the
    // groups' chains (modulation loads, absmax shuffles, scale divisions)
    // overlap.  A group's 8 lanes (one Q8_0 block) are all in or all out.
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int g = 32 * j + lane;
      const bool in = g < ng;
      float4 h = make_float4(__fmul_rn(v[j].x, rs), __fmul_rn(v[j].y, rs), __fmul_rn(v[j].z, rs),
                             __fmul_rn(v[j].w, rs));
      if (mscale && in) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(mscale) + g);
        if (affine) {  // gb_layer_norm's weight: ggml_mul
          h = make_float4(__fmul_rn(h.x, t.x), __fmul_rn(h.y, t.y), __fmul_rn(h.z, t.z), __fmul_rn(h.w, t.w));
        } else {       // modulate: ggml_add(ggml_mul(h, scale), h)
          h = make_float4(__fadd_rn(__fmul_rn(h.x, t.x), h.x), __fadd_rn(__fmul_rn(h.y, t.y), h.y),
                          __fadd_rn(__fmul_rn(h.z, t.z), h.z), __fadd_rn(__fmul_rn(h.w, t.w), h.w));
        }
      }
      if (mshift && in) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(mshift) + g);
        h = make_float4(__fadd_rn(h.x, t.x), __fadd_rn(h.y, t.y), __fadd_rn(h.z, t.z), __fadd_rn(h.w, t.w));
      }
      v[j] = h;
    }
    if (Q8) {
      float amax[NJ];
#pragma unroll
      for (int j = 0; j < NJ; ++j)
        amax[j] = fmaxf(fmaxf(0.0f, fmaxf(fabsf(v[j].x), fabsf(v[j].y))), fmaxf(fabsf(v[j].z), fabsf(v[j].w)));
#pragma unroll
      for (int o = 1; o < 8; o <<= 1)
#pragma unroll
        for (int j = 0; j < NJ; ++j) amax[j] = fmaxf(amax[j], __shfl_xor_sync(0xffffffffu, amax[j], o));
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int g = 32 * j + lane;
        float d, inv;
        q8_scale<VARIANT>(amax[j], d, inv);
        const uint32_t word = quantize_code<VARIANT>(v[j].x, inv) | (quantize_code<VARIANT>(v[j].y, inv) << 8) |
                              (quantize_code<VARIANT>(v[j].z, inv) << 16) | (quantize_code<VARIANT>(v[j].w, inv) << 24);
        if (g < ng) {
          reinterpret_cast<uint32_t*>(codes + row * static_cast<int64_t>(c))[g] = word;
          if ((lane & 7) == 0) qscales[(g / 8) * qld + row] = q8_split_scale(d);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < NJ; ++j)
        if (32 * j + lane < ng) reinterpret_cast<float4*>(y + row * ldy)[32 * j + lane] = v[j];
    }
  }
  if (PIPE) cp_async_wait<0>();  // the last (empty) prefetch group
}

template <int NJ, bool Q8, int VARIANT>
cudaError_t launch_kb(const float* x, int64_t m, int c, int64_t ldx, float eps, const float* ms, const float* sh,
                      float* y, int64_t ldy, int8_t* codes, float* qs, int64_t qld, bool affine, cudaStream_t s) {
  int sms = current_device_sms();
  if (sms <= 0) sms = 148;
  const int64_t blocks = (m + 7) / 8;  // 8 rows (warps) per block
  const bool pow2 = (c & (c - 1)) == 0;
  if constexpr (NJ == 8) {  // persistent warps, two resident blocks per SM, rows prefetched
    constexpr int smem = 8 * 2 * 32 * 8 * 16;
    auto kern = norm_modulate_kernel<8, Q8, VARIANT, true>;
    static bool attr_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      attr_set[dev] = true;
    }
    const int cap = sms * 2;
    const int grid = static_cast<int>(blocks < cap ? blocks : cap);
    kern<<<grid, 256, smem, s>>>(x, m, c, ldx, eps, ms, sh, y, ldy, codes, qs, qld, affine, pow2);
    return cudaGetLastError();
  } else {
    const int cap = sms * (NJ <= 16 ? 4 : 2);
    const int grid = static_cast<int>(blocks < cap ? blocks : cap);
    norm_modulate_kernel<NJ, Q8, VARIANT, false><<<grid, 256, 0, s>>>(x, m, c, ldx, eps, ms, sh, y, ldy, codes, qs,
                                                                       qld, affine, pow2);
    return cudaGetLastError();
  }
}

template <bool Q8, int VARIANT>
cudaError_t launch_q(const float* x, int64_t m, int c, int64_t ldx, float eps, const float* ms, const float* sh,
                     float* y, int64_t ldy, int8_t* codes, float* qs, int64_t qld, bool affine, cudaStream_t s) {
  if (c <= 1024) return launch_kb<8, Q8, VARIANT>(x, m, c, ldx, eps, ms, sh, y, ldy, codes, qs, qld, affine, s);
  if (c <= 2048) return launch_kb<16, Q8, VARIANT>(x, m, c, ldx, eps, ms, sh, y, ldy, codes, qs, qld, affine, s);
  return launch_kb<32, Q8, VARIANT>(x, m, c, ldx, eps, ms, sh, y, ldy, codes, qs, qld, affine, s);
}

}  // namespace

cudaError_t launch_norm_modulate(const float* x, int64_t m, int64_t c, int64_t ldx_floats, float eps,
                                 const float* mscale, const float* mshift, float* y, int64_t ldy_floats,
                                 int8_t* codes, float* qscales, int64_t qld, int variant, cudaStream_t s,
                                 bool affine) {
  if (m == 0) return cudaSuccess;
  if (c <= 0 || c % kQK != 0 || c > kNormMaxC) return cudaErrorInvalidValue;
  const int ci = static_cast<int>(c);
  if (!codes)
    return launch_q<false, 0>(x, m, ci, ldx_floats, eps, mscale, mshift, y, ldy_floats, nullptr, nullptr, 0, affine, s);
  if (variant == 0)
    return launch_q<true, 0>(x, m, ci, ldx_floats, eps, mscale, mshift, nullptr, 0, codes, qscales, qld, affine, s);
  return launch_q<true, 1>(x, m, ci, ldx_floats, eps, mscale, mshift, nullptr, 0, codes, qscales, qld, affine, s);
}

}  // namespace b2q
