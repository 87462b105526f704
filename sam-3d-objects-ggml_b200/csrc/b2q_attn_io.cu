// b2q_attn_io.cu -- the tensors on either side of the DiT self-attention core
// (cpp_ggml/src/ss_flow_graph.cpp:206-290, graph_builder.cpp:70-175):
//
//   qkv_heads:  the fused qkv projection output fp32 [B*T][3C] (C = H*D) ->
//               q, k, v as fp16 [B][H][T][D]; q and k go through the
//               per-head RMS norm with gamma first (gb_rms_norm_head:
//               ggml_rms_norm then ggml_mul by gamma[h][d]).  fp16 is the K/V
//               representation of the reference's flash-attention path
//               (gb_attention casts K and V to F16; the CPU kernel takes Q to
//               F16 for its K dots).
//   heads_q8:   the attention output o[b][h][t][d] (fp16, any strides) ->
//               the Q8_0 prepared activations of the output projection, rows
//               (b, t), K = H*D.  Every 32-value block lies inside one head
//               (D % 32 == 0), so a block is 32 contiguous d of one (b, h, t).
//
// RMS norm arithmetic (ggml_rms_norm, CPU backend): sum of x*x in double, mean
// = sum / D, scale = 1 / sqrtf(mean + eps) in float, y = x * scale, then
// y * gamma (ggml_mul), each one IEEE fp32 operation; fp16 conversion rounds
// to nearest even.  The double sums are exact for ordinary data, so the
// warp's order gives the sequential loop's value.
#include <cuda_fp16.h>

#include "b2q_internal.h"
#include "b2q_q8.cuh"

namespace b2q {

namespace {

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per (row, head); lane l holds d = l + 32 i (i < D / 32).  The row
// holds `parts` C-wide tensors (q, k, v of a fused projection, or fewer);
// part p goes to out[p] as fp16 [B][H][T][D], RMS-normed first when bit p of
// norm_mask is set (times gamma[p] when that is not null).
__device__ __forceinline__ void store_out(__half* p, float v) { *p = __float2half_rn(v); }
__device__ __forceinline__ void store_out(float* p, float v) { *p = v; }

template <int DPL, typename OutT>  // values per lane = D / 32; OutT: __half (rounded) or float
__global__ void __launch_bounds__(256) rows_to_heads_kernel(const float* __restrict__ qkv, int64_t rows, int64_t T,
                                                            int H, int64_t ldq, int parts, unsigned norm_mask,
                                                            const float* __restrict__ gq,
                                                            const float* __restrict__ gk, float eps,
                                                            OutT* __restrict__ q16, OutT* __restrict__ k16,
                                                            OutT* __restrict__ v16) {
  const int lane = threadIdx.x & 31;
  constexpr int D = DPL * 32;
  const int64_t C = static_cast<int64_t>(H) * D;
  const int64_t units = rows * H;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t u = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; u < units; u += warps) {
    const int64_t r = u / H;
    const int h = static_cast<int>(u - r * H);
    const int64_t b = r / T, t = r - b * T;
    const int64_t dst = ((b * H + h) * T + t) * D;
    const float* src = qkv + r * ldq + static_cast<int64_t>(h) * D;
    for (int part = 0; part < parts; ++part) {  // q, k, v
      float x[DPL];
#pragma unroll
      for (int i = 0; i < DPL; ++i) x[i] = __ldg(src + part * C + lane + 32 * i);
      OutT* out = part == 0 ? q16 : part == 1 ? k16 : v16;
      if ((norm_mask >> part) & 1u) {
        double s = 0.0;
#pragma unroll
        for (int i = 0; i < DPL; ++i) s += static_cast<double>(__fmul_rn(x[i], x[i]));
        s = warp_sum_d(s);
        const float mean = __double2float_rn(__ddiv_rn(s, static_cast<double>(D)));
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
        const float* g0 = part == 0 ? gq : gk;
        const float* g = g0 ? g0 + static_cast<int64_t>(h) * D : nullptr;
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          float y = __fmul_rn(x[i], scale);
          if (g) y = __fmul_rn(y, __ldg(g + lane + 32 * i));
          x[i] = y;
        }
      }
#pragma unroll
      for (int i = 0; i < DPL; ++i) store_out(out + dst + lane + 32 * i, x[i]);
    }
  }
}

// D = 64 (16 heads of C 1024): a warp takes two heads of one row, 16 lanes
// each, lane holding d = 4 (l % 16) .. + 3: one 512-byte float4 load per part
// and 8-byte fp16 stores (each head's 128-byte output row contiguous).  The
// double sum of squares is exact for ordinary data, so the 16-lane tree gives
// the same value as the 32-lane layout above.  Index math in 32 bits.
template <typename OutT>
__global__ void __launch_bounds__(256) rows_to_heads64_kernel(const float* __restrict__ qkv, uint32_t rows, uint32_t T,
                                                              uint32_t H, int64_t ldq, int parts, unsigned norm_mask,
                                                              const float* __restrict__ gq,
                                                              const float* __restrict__ gk, float eps,
                                                              OutT* __restrict__ q16, OutT* __restrict__ k16,
                                                              OutT* __restrict__ v16) {
  constexpr int D = 64;
  const int lane = threadIdx.x & 31;
  const int sub = lane >> 4, l16 = lane & 15;
  const int64_t C = static_cast<int64_t>(H) * D;
  const uint32_t hpairs = H / 2;
  const uint32_t units = rows * hpairs;
  const uint32_t warps = gridDim.x * (blockDim.x / 32);
  for (uint32_t u = (blockIdx.x * blockDim.x + threadIdx.x) / 32; u < units; u += warps) {
    const uint32_t r = u / hpairs;
    const uint32_t h = (u - r * hpairs) * 2 + sub;
    const uint32_t b = r / T, t = r - b * T;
    const int64_t dst = ((static_cast<int64_t>(b) * H + h) * T + t) * D + 4 * l16;
    const float* src = qkv + static_cast<int64_t>(r) * ldq + static_cast<int64_t>(h) * D + 4 * l16;
    for (int part = 0; part < parts; ++part) {  // q, k, v
      float4 x = __ldg(reinterpret_cast<const float4*>(src + part * C));
      OutT* out = part == 0 ? q16 : part == 1 ? k16 : v16;
      if ((norm_mask >> part) & 1u) {
        double s = static_cast<double>(__fmul_rn(x.x, x.x)) + static_cast<double>(__fmul_rn(x.y, x.y)) +
                   static_cast<double>(__fmul_rn(x.z, x.z)) + static_cast<double>(__fmul_rn(x.w, x.w));
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);  // within the 16 lanes
        const float mean = __double2float_rn(__ddiv_rn(s, static_cast<double>(D)));
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
        x.x = __fmul_rn(x.x, scale), x.y = __fmul_rn(x.y, scale), x.z = __fmul_rn(x.z, scale);
        x.w = __fmul_rn(x.w, scale);
        const float* g0 = part == 0 ? gq : gk;
        if (g0) {
          const float4 g = __ldg(reinterpret_cast<const float4*>(g0 + static_cast<int64_t>(h) * D + 4 * l16));
          x.x = __fmul_rn(x.x, g.x), x.y = __fmul_rn(x.y, g.y), x.z = __fmul_rn(x.z, g.z), x.w = __fmul_rn(x.w, g.w);
        }
      }
      if constexpr (sizeof(OutT) == 4) {
        *reinterpret_cast<float4*>(out + dst) = x;
      } else {
        __half2 lo = __floats2half2_rn(x.x, x.y), hi = __floats2half2_rn(x.z, x.w);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&lo);
        pk.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(out + dst) = pk;
      }
    }
  }
}

// One lane per (row, block): 32 contiguous fp16 of one head -> one Q8_0 block
// (the stand-alone quantizer's arithmetic on their fp32 values).
// Consecutive lanes take consecutive blocks of one token row: the attention
// output is token-major in memory, so a warp's loads are contiguous (a
// row-group mapping, with coalesced scale stores instead, measured slower).
template <int VARIANT>
__global__ void __launch_bounds__(256) heads_q8_kernel(const __half* __restrict__ o, int64_t rows, int64_t T,
                                                       int H, int D, int64_t sb, int64_t sh, int64_t st,
                                                       int8_t* __restrict__ codes, float* __restrict__ scales,
                                                       int64_t ld) {
  const int64_t kb = static_cast<int64_t>(H) * D / kQK;
  const int64_t units = rows * kb;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < units;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = u / kb, j = u - r * kb;
    const int64_t b = r / T, t = r - b * T;
    const int64_t c0 = j * kQK;
    const int h = static_cast<int>(c0 / D), d0 = static_cast<int>(c0 - static_cast<int64_t>(h) * D);
    const __half* src = o + b * sb + h * sh + t * st + d0;
    float v[kQK];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < kQK; ++i) {
      v[i] = __half2float(src[i]);
      amax = fmaxf(amax, fabsf(v[i]));
    }
    float d, inv;
    q8_scale<VARIANT>(amax, d, inv);
    uint32_t q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      q[i] = quantize_code<VARIANT>(v[4 * i], inv) | (quantize_code<VARIANT>(v[4 * i + 1], inv) << 8) |
             (quantize_code<VARIANT>(v[4 * i + 2], inv) << 16) | (quantize_code<VARIANT>(v[4 * i + 3], inv) << 24);
    uint4* dst = reinterpret_cast<uint4*>(codes + r * (kb * kQK) + c0);
    dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
    dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
    scales[j * ld + r] = q8_split_scale(d);
  }
}

int grid_for(int64_t work_items, int per_block, int cap_per_sm) {
  int sms = current_device_sms();
  if (sms <= 0) sms = 148;
  const int64_t blocks = (work_items + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(sms) * cap_per_sm;
  return static_cast<int>(blocks < cap ? blocks : cap);
}

template <typename OutT>
cudaError_t rows_to_heads_t(const float* src, int64_t B, int64_t T, int H, int D, int64_t ld_floats, int parts,
                            unsigned norm_mask, const float* g0, const float* g1, float eps, void* o0, void* o1,
                            void* o2, cudaStream_t s) {
  const int64_t rows = B * T;
  if (rows == 0) return cudaSuccess;
  if (parts < 1 || parts > 3 || (norm_mask >> 2) != 0) return cudaErrorInvalidValue;  // v is never normed
  const int grid = grid_for(rows * H, 8, 16);
  OutT *a = static_cast<OutT*>(o0), *b = static_cast<OutT*>(o1), *c = static_cast<OutT*>(o2);
  switch (D) {
    case 32:
      rows_to_heads_kernel<1, OutT><<<grid, 256, 0, s>>>(src, rows, T, H, ld_floats, parts, norm_mask, g0, g1, eps, a,
                                                         b, c);
      break;
    case 64:
      if (H % 2 == 0 && ld_floats % 4 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
          (!g0 || reinterpret_cast<uintptr_t>(g0) % 16 == 0) && (!g1 || reinterpret_cast<uintptr_t>(g1) % 16 == 0) &&
          rows * H <= 0xffffffffLL)
        rows_to_heads64_kernel<OutT><<<grid_for(rows * H / 2, 8, 16), 256, 0, s>>>(
            src, static_cast<uint32_t>(rows), static_cast<uint32_t>(T), static_cast<uint32_t>(H), ld_floats, parts,
            norm_mask, g0, g1, eps, a, b, c);
      else
        rows_to_heads_kernel<2, OutT><<<grid, 256, 0, s>>>(src, rows, T, H, ld_floats, parts, norm_mask, g0, g1, eps,
                                                           a, b, c);
      break;
    case 128:
      rows_to_heads_kernel<4, OutT><<<grid, 256, 0, s>>>(src, rows, T, H, ld_floats, parts, norm_mask, g0, g1, eps, a,
                                                         b, c);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_rows_to_heads(const float* src, int64_t B, int64_t T, int H, int D, int64_t ld_floats, int parts,
                                 unsigned norm_mask, const float* g0, const float* g1, float eps, void* o0, void* o1,
                                 void* o2, cudaStream_t s, bool f32_out) {
  return f32_out ? rows_to_heads_t<float>(src, B, T, H, D, ld_floats, parts, norm_mask, g0, g1, eps, o0, o1, o2, s)
                 : rows_to_heads_t<__half>(src, B, T, H, D, ld_floats, parts, norm_mask, g0, g1, eps, o0, o1, o2, s);
}

cudaError_t launch_heads_q8(const void* o16, int64_t B, int64_t T, int H, int D, int64_t sb, int64_t sh,
                            int64_t st, int8_t* codes, float* scales, int64_t ld, int variant, cudaStream_t s) {
  const int64_t rows = B * T;
  if (rows == 0) return cudaSuccess;
  const int grid = grid_for(rows * H * D / kQK, 256, 8);
  const __half* o = static_cast<const __half*>(o16);
  if (variant == 0)
    heads_q8_kernel<0><<<grid, 256, 0, s>>>(o, rows, T, H, D, sb, sh, st, codes, scales, ld);
  else
    heads_q8_kernel<1><<<grid, 256, 0, s>>>(o, rows, T, H, D, sb, sh, st, codes, scales, ld);
  return cudaGetLastError();
}

}  // namespace b2q
