// b2q_quantize.cu -- fp32 -> Q8_0 activation quantizer and the one-time GGUF
// weight re-layout.  Both are HBM-bound streaming kernels.
//
// Activation quantizer (ggml CPU from_float for GGML_TYPE_Q8_0, applied to
// every src1 row of GGML_OP_MUL_MAT): per 32-value block
//     amax = max |x|,  d = amax / 127  (stored as fp16, round to nearest even)
//     B2Q_ACT_X86: inverse = 127 / amax, code = round-half-even(x * inverse)
//     B2Q_ACT_REF: inverse = 1 / d,      code = round-half-away(x * inverse)
// Each division, product and rounding is one IEEE fp32 operation, so the codes
// and scales are bit-identical to the CPU's.
//
// Mapping: one lane per 32-value block, a warp per 32 rows x 1 block (see
// quantize_q8_0_kernel).
#include "b2q_internal.h"
#include "b2q_ptx.cuh"
#include "b2q_q8.cuh"

#include <cuda_fp16.h>

namespace b2q {

namespace {

template <bool VEC4>
__device__ __forceinline__ float4 load4(const float* p) {
  if (VEC4) return __ldg(reinterpret_cast<const float4*>(p));
  return make_float4(__ldg(p), __ldg(p + 1), __ldg(p + 2), __ldg(p + 3));
}

// One lane quantizes one whole 32-value block: lane i of a warp takes row
// 32*rg + i, so a warp covers one block column of 32 consecutive rows.  The
// block's absmax, scale and inverse are computed once (no cross-lane work and
// no per-lane duplicates), the 32 codes leave as two 16-byte stores, and the
// 32 lanes' scales of the split layout form one coalesced 128-byte store.
// Work units (row group, block) are spread over the grid's warps; all eight
// 16-byte loads of a unit are issued before any arithmetic.
template <int VARIANT, bool SPLIT, bool VEC4>
__global__ void __launch_bounds__(256) quantize_q8_0_kernel(const float* __restrict__ x, int64_t m,
                                                            int64_t k, int64_t ldx,
                                                            uint8_t* __restrict__ yb, int64_t ldy,
                                                            int8_t* __restrict__ codes,
                                                            float* __restrict__ scales, int64_t ld) {
  const int lane = threadIdx.x & 31;
  const int64_t kb = k / kQK;
  const int64_t units = (m + 31) / 32 * kb;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t u = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; u < units; u += warps) {
    const int64_t rg = u / kb;
    const int64_t b = u - rg * kb;
    const int64_t row = rg * 32 + lane;
    if (row >= m) continue;
    const float* src = x + row * ldx + b * kQK;
    float4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = load4<VEC4>(src + 4 * i);
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    float d, inv;
    q8_scale<VARIANT>(amax, d, inv);
    uint32_t q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      q[i] = quantize_code<VARIANT>(v[i].x, inv) | (quantize_code<VARIANT>(v[i].y, inv) << 8) |
             (quantize_code<VARIANT>(v[i].z, inv) << 16) | (quantize_code<VARIANT>(v[i].w, inv) << 24);
    const __half dh = __float2half_rn(d);
    if (SPLIT) {
      uint4* dst = reinterpret_cast<uint4*>(codes + row * k + b * kQK);
      dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
      dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
      scales[b * ld + row] = q8_split_scale(d);
    } else {
      // ggml block_q8_0: fp16 d then 32 codes; 34-byte blocks are 2-byte aligned
      uint16_t* dst = reinterpret_cast<uint16_t*>(yb + row * ldy + b * kQ8Bytes);
      dst[0] = __half_as_ushort(dh);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dst[1 + 2 * i] = static_cast<uint16_t>(q[i] & 0xffffu);
        dst[2 + 2 * i] = static_cast<uint16_t>(q[i] >> 16);
      }
    }
  }
}

template <bool SPLIT, bool VEC4>
cudaError_t launch_q(const float* x, int64_t m, int64_t k, int64_t ldx, uint8_t* yb, int64_t ldy,
                     int8_t* codes, float* scales, int64_t ld, int variant, cudaStream_t s) {
  const int64_t units = (m + 31) / 32 * (k / kQK);
  if (units == 0) return cudaSuccess;
  int sms = current_device_sms();
  if (sms <= 0) sms = 148;
  // 8 warps per block; at most 8 resident blocks per SM, one unit per warp when that fits
  const int64_t blocks_needed = (units + 7) / 8;
  const int grid = static_cast<int>(blocks_needed < sms * 8 ? blocks_needed : sms * 8);
  if (variant == 0)
    quantize_q8_0_kernel<0, SPLIT, VEC4><<<grid, 256, 0, s>>>(x, m, k, ldx, yb, ldy, codes, scales, ld);
  else
    quantize_q8_0_kernel<1, SPLIT, VEC4><<<grid, 256, 0, s>>>(x, m, k, ldx, yb, ldy, codes, scales, ld);
  return cudaGetLastError();
}

// ------------------------------------------------------------------- GELU
// y = gelu_ggml(x) elementwise over rows x cols (row pitches in floats).  Each
// thread takes 4 consecutive values of a row; 16-byte loads and stores when
// both pitches and bases allow (cols % 4 == 0 is required by the caller then).
template <bool VEC4>
__global__ void __launch_bounds__(256) gelu_kernel(const float* x, int64_t rows, int64_t cols, int64_t ldx,
                                                   float* y, int64_t ldy) {  // x == y allowed: no __restrict__
  const int64_t quads = (cols + 3) / 4;
  const int64_t total = rows * quads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / quads, c = (i - r * quads) * 4;
    if (VEC4) {
      const float4 v = *reinterpret_cast<const float4*>(x + r * ldx + c);
      *reinterpret_cast<float4*>(y + r * ldy + c) = make_float4(gelu_ggml(v.x), gelu_ggml(v.y), gelu_ggml(v.z),
                                                                gelu_ggml(v.w));
    } else {
      for (int64_t j = c; j < c + 4 && j < cols; ++j) y[r * ldy + j] = gelu_ggml(x[r * ldx + j]);
    }
  }
}

// ---------------------------------------------------------------- weights
// One thread per (row, block): raw GGUF block -> 32 int8 codes + fp32 scale
// (stored times 2^100, see b2q_internal.h).
template <int WTYPE>
__global__ void __launch_bounds__(256) pack_weights_kernel(const uint8_t* __restrict__ w, int64_t n,
                                                           int64_t k, int64_t ldw,
                                                           int8_t* __restrict__ codes,
                                                           float* __restrict__ scales, int64_t ld) {
  const int64_t kb = k / kQK;
  const int64_t total = n * kb;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / kb, b = i - row * kb;
    const uint8_t* blk = w + row * ldw + b * (WTYPE == kTypeQ8_0 ? kQ8Bytes : kQ4Bytes);
    const uint16_t* b16 = reinterpret_cast<const uint16_t*>(blk);
    const float d = __half2float(__ushort_as_half(b16[0]));
    uint32_t out[8];
    if (WTYPE == kTypeQ8_0) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        out[j] = static_cast<uint32_t>(b16[1 + 2 * j]) | (static_cast<uint32_t>(b16[2 + 2 * j]) << 16);
    } else {
      uint32_t nib[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        nib[j] = static_cast<uint32_t>(b16[1 + 2 * j]) | (static_cast<uint32_t>(b16[2 + 2 * j]) << 16);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // elements 4j..4j+3: low nibbles; elements 16+4j..: high nibbles; value - 8
        out[j] = __vsub4(nib[j] & 0x0f0f0f0fu, 0x08080808u);
        out[4 + j] = __vsub4((nib[j] >> 4) & 0x0f0f0f0fu, 0x08080808u);
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(codes + row * k + b * kQK);
    dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
    dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
    scales[b * ld + row] = d * kWeightScaleMul;
  }
}

// GGUF Q4_0 rows -> compact layout: one thread per (row, block) moves the 16
// nibble bytes to a 16-byte-aligned slot and the fp16 scale to the block-major
// scale table.
__global__ void __launch_bounds__(256) pack_q4c_kernel(const uint8_t* __restrict__ w, int64_t n, int64_t k,
                                                       int64_t ldw, uint8_t* __restrict__ nibbles,
                                                       uint16_t* __restrict__ scales, int64_t ld) {
  const int64_t kb = k / kQK;
  const int64_t total = n * kb;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / kb, b = i - row * kb;
    const uint16_t* b16 = reinterpret_cast<const uint16_t*>(w + row * ldw + b * kQ4Bytes);  // 18-byte blocks
    uint32_t q[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) q[j] = static_cast<uint32_t>(b16[1 + 2 * j]) | (static_cast<uint32_t>(b16[2 + 2 * j]) << 16);
    *reinterpret_cast<uint4*>(nibbles + row * (k / 2) + b * 16) = make_uint4(q[0], q[1], q[2], q[3]);
    scales[b * ld + row] = b16[0];
  }
}

}  // namespace

cudaError_t launch_pack_q4c(const uint8_t* w, int64_t n, int64_t k, int64_t ldw_bytes, uint8_t* nibbles,
                            uint16_t* scales, int64_t ld, cudaStream_t s) {
  const int64_t total = n * (k / kQK);
  if (total == 0) return cudaSuccess;
  int sms = current_device_sms();
  if (sms <= 0) sms = 148;
  const int64_t blocks = (total + 255) / 256;
  const int grid = static_cast<int>(blocks < sms * 16 ? blocks : sms * 16);
  pack_q4c_kernel<<<grid, 256, 0, s>>>(w, n, k, ldw_bytes, nibbles, scales, ld);
  return cudaGetLastError();
}

cudaError_t launch_quantize_q8_0_blocks(const float* x, int64_t m, int64_t k, int64_t ldx_floats,
                                        uint8_t* y, int64_t ldy_bytes, int variant, bool vec4,
                                        cudaStream_t s) {
  return vec4 ? launch_q<false, true>(x, m, k, ldx_floats, y, ldy_bytes, nullptr, nullptr, 0, variant, s)
              : launch_q<false, false>(x, m, k, ldx_floats, y, ldy_bytes, nullptr, nullptr, 0, variant, s);
}

cudaError_t launch_quantize_q8_0_split(const float* x, int64_t m, int64_t k, int64_t ldx_floats,
                                       int8_t* codes, float* scales, int64_t ld, int variant,
                                       bool vec4, cudaStream_t s) {
  return vec4 ? launch_q<true, true>(x, m, k, ldx_floats, nullptr, 0, codes, scales, ld, variant, s)
              : launch_q<true, false>(x, m, k, ldx_floats, nullptr, 0, codes, scales, ld, variant, s);
}

cudaError_t launch_gelu(const float* x, int64_t rows, int64_t cols, int64_t ldx_floats, float* y,
                        int64_t ldy_floats, cudaStream_t s) {
  const int64_t total = rows * ((cols + 3) / 4);
  if (total == 0) return cudaSuccess;
  int sms = current_device_sms();
  if (sms <= 0) sms = 148;
  const int64_t blocks = (total + 255) / 256;
  const int grid = static_cast<int>(blocks < sms * 16 ? blocks : sms * 16);
  const bool vec4 = cols % 4 == 0 && ldx_floats % 4 == 0 && ldy_floats % 4 == 0 &&
                    reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0;
  if (vec4)
    gelu_kernel<true><<<grid, 256, 0, s>>>(x, rows, cols, ldx_floats, y, ldy_floats);
  else
    gelu_kernel<false><<<grid, 256, 0, s>>>(x, rows, cols, ldx_floats, y, ldy_floats);
  return cudaGetLastError();
}

// ------------------------------------------------------------------- Q4_K
// fp32 activations -> Q8_K (ggml's reference quantizer, per 256 values: the
// value of largest |x|, first in scan order, sets iscale = -127/max; codes
// min(127, round-half-even(iscale * x)); d = 1/iscale; all-zero blocks give
// d = 0 and zero codes): codes int8 [M][K], d fp32 [K/256][ld].  The block
// sums of block_q8_K are not stored: the Q4_K GEMM gets them from its third
// weight plane.  One warp per (row, 256-value block), 8 values per lane.
template <bool VEC4>
__global__ void __launch_bounds__(256) quantize_q8k_kernel(const float* __restrict__ x, int64_t m, int64_t k,
                                                           int64_t ldx, int8_t* __restrict__ codes,
                                                           float* __restrict__ dq, int64_t ld) {
  const int lane = threadIdx.x & 31;
  const int64_t nsb = k / kQKK;
  const int64_t units = m * nsb;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t u = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; u < units; u += warps) {
    const int64_t row = u / nsb, sb = u - row * nsb;
    const float* src = x + row * ldx + sb * kQKK + 8 * lane;
    float v[8];
    if (VEC4) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(src)), b = __ldg(reinterpret_cast<const float4*>(src) + 1);
      v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = __ldg(src + t);
    }
    float amax = 0.0f, mx = 0.0f;
    int idx = 1 << 30;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float ax = fabsf(v[t]);
      if (ax > amax) {
        amax = ax;
        mx = v[t];
        idx = 8 * lane + t;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
      const float om = __shfl_xor_sync(0xffffffffu, mx, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (oa > amax || (oa == amax && oi < idx)) {
        amax = oa;
        mx = om;
        idx = oi;
      }
    }
    float d = 0.0f;
    uint32_t q0 = 0, q1 = 0;
    if (amax != 0.0f) {
      const float iscale = __fdiv_rn(-127.0f, mx);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int c = min(127, __float2int_rn(__fmul_rn(iscale, v[t])));
        const uint32_t byte = static_cast<uint32_t>(c) & 0xffu;
        if (t < 4)
          q0 |= byte << (8 * t);
        else
          q1 |= byte << (8 * (t - 4));
      }
      d = __fdiv_rn(1.0f, iscale);
    }
    *reinterpret_cast<uint2*>(codes + row * k + sb * kQKK + 8 * lane) = make_uint2(q0, q1);
    if (lane == 0) dq[sb * ld + row] = d;
  }
}

cudaError_t launch_quantize_q8_k(const float* x, int64_t m, int64_t k, int64_t ldx_floats, int8_t* codes,
                                 float* dq, int64_t ld, bool vec4, cudaStream_t s) {
  const int64_t units = m * (k / kQKK);
  if (units == 0) return cudaSuccess;
  int sms = current_device_sms();
  if (sms <= 0) sms = 148;
  const int64_t blocks = (units + 7) / 8;
  const int grid = static_cast<int>(blocks < sms * 8 ? blocks : sms * 8);
  if (vec4)
    quantize_q8k_kernel<true><<<grid, 256, 0, s>>>(x, m, k, ldx_floats, codes, dq, ld);
  else
    quantize_q8k_kernel<false><<<grid, 256, 0, s>>>(x, m, k, ldx_floats, codes, dq, ld);
  return cudaGetLastError();
}

// fp32 -> fp16 rows, round to nearest even: the src1 conversion of ggml's
// mul_mat against F16 weights (vec_dot_type F16; the CPU backend's F16C
// conversion with rounding mode 0).  Eight values per thread, one 16-byte store.
template <bool VEC4>
__global__ void __launch_bounds__(256) to_f16_kernel(const float* __restrict__ x, int64_t m, int64_t k, int64_t ldx,
                                                     __half* __restrict__ y, int64_t ldy) {
  const int64_t per_row = k / 8;
  const int64_t units = m * per_row;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < units;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = u / per_row, c = (u - r * per_row) * 8;
    const float* src = x + r * ldx + c;
    float v[8];
    if (VEC4) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(src));
      const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
      v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __ldg(src + i);
    }
    uint4 o;
    __half2 h;
    h = __floats2half2_rn(v[0], v[1]);
    o.x = *reinterpret_cast<uint32_t*>(&h);
    h = __floats2half2_rn(v[2], v[3]);
    o.y = *reinterpret_cast<uint32_t*>(&h);
    h = __floats2half2_rn(v[4], v[5]);
    o.z = *reinterpret_cast<uint32_t*>(&h);
    h = __floats2half2_rn(v[6], v[7]);
    o.w = *reinterpret_cast<uint32_t*>(&h);
    *reinterpret_cast<uint4*>(y + r * ldy + c) = o;
  }
}

cudaError_t launch_to_f16(const float* x, int64_t m, int64_t k, int64_t ldx_floats, void* y, int64_t ldy,
                          bool vec4, cudaStream_t s) {
  const int64_t units = m * (k / 8);
  if (units == 0) return cudaSuccess;
  int sms = current_device_sms();
  if (sms <= 0) sms = 148;
  const int64_t blocks = (units + 255) / 256;
  const int grid = static_cast<int>(blocks < sms * 8 ? blocks : sms * 8);
  __half* yh = static_cast<__half*>(y);
  if (vec4)
    to_f16_kernel<true><<<grid, 256, 0, s>>>(x, m, k, ldx_floats, yh, ldy);
  else
    to_f16_kernel<false><<<grid, 256, 0, s>>>(x, m, k, ldx_floats, yh, ldy);
  return cudaGetLastError();
}

cudaError_t launch_pack_weights(int wtype, const uint8_t* w, int64_t n, int64_t k,
                                int64_t ldw_bytes, int8_t* codes, float* scales, int64_t ld,
                                cudaStream_t s) {
  const int64_t total = n * (k / kQK);
  if (total == 0) return cudaSuccess;
  const int64_t blocks = (total + 255) / 256;
  const int grid = static_cast<int>(blocks < 65535 ? blocks : 65535);
  if (wtype == kTypeQ8_0)
    pack_weights_kernel<kTypeQ8_0><<<grid, 256, 0, s>>>(w, n, k, ldw_bytes, codes, scales, ld);
  else
    pack_weights_kernel<kTypeQ4_0><<<grid, 256, 0, s>>>(w, n, k, ldw_bytes, codes, scales, ld);
  return cudaGetLastError();
}

}  // namespace b2q
