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
// Mapping: a warp quantizes 128-value segments (4 blocks) of a row; each lane
// loads one 128-bit float4 per segment, so 8 lanes own one block and the
// block's absmax is three xor-shuffles inside that 8-lane group.
#include "b2q_internal.h"
#include "b2q_ptx.cuh"

#include <cuda_fp16.h>

namespace b2q {

namespace {

template <int VARIANT>
__device__ __forceinline__ int quantize_one(float v, float inv) {
  const float s = __fmul_rn(v, inv);
  if (VARIANT == 0) {
    int q = __float2int_rn(s);  // round to nearest, ties to even
    return max(-128, min(127, q));
  }
  return static_cast<int>(roundf(s));  // ties away from zero
}

struct BlockQuant {
  uint32_t packed;  // 4 codes of this lane, little-endian
  float d;          // fp32 block scale before the fp16 store
};

template <int VARIANT>
__device__ __forceinline__ BlockQuant quantize_lane(float4 v) {
  float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
  BlockQuant r;
  r.d = __fdiv_rn(amax, 127.0f);
  float inv;
  if (VARIANT == 0)
    inv = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
  else
    inv = r.d != 0.0f ? __fdiv_rn(1.0f, r.d) : 0.0f;
  const int q0 = quantize_one<VARIANT>(v.x, inv);
  const int q1 = quantize_one<VARIANT>(v.y, inv);
  const int q2 = quantize_one<VARIANT>(v.z, inv);
  const int q3 = quantize_one<VARIANT>(v.w, inv);
  r.packed = (static_cast<uint32_t>(q0) & 0xffu) | ((static_cast<uint32_t>(q1) & 0xffu) << 8) |
             ((static_cast<uint32_t>(q2) & 0xffu) << 16) | ((static_cast<uint32_t>(q3) & 0xffu) << 24);
  return r;
}

template <bool VEC4>
__device__ __forceinline__ float4 load4(const float* p) {
  if (VEC4) return __ldg(reinterpret_cast<const float4*>(p));
  return make_float4(__ldg(p), __ldg(p + 1), __ldg(p + 2), __ldg(p + 3));
}

// SPLIT = true : codes int8 [m][k] + fp32 scales [k/32][ld] (GEMM layout)
// SPLIT = false: ggml block_q8_0 rows (34-byte blocks)
// Each warp step handles kUnroll consecutive segments, all loads issued first,
// so every warp keeps kUnroll * 512 bytes in flight.
constexpr int kUnroll = 4;

template <int VARIANT, bool SPLIT, bool VEC4>
__global__ void __launch_bounds__(256) quantize_q8_0_kernel(const float* __restrict__ x, int64_t m,
                                                            int64_t k, int64_t ldx,
                                                            uint8_t* __restrict__ yb, int64_t ldy,
                                                            int8_t* __restrict__ codes,
                                                            float* __restrict__ scales, int64_t ld) {
  const int lane = threadIdx.x & 31;
  const int64_t segs = (k + 127) / 128;
  const int64_t total = m * segs;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t w0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32 * kUnroll;
       w0 < total; w0 += warps * kUnroll) {
    float4 v[kUnroll];
    int64_t row[kUnroll], k0[kUnroll];
    bool valid[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t w = w0 + u;
      row[u] = w / segs;
      k0[u] = (w - row[u] * segs) * 128 + lane * 4;
      valid[u] = w < total && k0[u] < k;  // k % 32 == 0: a block is all-valid or all-invalid
      v[u] = valid[u] ? load4<VEC4>(x + row[u] * ldx + k0[u]) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const BlockQuant q = quantize_lane<VARIANT>(v[u]);
      if (!valid[u]) continue;
      const int64_t blk = k0[u] / kQK;
      const int sub = lane & 7;
      const __half dh = __float2half_rn(q.d);
      if (SPLIT) {
        *reinterpret_cast<uint32_t*>(codes + row[u] * k + k0[u]) = q.packed;
        if (sub == 0) scales[blk * ld + row[u]] = __half2float(dh) * kActScaleMul;
      } else {
        uint8_t* b = yb + row[u] * ldy + blk * kQ8Bytes;
        uint16_t* b16 = reinterpret_cast<uint16_t*>(b + 2 + 4 * sub);
        b16[0] = static_cast<uint16_t>(q.packed & 0xffffu);
        b16[1] = static_cast<uint16_t>(q.packed >> 16);
        if (sub == 0) *reinterpret_cast<uint16_t*>(b) = __half_as_ushort(dh);
      }
    }
  }
}

template <bool SPLIT, bool VEC4>
cudaError_t launch_q(const float* x, int64_t m, int64_t k, int64_t ldx, uint8_t* yb, int64_t ldy,
                     int8_t* codes, float* scales, int64_t ld, int variant, cudaStream_t s) {
  const int64_t warps_needed = (m * ((k + 127) / 128) + kUnroll - 1) / kUnroll;
  if (warps_needed == 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks_needed = (warps_needed + 7) / 8;
  const int grid = static_cast<int>(blocks_needed < sms * 8 ? blocks_needed : sms * 8);
  if (variant == 0)
    quantize_q8_0_kernel<0, SPLIT, VEC4><<<grid, 256, 0, s>>>(x, m, k, ldx, yb, ldy, codes, scales, ld);
  else
    quantize_q8_0_kernel<1, SPLIT, VEC4><<<grid, 256, 0, s>>>(x, m, k, ldx, yb, ldy, codes, scales, ld);
  return cudaGetLastError();
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

}  // namespace

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
