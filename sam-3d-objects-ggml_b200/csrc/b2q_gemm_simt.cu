// b2q_gemm_simt.cu -- plain CUDA-core block GEMM that reproduces the ggml CPU
// backend's x86 accumulation order exactly (a check path, not a fast path).
//
// For one output y[m][n] the CPU dot keeps 8 fp32 lanes; lane l receives, per
// 32-value block, the int32 sum of products 4l..4l+3 (one dp4a here), converted
// to fp32 and added with one fused multiply-add by d = fp32(dw) * fp32(da); the
// lanes are then reduced as ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)).  With the
// same operand order every rounding matches, so the fp32 result is bit-exact.
//
// Inputs are raw ggml blocks: weights Q8_0 (34 B) or Q4_0 (18 B), activations
// Q8_0 (34 B).  Blocks are only 2-byte aligned, so words are assembled from
// 16-bit loads.
#include "b2q_internal.h"

#include <cuda_fp16.h>

namespace b2q {
namespace {

__device__ __forceinline__ uint32_t word_at(const uint16_t* p, int j) {
  return static_cast<uint32_t>(p[2 * j]) | (static_cast<uint32_t>(p[2 * j + 1]) << 16);
}

template <int WTYPE>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const uint8_t* __restrict__ w, int64_t ldw,
                                                        int64_t n, int64_t k,
                                                        const uint8_t* __restrict__ a, int64_t lda,
                                                        int64_t m, float* __restrict__ y,
                                                        int64_t ldy) {
  const int64_t col = static_cast<int64_t>(blockIdx.x) * 32 + (threadIdx.x & 31);
  const int64_t row = static_cast<int64_t>(blockIdx.y) * 8 + (threadIdx.x >> 5);
  if (col >= n || row >= m) return;
  const int64_t kb = k / kQK;
  const uint8_t* wr = w + col * ldw;
  const uint8_t* ar = a + row * lda;
  float lane[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) lane[l] = 0.0f;
  for (int64_t b = 0; b < kb; ++b) {
    const uint16_t* wb = reinterpret_cast<const uint16_t*>(wr + b * (WTYPE == kTypeQ8_0 ? kQ8Bytes : kQ4Bytes));
    const uint16_t* ab = reinterpret_cast<const uint16_t*>(ar + b * kQ8Bytes);
    const float d = __fmul_rn(__half2float(__ushort_as_half(wb[0])), __half2float(__ushort_as_half(ab[0])));
    uint32_t wq[8];
    if (WTYPE == kTypeQ8_0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) wq[j] = word_at(wb + 1, j);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t nib = word_at(wb + 1, j);
        wq[j] = __vsub4(nib & 0x0f0f0f0fu, 0x08080808u);
        wq[4 + j] = __vsub4((nib >> 4) & 0x0f0f0f0fu, 0x08080808u);
      }
    }
#pragma unroll
    for (int l = 0; l < 8; ++l) {
      const int s = __dp4a(static_cast<int>(wq[l]), static_cast<int>(word_at(ab + 1, l)), 0);
      lane[l] = __fmaf_rn(d, static_cast<float>(s), lane[l]);
    }
  }
  const float r0 = __fadd_rn(lane[4], lane[0]), r1 = __fadd_rn(lane[5], lane[1]);
  const float r2 = __fadd_rn(lane[6], lane[2]), r3 = __fadd_rn(lane[7], lane[3]);
  y[row * ldy + col] = __fadd_rn(__fadd_rn(r0, r2), __fadd_rn(r1, r3));
}

}  // namespace

cudaError_t launch_gemm_simt(int wtype, const uint8_t* w, int64_t ldw_bytes, int64_t n, int64_t k,
                             const uint8_t* a, int64_t lda_bytes, int64_t m, float* y,
                             int64_t ldy_floats, cudaStream_t s) {
  if (m == 0 || n == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>((n + 31) / 32), static_cast<unsigned>((m + 7) / 8));
  if (wtype == kTypeQ8_0)
    gemm_simt_kernel<kTypeQ8_0><<<grid, 256, 0, s>>>(w, ldw_bytes, n, k, a, lda_bytes, m, y, ldy_floats);
  else
    gemm_simt_kernel<kTypeQ4_0><<<grid, 256, 0, s>>>(w, ldw_bytes, n, k, a, lda_bytes, m, y, ldy_floats);
  return cudaGetLastError();
}

}  // namespace b2q
