// The dequantize-to-float form of the reference's linears: matmul_weight with
// keep_quant_gemm false (cpp_ggml/src/ss_flow_graph.cpp:13-34,
// slat_flow_graph.cpp:89-94) casts a quantized weight to F32 (as_f32) or to
// F32 then F16 (as_f16) with ggml_cast, and gb_linear (graph_builder.cpp:44-60)
// runs ggml_mul_mat on it with GGML_PREC_F32.
//
//   dequantize_kernel: GGUF Q8_0 / Q4_0 / Q4_K rows -> fp32 or fp16 rows, the
//     values ggml's dequantize_row_* produce (Q8_0 / Q4_0: fp32(d) * code;
//     Q4_K: (d * sc) * q - (dmin * m), each product and the difference rounded
//     separately), fp16 by one round-to-nearest-even of that fp32 value.
//   sgemm_kernel: the strict F32 mul_mat, y[m][n] = sum_k x[m][k] w[n][k]
//     (+ bias[n], one more rounding, ggml's separate ADD).  No tensor-core form
//     keeps fp32 products exact, so this is a CUDA-core kernel: 128 x 128
//     output tiles, 256 threads with 8 x 8 outputs each (packed fp32x2 FMAs),
//     16-deep k slabs double-buffered in shared memory, transposed so that the
//     inner loop reads 16-byte vectors.  Every output is one fp32 FMA chain in
//     k order.  Memory-light: at 128 x 128 tiles each operand byte is read
//     N/128 (or M/128) times, from L2.
#include "../../include/b2q.h"
#include "b2q_internal.h"
#include "b2q_ptx.cuh"

#include <cuda_fp16.h>

namespace b2q {
namespace {

// ------------------------------------------------------------ dequantize
// One thread per 32-value block (Q4_K: per 32-value sub-block of a 256-value
// super-block).
template <int WTYPE, bool F16OUT>
__global__ void dequantize_kernel(const uint8_t* __restrict__ w, int64_t ldw, int64_t n, int64_t k,
                                  void* __restrict__ out, int64_t ldo_elems) {
  const int64_t nbr = k / kQK;  // 32-value (sub-)blocks per row
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= n * nbr) return;
  const int64_t r = idx / nbr, b = idx % nbr;
  const uint8_t* row = w + r * ldw;
  float v[kQK];
  if (WTYPE == B2Q_TYPE_Q8_0 || WTYPE == B2Q_TYPE_Q4_0) {
    const int bytes = WTYPE == B2Q_TYPE_Q8_0 ? 34 : 18;
    const uint8_t* blk = row + b * bytes;
    const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] | (blk[1] << 8))));
#pragma unroll
    for (int j = 0; j < kQK; ++j) {
      int q;
      if (WTYPE == B2Q_TYPE_Q8_0) {
        q = static_cast<int8_t>(blk[2 + j]);
      } else {
        const uint8_t c = blk[2 + (j & 15)];
        q = static_cast<int>(j < 16 ? (c & 15) : (c >> 4)) - 8;
      }
      v[j] = __fmul_rn(static_cast<float>(q), d);
    }
  } else {  // Q4_K: 144-byte super-blocks {fp16 d, fp16 dmin, 12 scale bytes, 128 code bytes}
    const int64_t sb = b / 8;
    const int j = static_cast<int>(b % 8);
    const uint8_t* blk = row + sb * kQ4KBytes;
    const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] | (blk[1] << 8))));
    const float dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[2] | (blk[3] << 8))));
    const uint8_t* s = blk + 4;
    int sc, m;
    if (j < 4) {
      sc = s[j] & 63;
      m = s[j + 4] & 63;
    } else {
      sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
      m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
    const float d1 = __fmul_rn(d, static_cast<float>(sc)), m1 = __fmul_rn(dmin, static_cast<float>(m));
    // sub-block j: codes of bytes 32*(j/2) .. +31, low nibbles for even j, high for odd
    const uint8_t* qs = blk + 16 + 32 * (j / 2);
#pragma unroll
    for (int l = 0; l < kQK; ++l) {
      const int q = (j & 1) ? (qs[l] >> 4) : (qs[l] & 15);
      v[l] = __fsub_rn(__fmul_rn(d1, static_cast<float>(q)), m1);
    }
  }
  if (F16OUT) {
    __half* o = static_cast<__half*>(out) + r * ldo_elems + b * kQK;
#pragma unroll
    for (int j = 0; j < kQK; j += 2) *reinterpret_cast<__half2*>(o + j) = __floats2half2_rn(v[j], v[j + 1]);
  } else {
    float* o = static_cast<float*>(out) + r * ldo_elems + b * kQK;
#pragma unroll
    for (int j = 0; j < kQK; j += 4) *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  }
}

// ------------------------------------------------------------------ sgemm
constexpr int kSgBM = 128, kSgBN = 128, kSgBK = 16, kSgThreads = 256, kSgPad = 4;
constexpr int kSgLd = kSgBM + kSgPad;  // shared-memory row (one k) of a tile, floats

// Two 16-byte k-quads of this thread's rows of a [rows][k] operand tile into
// registers (zeros past the data).
__device__ __forceinline__ void sg_fetch(const float* __restrict__ a, int64_t lda, int64_t rows, int64_t k,
                                         int64_t r0, int64_t k0, int t, float4 (&v)[2]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int64_t r = r0 + t / 4 + 64 * h, kk = k0 + (t % 4) * 4;
    v[h] = (r < rows && kk < k) ? __ldg(reinterpret_cast<const float4*>(a + r * lda + kk))
                                : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
}

// ... and transposed into a [BK][ld] shared-memory slab.
__device__ __forceinline__ void sg_store(float* s, int t, const float4 (&v)[2]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = t / 4 + 64 * h, kq = (t % 4) * 4;
    s[(kq + 0) * kSgLd + r] = v[h].x;
    s[(kq + 1) * kSgLd + r] = v[h].y;
    s[(kq + 2) * kSgLd + r] = v[h].z;
    s[(kq + 3) * kSgLd + r] = v[h].w;
  }
}

__global__ void __launch_bounds__(kSgThreads, 1)
    sgemm_kernel(const float* __restrict__ x, int64_t ldx, int64_t M, const float* __restrict__ w, int64_t ldw,
                 int64_t N, int64_t K, const float* __restrict__ bias, float* __restrict__ y, int64_t ldy) {
  __shared__ __align__(16) float xs[2][kSgBK * kSgLd];
  __shared__ __align__(16) float ws[2][kSgBK * kSgLd];
  const int t = threadIdx.x, tx = t % 16, ty = t / 16;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kSgBM, n0 = static_cast<int64_t>(blockIdx.x) * kSgBN;
  float2 acc[8][4];  // rows ty*4+i (i<4) and 64+ty*4+i-4; column pairs tx*4+{0,2}, 64+tx*4+{0,2}
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = make_float2(0.0f, 0.0f);
  const int nk = static_cast<int>((K + kSgBK - 1) / kSgBK);
  float4 px[2], pw[2];
  sg_fetch(x, ldx, M, K, m0, 0, t, px);
  sg_fetch(w, ldw, N, K, n0, 0, t, pw);
  sg_store(xs[0], t, px);
  sg_store(ws[0], t, pw);
  __syncthreads();
  for (int kt = 0; kt < nk; ++kt) {
    const int cur = kt & 1;
    if (kt + 1 < nk) {  // the next slab's loads in flight during this slab's math
      sg_fetch(x, ldx, M, K, m0, static_cast<int64_t>(kt + 1) * kSgBK, t, px);
      sg_fetch(w, ldw, N, K, n0, static_cast<int64_t>(kt + 1) * kSgBK, t, pw);
    }
    const float* xc = xs[cur];
    const float* wc = ws[cur];
#pragma unroll
    for (int kk = 0; kk < kSgBK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(xc + kk * kSgLd + ty * 4);
      const float4 a1 = *reinterpret_cast<const float4*>(xc + kk * kSgLd + 64 + ty * 4);
      const float4 b0 = *reinterpret_cast<const float4*>(wc + kk * kSgLd + tx * 4);
      const float4 b1 = *reinterpret_cast<const float4*>(wc + kk * kSgLd + 64 + tx * 4);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float2 bv[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w), make_float2(b1.x, b1.y),
                            make_float2(b1.z, b1.w)};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = ffma2(make_float2(av[i], av[i]), bv[j], acc[i][j]);
    }
    if (kt + 1 < nk) {
      sg_store(xs[cur ^ 1], t, px);
      sg_store(ws[cur ^ 1], t, pw);
    }
    __syncthreads();
  }
  // ggml_add after the mul_mat: one more fp32 rounding per element.
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (m >= M) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t n = n0 + h * 64 + tx * 4;
      float v[4] = {acc[i][2 * h].x, acc[i][2 * h].y, acc[i][2 * h + 1].x, acc[i][2 * h + 1].y};
      float* yp = y + m * ldy + n;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (n + j < N) yp[j] = bias ? __fadd_rn(v[j], bias[n + j]) : v[j];
    }
  }
}

template <int WTYPE>
cudaError_t dequantize_t(const uint8_t* w, int64_t ldw, int64_t n, int64_t k, bool f16, void* out, int64_t ldo,
                         cudaStream_t s) {
  const int64_t units = n * (k / kQK);
  const int threads = 256;
  const int64_t blocks = (units + threads - 1) / threads;
  if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
  if (f16)
    dequantize_kernel<WTYPE, true><<<static_cast<unsigned>(blocks), threads, 0, s>>>(w, ldw, n, k, out, ldo);
  else
    dequantize_kernel<WTYPE, false><<<static_cast<unsigned>(blocks), threads, 0, s>>>(w, ldw, n, k, out, ldo);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_dequantize(int wtype, const void* w, int64_t ldw_bytes, int64_t n, int64_t k, bool f16_out,
                              void* out, int64_t ldo_elems, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const uint8_t* wb = static_cast<const uint8_t*>(w);
  switch (wtype) {
    case B2Q_TYPE_Q8_0: return dequantize_t<B2Q_TYPE_Q8_0>(wb, ldw_bytes, n, k, f16_out, out, ldo_elems, s);
    case B2Q_TYPE_Q4_0: return dequantize_t<B2Q_TYPE_Q4_0>(wb, ldw_bytes, n, k, f16_out, out, ldo_elems, s);
    case B2Q_TYPE_Q4_K: return dequantize_t<B2Q_TYPE_Q4_K>(wb, ldw_bytes, n, k, f16_out, out, ldo_elems, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_sgemm(const float* x, int64_t ldx, int64_t m, const float* w, int64_t ldw, int64_t n, int64_t k,
                         const float* bias, float* y, int64_t ldy, cudaStream_t s) {
  if (m == 0 || n == 0) return cudaSuccess;
  const int64_t gx = (n + kSgBN - 1) / kSgBN, gy = (m + kSgBM - 1) / kSgBM;
  if (gx > 0x7fffffff || gy > 65535) return cudaErrorInvalidValue;
  sgemm_kernel<<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)), kSgThreads, 0, s>>>(x, ldx, m, w, ldw,
                                                                                                 n, k, bias, y, ldy);
  return cudaGetLastError();
}

}  // namespace b2q
