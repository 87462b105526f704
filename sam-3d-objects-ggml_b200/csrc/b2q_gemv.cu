// b2q_gemv.cu -- the mul_mat for a handful of tokens (M <= 8): the adaLN
// projection (M = 1 per sample, cpp_ggml/src/ss_flow_graph.cpp:183-185) and
// the pose group's linears (M = 4).  At these sizes the tensor-core kernel
// runs one 64-token tile per 128 weight rows and is bound by its per-block
// pipeline latency; this kernel streams the weight once, on CUDA cores.
//
// Results are bit-identical to the tensor-core kernel's: per (row n, token m)
// the per-block terms are folded in the same order with the same roundings,
//     t_b = RN(S_b * dw_b)            (S_b: exact int32 block dot, via dp4a)
//     acc = RN(t_b * da_b + acc)      (fused multiply-add), b = 0, 1, ...
// followed by the same bias / gate / residual steps.  The tensor-core kernel
// computes t_b from the accumulator bits read as a subnormal (see
// b2q_gemm_tc.cu); the value is the same.
//
// Structure: a CTA owns R = 8 weight rows and walks K in chunks of KC blocks.
//   1. the chunk's weight scales [KC][R] and activation scales [M][KC] are
//      staged in shared memory (coalesced: each is a run of consecutive
//      floats in the block-major scale layout);
//   2. warp r takes weight row n0 + r, its lanes the chunk's blocks (every
//      code load of a warp is one contiguous run), and writes t_b for each
//      token to shared memory;
//   3. thread (r, m) continues its sequential fold over the chunk.
#include "b2q_internal.h"

namespace b2q {

namespace {

constexpr int kRows = 8;      // weight rows per CTA (one warp each in step 2)
constexpr int kChunk = 128;   // blocks of K per chunk
constexpr int kThreadsGemv = kRows * 32;

template <int MT>
__global__ void __launch_bounds__(kThreadsGemv) gemv_kernel(const int8_t* __restrict__ wc,
                                                            const float* __restrict__ ws, int64_t ldw, int64_t N,
                                                            const int8_t* __restrict__ ac,
                                                            const float* __restrict__ as, int64_t lda, int M,
                                                            int64_t K, const float* __restrict__ bias,
                                                            const float* __restrict__ gate,
                                                            const float* resid, int64_t ldr, float* y, int64_t ldy) {
  __shared__ float dws[kChunk][kRows];          // weight scales, unscaled (x 2^-100)
  __shared__ float das[MT][kChunk];             // activation scales, unscaled (x 2^-49)
  __shared__ float ts[kRows][MT][kChunk + 1];   // t_b per (row, token, block); +1: conflict-free column reads
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kRows;
  const int KB = static_cast<int>(K / kQK);
  // step-3 role: thread (fr, fm) folds row n0 + fr for token fm
  const int fr = tid / MT, fm = tid % MT;
  const bool folder = tid < kRows * MT && fm < M && n0 + fr < N;
  float acc = 0.0f;

  for (int b0 = 0; b0 < KB; b0 += kChunk) {
    const int kc = KB - b0 < kChunk ? KB - b0 : kChunk;
    // 1. scales of this chunk
    for (int i = tid; i < kc * kRows; i += kThreadsGemv) {
      const int b = i / kRows, r = i % kRows;
      dws[b][r] = n0 + r < N ? ws[static_cast<int64_t>(b0 + b) * ldw + n0 + r] * 0x1p-100f : 0.0f;
    }
    for (int i = tid; i < kc * M; i += kThreadsGemv) {
      const int b = i / M, m = i % M;
      das[m][b] = as[static_cast<int64_t>(b0 + b) * lda + m] * 0x1p-49f;
    }
    __syncthreads();
    // 2. block dots of row n0 + warp against every token, t_b = RN(S_b * dw_b)
    const int64_t n = n0 + warp;
    if (n < N) {
      const int8_t* wr = wc + n * K;
      for (int b = lane; b < kc; b += 32) {
        const int4* wp = reinterpret_cast<const int4*>(wr + static_cast<int64_t>(b0 + b) * kQK);
        const int4 w0 = __ldg(wp), w1 = __ldg(wp + 1);
        const float dw = dws[b][warp];
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m >= M) break;
          const int4* ap = reinterpret_cast<const int4*>(ac + static_cast<int64_t>(m) * K +
                                                         static_cast<int64_t>(b0 + b) * kQK);
          const int4 a0 = __ldg(ap), a1 = __ldg(ap + 1);
          int sdot = __dp4a(w0.x, a0.x, 0);
          sdot = __dp4a(w0.y, a0.y, sdot);
          sdot = __dp4a(w0.z, a0.z, sdot);
          sdot = __dp4a(w0.w, a0.w, sdot);
          sdot = __dp4a(w1.x, a1.x, sdot);
          sdot = __dp4a(w1.y, a1.y, sdot);
          sdot = __dp4a(w1.z, a1.z, sdot);
          sdot = __dp4a(w1.w, a1.w, sdot);
          ts[warp][m][b] = __fmul_rn(static_cast<float>(sdot), dw);
        }
      }
    }
    __syncthreads();
    // 3. the sequential fold over this chunk
    if (folder) {
#pragma unroll 8
      for (int b = 0; b < kc; ++b) acc = __fmaf_rn(ts[fr][fm][b], das[fm][b], acc);  // loads run ahead of the chain
    }
    __syncthreads();
  }
  if (!folder) return;
  const int64_t n = n0 + fr;
  float v = acc;
  if (bias) v = __fadd_rn(v, bias[n]);
  if (resid) {
    const float t = gate ? __fmul_rn(v, gate[n]) : v;
    v = __fadd_rn(resid[static_cast<int64_t>(fm) * ldr + n], t);
  }
  y[static_cast<int64_t>(fm) * ldy + n] = v;
}

}  // namespace

cudaError_t launch_gemv(const GemmArgs& g, cudaStream_t s) {
  if (g.M == 0 || g.N == 0) return cudaSuccess;
  if (g.M > kGemvMaxM) return cudaErrorInvalidValue;
  const int64_t grid = (g.N + kRows - 1) / kRows;
  if (grid > 0x7fffffff) return cudaErrorInvalidValue;
  const int M = static_cast<int>(g.M);
#define B2Q_GEMV(MT)                                                                                         \
  gemv_kernel<MT><<<static_cast<unsigned>(grid), kThreadsGemv, 0, s>>>(                                      \
      g.w.codes, g.w.scales, g.w.ld, g.N, g.a.codes, g.a.scales, g.a.ld, M, g.K, g.bias, g.gate, g.resid,    \
      g.ldr, g.y, g.ldy)
  if (M <= 1)
    B2Q_GEMV(1);
  else if (M <= 2)
    B2Q_GEMV(2);
  else if (M <= 4)
    B2Q_GEMV(4);
  else
    B2Q_GEMV(8);
#undef B2Q_GEMV
  return cudaGetLastError();
}

}  // namespace b2q
