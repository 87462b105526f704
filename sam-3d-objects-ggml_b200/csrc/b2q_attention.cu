// b2q_attention.cu -- the attention core of the SS-flow DiT blocks
// (gb_attention, cpp_ggml/src/graph_builder.cpp:139-175; called for the
// self-attention at ss_flow_graph.cpp:277,281 and the cross-attention at :346).
//
// F32 contract (this file's SIMT kernel): the reference's numeric-gate form of
// gb_attention -- ggml_flash_attn_ext with F32 K/V and GGML_PREC_F32, which on
// the CPU backend is a per-query online softmax in fp32: s = (q . k) * scale,
// running max m and sum l with expf, o = sum p v / l, every product and sum in
// IEEE fp32.  It is the diagnostic / parity form, not the speed path.
//
//   q    fp32 [B][H][Tq][D]          (contiguous, as b2q_qkv_heads_f32 writes it)
//   k, v fp32 [B][H][Tk][D]          keys 0 .. Tk-1
//   k2, v2 fp32 [B][H][Tk2][D]       optional second key source, keys Tk .. Tk+Tk2-1
//                                    (the pose group attends its own keys and the
//                                    shape group's, ss_flow_graph.cpp:262-275)
//   o    fp32 rows [B*Tq][H*D]       row (b, t), columns h*D + d: the layout the
//                                    output projection consumes
//
// Mapping: one CTA per 64 queries of one (b, h), 256 threads.  The CTA walks
// the keys in tiles of 64: K and V tiles in shared memory, each thread a 4 x 4
// block of the score tile (4 queries x 4 keys) and a 4 x D/16 block of the
// output.  A query row's 64 scores sit in 16 consecutive lanes, so the row max
// and row sum are 16-lane shuffles.
#include "b2q_internal.h"

#include <cmath>

namespace b2q {

namespace {

constexpr int kAttnBQ = 64;   // queries per CTA
constexpr int kAttnBK = 64;   // keys per tile
constexpr int kAttnThreads = 256;

template <int D>
struct AttnF32Smem {
  static constexpr int LD = D + 4;       // padded row (floats): conflict-free float4 column reads
  static constexpr int PLD = kAttnBK + 4;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + kAttnBQ * LD;
  static constexpr int V_OFF = K_OFF + kAttnBK * LD;
  static constexpr int P_OFF = V_OFF + kAttnBK * LD;
  static constexpr int FLOATS = P_OFF + kAttnBQ * PLD;
  static constexpr int BYTES = FLOATS * 4;
};

__device__ __forceinline__ float max16(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float sum16(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Loads rows [row0, row0 + 64) of a [T][D] fp32 matrix into smem (row pitch
// LD), zero rows at and past T.  Two sources: rows < T1 from a, the rest from b.
template <int D, int LD>
__device__ __forceinline__ void load_rows(float* dst, const float* a, int64_t T1, const float* b, int64_t T2,
                                          int64_t row0) {
  constexpr int V4 = D / 4;  // float4 per row
  for (int i = threadIdx.x; i < kAttnBK * V4; i += kAttnThreads) {
    const int r = i / V4, c = (i - r * V4) * 4;
    const int64_t t = row0 + r;
    float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (t < T1)
      x = __ldg(reinterpret_cast<const float4*>(a + t * D + c));
    else if (t < T1 + T2)
      x = __ldg(reinterpret_cast<const float4*>(b + (t - T1) * D + c));
    *reinterpret_cast<float4*>(dst + r * LD + c) = x;
  }
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads) attention_f32_kernel(const float* __restrict__ q,
                                                                     const float* __restrict__ k,
                                                                     const float* __restrict__ v,
                                                                     const float* __restrict__ k2,
                                                                     const float* __restrict__ v2, int H, int64_t Tq,
                                                                     int64_t Tk, int64_t Tk2, float scale,
                                                                     float* __restrict__ o, int64_t ldo) {
  using S = AttnF32Smem<D>;
  constexpr int LD = S::LD, PLD = S::PLD;
  constexpr int DC = D / 16;  // output dims per thread
  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);
  float* Qs = sm + S::Q_OFF;
  float* Ks = sm + S::K_OFF;
  float* Vs = sm + S::V_OFF;
  float* Ps = sm + S::P_OFF;

  const int h = blockIdx.y;
  const int64_t bh = static_cast<int64_t>(blockIdx.z) * H + h;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * kAttnBQ;
  const int t = threadIdx.x;
  const int rg = t >> 4, cg = t & 15;  // rows 4rg..4rg+3; score cols 4cg..4cg+3; output dims DC*cg..
  const float* qb = q + bh * Tq * D;
  const float* kb = k + bh * Tk * D;
  const float* vb = v + bh * Tk * D;
  const float* k2b = k2 ? k2 + bh * Tk2 * D : nullptr;
  const float* v2b = v2 ? v2 + bh * Tk2 * D : nullptr;
  const int64_t tk_all = Tk + (k2 ? Tk2 : 0);

  load_rows<D, LD>(Qs, qb, Tq, nullptr, 0, q0);

  float m[4], l[4], acc[4][DC];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.0f;
#pragma unroll
    for (int j = 0; j < DC; ++j) acc[i][j] = 0.0f;
  }

  for (int64_t k0 = 0; k0 < tk_all; k0 += kAttnBK) {
    __syncthreads();  // previous tile's K, V and P are no longer read
    load_rows<D, LD>(Ks, kb, Tk, k2b, k2 ? Tk2 : 0, k0);
    load_rows<D, LD>(Vs, vb, Tk, v2b, k2 ? Tk2 : 0, k0);
    __syncthreads();
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll 4
    for (int d = 0; d < D; d += 4) {
      float4 qa[4], ka[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qa[i] = *reinterpret_cast<const float4*>(Qs + (4 * rg + i) * LD + d);
#pragma unroll
      for (int j = 0; j < 4; ++j) ka[j] = *reinterpret_cast<const float4*>(Ks + (4 * cg + j) * LD + d);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = __fmaf_rn(qa[i].x, ka[j].x, s[i][j]);
          s[i][j] = __fmaf_rn(qa[i].y, ka[j].y, s[i][j]);
          s[i][j] = __fmaf_rn(qa[i].z, ka[j].z, s[i][j]);
          s[i][j] = __fmaf_rn(qa[i].w, ka[j].w, s[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float tmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][j] = (k0 + 4 * cg + j < tk_all) ? __fmul_rn(s[i][j], scale) : -INFINITY;
        tmax = fmaxf(tmax, s[i][j]);
      }
      tmax = max16(tmax);
      const float m_new = fmaxf(m[i], tmax);  // finite: every tile holds at least one key
      const float alpha = expf(m[i] - m_new);  // 0 on the first tile (m = -inf)
      float psum = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = expf(s[i][j] - m_new);
        Ps[(4 * rg + i) * PLD + 4 * cg + j] = p;
        psum = __fadd_rn(psum, p);
      }
      psum = sum16(psum);
      l[i] = __fmaf_rn(l[i], alpha, psum);
      m[i] = m_new;
#pragma unroll
      for (int jd = 0; jd < DC; ++jd) acc[i][jd] = __fmul_rn(acc[i][jd], alpha);
    }
    __syncthreads();  // P complete
#pragma unroll 4
    for (int kk = 0; kk < kAttnBK; ++kk) {
      float pr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pr[i] = Ps[(4 * rg + i) * PLD + kk];
      float vv[DC];
#pragma unroll
      for (int jd = 0; jd < DC; jd += 2) {
        const float2 x = *reinterpret_cast<const float2*>(Vs + kk * LD + DC * cg + jd);
        vv[jd] = x.x;
        vv[jd + 1] = x.y;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jd = 0; jd < DC; ++jd) acc[i][jd] = __fmaf_rn(pr[i], vv[jd], acc[i][jd]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t tq = q0 + 4 * rg + i;
    if (tq >= Tq) continue;
    const float inv = __fdiv_rn(1.0f, l[i]);
    float* dst = o + (static_cast<int64_t>(blockIdx.z) * Tq + tq) * ldo + static_cast<int64_t>(h) * D + DC * cg;
#pragma unroll
    for (int jd = 0; jd < DC; ++jd) dst[jd] = __fmul_rn(acc[i][jd], inv);
  }
}

template <int D>
cudaError_t launch_attention_f32_d(const float* q, const float* k, const float* v, const float* k2, const float* v2,
                                   int64_t B, int H, int64_t Tq, int64_t Tk, int64_t Tk2, float scale, float* o,
                                   int64_t ldo, cudaStream_t s) {
  using Sm = AttnF32Smem<D>;
  auto kern = attention_f32_kernel<D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Sm::BYTES);
  if (e != cudaSuccess) return e;
  const dim3 grid(static_cast<unsigned>((Tq + kAttnBQ - 1) / kAttnBQ), static_cast<unsigned>(H),
                  static_cast<unsigned>(B));
  kern<<<grid, kAttnThreads, Sm::BYTES, s>>>(q, k, v, k2, v2, H, Tq, Tk, Tk2, scale, o, ldo);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attention_f32(const float* q, const float* k, const float* v, const float* k2, const float* v2,
                                 int64_t B, int H, int64_t Tq, int64_t Tk, int64_t Tk2, int D, float scale, float* o,
                                 int64_t ldo_floats, cudaStream_t s) {
  if (B == 0 || Tq == 0) return cudaSuccess;
  switch (D) {
    case 32: return launch_attention_f32_d<32>(q, k, v, k2, v2, B, H, Tq, Tk, Tk2, scale, o, ldo_floats, s);
    case 64: return launch_attention_f32_d<64>(q, k, v, k2, v2, B, H, Tq, Tk, Tk2, scale, o, ldo_floats, s);
    case 128: return launch_attention_f32_d<128>(q, k, v, k2, v2, B, H, Tq, Tk, Tk2, scale, o, ldo_floats, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace b2q
