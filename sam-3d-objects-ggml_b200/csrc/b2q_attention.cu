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
// F16 form (attention_f16_kernel below): the production path of gb_attention
// (flash attention on F16 K/V), for D = 64, on the tensor cores.
//
// Mapping of the F32 kernel: one CTA per 64 queries of one (b, h), 256 threads.  The CTA walks
// the keys in tiles of 64: K and V tiles in shared memory, each thread a 4 x 4
// block of the score tile (4 queries x 4 keys) and a 4 x D/16 block of the
// output.  A query row's 64 scores sit in 16 consecutive lanes, so the row max
// and row sum are 16-lane shuffles.
#include "b2q_internal.h"
#include "b2q_ptx.cuh"
#include "b2q_q8.cuh"

#include <cuda_fp16.h>

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

// ----------------------------------------------------------------- F16 form
// Flash attention on the tensor cores for D = 64, fp16 q / k / v / o, fp32
// softmax.  One CTA per 256 queries (two 128-query tiles) of one (b, h);
// 384 threads = 3 warpgroups:
//   warp 0       TMA producer: both Q tiles once, then K and V tiles of 128 keys
//                (fp16, 128-byte swizzle) through a kFaStages ring shared by the
//                two query tiles
//   warp 1       TMEM allocator + MMA issuer: S_i = Q_i K^T (kind::f16, M 128,
//                N 128, K 64) and (P V)_i (M 128, N 64, K 128; P read from
//                tensor memory as the A operand, V as an MN-major operand
//                straight from its TMA tile), each issued as soon as its own
//                barriers complete (polled, S first)
//   warps 2, 3   idle (complete warpgroup 0, which runs on 56 registers)
//   warpgroups 1 and 2: softmax of query tile 0 and 1 (224 registers each):
//                thread t owns one query row (its TMEM lane) and reads the row's
//                128 scores, so the row max needs no shuffles (three-input max,
//                eight independent chains); exp2 of the scores (pre-multiplied
//                by scale * log2(e)) in fp32, two pairs in four on the MUFU
//                (ex2.approx) and two on the FMA pipe (fa_ex2_poly_f2), each
//                rounded once to fp16 and stored into tensor memory (row =
//                lane, two keys per column: the A layout of the P V MMA); the
//                row sum of P accumulates in fp32 from the unrounded values.
//                O accumulates in TMEM over the key tiles (the P V MMA adds
//                into it).  The row max used for the exps is raised only when a
//                tile's max exceeds it by more than 8 (so p <= 2^8, as exact in
//                fp16 as p <= 1); then the warp rescales its rows of O in TMEM
//                (and its row sum) between the previous P V and the next.
// While one warpgroup computes its softmax, the tensor core works on the other
// tile's S and P V.  Keys of a partial last tile of a source are masked to
// -inf.  Every wait is bounded; on give-up the CTA drains and frees TMEM.  A
// CTA whose second query tile lies wholly past Tq runs one tile.
__device__ unsigned int g_attn_status = 0;

constexpr int kFaBM = 128, kFaBN = 128, kFaD = 64, kFaStages = 4;
constexpr int kFaThreads = 384;
constexpr int kFaLaunchRegs = 168, kFaRegsControl = 56, kFaRegsSoftmax = 224;
static_assert(128 * kFaRegsControl + 256 * kFaRegsSoftmax <= kFaThreads * kFaLaunchRegs, "register split");
constexpr int kFaTile = 128 * 128;  // bytes of a 128-row x 64-fp16 tile
constexpr uint32_t kFaTmemCols = 512;
// TMEM columns: S_i at 128 i (fp32), O_i at 256 + 64 i (fp32), P_i at 384 + 64 i (fp16 pairs).
constexpr int kFaSOff = 0, kFaOOff = 256, kFaPOff = 384;
struct FaSmem {
  static constexpr int Q = 0;                            // Q_i at Q + i * tile
  static constexpr int KV = Q + 2 * kFaTile;             // stage s: K at KV + 2s * tile, V next
  static constexpr int BAR = KV + kFaStages * 2 * kFaTile;
  static constexpr int NBAR = 1 + 2 * kFaStages + 10 + 1;
  static constexpr int BYTES = BAR + NBAR * 8 + 16 + 1024;
};

struct FaParams {
  int n1, n2;          // key tiles of the first and second source
  int64_t Tq, Tk, Tk2;
  int H;
  float c2;            // scale * log2(e)
  __half* o;
  int64_t ldo;         // halves
  // Q8_0 form: the output projection's prepared activations (codes [B*Tq][H*64],
  // fp32 split scales [H*2][qld]) instead of o; qvar: the quantizer variant.
  int8_t* qc;
  float* qs;
  int64_t qld;
  int qvar;
};

__device__ __forceinline__ float fa_max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float fa_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// exp2 of two fp32 arguments, each rounded once to fp16 (P's type for the P V
// MMA).  The argument stays fp32: an fp16 argument near -10 carries an absolute
// error of 2^-8, 0.3% in p, six times the fp16 rounding of the result.
__device__ __forceinline__ uint32_t fa_pack_h2(float2 v) {
  const __half2 y = __floats2half2_rn(v.x, v.y);
  return *reinterpret_cast<const uint32_t*>(&y);
}

// exp2 of an fp32 pair on the FMA pipe (the MUFU pipe is the softmax's
// bottleneck).  Cody-Waite reduction
// 2^x = 2^n * 2^f with n = rint(x), f = x - n in [-0.5, 0.5]; 2^f by a cubic
// fitted here for least maximum relative error on [-0.5, 0.5] (Lawson's
// reweighted least squares on Chebyshev nodes): 7.5e-5 at most, under half
// an fp16 ulp (2^-12).  x <= 8 (scores minus a row max that trails the true
// one by at most 8); x is clamped at -125 so 2^n stays a normal exponent, and
// 2^-125 rounds to fp16 0 as the -inf of a masked key does.
__device__ __forceinline__ float2 fa_ex2_poly_f2(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23: x + kRound holds rint(x) in its low mantissa bits
  const float2 one = make_float2(1.0f, 1.0f), neg = make_float2(-1.0f, -1.0f);
  x = make_float2(fmaxf(x.x, -125.0f), fmaxf(x.y, -125.0f));
  const float2 r = ffma2(x, one, make_float2(kRound, kRound));
  const float2 n = ffma2(r, one, make_float2(-kRound, -kRound));
  const float2 f = ffma2(n, neg, x);
  float2 q = ffma2(make_float2(0.0551716685f, 0.0551716685f), f, make_float2(0.242611140f, 0.242611140f));
  q = ffma2(q, f, make_float2(0.693260968f, 0.693260968f));
  q = ffma2(q, f, make_float2(0.999928057f, 0.999928057f));
  // 2^n: n (two's complement in r's low bits) added to q's exponent field.
  const float ya = __uint_as_float(__float_as_uint(q.x) + (__float_as_uint(r.x) << 23));
  const float yb = __uint_as_float(__float_as_uint(q.y) + (__float_as_uint(r.y) << 23));
  return make_float2(ya, yb);
}

// Shared-memory descriptor for an MN-major operand with the 128-byte swizzle
// (MN atoms `lbo` bytes apart; V is one atom wide); 8-row K groups 1024 bytes
// apart.
__device__ __forceinline__ uint64_t smem_desc_mn_sw128(uint32_t addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3fffu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// One thread's row of one head (64 fp16-rounded outputs) -> two Q8_0 blocks of
// the prepared activations: the stand-alone quantizer's arithmetic on the same
// fp16 values, so the bytes equal b2q_heads_act_prepare of the fp16 output.
template <int VARIANT>
__device__ __forceinline__ void fa_store_q8(const float (&hv)[kFaD], int8_t* codes, float* scales, int64_t ld) {
#pragma unroll
  for (int j = 0; j < kFaD / kQK; ++j) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < kQK; ++i) amax = fmaxf(amax, fabsf(hv[j * kQK + i]));
    float d, inv;
    q8_scale<VARIANT>(amax, d, inv);
    uint32_t q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float* v = &hv[j * kQK + 4 * i];
      q[i] = quantize_code<VARIANT>(v[0], inv) | (quantize_code<VARIANT>(v[1], inv) << 8) |
             (quantize_code<VARIANT>(v[2], inv) << 16) | (quantize_code<VARIANT>(v[3], inv) << 24);
    }
    uint4* dst = reinterpret_cast<uint4*>(codes + j * kQK);
    dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
    dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
    scales[j * ld] = q8_split_scale(d);
  }
}

// EMU: of every 4 exp pairs, how many run as the FMA-pipe polynomial.  Q8: the
// output goes out as Q8_0 prepared activations (FaParams::qc / qs).
template <int EMU, bool Q8>
__global__ void __launch_bounds__(kFaThreads, 1)
    attention_f16_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_k2,
                         const __grid_constant__ CUtensorMap tm_v2, const FaParams p) {
  extern __shared__ uint8_t fa_smem_raw[];
  uint8_t* smem = fa_smem_raw + ((1024u - (smem_u32(fa_smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + FaSmem::BAR);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + kFaStages;
  uint64_t* s_full = kv_empty + kFaStages;  // [2] per query tile
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* p_empty = p_full + 2;
  uint64_t* pv_full = p_empty + 2;
  uint64_t* done = pv_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  unsigned int* status = &g_attn_status;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bh = static_cast<int64_t>(blockIdx.z) * p.H + blockIdx.y;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * 2 * kFaBM;
  const int nq = q0 + kFaBM < p.Tq ? 2 : 1;  // query tiles this CTA runs
  const int ntiles = p.n1 + p.n2;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kFaStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);  // one arrival per softmax warp
      mbar_init(&p_full[i], 4);
      mbar_init(&p_empty[i], 1);
      mbar_init(&pv_full[i], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    if (p.n2) {
      tma_prefetch_desc(&tm_k2);
      tma_prefetch_desc(&tm_v2);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kFaTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp < 4) {
    setmaxnreg_dec<kFaRegsControl>();
    if (warp == 0) {
      // ---------------------------------------------------------- producer
      if (elect_one()) {
        uint32_t issued = 0, issued_par = 0;
        mbar_arrive_expect_tx(q_full, nq * kFaTile);
        for (int i = 0; i < nq; ++i)
          tma_load_2d(smem + FaSmem::Q + i * kFaTile, &tm_q, q_full, 0, static_cast<int32_t>(bh * p.Tq + q0 + i * kFaBM));
        for (int t = 0; t < ntiles; ++t) {
          const int st = t % kFaStages;
          const uint32_t ph = (t / kFaStages) & 1u;
          if (!mbar_wait(&kv_empty[st], ph ^ 1u, status, kDevWaitProducer, abort_flag)) break;
          const bool second = t >= p.n1;
          const int64_t row = second ? bh * p.Tk2 + static_cast<int64_t>(t - p.n1) * kFaBN
                                     : bh * p.Tk + static_cast<int64_t>(t) * kFaBN;
          uint8_t* kd = smem + FaSmem::KV + 2 * st * kFaTile;
          mbar_arrive_expect_tx(&kv_full[st], 2 * kFaTile);
          tma_load_2d(kd, second ? &tm_k2 : &tm_k, &kv_full[st], 0, static_cast<int32_t>(row));
          tma_load_2d(kd + kFaTile, second ? &tm_v2 : &tm_v, &kv_full[st], 0, static_cast<int32_t>(row));
          issued |= 1u << st;
          issued_par = (issued_par & ~(1u << st)) | (ph << st);
        }
        // every issued copy lands before the CTA may exit
        mbar_wait(q_full, 0, status, kDevWaitDrain, nullptr);
        for (int st = 0; st < kFaStages; ++st)
          if ((issued >> st) & 1u) mbar_wait(&kv_full[st], (issued_par >> st) & 1u, status, kDevWaitDrain, nullptr);
      }
    } else if (warp == 1) {
      // -------------------------------------------------------- MMA issuer
      if (elect_one()) {
        constexpr uint32_t idesc_qk = idesc_f16(kFaBM, kFaBN);
        constexpr uint32_t idesc_pv = idesc_f16(kFaBM, kFaD) | (1u << 16);  // B (V) MN-major
        bool ok = mbar_wait(q_full, 0, status, kDevWaitMma, abort_flag);
        // S_i(t) = Q_i K(t)^T (issued once K(t) has landed and the softmax has read S_i(t-1)).
        auto issue_s = [&](int i, int t) {
          const int st = t % kFaStages;
          const uint32_t k_addr = smem_u32(smem + FaSmem::KV + 2 * st * kFaTile);
          const uint32_t q_addr = smem_u32(smem + FaSmem::Q + i * kFaTile);
#pragma unroll
          for (int kk = 0; kk < kFaD / 16; ++kk)
            mma_f16(tmem + kFaSOff + i * kFaBN, smem_desc_k_sw128(q_addr + kk * 32),
                    smem_desc_k_sw128(k_addr + kk * 32), idesc_qk, kk > 0 ? 1u : 0u);
          mma_commit(&s_full[i]);
        };
        // (P V)_i of key tile u (issued once P_i(u) is stored).
        auto issue_pv = [&](int i, int u) {
          const int st = u % kFaStages;
          const uint32_t v_addr = smem_u32(smem + FaSmem::KV + (2 * st + 1) * kFaTile);
#pragma unroll
          for (int kk = 0; kk < kFaBN / 16; ++kk)  // 16 keys (8 columns of P) per MMA; O accumulates over the key tiles
            mma_f16_ts(tmem + kFaOOff + i * kFaD, tmem + kFaPOff + i * (kFaBN / 2) + kk * 8,
                       smem_desc_mn_sw128(v_addr + kk * 2048, 0), idesc_pv, (kk > 0 || u > 0) ? 1u : 0u);
          mma_commit(&pv_full[i]);
          mma_commit(&p_empty[i]);
        };
        // Each query tile's chain advances on its own barriers: the issuer polls
        // them without blocking and issues whatever is ready, S before P V, so
        // that one softmax warpgroup's next S never waits behind the other's P.
        // A K / V stage is released once both tiles' P V of it are issued.  The
        // loop gives up (status kDevWaitMma) after kWaitBudgetNs without progress.
        int ns[2] = {0, 0}, npv[2] = {0, 0}, rel = 0;
        unsigned long long t_last = globaltimer_ns();
        uint32_t idle = 0;
        while (ok && rel < ntiles) {
          bool progress = false;
          for (int i = 0; i < nq; ++i) {
            const int t = ns[i];
            if (t < ntiles && mbar_test(&kv_full[t % kFaStages], (t / kFaStages) & 1u) &&
                mbar_test(&s_empty[i], (t & 1u) ^ 1u)) {
              tc_fence_after();
              issue_s(i, t);
              ns[i] = t + 1;
              progress = true;
            }
          }
          for (int i = 0; i < nq; ++i) {
            const int u = npv[i];
            if (u < ns[i] && mbar_test(&p_full[i], u & 1u)) {
              tc_fence_after();
              issue_pv(i, u);
              npv[i] = u + 1;
              progress = true;
            }
          }
          const int pv_done = nq > 1 ? min(npv[0], npv[1]) : npv[0];
          for (; rel < pv_done; ++rel) mma_commit(&kv_empty[rel % kFaStages]);
          if (progress) {
            t_last = globaltimer_ns();
            idle = 0;
          } else if ((++idle & 63u) == 0) {
            if (*abort_flag) {
              ok = false;
            } else if (globaltimer_ns() - t_last > kWaitBudgetNs) {
              record_device_error(status, kDevWaitMma);
              *abort_flag = 1;
              ok = false;
            }
          }
        }
        mma_commit(done);
        mbar_wait(done, 0, status, kDevWaitDrain, nullptr);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax
    setmaxnreg_inc<kFaRegsSoftmax>();
    const int i = (warp - 4) >> 2;     // query tile of this warpgroup
    const int qw = warp & 3;           // TMEM lane quarter
    const int row = qw * 32 + lane;    // query row within the tile
    if (i < nq) {
      const uint32_t lane_addr = static_cast<uint32_t>(qw * 32) << 16;
      const uint32_t ts = tmem + lane_addr + kFaSOff + i * kFaBN;
      const uint32_t tpv = tmem + lane_addr + kFaOOff + i * kFaD;
      const uint32_t tp = tmem + lane_addr + kFaPOff + i * (kFaBN / 2);
      float m = -INFINITY;
      float l = 0.0f;  // the row sum of P (fp32, unrounded values)
      bool ok = true;
      for (int t = 0; t < ntiles && ok; ++t) {
        const uint32_t par = t & 1u;
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[i], par, status, kDevWaitEpilogue, abort_flag));
        if (!ok) break;
        tc_fence_after();
        uint32_t sr[kFaBN];
#pragma unroll
        for (int c = 0; c < kFaBN; c += 32) tmem_ld_32x32b_x32(ts + c, *reinterpret_cast<uint32_t(*)[32]>(&sr[c]));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[i]);  // S_i is free for the next key tile's Q K^T
        const bool second = t >= p.n1;
        const int64_t valid64 = (second ? p.Tk2 : p.Tk) - static_cast<int64_t>(second ? t - p.n1 : t) * kFaBN;
        if (valid64 < kFaBN) {  // a partial last tile of its source: the missing keys score -inf
#pragma unroll
          for (int c = 0; c < kFaBN; ++c)
            if (c >= valid64) sr[c] = __float_as_uint(-INFINITY);
        }
        // Row max over raw scores (scale > 0 commutes with max): three-input
        // max, 8 independent chains.
        float mx8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) mx8[j] = __uint_as_float(sr[j]);
#pragma unroll
        for (int c = 8; c < kFaBN; c += 16)
#pragma unroll
          for (int j = 0; j < 8; ++j) mx8[j] = fa_max3(mx8[j], __uint_as_float(sr[c + j]), __uint_as_float(sr[c + 8 + j]));
        const float mx = fa_max3(fa_max3(mx8[0], mx8[1], mx8[2]), fa_max3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
        float m_new = fmaxf(m, __fmul_rn(mx, p.c2));
        bool grow = true;
        if (t > 0 && !(m_new > m + 8.0f)) {  // keep the row max: p stays <= 2^8
          m_new = m;
          grow = false;
        }
        const float alpha = grow ? fa_ex2(m - m_new) : 1.0f;
        // exp2 of the whole row into packed fp16 registers, EMU of every 4
        // pairs on the FMA pipe; only the stores wait for P_i to be free (the
        // previous key tile's P V MMA).
        uint32_t pk[kFaBN / 2];
        {
          const float2 c2 = make_float2(p.c2, p.c2), nm = make_float2(-m_new, -m_new), one = make_float2(1.0f, 1.0f);
          float2 ls[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                          make_float2(0.0f, 0.0f)};
#pragma unroll
          for (int c = 0; c < kFaBN; c += 2) {
            const float2 x = ffma2(make_float2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), c2, nm);
            const float2 y = (EMU > 0 && ((c >> 1) & 3) < EMU) ? fa_ex2_poly_f2(x) : make_float2(fa_ex2(x.x), fa_ex2(x.y));
            pk[c >> 1] = fa_pack_h2(y);
            ls[(c >> 1) & 3] = ffma2(y, one, ls[(c >> 1) & 3]);
          }
          l = __fmaf_rn(l, alpha, ((ls[0].x + ls[0].y) + (ls[1].x + ls[1].y)) + ((ls[2].x + ls[2].y) + (ls[3].x + ls[3].y)));
        }
        ok = __all_sync(0xffffffffu, mbar_wait(&p_empty[i], par ^ 1u, status, kDevWaitEpilogue, abort_flag));
        if (!ok) break;
        if (t > 0 && __any_sync(0xffffffffu, grow)) {
          // The previous P V is complete (p_empty): rescale this warp's rows of O
          // before the next P V adds into it (the row sum was rescaled above).
          tc_fence_after();
          uint32_t r[kFaD];
          tmem_ld_32x32b_x32(tpv, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
          tmem_ld_32x32b_x32(tpv + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
          tmem_wait_ld();
#pragma unroll
          for (int d = 0; d < kFaD; ++d) r[d] = __float_as_uint(__fmul_rn(__uint_as_float(r[d]), alpha));
          tmem_st_32x32b_x32(tpv, *reinterpret_cast<const uint32_t(*)[32]>(&r[0]));
          tmem_st_32x32b_x32(tpv + 32, *reinterpret_cast<const uint32_t(*)[32]>(&r[32]));
        }
        // P_i into tensor memory (row = lane, two keys per column), then to the MMA.
        tmem_st_32x32b_x32(tp, *reinterpret_cast<const uint32_t(*)[32]>(&pk[0]));
        tmem_st_32x32b_x32(tp + 32, *reinterpret_cast<const uint32_t(*)[32]>(&pk[32]));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[i]);
        m = m_new;
      }
      float o[kFaD + 1];  // o[64]: the row sum of P
      if (ok && ntiles > 0) {  // O from TMEM once the last P V is complete
        ok = __all_sync(0xffffffffu, mbar_wait(&pv_full[i], (ntiles - 1) & 1u, status, kDevWaitEpilogue, abort_flag));
        if (ok) {
          tc_fence_after();
          uint32_t r[kFaD];
          tmem_ld_32x32b_x32(tpv, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
          tmem_ld_32x32b_x32(tpv + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
          tmem_wait_ld();
#pragma unroll
          for (int d = 0; d < kFaD; ++d) o[d] = __uint_as_float(r[d]);
          o[kFaD] = l;
        }
      }
      const int64_t tq = q0 + i * kFaBM + row;
      if (Q8 && ok && tq < p.Tq) {
        const float inv = 1.0f / o[kFaD];
        float hv[kFaD];  // the fp16 output values, as the fp16 form stores them
#pragma unroll
        for (int d = 0; d < kFaD; ++d) hv[d] = __half2float(__float2half_rn(o[d] * inv));
        const int64_t r = static_cast<int64_t>(blockIdx.z) * p.Tq + tq;
        int8_t* codes = p.qc + r * (static_cast<int64_t>(p.H) * kFaD) + static_cast<int64_t>(blockIdx.y) * kFaD;
        float* scales = p.qs + static_cast<int64_t>(blockIdx.y) * (kFaD / kQK) * p.qld + r;
        if (p.qvar == 0)
          fa_store_q8<0>(hv, codes, scales, p.qld);
        else
          fa_store_q8<1>(hv, codes, scales, p.qld);
      } else if (ok && tq < p.Tq) {
        const float inv = 1.0f / o[kFaD];
        __half* dst = p.o + (static_cast<int64_t>(blockIdx.z) * p.Tq + tq) * p.ldo +
                      static_cast<int64_t>(blockIdx.y) * kFaD;
#pragma unroll
        for (int d = 0; d < kFaD; d += 8) {
          uint32_t pk[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const __half2 h2 = __floats2half2_rn(o[d + 2 * j] * inv, o[d + 2 * j + 1] * inv);
            pk[j] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          *reinterpret_cast<uint4*>(dst + d) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kFaTmemCols);
  }
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

namespace {

template <bool Q8>
cudaError_t launch_attention_f16_t(const void* q, const void* k, const void* v, const void* k2, const void* v2,
                                   int64_t B, int H, int64_t Tq, int64_t Tk, int64_t Tk2, float scale, FaParams p,
                                   cudaStream_t s) {
  if (B == 0 || Tq == 0) return cudaSuccess;
  CUtensorMap tq, tk, tv, tk2, tv2;
  const uint64_t bh = static_cast<uint64_t>(B) * H;
  auto map = [](CUtensorMap* m, const void* base, uint64_t rows) {
    return make_tensor_map_2d(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, base, kFaD, rows, kFaD * 2, kFaD, kFaBN,
                              CU_TENSOR_MAP_SWIZZLE_128B);
  };
  if (!map(&tq, q, bh * Tq) || !map(&tk, k, bh * Tk) || !map(&tv, v, bh * Tk)) return cudaErrorInvalidValue;
  const bool second = k2 && Tk2 > 0;
  if (!map(&tk2, second ? k2 : k, second ? bh * Tk2 : bh * Tk) || !map(&tv2, second ? v2 : v, second ? bh * Tk2 : bh * Tk))
    return cudaErrorInvalidValue;
  p.n1 = static_cast<int>((Tk + kFaBN - 1) / kFaBN);
  p.n2 = second ? static_cast<int>((Tk2 + kFaBN - 1) / kFaBN) : 0;
  p.Tq = Tq;
  p.Tk = Tk;
  p.Tk2 = second ? Tk2 : 0;
  p.H = H;
  p.c2 = scale * 1.4426950408889634f;  // log2(e)
  // Half of the exps on the FMA pipe.
  constexpr auto kernel = attention_f16_kernel<2, Q8>;
  static bool attr_set[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    // The register split needs the kernel compiled at exactly kFaLaunchRegs, or
    // setmaxnreg.inc could wait for registers that do not exist.
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != kFaLaunchRegs) return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FaSmem::BYTES);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const dim3 grid(static_cast<unsigned>((Tq + 2 * kFaBM - 1) / (2 * kFaBM)), static_cast<unsigned>(H),
                  static_cast<unsigned>(B));
  kernel<<<grid, kFaThreads, FaSmem::BYTES, s>>>(tq, tk, tv, tk2, tv2, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attention_f16(const void* q, const void* k, const void* v, const void* k2, const void* v2,
                                 int64_t B, int H, int64_t Tq, int64_t Tk, int64_t Tk2, float scale, void* o,
                                 int64_t ldo_halves, cudaStream_t s) {
  FaParams p{};
  p.o = static_cast<__half*>(o);
  p.ldo = ldo_halves;
  return launch_attention_f16_t<false>(q, k, v, k2, v2, B, H, Tq, Tk, Tk2, scale, p, s);
}

cudaError_t launch_attention_f16_q8(const void* q, const void* k, const void* v, const void* k2, const void* v2,
                                    int64_t B, int H, int64_t Tq, int64_t Tk, int64_t Tk2, float scale,
                                    int8_t* codes, float* scales, int64_t ld, int variant, cudaStream_t s) {
  FaParams p{};
  p.qc = codes;
  p.qs = scales;
  p.qld = ld;
  p.qvar = variant;
  return launch_attention_f16_t<true>(q, k, v, k2, v2, B, H, Tq, Tk, Tk2, scale, p, s);
}

cudaError_t read_attention_status(unsigned int* value, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_attn_status, sizeof(unsigned int));
  if (e != cudaSuccess || !clear) return e;
  const unsigned int zero = 0;
  return cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(unsigned int));
}

}  // namespace b2q
