// b2q_gemm_f16.cuh -- F16 weights x F32 activations (GGML_OP_MUL_MAT with
// src0 F16): the activations are rounded to fp16 first (ggml's CPU backend
// converts src1 to its vec_dot_type, F16, with round-to-nearest-even), then
//   y[m][n] = sum_k w16[n][k] * x16[m][k]   (fp32 accumulation)
// on the tensor cores: tcgen05.mma kind::f16 (A = B = F16, never BF16), fp32
// accumulators in TMEM carried over all of K.  No per-block scales, so this is
// a plain GEMM: the epilogue runs once per tile, not once per 32 values.
//
// Structure (persistent, one CTA per SM, 576 threads):
//   warp 0      TMA producer: weight tile [128 rows x 64 K] and activation
//               tile [256 tokens x 64 K] per stage (one 128-byte swizzle row
//               of fp16 each), 4 stages of 48 KB.  The MMA thread waits for
//               stage data ~58% of its time; 8 stages of 32 K (64-byte swizzle,
//               the same bytes in flight) measured slower (fc1 57.8 against
//               50.2 us): twice the per-stage barrier and issue work.
//   warp 1      TMEM allocator (512 columns) + single-thread MMA issuer:
//               4 MMAs (M 128, N 256, K 16) per stage into one of two
//               256-column accumulators, so a tile's epilogue overlaps the
//               next tile's MMAs
//   warps 2..17 epilogue: thread t of warp w owns weight row 32*(w%4) + t (its
//               TMEM lane) and 64 of the 256 token columns (warps 2-5 the
//               first quarter, 6-9 the second, ...); 32-column TMEM loads,
//               double-buffered, bias add, 128-byte coalesced stores.  The
//               stores set the pace: with one warp per lane quarter the
//               epilogue took ~19.8 k cycles per tile against ~8.2 k of MMA
//               (fc1 68.6 us); two per quarter 52.2 us, four 50.2 us.
// Tiles run weight-row-fastest, so the CTAs of one wave share activation tiles
// in L2.  Every wait is bounded; no TMA multicast.
//
// Included by b2q_gemm_tc.cu (same device status word, one translation unit).
#pragma once

namespace b2q {

namespace f16 {

constexpr int kBM = 128;             // weight rows per tile (MMA M, TMEM lanes)
constexpr int kBN = 256;             // tokens per tile (MMA N)
constexpr int kStageK = 64;          // fp16 values of K per stage (128 bytes)
constexpr int kMmaK = 16;            // K per kind::f16 MMA (32 bytes)
constexpr int kStages = 4;
constexpr CUtensorMapSwizzle kSwizzle = CU_TENSOR_MAP_SWIZZLE_128B;
constexpr int kAccs = 2;             // TMEM accumulators of kBN columns
constexpr uint32_t kTmemColsF = kAccs * kBN;
constexpr int kEpiWarp0 = 2, kEpiWarps = 16;
constexpr int kEpiCols = kBN / (kEpiWarps / 4);  // token columns per epilogue warp
constexpr int kThreadsF = (kEpiWarp0 + kEpiWarps) * 32;
constexpr int kABytes = kBM * kStageK * 2;  // 16 KB
constexpr int kBBytes = kBN * kStageK * 2;  // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kOffBars = kStages * kStageBytes;
constexpr int kNBars = 2 * kStages + 2 * kAccs + 1;  // full, empty, acc_full, acc_empty, done
constexpr int kSmemF = kOffBars + kNBars * 8 + 16 + 1024;  // + alignment slack
static_assert(kSmemF <= 227 * 1024, "shared memory per CTA");
static_assert(kStageBytes % 1024 == 0 && kABytes % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
static_assert(kTmemColsF <= 512, "TMEM columns");

struct F16Params {
  int M, N, kst, n_tiles, num_tiles;
  float* y;           // fp32 output [M][ldy], or
  __half* y16;        // fp16 output [M][ldy] (round to nearest even) when not null
  int64_t ldy;
  const float* bias;
  // Grouped form only (the planned sparse convolution): the number of
  // 256-row tiles of x is read from device memory (*m_tiles_dev), and tile j's
  // rows multiply the weight's K slice [k_group[j] * K, (k_group[j] + 1) * K).
  const int32_t* m_tiles_dev;
  const int32_t* k_group;
};

// OUT16: fp16 output (y16), else fp32 (y); one instantiation each, so the
// store loop carries no per-element branch on the output type.  GROUPED: the
// tile count and each token tile's weight K slice come from device memory.
template <bool OUT16, bool GROUPED = false>
__global__ void __launch_bounds__(kThreadsF, 1)
    gemm_f16_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                    const F16Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + kAccs;
  uint64_t* mma_done = acc_empty + kAccs;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < kAccs; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemColsF);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  int num_tiles = p.num_tiles, M = p.M;
  if constexpr (GROUPED) {  // written by an earlier kernel on this stream; clamped to the buffers' capacity
    const int cap = p.num_tiles / p.n_tiles;
    const int mt = min(max(__ldg(p.m_tiles_dev), 0), cap);
    num_tiles = p.n_tiles * mt;
    M = mt * kBN;
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      uint32_t stage = 0, phase = 0, issued_mask = 0, issued_par = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const int n0 = (tile % p.n_tiles) * kBM;
        const int m0 = (tile / p.n_tiles) * kBN;
        const int kw0 = GROUPED ? min(max(__ldg(p.k_group + tile / p.n_tiles), 0), 26) * p.kst * kStageK : 0;
        for (int ks = 0; ks < p.kst; ++ks) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, &g_device_status, kDevWaitProducer, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sb = smem + stage * kStageBytes;
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          tma_load_2d(sb, &tm_w, &full[stage], kw0 + ks * kStageK, n0);  // x * 2 bytes: multiples of 128
          tma_load_2d(sb + kABytes, &tm_x, &full[stage], ks * kStageK, m0);
          issued_mask |= 1u << stage;
          issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      for (int s = 0; s < kStages; ++s)  // every issued copy lands before the CTA may exit
        if ((issued_mask >> s) & 1u)
          mbar_wait(&full[s], (issued_par >> s) & 1u, &g_device_status, kDevWaitDrain, nullptr);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_f16(kBM, kBN);
      uint32_t stage = 0, phase = 0, t = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++t) {
        const uint32_t a = t & (kAccs - 1), apar = (t / kAccs) & 1u;
        if (!mbar_wait(&acc_empty[a], apar ^ 1u, &g_device_status, kDevWaitMma, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + a * kBN;
        for (int ks = 0; ks < p.kst; ++ks) {
          if (!mbar_wait(&full[stage], phase, &g_device_status, kDevWaitMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + stage * kStageBytes);
          const uint32_t b_base = a_base + kABytes;
#pragma unroll
          for (int j = 0; j < kStageK / kMmaK; ++j)
            mma_f16(d, smem_desc_k_sw128(a_base + j * kMmaK * 2), smem_desc_k_sw128(b_base + j * kMmaK * 2), idesc,
                    (ks | j) != 0 ? 1u : 0u);
          mma_commit(&empty[stage]);  // the stage goes back once its MMAs have read it
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) mma_commit(&acc_full[a]);
      }
      mma_commit(mma_done);  // all issued MMAs complete before TMEM is released
      mbar_wait(mma_done, 0, &g_device_status, kDevWaitDrain, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const int col0 = ((warp - kEpiWarp0) >> 2) * kEpiCols;  // this warp's first token column
    const uint32_t tlane = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    uint32_t t = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t) {
      const uint32_t a = t & (kAccs - 1), apar = (t / kAccs) & 1u;
      if (!mbar_wait(&acc_full[a], apar, &g_device_status, kDevWaitEpilogue, abort_flag)) break;
      tc_fence_after();
      const int64_t n = static_cast<int64_t>(tile % p.n_tiles) * kBM + row;
      const int64_t m0 = static_cast<int64_t>(tile / p.n_tiles) * kBN + col0;
      const bool nv = n < p.N;
      const float bv = (p.bias && nv) ? p.bias[n] : 0.0f;
      float* yp = p.y + m0 * p.ldy + n;
      __half* yp16 = p.y16 + m0 * p.ldy + n;
      uint32_t buf[2][32];
      const uint32_t tacc = tlane + a * kBN + col0;
      tmem_ld_32x32b_x32(tacc, buf[0]);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < kEpiCols / 32; ++c) {
        if (c + 1 < kEpiCols / 32) tmem_ld_32x32b_x32(tacc + (c + 1) * 32, buf[(c + 1) & 1]);
        if (nv) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int64_t m = m0 + c * 32 + i;
            const float v = __uint_as_float(buf[c & 1][i]);
            const float o = p.bias ? __fadd_rn(v, bv) : v;  // gb_linear's ggml_add
            if (m < M) {
              if constexpr (OUT16)
                yp16[(c * 32 + i) * p.ldy] = __float2half_rn(o);
              else
                yp[(c * 32 + i) * p.ldy] = o;
            }
          }
        }
        tmem_wait_ld();
        if (c == kEpiCols / 32 - 2) {  // the last chunk is in registers: the accumulator goes back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[a]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemColsF);
  }
}


// ---------------------------------------------------------------- CTA pairs
// The same GEMM on CTA pairs (cta_group::2): a cluster of two CTAs runs one
// tile of 256 weight rows x 256 tokens with MMAs of M 256, N 256, K 16 issued
// by the pair leader (cluster rank 0).  Each CTA's TMA brings, per stage, its
// own 128 weight rows and its own 128 of the 256 tokens (32 KB; the MMA reads
// A and B halves from both CTAs' shared memory at the same offsets), counted
// on the leader's `full` barrier.  Per SM that is 32 KB of L2 reads per 512
// cycles of MMA, against 48 KB for the single-CTA 128 x 256 tile -- whose
// per-SM L2 read rate (~64 B/clk) left its MMA waiting for data.  Each CTA's
// TMEM holds its 128 rows of the two 256-column accumulators; its 16 epilogue
// warps read them and release an accumulator to the leader with remote
// arrivals.  No load has a multicast qualifier: only the leader's commits are
// multicast, to the barrier at the same offset in both CTAs.
constexpr int kPairStages = 6;
constexpr int kPairABytes = kBM * kStageK * 2;        // 16 KB: this CTA's 128 weight rows
constexpr int kPairBBytes = (kBN / 2) * kStageK * 2;  // 16 KB: this CTA's 128 tokens
constexpr int kPairStageBytes = kPairABytes + kPairBBytes;
constexpr int kPairOffBars = kPairStages * kPairStageBytes;
constexpr int kPairNBars = 2 * kPairStages + 2 * kAccs + 1;
constexpr int kPairSmem = kPairOffBars + kPairNBars * 8 + 16 + 1024;
static_assert(kPairSmem <= 227 * 1024, "shared memory per CTA");
static_assert(kPairStageBytes % 1024 == 0 && kPairABytes % 1024 == 0, "swizzle atoms stay 1024-byte aligned");

template <bool OUT16>
__global__ void __launch_bounds__(kThreadsF, 1)
    gemm_f16_pair_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                         const F16Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPairOffBars);  // used in the leader
  uint64_t* empty = full + kPairStages;
  uint64_t* acc_full = empty + kPairStages;
  uint64_t* acc_empty = acc_full + kAccs;  // used in the leader: both CTAs' epilogue warps
  uint64_t* mma_done = acc_empty + kAccs;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < kAccs; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, kTmemColsF);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before any arrival crosses the pair
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      const uint32_t full0 = cluster_addr(full, 0);  // the leader's full[0]
      uint32_t stage = 0, phase = 0, issued_mask = 0, issued_par = 0;
      bool ok = true;
      for (int tile = cluster; ok && tile < p.num_tiles; tile += nclusters) {
        const int n0 = (tile % p.n_tiles) * (2 * kBM) + static_cast<int>(rank) * kBM;
        const int m0 = (tile / p.n_tiles) * kBN + static_cast<int>(rank) * (kBN / 2);
        for (int ks = 0; ks < p.kst; ++ks) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, &g_device_status, kDevWaitProducer, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sb = smem + stage * kPairStageBytes;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * kPairStageBytes);  // both CTAs' bytes
          const uint32_t fb = full0 + stage * 8;
          tma_load_2d_pair(sb, &tm_w, fb, ks * kStageK, n0);
          tma_load_2d_pair(sb + kPairABytes, &tm_x, fb, ks * kStageK, m0);
          issued_mask |= 1u << stage;
          issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (leader)  // every issued copy of both CTAs lands before the pair may exit
        for (int s = 0; s < kPairStages; ++s)
          if ((issued_mask >> s) & 1u)
            mbar_wait(&full[s], (issued_par >> s) & 1u, &g_device_status, kDevWaitDrain, nullptr);
    }
  } else if (warp == 1) {
    // ------------------------------------------------- MMA issuer (leader)
    if (leader && elect_one()) {
      constexpr uint32_t idesc = idesc_f16(2 * kBM, kBN);
      uint32_t stage = 0, phase = 0, t = 0;
      bool ok = true;
      for (int tile = cluster; ok && tile < p.num_tiles; tile += nclusters, ++t) {
        const uint32_t a = t & (kAccs - 1), apar = (t / kAccs) & 1u;
        if (!mbar_wait_cluster(&acc_empty[a], apar ^ 1u, &g_device_status, kDevWaitMma, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + a * kBN;
        for (int ks = 0; ks < p.kst; ++ks) {
          if (!mbar_wait(&full[stage], phase, &g_device_status, kDevWaitMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + stage * kPairStageBytes);
          const uint32_t b_base = a_base + kPairABytes;
#pragma unroll
          for (int j = 0; j < kStageK / kMmaK; ++j)
            mma_f16_pair(d, smem_desc_k_sw128(a_base + j * kMmaK * 2), smem_desc_k_sw128(b_base + j * kMmaK * 2),
                         idesc, (ks | j) != 0 ? 1u : 0u);
          mma_commit_pair(&empty[stage], 0x3);  // both CTAs' stage goes back once the MMAs have read it
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) mma_commit_pair(&acc_full[a], 0x3);
      }
      mma_commit_pair(mma_done, 0x1);  // all issued MMAs complete before TMEM is released
      mbar_wait(mma_done, 0, &g_device_status, kDevWaitDrain, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int col0 = ((warp - kEpiWarp0) >> 2) * kEpiCols;
    const uint32_t tlane = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    uint32_t t = 0;
    for (int tile = cluster; tile < p.num_tiles; tile += nclusters, ++t) {
      const uint32_t a = t & (kAccs - 1), apar = (t / kAccs) & 1u;
      if (!mbar_wait(&acc_full[a], apar, &g_device_status, kDevWaitEpilogue, abort_flag)) break;
      tc_fence_after();
      const int64_t n = static_cast<int64_t>(tile % p.n_tiles) * (2 * kBM) + rank * kBM + row;
      const int64_t m0 = static_cast<int64_t>(tile / p.n_tiles) * kBN + col0;
      const bool nv = n < p.N;
      const float bv = (p.bias && nv) ? p.bias[n] : 0.0f;
      float* yp = p.y + m0 * p.ldy + n;
      __half* yp16 = p.y16 + m0 * p.ldy + n;
      uint32_t buf[2][32];
      const uint32_t tacc = tlane + a * kBN + col0;
      tmem_ld_32x32b_x32(tacc, buf[0]);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < kEpiCols / 32; ++c) {
        if (c + 1 < kEpiCols / 32) tmem_ld_32x32b_x32(tacc + (c + 1) * 32, buf[(c + 1) & 1]);
        if (nv) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int64_t m = m0 + c * 32 + i;
            const float v = __uint_as_float(buf[c & 1][i]);
            const float o = p.bias ? __fadd_rn(v, bv) : v;  // gb_linear's ggml_add
            if (m < p.M) {
              if constexpr (OUT16)
                yp16[(c * 32 + i) * p.ldy] = __float2half_rn(o);
              else
                yp[(c * 32 + i) * p.ldy] = o;
            }
          }
        }
        tmem_wait_ld();
        if (c == kEpiCols / 32 - 2) {  // the last chunk is in registers: the accumulator goes back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(cluster_addr(&acc_empty[a], 0));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the leader's MMAs into this CTA's TMEM and its reads of this CTA's stages are over
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemColsF);
  }
}

}  // namespace f16

// The plain F16 mul_mat runs on CTA pairs (f16::gemm_f16_pair_kernel), one
// persistent pair per co-resident cluster slot.
cudaError_t launch_gemm_f16(const void* w, int64_t ldw_bytes, const void* x16, int64_t ldx_bytes, int64_t M,
                            int64_t N, int64_t K, float* y, int64_t ldy, const float* bias, int num_sms,
                            cudaStream_t s, void* y16) {
  (void)num_sms;
  if (M == 0 || N == 0) return cudaSuccess;
  if (K <= 0 || K % 8 != 0 || M > INT32_MAX || N > INT32_MAX) return cudaErrorInvalidValue;
  CUtensorMap tm_w, tm_x;  // per CTA: 128 weight rows and 128 tokens per stage
  if (!make_tensor_map_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w, K, N, ldw_bytes, f16::kStageK, f16::kBM,
                          f16::kSwizzle) ||
      !make_tensor_map_2d(&tm_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x16, K, M, ldx_bytes, f16::kStageK, f16::kBN / 2,
                          f16::kSwizzle))
    return cudaErrorInvalidValue;
  f16::F16Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.kst = static_cast<int>((K + f16::kStageK - 1) / f16::kStageK);
  p.n_tiles = static_cast<int>((N + 2 * f16::kBM - 1) / (2 * f16::kBM));
  const int64_t tiles = static_cast<int64_t>(p.n_tiles) * ((M + f16::kBN - 1) / f16::kBN);
  if (tiles > INT32_MAX) return cudaErrorInvalidValue;
  p.num_tiles = static_cast<int>(tiles);
  p.y = y;
  p.y16 = static_cast<__half*>(y16);
  p.ldy = ldy;
  p.bias = bias;
  auto kernel = p.y16 ? f16::gemm_f16_pair_kernel<true> : f16::gemm_f16_pair_kernel<false>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(f16::kThreadsF);
  cfg.dynamicSmemBytes = f16::kPairSmem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Set up once per device: shared memory attribute, and how many pairs can be
  // resident at once (SMs pair up within a GPC).
  static std::atomic<uint64_t> ready{0};
  static int max_clusters[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const uint64_t bit = uint64_t{1} << dev;
  if (!(ready.load(std::memory_order_acquire) & bit)) {
    for (auto k : {f16::gemm_f16_pair_kernel<false>, f16::gemm_f16_pair_kernel<true>}) {
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, f16::kPairSmem);
      if (e != cudaSuccess) return e;
    }
    cfg.gridDim = dim3(2);
    int n = 0;
    cudaError_t e = cudaOccupancyMaxActiveClusters(&n, f16::gemm_f16_pair_kernel<false>, &cfg);
    if (e != cudaSuccess) return e;
    if (n < 1) return cudaErrorInvalidConfiguration;
    max_clusters[dev] = n;
    ready.fetch_or(bit, std::memory_order_acq_rel);
  }
  const int clusters = p.num_tiles < max_clusters[dev] ? p.num_tiles : max_clusters[dev];
  cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters));
  return cudaLaunchKernelEx(&cfg, kernel, tm_w, tm_x, p);
}

cudaError_t launch_gemm_f16_grouped(const void* w, int64_t ldw_bytes, int64_t Kw, const void* x16, int64_t ldx_bytes,
                                    int64_t M_cap, int64_t N, int64_t K, float* y, int64_t ldy,
                                    const int32_t* m_tiles_dev, const int32_t* k_group, int64_t max_m_tiles,
                                    int num_sms, cudaStream_t s) {
  if (N == 0 || max_m_tiles == 0) return cudaSuccess;
  // Every group's K slice must be whole stages, so a tile never reads into the next slice.
  if (K <= 0 || K % f16::kStageK != 0 || Kw % K != 0 || M_cap < max_m_tiles * f16::kBN || N > INT32_MAX ||
      M_cap > INT32_MAX)
    return cudaErrorInvalidValue;
  CUtensorMap tm_w, tm_x;
  if (!make_tensor_map_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w, Kw, N, ldw_bytes, f16::kStageK, f16::kBM,
                          f16::kSwizzle) ||
      !make_tensor_map_2d(&tm_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x16, K, M_cap, ldx_bytes, f16::kStageK, f16::kBN,
                          f16::kSwizzle))
    return cudaErrorInvalidValue;
  f16::F16Params p{};
  p.M = static_cast<int>(M_cap);
  p.N = static_cast<int>(N);
  p.kst = static_cast<int>(K / f16::kStageK);
  p.n_tiles = static_cast<int>((N + f16::kBM - 1) / f16::kBM);
  const int64_t tiles = static_cast<int64_t>(p.n_tiles) * max_m_tiles;
  if (tiles > INT32_MAX) return cudaErrorInvalidValue;
  p.num_tiles = static_cast<int>(tiles);  // upper bound; the kernel reads the real count
  p.y = y;
  p.y16 = nullptr;
  p.ldy = ldy;
  p.bias = nullptr;
  p.m_tiles_dev = m_tiles_dev;
  p.k_group = k_group;
  static std::atomic<uint64_t> ready{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  const uint64_t bit = dev < 64 ? (uint64_t{1} << dev) : 0;
  if (!bit || !(ready.load(std::memory_order_acquire) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(f16::gemm_f16_kernel<false, true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, f16::kSmemF);
    if (e != cudaSuccess) return e;
    ready.fetch_or(bit, std::memory_order_acq_rel);
  }
  const int grid = p.num_tiles < num_sms ? p.num_tiles : num_sms;
  f16::gemm_f16_kernel<false, true><<<grid, f16::kThreadsF, f16::kSmemF, s>>>(tm_w, tm_x, p);
  return cudaGetLastError();
}

}  // namespace b2q
