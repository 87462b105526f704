// b2q_gemm_q4k.cu -- Q4_K weights x Q8_K activations on the tensor cores,
// using the integer structure of the k-quants.
//
// In a Q4_K super-block (256 values) the per-sub-block scales sc_j and mins
// m_j are 6-bit integers under one fp16 d / dmin, and the Q8_K activation has
// one fp32 scale per 256 values.  So the whole super-block's dot is integer
// until two fp32 products (ggml's own dot keeps it in int32 the same way):
//   sum_j sc_j * S_j  = A1 + 8 * A2,   A1 = sum (q4 * (sc & 7)) * q8,
//                                      A2 = sum (q4 * (sc >> 3)) * q8,
//   sum_j m_j * B_j   = A3,            A3 = sum  m_j * q8,
// where every weight operand (q4*(sc&7), q4*(sc>>3) <= 105; m <= 63) fits
// int8.  The packed weight therefore holds three int8 planes; the tensor core
// accumulates A1, A2, A3 in TMEM over all 8 sub-blocks (24 MMAs per
// super-block), and the epilogue folds once per super-block:
//   acc += RN(A1*d)*da + RN(A2*8d)*da + RN(-A3*dmin)*da
// instead of once per 32 values.  |A| < 2^22, so A + 0x4B400000 read as fp32
// is 1.5*2^23 + A exactly, and one FMA with -1.5*2^23*s gives RN(A*s).
//
// Structure (persistent, one CTA per SM, 384 threads): warp 0 issues TMA,
// warp 1 issues the MMAs, warps 4-11 run the epilogue.  Tiles are 128 weight
// rows x 64 tokens; a pipeline stage holds 4 sub-blocks of the three planes
// and of the activation codes and is released by the MMA's commit; the
// super-block scales (d, dmin per row, da per token) sit in a two-slot ring
// released by the epilogue; TMEM holds two super-block groups of three
// 64-column accumulators.  No TMA multicast.
//
// Included by b2q_gemm_tc.cu: the kernel records bounded-wait failures in the
// same device status word (one translation unit, no relocatable device code).
#pragma once

namespace b2q {

namespace q4k {

constexpr int kBM = 128;
constexpr int kSubPerStage = 4;               // 32-value sub-blocks per stage
constexpr int kStageK = kSubPerStage * kQK;   // 128 bytes of K per row
constexpr int kStages = 3;
constexpr int kPlanes = 3;
constexpr int kScaleSlots = 2;                // super-block scale ring
constexpr uint32_t kTmemColsQ = 512;
constexpr int kEpiWarps = 8, kEpiWarp0 = 4;
constexpr int kThreadsQ = (kEpiWarp0 + kEpiWarps) * 32;
constexpr int kLaunchRegsQ = 168, kRegsControlQ = 40, kRegsEpilogueQ = 232;
static_assert(128 * kRegsControlQ + 256 * kRegsEpilogueQ <= kThreadsQ * kLaunchRegsQ, "register split");
constexpr int kPlaneBytes = kBM * kStageK;             // 16 KB
constexpr int kABytes = kPlanes * kPlaneBytes;         // 48 KB

// BN tokens per tile.  TMEM holds GROUPS super-block groups of three BN-column
// accumulators: two groups at BN = 64 (the MMA runs one super-block ahead of
// the epilogue), one at BN = 128 (twice the tokens per weight tile, so half
// the weight-plane traffic from L2; the MMA waits only for the epilogue's
// TMEM loads, not for its arithmetic).
template <int BN>
struct QCfg {
  static_assert(BN == 64 || BN == 128, "tile width");
  static constexpr int COLS = BN / 2;                               // token columns per epilogue thread
  static constexpr int GROUPS = 2 * kPlanes * BN <= int(kTmemColsQ) ? 2 : 1;
  static constexpr int GROUP_COLS = GROUPS == 2 ? 256 : 512;
  static constexpr int B_BYTES = BN * kStageK;
  static constexpr int STAGE_TX = kABytes + B_BYTES;
  static constexpr int STAGE_PITCH = (STAGE_TX + 1023) / 1024 * 1024;
  static constexpr int SLOT_BYTES = (2 * kBM + BN) * 4;            // d[128], dmin[128], da[BN]
  static constexpr int OFF_SCALES = kStages * STAGE_PITCH;
  static constexpr int OFF_BARS = OFF_SCALES + kScaleSlots * SLOT_BYTES;
  // full[S], empty[S], sfull[2], sempty[2], acc_full[G], acc_empty[G][3 planes], done
  static constexpr int NBARS = 2 * kStages + 2 * kScaleSlots + GROUPS + GROUPS * kPlanes + 1;
  static constexpr int SMEM = OFF_BARS + NBARS * 8 + 16 + 1024;
  static_assert(STAGE_PITCH % 1024 == 0, "swizzle alignment");
  static_assert(SLOT_BYTES % 128 == 0, "TMA destinations");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

constexpr uint32_t kMagicBits = 0x4B400000u;  // 1.5 * 2^23
constexpr float kMagic = 12582912.0f;

struct Q4kParams {
  int M, N, KSB, n_tiles, num_tiles;
  float* y;
  int64_t ldy;
  const float* bias;
  const float* gate;
  const float* resid;
  int64_t ldr;
};

// This thread's COLS columns of one plane accumulator, 32 columns per load.
template <int COLS>
__device__ __forceinline__ void load_plane(uint32_t taddr, uint32_t (&r)[COLS]) {
#pragma unroll
  for (int c = 0; c < COLS; c += 32) tmem_ld_32x32b_x32(taddr + c, *reinterpret_cast<uint32_t(*)[32]>(&r[c]));
}

// acc += RN(A * s) * da for one plane: A + 1.5*2^23 read as fp32, then
// fma(v, s, -1.5*2^23*s) = RN(A * s) exactly, then the fused accumulate.
template <int COLS>
__device__ __forceinline__ void fold_plane(const uint32_t (&r)[COLS], float s, const float* da, float2 (&acc)[COLS / 2]) {
  const float2 S = make_float2(s, s), C = make_float2(-kMagic * s, -kMagic * s);
  const float4* da4 = reinterpret_cast<const float4*>(da);
#pragma unroll
  for (int i = 0; i < COLS / 4; ++i) {
    const float4 q = da4[i];
    const float2 v0 = make_float2(__uint_as_float(r[4 * i] + kMagicBits), __uint_as_float(r[4 * i + 1] + kMagicBits));
    const float2 v1 = make_float2(__uint_as_float(r[4 * i + 2] + kMagicBits), __uint_as_float(r[4 * i + 3] + kMagicBits));
    acc[2 * i] = ffma2(ffma2(v0, S, C), make_float2(q.x, q.y), acc[2 * i]);
    acc[2 * i + 1] = ffma2(ffma2(v1, S, C), make_float2(q.z, q.w), acc[2 * i + 1]);
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreadsQ, 1)
    gemm_q4k_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                    const __grid_constant__ CUtensorMap tm_sd, const __grid_constant__ CUtensorMap tm_sm,
                    const __grid_constant__ CUtensorMap tm_sa, const Q4kParams p) {
  using C = QCfg<BN>;
  constexpr int COLS = C::COLS, GROUPS = C::GROUPS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BARS);
  uint64_t* empty = full + kStages;
  uint64_t* sfull = empty + kStages;
  uint64_t* sempty = sfull + kScaleSlots;
  uint64_t* acc_full = sempty + kScaleSlots;
  uint64_t* acc_empty = acc_full + GROUPS;  // [group][plane]: each plane goes back to the MMA when loaded
  uint64_t* mma_done = acc_empty + GROUPS * kPlanes;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);  // the MMA issuer's commit
    }
    for (int g = 0; g < kScaleSlots; ++g) {
      mbar_init(&sfull[g], 1);
      mbar_init(&sempty[g], kEpiWarps);  // one arrive per epilogue warp
    }
    for (int g = 0; g < GROUPS; ++g) {
      mbar_init(&acc_full[g], 1);
      for (int pl = 0; pl < kPlanes; ++pl) mbar_init(&acc_empty[g * kPlanes + pl], kEpiWarps * 32);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_sd);
    tma_prefetch_desc(&tm_sm);
    tma_prefetch_desc(&tm_sa);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemColsQ);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp < kEpiWarp0) {
    // ------------------------------------------------- warpgroup 0 (control)
    setmaxnreg_dec<kRegsControlQ>();
    if (warp == 0) {
      // ---------------------------------------------------------- producer
      if (elect_one()) {
        uint32_t stage = 0, phase = 0, issued_mask = 0, issued_par = 0, sbc = 0, s_mask = 0, s_par = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
          const int n0 = (tile % p.n_tiles) * kBM, m0 = (tile / p.n_tiles) * BN;
          for (int sb = 0; ok && sb < p.KSB; ++sb, ++sbc) {
            const uint32_t g = sbc & 1u, gpar = (sbc >> 1) & 1u;  // scale slot
            if (!mbar_wait(&sempty[g], gpar ^ 1u, &g_device_status, kDevWaitProducer, abort_flag)) {
              ok = false;
              break;
            }
            uint8_t* sl = smem + C::OFF_SCALES + g * C::SLOT_BYTES;
            mbar_arrive_expect_tx(&sfull[g], C::SLOT_BYTES);
            tma_load_2d(sl, &tm_sd, &sfull[g], n0, sb);
            tma_load_2d(sl + kBM * 4, &tm_sm, &sfull[g], n0, sb);
            tma_load_2d(sl + 2 * kBM * 4, &tm_sa, &sfull[g], m0, sb);
            s_mask |= 1u << g;
            s_par = (s_par & ~(1u << g)) | (gpar << g);
            for (int h = 0; h < 2; ++h) {
              if (!mbar_wait(&empty[stage], phase ^ 1u, &g_device_status, kDevWaitProducer, abort_flag)) {
                ok = false;
                break;
              }
              uint8_t* st = smem + stage * C::STAGE_PITCH;
              mbar_arrive_expect_tx(&full[stage], C::STAGE_TX);
              const int kx = (2 * sb + h) * kStageK;
#pragma unroll
              for (int pl = 0; pl < kPlanes; ++pl)
                tma_load_2d(st + pl * kPlaneBytes, &tm_w, &full[stage], kx, pl * p.N + n0);
              tma_load_2d(st + kABytes, &tm_a, &full[stage], kx, m0);
              issued_mask |= 1u << stage;
              issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
              if (++stage == kStages) {
                stage = 0;
                phase ^= 1u;
              }
            }
          }
        }
        // Every issued copy lands before the CTA may exit.
        for (int s = 0; s < kStages; ++s)
          if ((issued_mask >> s) & 1u)
            mbar_wait(&full[s], (issued_par >> s) & 1u, &g_device_status, kDevWaitDrain, nullptr);
        for (int g = 0; g < kScaleSlots; ++g)
          if ((s_mask >> g) & 1u)
            mbar_wait(&sfull[g], (s_par >> g) & 1u, &g_device_status, kDevWaitDrain, nullptr);
      }
    } else if (warp == 1) {
      // -------------------------------------------------------- MMA issuer
      if (elect_one()) {
        constexpr uint32_t idesc = idesc_i8(kBM, BN);
        uint32_t stage = 0, phase = 0, sbc = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
          for (int sb = 0; ok && sb < p.KSB; ++sb, ++sbc) {
            const uint32_t g = GROUPS == 2 ? (sbc & 1u) : 0u;
            const uint32_t gpar = GROUPS == 2 ? ((sbc >> 1) & 1u) : (sbc & 1u);
            const uint32_t dbase = tmem_base + g * C::GROUP_COLS;
            for (int h = 0; ok && h < 2; ++h) {
              if (!mbar_wait(&full[stage], phase, &g_device_status, kDevWaitMma, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t a0 = smem_u32(smem + stage * C::STAGE_PITCH);
              const uint32_t b0 = a0 + kABytes;
              // Plane-major: the first stage of a super-block waits for each
              // plane's accumulator separately, so it can start on plane 0
              // while the epilogue is still loading plane 2.
#pragma unroll
              for (int pl = 0; pl < kPlanes; ++pl) {
                if (h == 0) {
                  if (!mbar_wait(&acc_empty[g * kPlanes + pl], gpar ^ 1u, &g_device_status, kDevWaitMma, abort_flag)) {
                    ok = false;
                    break;
                  }
                  tc_fence_after();
                }
#pragma unroll
                for (int j = 0; j < kSubPerStage; ++j)
                  mma_i8(dbase + pl * BN, smem_desc_k_sw128(a0 + pl * kPlaneBytes + j * kQK),
                         smem_desc_k_sw128(b0 + j * kQK), idesc, (h | j) ? 1u : 0u);
              }
              mma_commit(&empty[stage]);  // the stage is free once these MMAs have read it
              if (++stage == kStages) {
                stage = 0;
                phase ^= 1u;
              }
            }
            if (ok) mma_commit(&acc_full[g]);
          }
        }
        // All issued MMAs complete before TMEM is released.
        mma_commit(mma_done);
        mbar_wait(mma_done, 0, &g_device_status, kDevWaitDrain, nullptr);
      }
    }
  } else {
    // ------------------------------------------------ warpgroups 1-2: epilogue
    setmaxnreg_inc<kRegsEpilogueQ>();
    const int quarter = warp & 3;               // TMEM lane quarter this warp may access
    const int chalf = (warp - kEpiWarp0) >> 2;  // which half of the BN token columns
    const int row = quarter * 32 + lane;        // this thread's weight row (TMEM lane)
    const uint32_t tlane = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + chalf * COLS;
    uint32_t sbc = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
      float2 acc[COLS / 2];
#pragma unroll
      for (int c = 0; c < COLS / 2; ++c) acc[c] = make_float2(0.0f, 0.0f);
      for (int sb = 0; sb < p.KSB; ++sb, ++sbc) {
        const uint32_t s = sbc & 1u, spar = (sbc >> 1) & 1u;
        const uint32_t g = GROUPS == 2 ? (sbc & 1u) : 0u;
        const uint32_t gpar = GROUPS == 2 ? ((sbc >> 1) & 1u) : (sbc & 1u);
        if (!mbar_wait(&sfull[s], spar, &g_device_status, kDevWaitEpilogue, abort_flag) ||
            !mbar_wait(&acc_full[g], gpar, &g_device_status, kDevWaitEpilogue, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tb = tlane + g * C::GROUP_COLS;
        const float* sl = reinterpret_cast<const float*>(smem + C::OFF_SCALES + s * C::SLOT_BYTES);
        const float d = sl[row], dmin = sl[kBM + row];
        const float* da = sl + 2 * kBM + chalf * COLS;
        // Planes 0 and 1 in flight together, plane 2 streams in while plane 0
        // is folded; TMEM goes back to the MMA as soon as all three are loaded.
        uint32_t ra[COLS], rb[COLS];
        load_plane<COLS>(tb, ra);
        load_plane<COLS>(tb + BN, rb);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&acc_empty[g * kPlanes + 0]);
        mbar_arrive(&acc_empty[g * kPlanes + 1]);
        fold_plane<COLS>(ra, d, da, acc);
        load_plane<COLS>(tb + 2 * BN, ra);
        fold_plane<COLS>(rb, 8.0f * d, da, acc);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&acc_empty[g * kPlanes + 2]);
        fold_plane<COLS>(ra, -dmin, da, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sempty[s]);  // the slot's scales are read
      }
      if (!ok) break;
      const int64_t n = static_cast<int64_t>(tile % p.n_tiles) * kBM + row;
      const int64_t m0 = static_cast<int64_t>(tile / p.n_tiles) * BN + chalf * COLS;
      if (n < p.N) {
        const float bv = p.bias ? p.bias[n] : 0.0f;
        const float2 b2 = make_float2(bv, bv), one = make_float2(1.0f, 1.0f);
#pragma unroll
        for (int c = 0; c < COLS / 2; ++c) acc[c] = ffma2(acc[c], one, b2);  // ggml_add: x*1 + b, one rounding
        float* yp = p.y + m0 * p.ldy + n;
        if (p.resid) {
          const float gv = p.gate ? p.gate[n] : 1.0f;
          const float* rp = p.resid + m0 * p.ldr + n;
#pragma unroll
          for (int c = 0; c < COLS; ++c) {
            if (m0 + c < p.M) {
              const float h = (c & 1) ? acc[c / 2].y : acc[c / 2].x;
              yp[c * p.ldy] = __fadd_rn(rp[c * p.ldr], p.gate ? __fmul_rn(h, gv) : h);
            }
          }
        } else {
#pragma unroll
          for (int c = 0; c < COLS / 2; ++c) {
            if (m0 + 2 * c < p.M) yp[(2 * c) * p.ldy] = acc[c].x;
            if (m0 + 2 * c + 1 < p.M) yp[(2 * c + 1) * p.ldy] = acc[c].y;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemColsQ);
  }
}

template <int BN>
cudaError_t launch_bn(const Q4kArgs& g, int num_sms, cudaStream_t s) {
  using C = QCfg<BN>;
  const int64_t KSB = g.K / kQKK;
  CUtensorMap tm_w, tm_a, tm_sd, tm_sm, tm_sa;
  if (!make_tensor_map_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.w_codes, g.K, 3 * g.N, g.K, kStageK, kBM,
                          CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tensor_map_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.a_codes, g.K, g.M, g.K, kStageK, BN,
                          CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tensor_map_2d(&tm_sd, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.w_d, g.ldw, KSB, g.ldw * 4, kBM, 1,
                          CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tensor_map_2d(&tm_sm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.w_dmin, g.ldw, KSB, g.ldw * 4, kBM, 1,
                          CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tensor_map_2d(&tm_sa, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.a_d, g.lda, KSB, g.lda * 4, BN, 1,
                          CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  Q4kParams p;
  p.M = static_cast<int>(g.M);
  p.N = static_cast<int>(g.N);
  p.KSB = static_cast<int>(KSB);
  p.n_tiles = static_cast<int>((g.N + kBM - 1) / kBM);
  const int m_tiles = static_cast<int>((g.M + BN - 1) / BN);
  if (static_cast<int64_t>(p.n_tiles) * m_tiles > INT32_MAX) return cudaErrorInvalidValue;
  p.num_tiles = p.n_tiles * m_tiles;
  p.y = g.y;
  p.ldy = g.ldy;
  p.bias = g.bias;
  p.gate = g.gate;
  p.resid = g.resid;
  p.ldr = g.ldr;
  auto kern = gemm_q4k_kernel<BN>;
  static std::atomic<uint64_t> ready{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  const uint64_t bit = dev < 64 ? (uint64_t{1} << dev) : 0;
  if (!bit || !(ready.load(std::memory_order_acquire) & bit)) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != kLaunchRegsQ) return cudaErrorInvalidConfiguration;  // the register split needs it
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    ready.fetch_or(bit, std::memory_order_acq_rel);
  }
  const int grid = p.num_tiles < num_sms ? p.num_tiles : num_sms;
  kern<<<grid, kThreadsQ, C::SMEM, s>>>(tm_w, tm_a, tm_sd, tm_sm, tm_sa, p);
  return cudaGetLastError();
}

}  // namespace q4k

cudaError_t launch_gemm_q4k(const Q4kArgs& g, int num_sms, cudaStream_t s) {
  if (g.M == 0 || g.N == 0) return cudaSuccess;
  if (g.K % kQKK != 0 || g.M > INT32_MAX || g.N > INT32_MAX / 3) return cudaErrorInvalidValue;
  // Wide tiles halve the weight-plane traffic; narrow ones keep small token
  // counts from leaving SMs idle.
  const int64_t n_tiles = (g.N + q4k::kBM - 1) / q4k::kBM;
  if (n_tiles * ((g.M + 127) / 128) >= num_sms) return q4k::launch_bn<128>(g, num_sms, s);
  return q4k::launch_bn<64>(g, num_sms, s);
}

}  // namespace b2q
