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
// The planes are built on chip: the packed weight is the Q4_K rows
// themselves (0.5625 bytes per value); per super-block the TMA brings the 128
// rows' 144-byte blocks, two converter warps unpack them into the three
// planes in shared memory (in the 128-byte-swizzled K-major layout the MMA
// descriptors expect), and the planes never cross L2.
//
// Structure (persistent, one CTA per SM, 384 threads): warp 0 issues TMA,
// warp 1 issues the MMAs, warps 2-3 convert, warps 4-11 run the epilogue.
// Tiles are 128 weight rows x BN tokens.  Rings: a two-slot super-block ring
// (the raw Q4_K tile and the tokens' Q8_K scales; released by the converters
// and the epilogue), two plane stages of 4 sub-blocks (converters fill, the
// MMA's commit releases), three activation-code stages (TMA fills, the MMA's
// commit releases).  TMEM holds GROUPS super-block groups of three BN-column
// accumulators; each plane's accumulator goes back to the MMA as soon as the
// epilogue has loaded it.  No TMA multicast.
//
// Included by b2q_gemm_tc.cu: the kernel records bounded-wait failures in the
// same device status word (one translation unit, no relocatable device code).
#pragma once

namespace b2q {

namespace q4k {

constexpr int kBM = 128;
constexpr int kSubPerStage = 4;               // 32-value sub-blocks per stage
constexpr int kStageK = kSubPerStage * kQK;   // 128 bytes of K per row
constexpr int kPStages = 2;                   // plane stages (one super-block)
constexpr int kBStages = 3;                   // activation-code stages
constexpr int kPlanes = 3;
constexpr int kSlots = 2;                     // super-block ring: raw Q4_K tile + da
constexpr uint32_t kTmemColsQ = 512;
constexpr int kConvWarp0 = 4, kConvWarps = 4;  // warpgroup 1: one weight row per thread
constexpr int kEpiWarps = 8, kEpiWarp0 = 8;    // warpgroups 2-3
constexpr int kThreadsQ = (kEpiWarp0 + kEpiWarps) * 32;
// Register split per warpgroup (setmaxnreg): control, converters, epilogue.
constexpr int kLaunchRegsQ = 128, kRegsControlQ = 40, kRegsConvQ = 56, kRegsEpilogueQ = 208;
static_assert(128 * kRegsControlQ + 128 * kRegsConvQ + 256 * kRegsEpilogueQ <= kThreadsQ * kLaunchRegsQ,
              "register split");
constexpr int kPlaneBytes = kBM * kStageK;             // 16 KB
constexpr int kPStageBytes = kPlanes * kPlaneBytes;    // 48 KB
constexpr int kRawBytes = kBM * kQ4KBytes;             // 18 KB: 128 rows x one 144-byte block

// BN tokens per tile.  TMEM holds GROUPS super-block groups of three BN-column
// accumulators: two groups at BN = 64, one at BN = 128 (twice the tokens per
// weight tile).
template <int BN>
struct QCfg {
  static_assert(BN == 64 || BN == 128, "tile width");
  static constexpr int COLS = BN / 2;                               // token columns per epilogue thread
  static constexpr int GROUPS = 2 * kPlanes * BN <= int(kTmemColsQ) ? 2 : 1;
  static constexpr int GROUP_COLS = GROUPS == 2 ? 256 : 512;
  static constexpr int B_BYTES = BN * kStageK;
  static constexpr int SLOT_BYTES = kRawBytes + BN * 4;            // raw tile, then da[BN]
  static constexpr int OFF_P = 0;                                   // plane stages (1024-aligned)
  static constexpr int OFF_B = OFF_P + kPStages * kPStageBytes;     // activation-code stages
  static constexpr int OFF_SLOTS = OFF_B + kBStages * B_BYTES;
  static constexpr int OFF_BARS = OFF_SLOTS + kSlots * SLOT_BYTES;
  // slot_full/empty[2], b_full/empty[3], p_full/empty[2], acc_full[G], acc_empty[G][3], done
  static constexpr int NBARS = 2 * kSlots + 2 * kBStages + 2 * kPStages + GROUPS + GROUPS * kPlanes + 1;
  static constexpr int SMEM = OFF_BARS + NBARS * 8 + 16 + 1024;
  static_assert(B_BYTES % 1024 == 0 && kPStageBytes % 1024 == 0, "swizzle alignment");
  static_assert(SLOT_BYTES % 128 == 0 && kRawBytes % 128 == 0, "TMA destinations");
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

// Converts one weight row's 4 sub-blocks (stage h of its super-block) from the
// raw 144-byte Q4_K block `rb` into the three plane tiles at `pst`: row r's
// 128 bytes of each plane in the 128-byte-swizzled K-major layout (8-row
// atoms of 1024 bytes; 16-byte chunk c of row r at chunk c ^ (r % 8)).
// Quant bytes hold two sub-blocks: the low nibbles are sub-block 2g, the high
// nibbles 2g+1; a 32-bit multiply by a 3-bit scale half scales 4 quants at
// once (each product <= 105 stays inside its byte).
__device__ __forceinline__ void convert_row(const uint8_t* rb, int r, int h, uint8_t* pst) {
  const uint8_t* sm = rb + 4;
  uint8_t* rowp = pst + (r >> 3) * 1024 + (r & 7) * 128;
  const int sw = r & 7;
#pragma unroll
  for (int jl = 0; jl < 4; ++jl) {  // sub-block within the stage
    const int j = 4 * h + jl;       // within the super-block
    int sc, mn;
    if (j < 4) {
      sc = sm[j] & 63;
      mn = sm[j + 4] & 63;
    } else {
      sc = (sm[j + 4] & 15) | ((sm[j - 4] >> 6) << 4);
      mn = (sm[j + 4] >> 4) | ((sm[j] >> 6) << 4);
    }
    const uint32_t lo = static_cast<uint32_t>(sc & 7), hi = static_cast<uint32_t>(sc >> 3);
    const uint32_t m4 = static_cast<uint32_t>(mn) * 0x01010101u;
    const int shift = (j & 1) * 4;  // sub-block 2g: low nibbles, 2g+1: high nibbles
    const uint4* q = reinterpret_cast<const uint4*>(rb + 16 + 32 * (j >> 1));
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {  // the sub-block's two 16-value chunks
      const uint4 w = q[cc];
      const uint32_t v0 = (w.x >> shift) & 0x0F0F0F0Fu, v1 = (w.y >> shift) & 0x0F0F0F0Fu;
      const uint32_t v2 = (w.z >> shift) & 0x0F0F0F0Fu, v3 = (w.w >> shift) & 0x0F0F0F0Fu;
      const int off = ((2 * jl + cc) ^ sw) << 4;
      *reinterpret_cast<uint4*>(rowp + off) = make_uint4(v0 * lo, v1 * lo, v2 * lo, v3 * lo);
      *reinterpret_cast<uint4*>(rowp + kPlaneBytes + off) = make_uint4(v0 * hi, v1 * hi, v2 * hi, v3 * hi);
      *reinterpret_cast<uint4*>(rowp + 2 * kPlaneBytes + off) = make_uint4(m4, m4, m4, m4);
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreadsQ, 1)
    gemm_q4k_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                    const __grid_constant__ CUtensorMap tm_sa, const Q4kParams p) {
  using C = QCfg<BN>;
  constexpr int COLS = C::COLS, GROUPS = C::GROUPS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* slot_full = reinterpret_cast<uint64_t*>(smem + C::OFF_BARS);
  uint64_t* slot_empty = slot_full + kSlots;
  uint64_t* b_full = slot_empty + kSlots;
  uint64_t* b_empty = b_full + kBStages;
  uint64_t* p_full = b_empty + kBStages;
  uint64_t* p_empty = p_full + kPStages;
  uint64_t* acc_full = p_empty + kPStages;
  uint64_t* acc_empty = acc_full + GROUPS;  // [group][plane]
  uint64_t* mma_done = acc_empty + GROUPS * kPlanes;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&slot_full[s], 1);
      mbar_init(&slot_empty[s], kConvWarps + kEpiWarps);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&p_full[s], kConvWarps);  // one arrive per converter warp
      mbar_init(&p_empty[s], 1);
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

  if (warp < kConvWarp0) {
    // ------------------------------------------------- warpgroup 0 (control)
    setmaxnreg_dec<kRegsControlQ>();
    if (warp == 0) {
      // ---------------------------------------------------------- producer
      if (elect_one()) {
        uint32_t bs = 0, bph = 0, b_mask = 0, b_par = 0, sbc = 0, s_mask = 0, s_par = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
          const int n0 = (tile % p.n_tiles) * kBM, m0 = (tile / p.n_tiles) * BN;
          for (int sb = 0; ok && sb < p.KSB; ++sb, ++sbc) {
            const uint32_t rs = sbc & 1u, rpar = (sbc >> 1) & 1u;
            if (!mbar_wait(&slot_empty[rs], rpar ^ 1u, &g_device_status, kDevWaitProducer, abort_flag)) {
              ok = false;
              break;
            }
            uint8_t* sl = smem + C::OFF_SLOTS + rs * C::SLOT_BYTES;
            mbar_arrive_expect_tx(&slot_full[rs], C::SLOT_BYTES);
            tma_load_2d(sl, &tm_w, &slot_full[rs], sb * kQ4KBytes, n0);
            tma_load_2d(sl + kRawBytes, &tm_sa, &slot_full[rs], m0, sb);
            s_mask |= 1u << rs;
            s_par = (s_par & ~(1u << rs)) | (rpar << rs);
            for (int h = 0; h < 2; ++h) {
              if (!mbar_wait(&b_empty[bs], bph ^ 1u, &g_device_status, kDevWaitProducer, abort_flag)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&b_full[bs], C::B_BYTES);
              tma_load_2d(smem + C::OFF_B + bs * C::B_BYTES, &tm_a, &b_full[bs], (2 * sb + h) * kStageK, m0);
              b_mask |= 1u << bs;
              b_par = (b_par & ~(1u << bs)) | (bph << bs);
              if (++bs == kBStages) {
                bs = 0;
                bph ^= 1u;
              }
            }
          }
        }
        // Every issued copy lands before the CTA may exit.
        for (int s = 0; s < kBStages; ++s)
          if ((b_mask >> s) & 1u) mbar_wait(&b_full[s], (b_par >> s) & 1u, &g_device_status, kDevWaitDrain, nullptr);
        for (int s = 0; s < kSlots; ++s)
          if ((s_mask >> s) & 1u)
            mbar_wait(&slot_full[s], (s_par >> s) & 1u, &g_device_status, kDevWaitDrain, nullptr);
      }
    } else if (warp == 1) {
      // -------------------------------------------------------- MMA issuer
      if (elect_one()) {
        constexpr uint32_t idesc = idesc_i8(kBM, BN);
        uint32_t bs = 0, bph = 0, ps = 0, pph = 0, sbc = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
          for (int sb = 0; ok && sb < p.KSB; ++sb, ++sbc) {
            const uint32_t g = GROUPS == 2 ? (sbc & 1u) : 0u;
            const uint32_t gpar = GROUPS == 2 ? ((sbc >> 1) & 1u) : (sbc & 1u);
            const uint32_t dbase = tmem_base + g * C::GROUP_COLS;
            for (int h = 0; ok && h < 2; ++h) {
              if (!mbar_wait(&p_full[ps], pph, &g_device_status, kDevWaitMma, abort_flag) ||
                  !mbar_wait(&b_full[bs], bph, &g_device_status, kDevWaitMma, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t a0 = smem_u32(smem + C::OFF_P + ps * kPStageBytes);
              const uint32_t b0 = smem_u32(smem + C::OFF_B + bs * C::B_BYTES);
              // Plane-major: the first stage of a super-block waits for each
              // plane's accumulator separately.
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
              mma_commit(&p_empty[ps]);  // both stages are free once these MMAs have read them
              mma_commit(&b_empty[bs]);
              if (++ps == kPStages) {
                ps = 0;
                pph ^= 1u;
              }
              if (++bs == kBStages) {
                bs = 0;
                bph ^= 1u;
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
  } else if (warp < kEpiWarp0) {
    // ------------------------------------------- warpgroup 1: converters
    setmaxnreg_dec<kRegsConvQ>();
    {
      const int ct = (warp - kConvWarp0) * 32 + lane;  // this thread's weight row
      uint32_t ps = 0, pph = 0, sbc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        for (int sb = 0; ok && sb < p.KSB; ++sb, ++sbc) {
          const uint32_t rs = sbc & 1u, rpar = (sbc >> 1) & 1u;
          if (!mbar_wait(&slot_full[rs], rpar, &g_device_status, kDevWaitProducer, abort_flag)) {
            ok = false;
            break;
          }
          const uint8_t* raw = smem + C::OFF_SLOTS + rs * C::SLOT_BYTES;
          for (int h = 0; h < 2; ++h) {
            if (!mbar_wait(&p_empty[ps], pph ^ 1u, &g_device_status, kDevWaitProducer, abort_flag)) {
              ok = false;
              break;
            }
            uint8_t* pst = smem + C::OFF_P + ps * kPStageBytes;
            convert_row(raw + ct * kQ4KBytes, ct, h, pst);
            fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[ps]);
            if (++ps == kPStages) {
              ps = 0;
              pph ^= 1u;
            }
          }
          __syncwarp();
          if (ok && lane == 0) mbar_arrive(&slot_empty[rs]);
        }
      }
    }
  } else {
    // ------------------------------------------------ warpgroups 2-3: epilogue
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
        const uint32_t rs = sbc & 1u, rpar = (sbc >> 1) & 1u;
        const uint32_t g = GROUPS == 2 ? (sbc & 1u) : 0u;
        const uint32_t gpar = GROUPS == 2 ? ((sbc >> 1) & 1u) : (sbc & 1u);
        if (!mbar_wait(&slot_full[rs], rpar, &g_device_status, kDevWaitEpilogue, abort_flag) ||
            !mbar_wait(&acc_full[g], gpar, &g_device_status, kDevWaitEpilogue, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tb = tlane + g * C::GROUP_COLS;
        const uint8_t* sl = smem + C::OFF_SLOTS + rs * C::SLOT_BYTES;
        const uint32_t dd = *reinterpret_cast<const uint32_t*>(sl + row * kQ4KBytes);  // fp16 d, fp16 dmin
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(dd & 0xffffu)));
        const float dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(dd >> 16)));
        const float* da = reinterpret_cast<const float*>(sl + kRawBytes) + chalf * COLS;
        if constexpr (COLS <= 32) {
          // Planes 0 and 1 in flight together, plane 2 streams in while plane 1 is folded.
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
        } else {
          // One plane at a time (the registers hold one 64-column plane beside
          // the accumulators); each plane goes back to the MMA once loaded.
          const float sc[kPlanes] = {d, 8.0f * d, -dmin};
#pragma unroll
          for (int pl = 0; pl < kPlanes; ++pl) {
            uint32_t ra[COLS];
            load_plane<COLS>(tb + pl * BN, ra);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(&acc_empty[g * kPlanes + pl]);
            fold_plane<COLS>(ra, sc[pl], da, acc);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&slot_empty[rs]);  // this super-block's scales are read
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
              const float hv = (c & 1) ? acc[c / 2].y : acc[c / 2].x;
              yp[c * p.ldy] = __fadd_rn(rp[c * p.ldr], p.gate ? __fmul_rn(hv, gv) : hv);
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
  CUtensorMap tm_w, tm_a, tm_sa;
  if (!make_tensor_map_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.w_raw, KSB * kQ4KBytes, g.N, g.ldw_bytes,
                          kQ4KBytes, kBM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_tensor_map_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.a_codes, g.K, g.M, g.K, kStageK, BN,
                          CU_TENSOR_MAP_SWIZZLE_128B) ||
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
  kern<<<grid, kThreadsQ, C::SMEM, s>>>(tm_w, tm_a, tm_sa, p);
  return cudaGetLastError();
}

}  // namespace q4k

cudaError_t launch_gemm_q4k(const Q4kArgs& g, int num_sms, cudaStream_t s) {
  if (g.M == 0 || g.N == 0) return cudaSuccess;
  if (g.K % kQKK != 0 || g.M > INT32_MAX || g.N > INT32_MAX) return cudaErrorInvalidValue;
  // Wide tiles halve the weight reads per token; narrow ones keep small token
  // counts from leaving SMs idle.
  const int64_t n_tiles = (g.N + q4k::kBM - 1) / q4k::kBM;
  if (n_tiles * ((g.M + 127) / 128) >= num_sms) return q4k::launch_bn<128>(g, num_sms, s);
  return q4k::launch_bn<64>(g, num_sms, s);
}

}  // namespace b2q
