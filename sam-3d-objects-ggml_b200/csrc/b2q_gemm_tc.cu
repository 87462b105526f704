// b2q_gemm_tc.cu -- tcgen05 int8 block GEMM with the per-block scale epilogue.
//
//   y[m][n] = sum_b  dw[n,b] * da[m,b] * S_b(n,m),   S_b = sum_{i<32} qw[n,32b+i] * qa[m,32b+i]
//
// Per 32-value block b, one tcgen05.mma (kind::i8, M = 128 weight rows, N = BN
// tokens, K = 32) computes that block's int32 dots S_b into a fresh TMEM
// accumulator slot.  Scales change every 32 of K, so int32 cannot be carried
// across blocks; epilogue warps drain every slot and apply the scales in fp32,
// while the tensor core fills the next slots.  The epilogue's per-(n, m, b)
// arithmetic, not the tensor core, bounds this kernel.
//
// Exact int32 -> fp32 fold without any conversion instruction:
//   a second, constant MMA (kind::i8, unsigned x unsigned, both operands one 4 KB
//   smem tile in which every 16-byte chunk is P with sum_j P_j^2 = 2^19) adds
//   exactly 2^20 to every accumulator element, so D = S + 2^20 lies in
//   [2^19, 3*2^19] and its bits, read as fp32, are the subnormal D * 2^-149.
//   With dw' = dw * 2^100 (weight scales are stored pre-scaled) and
//   c = -dw * 2^-29 (= -2^20 * dw' * 2^-149, exact):
//       t   = fma(bits(D), dw', c)  = round(S * dw) * 2^-49   (one rounding)
//       acc = fma(t, da', acc)      with da' = da * 2^49 (stored pre-scaled)
//   i.e. two fp32 FMAs per (row, token, block) -- issued as packed f32x2 pairs --
//   the same two roundings as round(S*dw)*da, with every intermediate normal.
//
// TMEM access: each epilogue warp reads its 32 rows x 64 columns of a slot with
// two tcgen05.ld.16x256b.x8 (thread i: rows i/4, i/4+8 (+16, +24), columns
// 8g + 2(i%4) + {0,1}), so a thread needs 16 activation scales (8 LDS.64 with
// 4 distinct addresses per warp) and 4 weight scales per block.  The two halves
// are software-pipelined: each load is in flight while the other half is
// scaled, and a slot is released as soon as both halves are in registers.
//
// Roles (384 threads = 3 warpgroups, 1 CTA per SM, persistent over tiles):
//   warp 0      TMA producer: weight codes [128 x 128B], activation codes
//               [BN x 128B] (128B swizzle), weight scales [4 x 128] and
//               activation scales [4 x BN] fp32 per stage (4 blocks of K)
//   warp 1      TMEM allocator + single-thread MMA issuer
//   warps 2,3   idle (complete warpgroup 0, which runs on 40 registers)
//   warps 4..11 epilogue (232 registers): warp w owns TMEM lanes 32*(w%4)..
//               (weight rows) and half of the BN accumulator columns (tokens)
// Every wait is bounded (b2q_ptx.cuh); on give-up the CTA drains its in-flight
// copies and MMAs, frees TMEM and exits, leaving a code in g_device_status.
#include "b2q_internal.h"
#include "b2q_ptx.cuh"

namespace b2q {

// Device status word of this library's kernels (0 = ok, else the first
// kDevWait* code recorded by a bounded wait that gave up).
__device__ unsigned int g_device_status = 0;

namespace {

constexpr int kBM = 128;             // weight rows per tile (MMA M, TMEM lanes)
constexpr int kKBS = 4;              // 32-value blocks per pipeline stage
constexpr int kStageK = kKBS * kQK;  // 128 bytes of K per operand row per stage
constexpr int kEpiWarps = 8;
constexpr int kEpiWarp0 = 4;  // epilogue = warpgroups 1 and 2
constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * 32;
// Register split (setmaxnreg works per warpgroup).  The kernel is compiled for
// 384 threads at kLaunchRegs registers each (the per-SM-subpartition cap for
// 3 warps per subpartition); warpgroup 0 gives registers back, the two
// epilogue warpgroups take them: 128*40 + 256*232 = 384*168.  The host refuses
// to launch unless the compiled count is kLaunchRegs, so the increase can
// never wait on registers that do not exist.
constexpr int kLaunchRegs = 168;
constexpr int kRegsControl = 40;
constexpr int kRegsEpilogue = 232;
static_assert(128 * kRegsControl + 256 * kRegsEpilogue <= kThreads * kLaunchRegs, "register split");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kOffset = 1u << 20;        // added to every S by the constant MMA
constexpr int kOffsetTileBytes = 4096;        // 128 rows x 32 bytes, every 16-byte chunk = P
constexpr float kNegTwoPowM129 = -0x1p-129f;  // subnormal, exact

template <int BN, int STAGES>
struct Cfg {
  static constexpr int A_BYTES = kBM * kStageK;
  static constexpr int B_BYTES = BN * kStageK;
  static constexpr int SW_BYTES = kKBS * kBM * 4;
  static constexpr int SA_BYTES = kKBS * BN * 4;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SW_BYTES + SA_BYTES;
  static constexpr int ACC_SLOTS = static_cast<int>(kTmemCols) / BN;
  static constexpr int COLS = BN / 2;  // accumulator columns per epilogue warp
  static constexpr int OFF_TILE = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = OFF_TILE + kOffsetTileBytes;
  static constexpr int NBARS = 2 * STAGES + 2 * ACC_SLOTS + 1;
  static constexpr int SMEM = BAR_OFF + NBARS * 8 + 16 + 1024;  // + alignment slack
  static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte swizzle alignment");
  static_assert(STAGES <= 16, "stage bitmasks");
  static_assert(BN == 128, "the epilogue drains 64 columns per warp");
};

struct TcParams {
  int M, N, KB, n_tiles, num_tiles;
  float* y;
  int64_t ldy;
  const float* bias;
  int32_t* dots;
};

// Shared-memory descriptor for the constant offset tile: K-major, no swizzle,
// core matrices (8 rows x 16 bytes) 128 bytes apart along K and 256 bytes apart
// along M/N.  Every 16-byte chunk of the tile holds the same pattern, so every
// row and k position reads P whatever the core-matrix order.
__device__ __forceinline__ uint64_t smem_desc_k_noswz(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3fffu);
  d |= static_cast<uint64_t>(128u >> 4) << 16;  // leading (K) byte offset
  d |= static_cast<uint64_t>(256u >> 4) << 32;  // stride (M/N) byte offset
  d |= static_cast<uint64_t>(1u) << 46;         // descriptor version
  return d;                                     // layout type 0: no swizzle
}

// kind::i8, unsigned A and B, int32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_u8(int m, int n) {
  return (2u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// 16 lanes x 256 bits x 8: thread i receives, for g = 0..7,
//   r[4g+0], r[4g+1] = lane (base + i/4),     columns 8g + 2(i%4) + {0, 1}
//   r[4g+2], r[4g+3] = lane (base + 8 + i/4), same columns
__device__ __forceinline__ void tmem_ld_16x256b_x8(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Scale and accumulate one 16-lane half: rows (ra, rb) = (i/4, i/4+8) of the
// half; acc[8*k + g] holds row k (0..3 over both halves) and columns
// 8g + 2(i%4) + {0, 1}.
__device__ __forceinline__ void fold_half(float2 (&acc)[32], int k0, const uint32_t (&r)[32],
                                          const float2 (&da)[8], float2 wa, float2 ca, float2 wb,
                                          float2 cb) {
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    const float2 ta = ffma2(make_float2(__uint_as_float(r[4 * g]), __uint_as_float(r[4 * g + 1])), wa, ca);
    const float2 tb = ffma2(make_float2(__uint_as_float(r[4 * g + 2]), __uint_as_float(r[4 * g + 3])), wb, cb);
    acc[8 * k0 + g] = ffma2(ta, da[g], acc[8 * k0 + g]);
    acc[8 * (k0 + 1) + g] = ffma2(tb, da[g], acc[8 * (k0 + 1) + g]);
  }
}

// Debug path: raw int32 block dots S = D - 2^20 of one 16-lane half.
__device__ __forceinline__ void dump_half(const TcParams& p, const uint32_t (&r)[32], int64_t n_a,
                                          int64_t m_base, int KB, int blk) {
  for (int g = 0; g < 8; ++g)
    for (int k = 0; k < 4; ++k) {
      const int64_t n = n_a + ((k & 2) ? 8 : 0);
      const int64_t m = m_base + 8 * g + (k & 1);
      if (n < p.N && m < p.M) p.dots[(m * p.N + n) * KB + blk] = static_cast<int32_t>(r[4 * g + k] - kOffset);
    }
}

template <int BN, int STAGES, bool DUMP>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_wc, const __grid_constant__ CUtensorMap tm_ac,
                   const __grid_constant__ CUtensorMap tm_ws, const __grid_constant__ CUtensorMap tm_as,
                   const TcParams p) {
  using C = Cfg<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + C::ACC_SLOTS;
  uint64_t* mma_done = acc_empty + C::ACC_SLOTS;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kEpiWarps);
    }
    for (int a = 0; a < C::ACC_SLOTS; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  {
    // Offset tile: every 16-byte chunk = P, sum_j P_j^2 = 8*255^2 + 63^2 + 10^2
    // + 4^2 + 3*1^2 = 2^19, so one K = 32 u8 x u8 MMA adds exactly 2^20.
    const uint4 pattern = make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0x01040A3Fu, 0x00000101u);
    uint4* tile = reinterpret_cast<uint4*>(smem + C::OFF_TILE);
    for (int i = threadIdx.x; i < kOffsetTileBytes / 16; i += kThreads) tile[i] = pattern;
    fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_wc);
    tma_prefetch_desc(&tm_ac);
    tma_prefetch_desc(&tm_ws);
    tma_prefetch_desc(&tm_as);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  const int KB = p.KB;
  const int n_ks = (KB + kKBS - 1) / kKBS;

  if (warp < kEpiWarp0) {
    // ------------------------------------------------- warpgroup 0 (control)
    setmaxnreg_dec<kRegsControl>();
    if (warp == 0) {
      // ---------------------------------------------------------- producer
      if (elect_one()) {
        uint32_t stage = 0, phase = 0, issued_mask = 0, issued_par = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
          const int n0 = (tile % p.n_tiles) * kBM;
          const int m0 = (tile / p.n_tiles) * BN;
          for (int ks = 0; ks < n_ks; ++ks) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, &g_device_status, kDevWaitProducer, abort_flag)) {
              ok = false;
              break;
            }
            uint8_t* sb = smem + stage * C::STAGE_BYTES;
            mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
            tma_load_2d(sb, &tm_wc, &full[stage], ks * kStageK, n0);
            tma_load_2d(sb + C::A_BYTES, &tm_ac, &full[stage], ks * kStageK, m0);
            tma_load_2d(sb + C::A_BYTES + C::B_BYTES, &tm_ws, &full[stage], n0, ks * kKBS);
            tma_load_2d(sb + C::A_BYTES + C::B_BYTES + C::SW_BYTES, &tm_as, &full[stage], m0, ks * kKBS);
            issued_mask |= 1u << stage;
            issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
        // Every issued copy lands before the CTA may exit.
        for (int s = 0; s < STAGES; ++s)
          if ((issued_mask >> s) & 1u)
            mbar_wait(&full[s], (issued_par >> s) & 1u, &g_device_status, kDevWaitDrain, nullptr);
      }
    } else if (warp == 1) {
      // -------------------------------------------------------- MMA issuer
      if (elect_one()) {
        constexpr uint32_t idesc = idesc_i8(kBM, BN);
        constexpr uint32_t idesc_off = idesc_u8(kBM, BN);
        const uint64_t off_desc = smem_desc_k_noswz(smem_u32(smem + C::OFF_TILE));
        uint32_t stage = 0, phase = 0, slot = 0, acc_phase = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
          for (int ks = 0; ok && ks < n_ks; ++ks) {
            if (!mbar_wait(&full[stage], phase, &g_device_status, kDevWaitMma, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(smem + stage * C::STAGE_BYTES);
            const uint32_t b_base = a_base + C::A_BYTES;
            const int nblk = min(kKBS, KB - ks * kKBS);
            for (int j = 0; j < nblk; ++j) {
              if (!mbar_wait(&acc_empty[slot], acc_phase ^ 1u, &g_device_status, kDevWaitMma, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t d = tmem_base + slot * BN;
              mma_i8(d, smem_desc_k_sw128(a_base + j * kQK), smem_desc_k_sw128(b_base + j * kQK), idesc, 0u);
              mma_i8(d, off_desc, off_desc, idesc_off, 1u);
              mma_commit(&acc_full[slot]);
              if (++slot == C::ACC_SLOTS) {
                slot = 0;
                acc_phase ^= 1u;
              }
            }
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
        // All issued MMAs complete before TMEM is released.
        mma_commit(mma_done);
        mbar_wait(mma_done, 0, &g_device_status, kDevWaitDrain, nullptr);
      }
    }
  } else {
    // ------------------------------------------------ warpgroups 1-2: epilogue
    setmaxnreg_inc<kRegsEpilogue>();
    const int quarter = warp & 3;               // TMEM lane quarter this warp may access
    const int chalf = (warp - kEpiWarp0) >> 2;  // which half of the BN columns
    const int row0 = quarter * 32 + (lane >> 2);  // this thread's rows: row0 + {0, 8, 16, 24}
    const int col0 = chalf * C::COLS + 2 * (lane & 3);  // columns col0 + 8g + {0, 1}
    const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + chalf * C::COLS;
    // Half-slot software pipeline: the first 16-lane half of a block's slot is
    // loaded while the previous block is still being scaled; the slot is handed
    // back to the MMA as soon as both halves sit in registers.
    const int my_tiles = (p.num_tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                         static_cast<int>(gridDim.x);
    const int total = my_tiles * KB;
    uint32_t stage = 0, phase = 0, slot = 0, acc_phase = 0;
    uint32_t r0[32], r1[32];
    bool ok = total > 0 && mbar_wait(&acc_full[0], 0, &g_device_status, kDevWaitEpilogue, abort_flag);
    if (ok) {
      tc_fence_after();
      tmem_ld_16x256b_x8(tbase, r0);
      tmem_wait_ld();
    }
    int g = 0;
    for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
      const int n0 = (tile % p.n_tiles) * kBM;
      const int m0 = (tile / p.n_tiles) * BN;
      float2 acc[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) acc[c] = make_float2(0.0f, 0.0f);
      for (int ks = 0; ok && ks < n_ks; ++ks) {
        if (!mbar_wait(&full[stage], phase, &g_device_status, kDevWaitEpilogue, abort_flag)) {
          ok = false;
          break;
        }
        const uint8_t* sb = smem + stage * C::STAGE_BYTES;
        const float* sw = reinterpret_cast<const float*>(sb + C::A_BYTES + C::B_BYTES);
        const float* sa = sw + kKBS * kBM;
        const int nblk = min(kKBS, KB - ks * kKBS);
        for (int j = 0; j < nblk; ++j, ++g) {
          const uint32_t taddr = tbase + slot * BN;
          tmem_ld_16x256b_x8(taddr + (16u << 16), r1);  // second half of this block
          const float* swj = sw + j * kBM + row0;
          const float w0 = swj[0], w1 = swj[8], w2 = swj[16], w3 = swj[24];
          const float2* saj = reinterpret_cast<const float2*>(sa + j * BN + col0);
          float2 da[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) da[q] = saj[4 * q];
          if (DUMP) dump_half(p, r0, n0 + row0, m0 + col0, KB, ks * kKBS + j);
          fold_half(acc, 0, r0, da, make_float2(w0, w0), make_float2(w0 * kNegTwoPowM129, w0 * kNegTwoPowM129),
                    make_float2(w1, w1), make_float2(w1 * kNegTwoPowM129, w1 * kNegTwoPowM129));
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[slot]);  // both halves are in registers
          if (++slot == C::ACC_SLOTS) {
            slot = 0;
            acc_phase ^= 1u;
          }
          if (g + 1 < total) {  // prefetch the next block's first half
            if (!mbar_wait(&acc_full[slot], acc_phase, &g_device_status, kDevWaitEpilogue, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            tmem_ld_16x256b_x8(tbase + slot * BN, r0);
          }
          if (DUMP) dump_half(p, r1, n0 + row0 + 16, m0 + col0, KB, ks * kKBS + j);
          fold_half(acc, 2, r1, da, make_float2(w2, w2), make_float2(w2 * kNegTwoPowM129, w2 * kNegTwoPowM129),
                    make_float2(w3, w3), make_float2(w3 * kNegTwoPowM129, w3 * kNegTwoPowM129));
          tmem_wait_ld();
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (p.y) {
        // acc[8k + g] = rows row0 + 8k, columns col0 + 8g + {0, 1}
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int64_t n = static_cast<int64_t>(n0) + row0 + 8 * k;
          if (n >= p.N) continue;
          const float bv = p.bias ? p.bias[n] : 0.0f;
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            const int64_t m = static_cast<int64_t>(m0) + col0 + 8 * g;
            const float2 v = acc[8 * k + g];
            if (m < p.M) p.y[m * p.ldy + n] = p.bias ? v.x + bv : v.x;
            if (m + 1 < p.M) p.y[(m + 1) * p.ldy + n] = p.bias ? v.y + bv : v.y;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------------ host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

bool make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                 uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int STAGES, bool DUMP>
cudaError_t launch_cfg(const GemmArgs& g, int num_sms, cudaStream_t s) {
  using C = Cfg<BN, STAGES>;
  const int64_t KB = g.K / kQK;
  CUtensorMap tm_wc, tm_ac, tm_ws, tm_as;
  if (!make_map_2d(&tm_wc, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.w.codes, g.K, g.N, g.K, kStageK, kBM,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tm_ac, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.a.codes, g.K, g.M, g.K, kStageK, BN,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tm_ws, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.w.scales, g.N, KB, g.w.ld * 4, kBM,
                   kKBS, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map_2d(&tm_as, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.a.scales, g.M, KB, g.a.ld * 4, BN,
                   kKBS, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  TcParams p;
  p.M = static_cast<int>(g.M);
  p.N = static_cast<int>(g.N);
  p.KB = static_cast<int>(KB);
  p.n_tiles = static_cast<int>((g.N + kBM - 1) / kBM);
  const int m_tiles = static_cast<int>((g.M + BN - 1) / BN);
  p.num_tiles = p.n_tiles * m_tiles;
  p.y = g.y;
  p.ldy = g.ldy;
  p.bias = g.bias;
  p.dots = g.dots;
  auto kern = gemm_tc_kernel<BN, STAGES, DUMP>;
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, kern);
  if (e != cudaSuccess) return e;
  if (fa.numRegs != kLaunchRegs) return cudaErrorInvalidConfiguration;  // see the register split
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int grid = p.num_tiles < num_sms ? p.num_tiles : num_sms;
  kern<<<grid, kThreads, C::SMEM, s>>>(tm_wc, tm_ac, tm_ws, tm_as, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t read_device_status(unsigned int* value, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_device_status, sizeof(unsigned int));
  if (e != cudaSuccess || !clear) return e;
  const unsigned int zero = 0;
  return cudaMemcpyToSymbol(g_device_status, &zero, sizeof(unsigned int));
}

cudaError_t launch_gemm_tc(const GemmArgs& g, int num_sms, cudaStream_t s) {
  if (g.M == 0 || g.N == 0) return cudaSuccess;
  if (g.dots) return launch_cfg<128, 4, true>(g, num_sms, s);
  return launch_cfg<128, 4, false>(g, num_sms, s);
}

}  // namespace b2q
