// b2q_gemm_tc.cu -- tcgen05 int8 block GEMM with the per-block scale epilogue.
//
//   y[m][n] = sum_b  dw[n,b] * da[m,b] * S_b(n,m),   S_b = sum_{i<32} qw[n,32b+i] * qa[m,32b+i]
//
// One tcgen05.mma (kind::i8, M=128 weight rows x N=BN tokens x K=32) computes
// exactly one block's int32 dots S_b into a fresh TMEM accumulator; the epilogue
// warps drain it, scale and accumulate in fp32 registers, while the tensor core
// already fills the next accumulator slot.  Scales change every 32 of K, so int32
// cannot be carried across blocks: the epilogue's per-(m,n,b) arithmetic, not
// the tensor core, bounds this kernel.
//
// Epilogue arithmetic per element and block (exact int -> fp32 fold):
//   f = bits(S + 0x4B400000)       = 1.5*2^23 + S exactly (|S| <= 32*127*128 < 2^22)
//   t = fma(f, dw, -1.5*2^23*dw)   = round(S * dw)   (the constant term is exact:
//                                     dw has an 11-bit fp16 significand)
//   acc = fma(t, da, acc)
//
// Roles (320 threads, 1 CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: weight codes [128 x 128B], activation codes
//               [BN x 128B] (128B swizzle), weight scales [4 x 128] and
//               activation scales [4 x BN] fp32 per stage (4 blocks of K)
//   warp 1      TMEM allocator + single-thread MMA issuer
//   warps 2..9  epilogue: warp w owns TMEM lanes 32*(w%4).. (weight rows) and
//               half of the BN accumulator columns (tokens)
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
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr uint32_t kMagicBits = 0x4B400000u;
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
constexpr uint32_t kTmemCols = 512;

template <int BN, int STAGES>
struct Cfg {
  static constexpr int A_BYTES = kBM * kStageK;
  static constexpr int B_BYTES = BN * kStageK;
  static constexpr int SW_BYTES = kKBS * kBM * 4;
  static constexpr int SA_BYTES = kKBS * BN * 4;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SW_BYTES + SA_BYTES;
  static constexpr int ACC_SLOTS = static_cast<int>(kTmemCols) / BN;
  static constexpr int COLS = BN / 2;  // accumulator columns per epilogue warp
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
  static constexpr int NBARS = 2 * STAGES + 2 * ACC_SLOTS + 1;
  static constexpr int SMEM = BAR_OFF + NBARS * 8 + 16 + 1024;  // + alignment slack
  static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte swizzle alignment");
  static_assert(STAGES <= 16, "stage bitmasks");
};

struct TcParams {
  int M, N, KB, n_tiles, num_tiles;
  float* y;
  int64_t ldy;
  const float* bias;
  int32_t* dots;
};

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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
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
        if ((issued_mask >> s) & 1u) mbar_wait(&full[s], (issued_par >> s) & 1u, &g_device_status, kDevWaitDrain, nullptr);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_i8(kBM, BN);
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
            mma_i8(tmem_base + slot * BN, smem_desc_k_sw128(a_base + j * kQK),
                   smem_desc_k_sw128(b_base + j * kQK), idesc, 0u);
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
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int chalf = ew >> 2;     // which half of the BN columns
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    uint32_t stage = 0, phase = 0, slot = 0, acc_phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
      const int n0 = (tile % p.n_tiles) * kBM;
      const int m0 = (tile / p.n_tiles) * BN;
      float acc[C::COLS];
#pragma unroll
      for (int c = 0; c < C::COLS; ++c) acc[c] = 0.0f;
      for (int ks = 0; ok && ks < n_ks; ++ks) {
        if (!mbar_wait(&full[stage], phase, &g_device_status, kDevWaitEpilogue, abort_flag)) {
          ok = false;
          break;
        }
        const uint8_t* sb = smem + stage * C::STAGE_BYTES;
        const float* sw = reinterpret_cast<const float*>(sb + C::A_BYTES + C::B_BYTES);
        const float* sa = sw + kKBS * kBM;
        const int nblk = min(kKBS, KB - ks * kKBS);
        for (int j = 0; j < nblk; ++j) {
          if (!mbar_wait(&acc_full[slot], acc_phase, &g_device_status, kDevWaitEpilogue, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t taddr = tmem_base + lane_off + slot * BN + chalf * C::COLS;
          const float dw = sw[j * kBM + row];
          const float cw = -kMagic * dw;
          const float4* da4 = reinterpret_cast<const float4*>(sa + j * BN + chalf * C::COLS);
#pragma unroll
          for (int c0 = 0; c0 < C::COLS; c0 += 32) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(taddr + c0, r);
            tmem_wait_ld();
            if (c0 + 32 == C::COLS) {  // accumulator slot fully read: hand it back
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&acc_empty[slot]);
            }
#pragma unroll
            for (int c = 0; c < 32; c += 4) {
              const float4 da = da4[(c0 + c) >> 2];
              acc[c0 + c + 0] = fmaf(fmaf(__uint_as_float(r[c + 0] + kMagicBits), dw, cw), da.x, acc[c0 + c + 0]);
              acc[c0 + c + 1] = fmaf(fmaf(__uint_as_float(r[c + 1] + kMagicBits), dw, cw), da.y, acc[c0 + c + 1]);
              acc[c0 + c + 2] = fmaf(fmaf(__uint_as_float(r[c + 2] + kMagicBits), dw, cw), da.z, acc[c0 + c + 2]);
              acc[c0 + c + 3] = fmaf(fmaf(__uint_as_float(r[c + 3] + kMagicBits), dw, cw), da.w, acc[c0 + c + 3]);
            }
            if (DUMP) {
              const int64_t n = n0 + row;
              const int blk = ks * kKBS + j;
              if (n < p.N) {
#pragma unroll 4
                for (int c = 0; c < 32; ++c) {
                  const int64_t mm = m0 + chalf * C::COLS + c0 + c;
                  if (mm < p.M) p.dots[(mm * p.N + n) * KB + blk] = static_cast<int32_t>(r[c]);
                }
              }
            }
          }
          if (++slot == C::ACC_SLOTS) {
            slot = 0;
            acc_phase ^= 1u;
          }
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
      const int64_t n = static_cast<int64_t>(n0) + row;
      if (p.y && n < p.N) {
        const int mbase = m0 + chalf * C::COLS;
        const int mcount = min(C::COLS, p.M - mbase);
        float* yp = p.y + static_cast<int64_t>(mbase) * p.ldy + n;
        const float bv = p.bias ? p.bias[n] : 0.0f;
        const bool add_bias = p.bias != nullptr;
#pragma unroll
        for (int c = 0; c < C::COLS; ++c) {
          if (c < mcount) *yp = add_bias ? acc[c] + bv : acc[c];
          yp += p.ldy;
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

bool make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base,
                 uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  (void)esize;
  return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int STAGES, bool DUMP>
cudaError_t launch_cfg(const GemmArgs& g, int num_sms, cudaStream_t s) {
  using C = Cfg<BN, STAGES>;
  const int64_t KB = g.K / kQK;
  CUtensorMap tm_wc, tm_ac, tm_ws, tm_as;
  if (!make_map_2d(&tm_wc, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.w.codes, g.K, g.N, g.K, kStageK, kBM,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tm_ac, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.a.codes, g.K, g.M, g.K, kStageK, BN,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tm_ws, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, g.w.scales, g.N, KB, g.w.ld * 4, kBM,
                   kKBS, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map_2d(&tm_as, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, g.a.scales, g.M, KB, g.a.ld * 4, BN,
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
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
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
