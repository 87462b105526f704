// b2q_gemm_tc.cu -- tcgen05 int8 block GEMM with the per-block scale epilogue.
//
//   y[m][n] = sum_b  dw[n,b] * da[m,b] * S_b(n,m),   S_b = sum_{i<32} qw[n,32b+i] * qa[m,32b+i]
//
// Per 32-value block b, one tcgen05.mma (kind::i8, M = 128 weight rows, N = 128
// tokens, K = 32) computes that block's int32 dots S_b into its own TMEM
// accumulator slot.  Scales change every 32 of K, so int32 cannot be carried
// across blocks; epilogue warps read every slot and apply the scales in fp32,
// while the tensor core fills the next slots.  The per-(n, m, b) epilogue --
// TMEM reads and two FMAs per element -- not the tensor core, bounds the kernel.
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
// Epilogue data path: thread t of epilogue warp w owns weight row 32*(w%4) + t
// (its TMEM lane) and 64 of the 128 token columns, read with two
// tcgen05.ld.32x32b.x32 (the widest-bandwidth load shape).  Its weight scale is
// one scalar per block; the 64 activation scales are warp-uniform broadcast
// loads.  Hand-off per block and per slot: the MMA thread commits each block to
// its slot's barrier; an epilogue warp waits for the block, loads it, scales it
// into its accumulators and only then hands the slot back (one arrival per
// warp).  What bounds this loop, measured on B200: a block's MMA result becomes
// visible to a waiting thread ~1300 cycles after issue with 4 slots in flight
// (a ping-pong with no epilogue work at all runs at ~330-400 cycles per block),
// and TMEM holds only 4 blocks of int32 accumulators, so the chain, not the
// FMA work (256 cycles per block), sets the pace.  Register double buffering
// (loading block g+1 while scaling g) and releasing a slot before scaling both
// measured slower than this single-buffered, release-after-scaling order.
// K is padded to whole stages (the padding blocks read zero codes and scales
// through the tensor maps' out-of-bounds fill and add exactly nothing).
// Output stores, bias fused: when y's rows are 16-byte aligned and N is a
// multiple of 32, each epilogue warp writes its 32 rows x BN/2 tokens into its
// own shared-memory box and leaves it by one TMA store (the gate + residual
// form first TMA-loads the residual box during the tile); otherwise, for each
// token, the 32 threads of a warp write 32 consecutive floats of y's row
// (128-byte coalesced).  Other tile ends: GELU + Q8_0 of the next layer's
// input, fp16 attention heads, the column-parallel peer stores.
//
// Roles (384 threads = 3 warpgroups, 1 CTA per SM, persistent over tiles):
//   warp 0      TMA producer: weight codes [128 x 128B], activation codes
//               [128 x 128B] (128B swizzle), weight scales [4 x 128] and
//               activation scales [4 x 128] fp32 per stage (4 blocks of K)
//   warp 1      TMEM allocator + single-thread MMA issuer
//   warps 2,3   idle (complete warpgroup 0, which runs on 40 registers)
//   warps 4..11 epilogue (232 registers)
// Every wait is bounded (b2q_ptx.cuh); on give-up the CTA drains its in-flight
// copies and MMAs, frees TMEM and exits, leaving a code in g_device_status.
#include <atomic>

#include <cuda_fp16.h>

#include "b2q_internal.h"
#include "b2q_ptx.cuh"
#include "b2q_q8.cuh"

namespace b2q {

// Device status word of this library's kernels (0 = ok, else the first
// kDevWait* code recorded by a bounded wait that gave up).
__device__ unsigned int g_device_status = 0;

namespace {

constexpr int kBM = 128;             // weight rows per tile (MMA M, TMEM lanes)
constexpr int kMaxBN = 128;          // the widest tile (MMA N)
constexpr int kKBS = 4;              // 32-value blocks per pipeline stage
constexpr int kStageK = kKBS * kQK;  // 128 bytes of K per operand row per stage
constexpr int kEpiWarps = 8;
constexpr int kEpiWarp0 = 4;         // epilogue = warpgroups 1 and 2
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

// BN: tokens per tile (MMA N), 64..128 in steps of 16; the host picks it per
// shape so that the tiles spread evenly over the SMs (see pick_bn).
template <int STAGES, int BN, bool Q4C = false>
struct Cfg {
  static_assert(BN % 16 == 0 && BN >= 64 && BN <= kMaxBN, "tile width");
  static constexpr int COLS = BN / 2;  // token columns per epilogue thread
  // Accumulator slots (blocks in flight): as many BN-column slots as TMEM
  // holds.  A block's MMA-to-epilogue round trip takes about the same time
  // whatever its width, so the blocks in flight set the rate: 4 at BN 128 or
  // 112, 5 at 96, 6 at 80, 8 at 64.
  static constexpr int SLOTS = static_cast<int>(kTmemCols) / BN;
  static constexpr int A_BYTES = kBM * kStageK;
  static constexpr int B_BYTES = BN * kStageK;
  static constexpr int SW_BYTES = kKBS * kBM * 4;
  static constexpr int SA_BYTES = kKBS * BN * 4;
  // Compact Q4_0 weights: the TMA brings the stage's nibble blocks (128 rows x
  // 64 bytes) and fp16 scales (4 x 128); the converter warps widen them into the
  // A (int8 codes) and SW (fp32 scales) regions that the other roles read.
  static constexpr int PK_OFF = A_BYTES + B_BYTES + SW_BYTES + SA_BYTES;
  static constexpr int PK_BYTES = Q4C ? kBM * kStageK / 2 : 0;
  static constexpr int SWH_OFF = PK_OFF + PK_BYTES;
  static constexpr int SWH_BYTES = Q4C ? kKBS * kBM * 2 : 0;
  // bytes the TMA delivers per stage
  static constexpr int TX_BYTES = Q4C ? B_BYTES + SA_BYTES + PK_BYTES + SWH_BYTES
                                      : A_BYTES + B_BYTES + SW_BYTES + SA_BYTES;
  static constexpr int STAGE_BYTES = (SWH_OFF + SWH_BYTES + 1023) / 1024 * 1024;  // stage pitch in smem
  static constexpr int OFF_TILE = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = OFF_TILE + kOffsetTileBytes;
  // stage full / empty (+ converted), slot full / empty, MMA drain, one
  // residual-box barrier per epilogue warp
  static constexpr int NBARS = (Q4C ? 3 : 2) * STAGES + 2 * SLOTS + 1 + kEpiWarps;
  static constexpr int SMEM = BAR_OFF + NBARS * 8 + 16 + 1024;  // + alignment slack
  // GELU + Q8_0 variant only: a 32 x 33 fp32 transpose buffer per epilogue warp.
  static constexpr int XPOSE_OFF = (BAR_OFF + NBARS * 8 + 16 + 127) / 128 * 128;
  static constexpr int XPOSE_FLOATS = 32 * 33;
  static constexpr int SMEM_XPOSE = XPOSE_OFF + 8 * XPOSE_FLOATS * 4 + 1024;
  // Plain tile end through TMA stores only: one [COLS tokens][32 rows] fp32 box
  // per epilogue warp (128-byte rows, the layout of y), stored asynchronously.
  static constexpr int STO_OFF = XPOSE_OFF;
  static constexpr int STO_WARP_FLOATS = COLS * 32;
  static constexpr int SMEM_STO = STO_OFF + kEpiWarps * STO_WARP_FLOATS * 4 + 1024;
  static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte swizzle alignment");
  static_assert(STAGES <= 16, "stage bitmasks");
};

struct TcParams {
  int M, N, KB, n_tiles, num_tiles;  // KB: blocks of K per tile, rounded up to whole stages
  int KB_real;                       // blocks of K in the data (the rest read as zeros)
  float* y;
  int64_t ldy;
  const float* bias;
  int32_t* dots;
};

// Kernel variants (one instantiation each, so the plain kernel carries none of
// the others' code or parameters).
enum Mode : int {
  kModePlain = 0,   // y = w . x (+ bias)
  kModeDump = 1,    // raw int32 block dots of every block (debug / parity)
  kModePeers = 2,   // column-parallel: the tile goes into every rank's y buffer
  kModeStall = 3,   // failure-path self-test: the producer withholds every stage
  kModeGeluQ8 = 4,  // fused GELU + Q8_0 quantize of the output (next layer's input)
  kModeGateRes = 5, // y = resid + gate * (w . x + bias): the DiT branch's gated residual
  kModeGeluQ8Peers = 6,  // column-parallel GELU + Q8_0: the quantized tile goes into every rank's activations
  kModeStoreTma = 7,     // as plain, each epilogue warp's part of the tile leaves by one TMA store
  kModeHeadsF16 = 8,     // as plain, each output rounded to fp16 into its attention head's [T][64] rows
  kModeGateResTma = 9,   // as gate + residual, the residual box loaded and the result box stored by TMA
};

// Output arguments of the non-plain variants, a separate kernel parameter:
// growing TcParams by such fields slowed the plain kernel's tile loop by 8%.
//   peers: every element goes to ptr[q][m * ldy + col0 + n] for each q -- this
//          rank's slice of the output columns, written straight into every
//          rank's full-width buffer (P2P-mapped memory of the other GPUs);
//   gelu+q8: quantize_q8_0(gelu(y)) into the split layout of the next
//          mul_mat's activations: codes q_codes[m * q_k + n], scales
//          q_scales[(n / 32) * q_ld + m];
//   gate+residual: y[m * ldy + n] = resid[m * ldr + n] + gate[n] * (w . x + bias)[m][n],
//          each step rounded as ggml's separate mul and add (gate may be null);
//   gelu+q8 peers: as gelu+q8, into every rank's split activation buffer:
//          codes at ptr[q] + q_code_off (this rank's first column of the next
//          layer's K), scales at ptr[q] + q_scale_off (its first scale row),
//          codes row pitch q_k = the whole next-layer K.
struct OutParams {
  int n;
  int64_t col0;
  float* ptr[kMaxPeers];
  int8_t* q_codes;
  float* q_scales;
  int64_t q_ld, q_k;
  int q_variant;
  const float* gate;
  const float* resid;
  int64_t ldr;
  int64_t q_code_off, q_scale_off;
  __half* heads[2];  // heads tile end: the [B][H][T][64] fp16 outputs of column parts 0 and 1
  int64_t heads_T;
  int heads_H;
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

// This thread's COLS columns of one accumulator slot, in 32/16/8-column loads.
template <int COLS>
__device__ __forceinline__ void load_slot(uint32_t taddr, uint32_t (&r)[COLS]) {
  static_assert(COLS % 8 == 0, "slot columns");
  int c = 0;
#pragma unroll
  for (; c + 32 <= COLS; c += 32) tmem_ld_32x32b_x32(taddr + c, *reinterpret_cast<uint32_t(*)[32]>(&r[c]));
  if (c + 16 <= COLS) {
    tmem_ld_32x32b_x16(taddr + c, &r[c]);
    c += 16;
  }
  if (c + 8 <= COLS) tmem_ld_32x32b_x8(taddr + c, &r[c]);
}

// One block of the epilogue: wait for block g in accumulator slot `slot`,
// load this thread's COLS columns, scale them into acc, then hand the slot
// back.  j: block within the stage (selects the stage's scales).  Returns
// false when a bounded wait gave up.
template <int STAGES, int BN, bool DUMP, bool Q4C, int COLS = BN / 2>
__device__ __forceinline__ bool epi_block(uint32_t (&cur)[COLS], float2 (&acc)[COLS / 2], int slot, uint32_t sphase,
                                          int j, int kb, int tile, const TcParams& p, const uint8_t* sb,
                                          uint64_t* acc_full, uint64_t* acc_empty, volatile int* abort_flag,
                                          uint32_t tbase, int row, int chalf, int lane) {
  using C = Cfg<STAGES, BN, Q4C>;
  if (!mbar_wait(&acc_full[slot], sphase, &g_device_status, kDevWaitEpilogue, abort_flag)) return false;
  tc_fence_after();
  load_slot<COLS>(tbase + slot * BN, cur);
  const float* sw = reinterpret_cast<const float*>(sb + C::A_BYTES + C::B_BYTES);
  const float* sa = sw + kKBS * kBM;
  const float w = sw[j * kBM + row];
  const float2 w2 = make_float2(w, w);
  const float2 c2 = make_float2(w * kNegTwoPowM129, w * kNegTwoPowM129);
  const float4* da4 = reinterpret_cast<const float4*>(sa + j * BN + chalf * COLS);
  tmem_wait_ld();
  if (DUMP && kb < p.KB_real) {
    const int64_t n = static_cast<int64_t>(tile % p.n_tiles) * kBM + row;
    const int64_t m0 = static_cast<int64_t>(tile / p.n_tiles) * BN + chalf * COLS;
    for (int c = 0; c < COLS; ++c) {
      const int64_t m = m0 + c;
      if (n < p.N && m < p.M) p.dots[(m * p.N + n) * p.KB_real + kb] = static_cast<int32_t>(cur[c] - kOffset);
    }
  }
#pragma unroll
  for (int i = 0; i < COLS / 4; ++i) {
    const float4 d = da4[i];
    const float2 t0 = ffma2(make_float2(__uint_as_float(cur[4 * i]), __uint_as_float(cur[4 * i + 1])), w2, c2);
    const float2 t1 = ffma2(make_float2(__uint_as_float(cur[4 * i + 2]), __uint_as_float(cur[4 * i + 3])), w2, c2);
    acc[2 * i] = ffma2(t0, make_float2(d.x, d.y), acc[2 * i]);
    acc[2 * i + 1] = ffma2(t1, make_float2(d.z, d.w), acc[2 * i + 1]);
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(&acc_empty[slot]);
  return true;
}

// Fused GELU + Q8_0 quantize of token columns m0+CB .. m0+CB+W-1 of one warp's
// accumulators.  The warp's 32 lanes hold one 32-value block (lane = position
// in the block) of each token's next-layer activations.  The GELU values go
// through a 32 x 33 shared-memory transpose (conflict-free both ways), after
// which lane c holds the whole block of column CB+c and quantizes it exactly as
// the stand-alone quantizer does: fmaxf absmax from 0, one scale, 32 codes as
// two 16-byte stores, and the lanes' scales as one coalesced store.
template <int VARIANT, int CB, int W, bool PQ, int NACC>
__device__ __forceinline__ void geluq_chunk(const float2 (&acc)[NACC], float bv, bool has_bias, int64_t m0,
                                            int64_t M, int lane, int8_t* codes, int64_t q_k, float* qs, float* xp,
                                            const OutParams& pp, int64_t nq) {
#pragma unroll
  for (int c = 0; c < W; ++c) {
    const float v = ((CB + c) & 1) ? acc[(CB + c) / 2].y : acc[(CB + c) / 2].x;
    xp[c * 33 + lane] = gelu_ggml(has_bias ? v + bv : v);
  }
  __syncwarp();
  const int64_t m = m0 + CB + lane;
  if (lane < W && m < M) {
    float z[kQK];
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < kQK; ++j) {
      z[j] = xp[lane * 33 + j];
      amax = fmaxf(amax, fabsf(z[j]));
    }
    float d, inv;
    q8_scale<VARIANT>(amax, d, inv);
    uint32_t q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      q[i] = quantize_code<VARIANT>(z[4 * i], inv) | (quantize_code<VARIANT>(z[4 * i + 1], inv) << 8) |
             (quantize_code<VARIANT>(z[4 * i + 2], inv) << 16) | (quantize_code<VARIANT>(z[4 * i + 3], inv) << 24);
    if constexpr (!PQ) {
      uint4* dst = reinterpret_cast<uint4*>(codes + m * q_k);
      dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
      dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
      qs[m] = q8_split_scale(d);
    } else {
      // The same 36 bytes into every rank's activations (NVLink stores for the
      // peers): the exchange is the next layer's Q8_0 input, not fp32.
      const float sc = q8_split_scale(d);
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r) {  // static indices: the pointers stay in the param bank
        if (r >= pp.n) break;
        uint8_t* base = reinterpret_cast<uint8_t*>(pp.ptr[r]);
        uint4* dst = reinterpret_cast<uint4*>(base + pp.q_code_off + nq + m * q_k);
        dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
        dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
        reinterpret_cast<float*>(base + pp.q_scale_off)[(nq / kQK) * pp.q_ld + m] = sc;
      }
    }
  }
  __syncwarp();
}

template <int VARIANT, int COLS, bool PQ, int NACC>
__device__ __forceinline__ void geluq_cols(const float2 (&acc)[NACC], float bv, bool has_bias, int64_t m0, int64_t M,
                                           int lane, int8_t* codes, int64_t q_k, float* qs, float* xp,
                                           const OutParams& pp, int64_t nq) {
  geluq_chunk<VARIANT, 0, (COLS < 32 ? COLS : 32), PQ>(acc, bv, has_bias, m0, M, lane, codes, q_k, qs, xp, pp, nq);
  if constexpr (COLS > 32)
    geluq_chunk<VARIANT, 32, COLS - 32, PQ>(acc, bv, has_bias, m0, M, lane, codes, q_k, qs, xp, pp, nq);
}

template <int STAGES, int BN, int MODE, bool Q4C>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_wc, const __grid_constant__ CUtensorMap tm_ac,
                   const __grid_constant__ CUtensorMap tm_ws, const __grid_constant__ CUtensorMap tm_as,
                   const __grid_constant__ CUtensorMap tm_y, const __grid_constant__ CUtensorMap tm_r, const TcParams p,
                   const __grid_constant__ OutParams pp) {
  constexpr bool DUMP = MODE == kModeDump, PEERS = MODE == kModePeers, STALL = MODE == kModeStall;
  constexpr bool TST = MODE == kModeStoreTma;
  constexpr bool HEADS = MODE == kModeHeadsF16;
  constexpr bool GRT = MODE == kModeGateResTma;  // TMA residual box in, TMA result box out
  static_assert(!(GRT && Q4C), "the compact Q4_0 stages leave no room for the boxes");
  static_assert(!(TST && Q4C), "the compact Q4_0 stages leave no room for the store boxes");
  constexpr bool PQ = MODE == kModeGeluQ8Peers;
  constexpr bool GELUQ = MODE == kModeGeluQ8 || PQ, GATERES = MODE == kModeGateRes;
  using C = Cfg<STAGES, BN, Q4C>;
  constexpr int COLS = C::COLS;
  extern __shared__ uint8_t smem_raw[];
  // Offset arithmetic on the __shared__ array itself (no integer round trip), so
  // the compiler keeps the shared address space and emits shared-memory loads.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + C::SLOTS;
  uint64_t* mma_done = acc_empty + C::SLOTS;
  uint64_t* conv = mma_done + 1;  // Q4C: the stage's weight codes and scales are widened
  uint64_t* rbar = conv + (Q4C ? STAGES : 0);  // [kEpiWarps]: each warp's residual box landed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(rbar + kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  // The MMA and the epilogue read a stage once it is complete: its copies landed
  // and, for compact Q4_0 weights, its codes and scales are widened.
  uint64_t* ready = Q4C ? conv : full;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kEpiWarps);
    }
    for (int a = 0; a < C::SLOTS; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(mma_done, 1);
    for (int w = 0; w < kEpiWarps; ++w) mbar_init(&rbar[w], 1);
    if (Q4C)
      for (int st = 0; st < STAGES; ++st) mbar_init(&conv[st], 2);  // the two converter warps
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
  const int n_ks = KB / kKBS;

  if (warp < kEpiWarp0) {
    // ------------------------------------------------- warpgroup 0 (control)
    setmaxnreg_dec<kRegsControl>();
    if (warp == 0) {
      // ---------------------------------------------------------- producer
      if (elect_one()) {
        uint32_t stage = 0, phase = 0, issued_mask = 0, issued_par = 0;
        bool ok = !STALL;  // self-test: withheld stages leave the consumers' waits to run out
        for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
          const int n0 = (tile % p.n_tiles) * kBM;
          const int m0 = (tile / p.n_tiles) * BN;
          for (int ks = 0; ks < n_ks; ++ks) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, &g_device_status, kDevWaitProducer, abort_flag)) {
              ok = false;
              break;
            }
            uint8_t* sb = smem + stage * C::STAGE_BYTES;
            mbar_arrive_expect_tx(&full[stage], C::TX_BYTES);
            if (Q4C) {  // nibble blocks and fp16 scales; the converters fill A and SW
              tma_load_2d(sb + C::PK_OFF, &tm_wc, &full[stage], ks * kStageK / 2, n0);
              tma_load_2d(sb + C::SWH_OFF, &tm_ws, &full[stage], n0, ks * kKBS);
            } else {
              tma_load_2d(sb, &tm_wc, &full[stage], ks * kStageK, n0);
              tma_load_2d(sb + C::A_BYTES + C::B_BYTES, &tm_ws, &full[stage], n0, ks * kKBS);
            }
            tma_load_2d(sb + C::A_BYTES, &tm_ac, &full[stage], ks * kStageK, m0);
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
        uint32_t stage = 0, phase = 0;
        uint32_t slot = 0, sphase = 0;  // block q fills slot q % SLOTS; sphase = (q / SLOTS) & 1
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
          for (int ks = 0; ok && ks < n_ks; ++ks) {
            if (!mbar_wait(&ready[stage], phase, &g_device_status, kDevWaitMma, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(smem + stage * C::STAGE_BYTES);
            const uint32_t b_base = a_base + C::A_BYTES;
            for (int j = 0; j < kKBS; ++j) {
              if (!mbar_wait(&acc_empty[slot], sphase ^ 1u, &g_device_status, kDevWaitMma, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t d = tmem_base + slot * BN;
              mma_i8(d, smem_desc_k_sw128(a_base + j * kQK), smem_desc_k_sw128(b_base + j * kQK), idesc, 0u);
              mma_i8(d, off_desc, off_desc, idesc_off, 1u);
              mma_commit(&acc_full[slot]);
              if (++slot == C::SLOTS) {
                slot = 0;
                sphase ^= 1u;
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
    } else if (Q4C) {
      // -------------------------------------------- warps 2, 3: Q4_0 converters
      // Per stage: 128 rows x 4 blocks of nibbles -> int8 codes (value - 8) in
      // the 128-byte-swizzled K-major tile the MMA reads (chunk c of row r at
      // chunk c ^ (r % 8) of its 8-row atom), and the fp16 scales -> fp32 times
      // 2^100 (the stored form of the int8 layout's weight scales).  Consecutive
      // threads read consecutive 16-byte nibble blocks.
      const int ct = threadIdx.x - 64;  // 0..63
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        for (int ks = 0; ks < n_ks; ++ks) {
          if (!mbar_wait(&full[stage], phase, &g_device_status, kDevWaitProducer, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sb = smem + stage * C::STAGE_BYTES;
#pragma unroll 2
          for (int i = 0; i < 8; ++i) {
            const int u = ct + 64 * i;
            const int row = u >> 2, blk = u & 3;
            const uint4 nb = *reinterpret_cast<const uint4*>(sb + C::PK_OFF + row * (kStageK / 2) + blk * 16);
            uint8_t* arow = sb + row * kStageK;  // row r of the 1024-byte-aligned tile: r * 128
            const uint4 lo = make_uint4(__vsub4(nb.x & 0x0f0f0f0fu, 0x08080808u), __vsub4(nb.y & 0x0f0f0f0fu, 0x08080808u),
                                        __vsub4(nb.z & 0x0f0f0f0fu, 0x08080808u), __vsub4(nb.w & 0x0f0f0f0fu, 0x08080808u));
            const uint4 hi = make_uint4(__vsub4((nb.x >> 4) & 0x0f0f0f0fu, 0x08080808u),
                                        __vsub4((nb.y >> 4) & 0x0f0f0f0fu, 0x08080808u),
                                        __vsub4((nb.z >> 4) & 0x0f0f0f0fu, 0x08080808u),
                                        __vsub4((nb.w >> 4) & 0x0f0f0f0fu, 0x08080808u));
            *reinterpret_cast<uint4*>(arow + (((2 * blk) ^ (row & 7)) << 4)) = lo;
            *reinterpret_cast<uint4*>(arow + (((2 * blk + 1) ^ (row & 7)) << 4)) = hi;
          }
          const __half* swh = reinterpret_cast<const __half*>(sb + C::SWH_OFF);
          float* sw = reinterpret_cast<float*>(sb + C::A_BYTES + C::B_BYTES);
#pragma unroll
          for (int i = 0; i < 8; ++i) sw[ct + 64 * i] = __half2float(swh[ct + 64 * i]) * kWeightScaleMul;
          fence_proxy_async_smem();  // the codes (generic-proxy writes) -> visible to the tensor core
          __syncwarp();
          if (lane == 0) mbar_arrive(&conv[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------ warpgroups 1-2: epilogue
    setmaxnreg_inc<kRegsEpilogue>();
    const int quarter = warp & 3;               // TMEM lane quarter this warp may access
    const int chalf = (warp - kEpiWarp0) >> 2;  // which 64 of the 128 token columns
    const int row = quarter * 32 + lane;        // this thread's weight row (TMEM lane)
    const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + chalf * COLS;
    uint32_t ra[COLS];
    float2 acc[COLS / 2];
    uint32_t stage = 0, phase = 0;
    uint32_t slot = 0, sphase = 0;  // accumulator slot and its parity, as the MMA issuer's
    bool ok = true;
    // GRT: this warp's box, its residual barrier's parity, a residual load in flight.
    float* rbox = reinterpret_cast<float*>(smem + C::STO_OFF) + (warp - kEpiWarp0) * C::STO_WARP_FLOATS;
    uint64_t* my_rbar = &rbar[warp - kEpiWarp0];
    uint32_t rphase = 0;
    bool rpending = false;
    for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
#pragma unroll
      for (int c = 0; c < COLS / 2; ++c) acc[c] = make_float2(0.0f, 0.0f);
      for (int ks = 0; ks < n_ks; ++ks) {
        // The stage's scales are read from shared memory: wait for the stage.
        if (!mbar_wait(&ready[stage], phase, &g_device_status, kDevWaitEpilogue, abort_flag)) {
          ok = false;
          break;
        }
        const uint8_t* sb = smem + stage * C::STAGE_BYTES;
#pragma unroll
        for (int j = 0; j < kKBS; ++j) {
          if (!epi_block<STAGES, BN, DUMP, Q4C>(ra, acc, static_cast<int>(slot), sphase, j, ks * kKBS + j, tile, p, sb,
                                           acc_full, acc_empty, abort_flag, tbase, row, chalf, lane)) {
            ok = false;
            break;
          }
          if (++slot == C::SLOTS) {
            slot = 0;
            sphase ^= 1u;
          }
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
        if (GRT && ks == 0) {
          // The tile's residual box is fetched once the first stage is done (the
          // previous tile's result box has long left it by then).
          const int rnq = (tile % p.n_tiles) * kBM + quarter * 32;
          const int rm0 = (tile / p.n_tiles) * BN + chalf * COLS;
          if (rnq < p.N && rm0 < p.M) {
            if (lane == 0) {
              bulk_wait_read_all();  // the previous result box has been read out
              mbar_arrive_expect_tx(my_rbar, C::STO_WARP_FLOATS * 4);
              tma_load_2d(rbox, &tm_r, my_rbar, rnq, rm0);
            }
            rpending = true;
          }
        }
      }
      if (!ok || (!GELUQ && !HEADS && !p.y)) continue;
      const int64_t n = static_cast<int64_t>(tile % p.n_tiles) * kBM + row;
      const int64_t m0 = static_cast<int64_t>(tile / p.n_tiles) * BN + chalf * COLS;
      if (HEADS) {
        // Column n is dimension d of head h of part `part` (the cross-attention's
        // q, or its k | v): bias added as the plain tile end adds it (one fp32
        // rounding), then one fp16 rounding as b2q_rows_to_heads stores it.  For
        // each token the warp's 32 lanes write 32 consecutive halves of one row.
        if (n < p.N && m0 < p.M) {
          const int64_t C = static_cast<int64_t>(pp.heads_H) * 64;
          const int part = n >= C ? 1 : 0;
          const int64_t nc = n - part * C;
          const int64_t T = pp.heads_T;
          __half* base = pp.heads[part] + (nc >> 6) * T * 64 + (nc & 63);
          const int64_t b = m0 / T;
          int64_t t = m0 - b * T;
          int64_t off = (b * pp.heads_H * T + t) * 64;  // of token m0
          const float bv = p.bias ? p.bias[n] : 0.0f;
          const float2 b2 = make_float2(bv, bv), one = make_float2(1.0f, 1.0f);
#pragma unroll
          for (int c = 0; c < COLS; ++c) {
            if (m0 + c >= p.M) break;
            if ((c & 1) == 0) acc[c / 2] = ffma2(acc[c / 2], one, b2);
            base[off] = __float2half_rn((c & 1) ? acc[c / 2].y : acc[c / 2].x);
            off += 64;
            if (++t == T) {  // the next token is the next sequence's first
              t = 0;
              off += (static_cast<int64_t>(pp.heads_H) - 1) * T * 64;
            }
          }
        }
        continue;
      }
      if (GRT) {
        // y = resid + gate * (w.x + bias) as the gate + residual tile end rounds
        // it (bias by the packed FMA, __fmul_rn by the row's gate, __fadd_rn of
        // the residual), with the residual read from the warp's box (TMA-loaded
        // during the tile) and the result written back into it for one TMA store.
        // y may be the residual itself: each box is read before it is stored.
        const int64_t rnq = static_cast<int64_t>(tile % p.n_tiles) * kBM + quarter * 32;
        if (rnq < p.N && m0 < p.M) {
          if (!__all_sync(0xffffffffu, mbar_wait(my_rbar, rphase, &g_device_status, kDevWaitEpilogue, abort_flag))) {
            ok = false;
            continue;
          }
          rphase ^= 1u;
          rpending = false;
          const float bv = p.bias ? p.bias[n] : 0.0f;
          const float gv = pp.gate ? pp.gate[n] : 1.0f;
          const float2 b2 = make_float2(bv, bv), one = make_float2(1.0f, 1.0f);
#pragma unroll
          for (int c = 0; c < COLS / 2; ++c) {
            const float2 h = ffma2(acc[c], one, b2);
            const float t0 = pp.gate ? __fmul_rn(h.x, gv) : h.x;
            const float t1 = pp.gate ? __fmul_rn(h.y, gv) : h.y;
            rbox[(2 * c) * 32 + lane] = __fadd_rn(rbox[(2 * c) * 32 + lane], t0);
            rbox[(2 * c + 1) * 32 + lane] = __fadd_rn(rbox[(2 * c + 1) * 32 + lane], t1);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tm_y, rbox, static_cast<int32_t>(rnq), static_cast<int32_t>(m0));
            bulk_commit();
          }
        }
        continue;
      }
      if (TST) {
        // The warp's 32 rows x COLS tokens go through its own box in shared
        // memory and leave by one TMA store, so the next tile's blocks start at
        // once instead of behind 2*COLS global stores per thread.  N % 32 == 0:
        // the warp's rows are all valid or all not; rows and tokens past the
        // tensor's edge are not written by the store.
        const int64_t nq = static_cast<int64_t>(tile % p.n_tiles) * kBM + quarter * 32;
        if (nq < p.N && m0 < p.M) {
          float* st = reinterpret_cast<float*>(smem + C::STO_OFF) + (warp - kEpiWarp0) * C::STO_WARP_FLOATS;
          const float bv = p.bias ? p.bias[n] : 0.0f;
          const float2 b2 = make_float2(bv, bv), one = make_float2(1.0f, 1.0f);  // as the plain tile end
          if (lane == 0) bulk_wait_read_all();  // the warp's previous box has left shared memory
          __syncwarp();
#pragma unroll
          for (int c = 0; c < COLS / 2; ++c) {
            const float2 v = ffma2(acc[c], one, b2);
            st[(2 * c) * 32 + lane] = v.x;
            st[(2 * c + 1) * 32 + lane] = v.y;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tm_y, st, static_cast<int32_t>(nq), static_cast<int32_t>(m0));
            bulk_commit();
          }
        }
        continue;
      }
      if (GELUQ) {
        // The warp's 32 weight rows are one Q8_0 block of the next layer's K
        // (N % 32 == 0, so they are all valid or all not).
        const int64_t nq = static_cast<int64_t>(tile % p.n_tiles) * kBM + quarter * 32;
        if (nq < p.N && m0 < p.M) {
          const float bv = p.bias ? p.bias[n] : 0.0f;
          int8_t* codes = PQ ? nullptr : pp.q_codes + nq;
          float* qs = PQ ? nullptr : pp.q_scales + (nq / kQK) * pp.q_ld;
          float* xp = reinterpret_cast<float*>(smem + C::XPOSE_OFF) + (warp - kEpiWarp0) * C::XPOSE_FLOATS;
          if (pp.q_variant == 0)
            geluq_cols<0, COLS, PQ>(acc, bv, p.bias != nullptr, m0, p.M, lane, codes, pp.q_k, qs, xp, pp, nq);
          else
            geluq_cols<1, COLS, PQ>(acc, bv, p.bias != nullptr, m0, p.M, lane, codes, pp.q_k, qs, xp, pp, nq);
        }
      } else if (n < p.N) {
        const float bv = p.bias ? p.bias[n] : 0.0f;
        if (!PEERS) {  // the column-parallel store is its own instantiation: it slows this loop
          // ggml_add after the mul_mat: one fp32 rounding per element (x * 1 + b), in one
          // packed pass (a select per store costs this kernel 10%).  Without a bias
          // bv = +0, an identity here: the sums start at +0, so none is -0.
          const float2 b2 = make_float2(bv, bv), one = make_float2(1.0f, 1.0f);
#pragma unroll
          for (int c = 0; c < COLS / 2; ++c) acc[c] = ffma2(acc[c], one, b2);
          float* yp = p.y + m0 * p.ldy + n;
          if (GATERES) {
            // ggml_mul(h, gate) then ggml_add(resid, h): two roundings.  The
            // residual is read 16 columns at a time (its loads in flight together).
            const float gv = pp.gate ? pp.gate[n] : 1.0f;
            const float* rp = pp.resid + m0 * pp.ldr + n;
#pragma unroll
            for (int c0 = 0; c0 < COLS; c0 += 16) {
              float r[16];
#pragma unroll
              for (int c = 0; c < 16 && c0 + c < COLS; ++c) r[c] = m0 + c0 + c < p.M ? rp[(c0 + c) * pp.ldr] : 0.0f;
#pragma unroll
              for (int c = 0; c < 16 && c0 + c < COLS; ++c) {
                const int cc = c0 + c;
                const float h = (cc & 1) ? acc[cc / 2].y : acc[cc / 2].x;
                const float t = pp.gate ? __fmul_rn(h, gv) : h;
                if (m0 + cc < p.M) yp[cc * p.ldy] = __fadd_rn(r[c], t);
              }
            }
          } else {
#pragma unroll
            for (int c = 0; c < COLS / 2; ++c) {
              if (m0 + 2 * c < p.M) yp[(2 * c) * p.ldy] = acc[c].x;
              if (m0 + 2 * c + 1 < p.M) yp[(2 * c + 1) * p.ldy] = acc[c].y;
            }
          }
        } else {
          // Gather fused into the epilogue: the tile goes to every rank's buffer
          // (NVLink stores for the peers), overlapping with the next tiles' math.
          const int64_t off = m0 * p.ldy + pp.col0 + n;
#pragma unroll
          for (int q = 0; q < kMaxPeers; ++q) {  // static indices: the pointers stay in the param bank
            if (q >= pp.n) break;
            float* yp = pp.ptr[q] + off;
#pragma unroll
            for (int c = 0; c < COLS / 2; ++c) {
              if (m0 + 2 * c < p.M) yp[(2 * c) * p.ldy] = p.bias ? acc[c].x + bv : acc[c].x;
              if (m0 + 2 * c + 1 < p.M) yp[(2 * c + 1) * p.ldy] = p.bias ? acc[c].y + bv : acc[c].y;
            }
          }
        }
      }
    }
    // A residual load still in flight (a wait gave up) lands before the CTA exits.
    if (GRT && rpending) mbar_wait(my_rbar, rphase, &g_device_status, kDevWaitDrain, nullptr);
    if ((TST || GRT) && lane == 0) bulk_wait_all();  // the warp's stores complete before the CTA exits
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

template <int STAGES, int BN, int MODE, bool Q4C>
cudaError_t launch_cfg(const GemmArgs& g, int num_sms, cudaStream_t s) {
  constexpr bool PEERS = MODE == kModePeers || MODE == kModeGeluQ8Peers;
  using C = Cfg<STAGES, BN, Q4C>;
  const int64_t KB = g.K / kQK;
  CUtensorMap tm_wc, tm_ac, tm_ws, tm_as;
  const bool wmaps =
      Q4C ? make_map_2d(&tm_wc, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.q4c.nibbles, g.K / 2, g.N, g.K / 2, kStageK / 2, kBM,
                        CU_TENSOR_MAP_SWIZZLE_NONE) &&
                make_map_2d(&tm_ws, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, g.q4c.scales, g.N, KB, g.q4c.ld * 2, kBM, kKBS,
                            CU_TENSOR_MAP_SWIZZLE_NONE)
          : make_map_2d(&tm_wc, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.w.codes, g.K, g.N, g.K, kStageK, kBM,
                        CU_TENSOR_MAP_SWIZZLE_128B) &&
                make_map_2d(&tm_ws, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.w.scales, g.N, KB, g.w.ld * 4, kBM, kKBS,
                            CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!wmaps ||
      !make_map_2d(&tm_ac, CU_TENSOR_MAP_DATA_TYPE_UINT8, g.a.codes, g.K, g.M, g.K, kStageK, BN,
                   CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tm_as, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.a.scales, g.M, KB, g.a.ld * 4, BN,
                   kKBS, CU_TENSOR_MAP_SWIZZLE_NONE))
    return cudaErrorInvalidValue;
  TcParams p;
  p.M = static_cast<int>(g.M);
  p.N = static_cast<int>(g.N);
  p.KB = static_cast<int>((KB + kKBS - 1) / kKBS * kKBS);
  p.KB_real = static_cast<int>(KB);
  p.n_tiles = static_cast<int>((g.N + kBM - 1) / kBM);
  const int m_tiles = static_cast<int>((g.M + BN - 1) / BN);
  p.num_tiles = p.n_tiles * m_tiles;
  p.y = g.y;
  p.ldy = g.ldy;
  p.bias = g.bias;
  p.dots = g.dots;
  OutParams pp;
  pp.n = PEERS ? g.n_peers : 0;
  pp.col0 = g.y_col0;
  for (int q = 0; q < kMaxPeers; ++q) pp.ptr[q] = q < pp.n ? g.y_peer[q] : nullptr;
  pp.q_codes = g.q_codes;
  pp.q_scales = g.q_scales;
  pp.q_ld = g.q_ld;
  pp.q_k = MODE == kModeGeluQ8Peers ? g.q_k : g.N;
  pp.q_code_off = g.q_code_off;
  pp.q_scale_off = g.q_scale_off;
  pp.q_variant = g.q_variant;
  pp.gate = g.gate;
  pp.resid = g.resid;
  pp.ldr = g.ldr;
  pp.heads[0] = static_cast<__half*>(g.heads[0]);
  pp.heads[1] = static_cast<__half*>(g.heads[1]);
  pp.heads_T = g.heads_T;
  pp.heads_H = g.heads_H;
  CUtensorMap tm_y{}, tm_r{};
  if constexpr (MODE == kModeStoreTma) {
    // y as [M][ldy] fp32, one box = one epilogue warp's 32 rows x COLS tokens.
    // A shape the map cannot describe takes the plain tile end instead.
    if (!make_map_2d(&tm_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.y, g.N, g.M, g.ldy * 4, 32, C::COLS,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
      return launch_cfg<STAGES, BN, kModePlain, Q4C>(g, num_sms, s);
  }
  if constexpr (MODE == kModeGateResTma) {
    // y and the residual as [M][ld] fp32, the same boxes; else the global-memory form.
    if (!make_map_2d(&tm_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.y, g.N, g.M, g.ldy * 4, 32, C::COLS,
                     CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_2d(&tm_r, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.resid, g.N, g.M, g.ldr * 4, 32, C::COLS,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
      return launch_cfg<STAGES, BN, kModeGateRes, Q4C>(g, num_sms, s);
  }
  auto kern = gemm_tc_kernel<STAGES, BN, MODE, Q4C>;
  constexpr bool GELUQ = MODE == kModeGeluQ8 || MODE == kModeGeluQ8Peers;
  constexpr int smem_bytes = GELUQ ? C::SMEM_XPOSE
                             : (MODE == kModeStoreTma || MODE == kModeGateResTma) ? C::SMEM_STO
                                                                               : C::SMEM;
  static_assert(smem_bytes <= 227 * 1024, "shared memory per CTA");
  // Checked and set once per device (a bit per device; the calls cost more
  // host time than the rest of the launch).
  static std::atomic<uint64_t> ready{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  const uint64_t bit = dev < 64 ? (uint64_t{1} << dev) : 0;
  if (!bit || !(ready.load(std::memory_order_acquire) & bit)) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != kLaunchRegs) return cudaErrorInvalidConfiguration;  // see the register split
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e != cudaSuccess) return e;
    ready.fetch_or(bit, std::memory_order_acq_rel);
  }
  const int grid = p.num_tiles < num_sms ? p.num_tiles : num_sms;
  kern<<<grid, kThreads, smem_bytes, s>>>(tm_wc, tm_ac, tm_ws, tm_as, tm_y, tm_r, p, pp);
  return cudaGetLastError();
}

// Tile width for an M x N problem: the candidate whose busiest SM finishes
// first.  One tile costs about (0.3 + 0.7 * BN / 128) of a 128-wide tile (the
// per-block hand-offs and MMA issue do not shrink with the width); ties go to
// the wider tile.  Wide problems keep 128 (fc1-like shapes fill every wave);
// narrow or short ones (few tiles per SM) trade width for balance.
int pick_bn(int64_t m, int64_t n, int num_sms) {
  static const int cands[] = {128, 112, 96, 80, 64};
  const int64_t n_tiles = (n + kBM - 1) / kBM;
  int best = 128;
  double best_cost = 1e300;
  for (int bn : cands) {
    const int64_t tiles = n_tiles * ((m + bn - 1) / bn);
    const int64_t rounds = (tiles + num_sms - 1) / num_sms;
    const double cost = static_cast<double>(rounds) * (0.3 + 0.7 * bn / 128.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

}  // namespace

cudaError_t read_device_status(unsigned int* value, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_device_status, sizeof(unsigned int));
  if (e != cudaSuccess || !clear) return e;
  const unsigned int zero = 0;
  return cudaMemcpyToSymbol(g_device_status, &zero, sizeof(unsigned int));
}

template <int MODE, bool Q4C = false>
cudaError_t launch_picked(const GemmArgs& g, int num_sms, cudaStream_t s) {
  switch (pick_bn(g.M, g.N, num_sms)) {
    case 112: return launch_cfg<4, 112, MODE, Q4C>(g, num_sms, s);
    case 96: return launch_cfg<4, 96, MODE, Q4C>(g, num_sms, s);
    case 80: return launch_cfg<4, 80, MODE, Q4C>(g, num_sms, s);
    case 64: return launch_cfg<4, 64, MODE, Q4C>(g, num_sms, s);
    default: return launch_cfg<4, 128, MODE, Q4C>(g, num_sms, s);
  }
}

bool make_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                        uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swz) {
  return make_map_2d(map, dt, base, inner, outer, row_stride_bytes, box_inner, box_outer, swz);
}

cudaError_t launch_gemm_tc(const GemmArgs& g, int num_sms, cudaStream_t s) {
  if (g.M == 0 || g.N == 0) return cudaSuccess;
  if (g.q4c.nibbles) {  // compact Q4_0 weights: plain, bias, gate + residual and GELU + Q8_0 tile ends
    if (g.dots || g.inject_stall || g.n_peers > 0) return cudaErrorInvalidValue;
    if (g.q_codes) {
      if (g.N % kQK != 0 || !g.q_scales) return cudaErrorInvalidValue;
      return launch_picked<kModeGeluQ8, true>(g, num_sms, s);
    }
    if (g.resid) return launch_picked<kModeGateRes, true>(g, num_sms, s);
    return launch_picked<kModePlain, true>(g, num_sms, s);
  }
  if (g.dots) return launch_cfg<4, 128, kModeDump, false>(g, num_sms, s);
  if (g.inject_stall) return launch_cfg<4, 128, kModeStall, false>(g, num_sms, s);
  if (g.q_codes) {
    if (g.N % kQK != 0 || !g.q_scales) return cudaErrorInvalidValue;
    return launch_picked<kModeGeluQ8>(g, num_sms, s);
  }
  if (g.q_peers) {  // column-parallel GELU + Q8_0: q_code_off, q_scale_off and q_k describe the buffers
    if (g.N % kQK != 0 || g.q_k % kQK != 0 || g.n_peers < 1) return cudaErrorInvalidValue;
    return launch_picked<kModeGeluQ8Peers>(g, num_sms, s);
  }
  if (g.heads[0]) {  // tensor-core tiles only (the caller checks the shape)
    if (g.M <= kGemvMaxM || g.resid || g.n_peers > 0 || g.heads_T <= 0 || g.heads_H <= 0)
      return cudaErrorInvalidValue;
    return launch_picked<kModeHeadsF16>(g, num_sms, s);
  }
  // A handful of tokens: the weight streamed once on CUDA cores, same bits.
  if (g.M <= kGemvMaxM && g.n_peers == 0) return launch_gemv(g, s);
  if (g.resid) {
    // TMA boxes when y's and the residual's rows are 16-byte aligned and whole 32-row boxes.
    if (g.y && reinterpret_cast<uintptr_t>(g.y) % 16 == 0 && g.ldy % 4 == 0 &&
        reinterpret_cast<uintptr_t>(g.resid) % 16 == 0 && g.ldr % 4 == 0 && g.N % 32 == 0)
      return launch_picked<kModeGateResTma>(g, num_sms, s);
    return launch_picked<kModeGateRes>(g, num_sms, s);
  }
  if (g.n_peers > 0) return launch_picked<kModePeers>(g, num_sms, s);
  // TMA-stored tile ends when y's rows are 16-byte aligned and whole 32-row boxes.
  if (g.y && reinterpret_cast<uintptr_t>(g.y) % 16 == 0 && g.ldy % 4 == 0 && g.N % 32 == 0)
    return launch_picked<kModeStoreTma>(g, num_sms, s);
  return launch_picked<kModePlain>(g, num_sms, s);
}

}  // namespace b2q

// The Q4_K and F16 kernels share this translation unit (and g_device_status).
#include "b2q_gemm_q4k.cuh"
#include "b2q_gemm_f16.cuh"
