// b2q_internal.h -- shared declarations between the C-ABI layer (b2q_api.cu)
// and the kernel translation units.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace b2q {

// Device status codes (g_device_status).
enum : unsigned int {
  kDevOk = 0,
  kDevWaitProducer = 0x101,  // TMA producer gave up waiting for a free stage
  kDevWaitMma = 0x102,       // MMA issuer gave up waiting for data / a free accumulator
  kDevWaitEpilogue = 0x103,  // epilogue gave up waiting for an accumulator
  kDevWaitDrain = 0x104,     // teardown gave up waiting for in-flight copies / MMAs
};

constexpr int kQK = 32;
constexpr int kQ8Bytes = 34;
constexpr int kQ4Bytes = 18;
constexpr int kTypeQ4_0 = 2;
constexpr int kTypeQ8_0 = 8;
constexpr int kTypeQ4_K = 12;  // ggml's k-quant, 256-value super-blocks (144 bytes)
constexpr int kQKK = 256;
constexpr int kQ4KBytes = 144;
// Q4_K packed layout: the GGUF block_q4_K rows themselves, contiguous
// (k/256 * 144 bytes per row), base 256-byte aligned; the GEMM unpacks them on
// chip.  Q8_K prepared activations: codes int8 [m][k] | d fp32 [k/256][scale_ld(m)].
struct Q4kWeight {
  const uint8_t* raw;
  int64_t row_bytes;
};
struct Q8kAct {
  int8_t* codes;
  float* d;
  int64_t ld;
};

inline int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// Layout of the GEMM operands in HBM ("split" layout):
//   codes  int8  [rows][K]          row stride K bytes
//   scales fp32  [K/32][ld]         ld = round_up(rows, 4)  (16-byte TMA strides)
// The fp32 scales are stored pre-multiplied by a power of two (exact for fp16
// values): weights by 2^kWeightScaleExp2, activations by 2^kActScaleExp2.  The
// GEMM epilogue relies on these factors to fold int32 dots read as fp32
// subnormals into normal fp32 values (see b2q_gemm_tc.cu).
constexpr float kWeightScaleMul = 0x1p100f;  // 2^100
constexpr float kActScaleMul = 0x1p49f;      // 2^49
struct SplitOperand {
  const int8_t* codes;
  const float* scales;
  int64_t rows;
  int64_t ld;  // scale row stride in elements
};

inline int64_t scale_ld(int64_t rows) { return round_up(rows, 4); }

// Compact Q4_0 weight layout (the GGUF footprint, 0.5625 bytes per value): the
// 16 nibble bytes of every block, rows of k/2 bytes (GGUF order inside a block:
// byte j holds element j low and element j + 16 high), then the fp16 scales
// block-major [k/32][ld] with ld = round_up(n, 8) (16-byte TMA strides).  The
// GEMM widens the nibbles on chip.
inline int64_t q4c_scale_ld(int64_t n) { return round_up(n, 8); }
inline size_t q4c_bytes(int64_t n, int64_t k) {
  return static_cast<size_t>(round_up(n * (k / 2), 256) + round_up((k / kQK) * q4c_scale_ld(n) * 2, 256));
}
struct Q4cWeight {
  const uint8_t* nibbles;  // [n][k/2]
  const uint16_t* scales;  // fp16 [k/32][ld]
  int64_t ld;
};
inline Q4cWeight q4c_at(const uint8_t* base, int64_t n, int64_t k) {
  Q4cWeight w;
  w.nibbles = base;
  w.scales = reinterpret_cast<const uint16_t*>(base + round_up(n * (k / 2), 256));
  w.ld = q4c_scale_ld(n);
  return w;
}
inline size_t split_bytes(int64_t rows, int64_t k) {
  return static_cast<size_t>(round_up(rows * k, 256) + round_up((k / kQK) * scale_ld(rows) * 4, 256));
}
inline size_t q4k_bytes(int64_t n, int64_t k) { return static_cast<size_t>(round_up(n * (k / kQKK) * kQ4KBytes, 256)); }
inline size_t q8k_bytes(int64_t m, int64_t k) {
  return static_cast<size_t>(round_up(m * k, 256) + round_up((k / kQKK) * scale_ld(m) * 4, 256));
}
inline Q4kWeight q4k_at(const uint8_t* base, int64_t n, int64_t k) {
  (void)n;
  Q4kWeight w;
  w.raw = base;
  w.row_bytes = (k / kQKK) * kQ4KBytes;
  return w;
}
inline Q8kAct q8k_at(uint8_t* base, int64_t m, int64_t k) {
  Q8kAct a;
  a.codes = reinterpret_cast<int8_t*>(base);
  a.d = reinterpret_cast<float*>(base + round_up(m * k, 256));
  a.ld = scale_ld(m);
  return a;
}

// The current device and its SM count, cached per device after the first
// query (the launch paths call this on every call).  Returns the SM count;
// 0 when the device is not compute capability 10.0; -1 when a query failed.
int current_device_sms(int* device = nullptr);

// ---- launchers (return cudaSuccess or the launch error) ----
cudaError_t launch_quantize_q8_0_blocks(const float* x, int64_t m, int64_t k, int64_t ldx_floats,
                                        uint8_t* y, int64_t ldy_bytes, int variant, bool vec4,
                                        cudaStream_t s);
cudaError_t launch_quantize_q8_0_split(const float* x, int64_t m, int64_t k, int64_t ldx_floats,
                                       int8_t* codes, float* scales, int64_t ld, int variant,
                                       bool vec4, cudaStream_t s);
cudaError_t launch_quantize_q8_k(const float* x, int64_t m, int64_t k, int64_t ldx_floats, int8_t* codes,
                                 float* dq, int64_t ld, bool vec4, cudaStream_t s);

cudaError_t launch_pack_weights(int wtype, const uint8_t* w, int64_t n, int64_t k,
                                int64_t ldw_bytes, int8_t* codes, float* scales, int64_t ld,
                                cudaStream_t s);
// GGUF Q4_0 rows -> the compact layout above.
cudaError_t launch_pack_q4c(const uint8_t* w, int64_t n, int64_t k, int64_t ldw_bytes, uint8_t* nibbles,
                            uint16_t* scales, int64_t ld, cudaStream_t s);
cudaError_t launch_gemm_simt(int wtype, const uint8_t* w, int64_t ldw_bytes, int64_t n, int64_t k,
                             const uint8_t* a, int64_t lda_bytes, int64_t m, float* y,
                             int64_t ldy_floats, cudaStream_t s);

// ggml_norm + adaLN modulate, fp32 out (codes == nullptr) or Q8_0 split out.
constexpr int64_t kNormMaxC = 4096;
cudaError_t launch_norm_modulate(const float* x, int64_t m, int64_t c, int64_t ldx_floats, float eps,
                                 const float* mscale, const float* mshift, float* y, int64_t ldy_floats,
                                 int8_t* codes, float* qscales, int64_t qld, int variant, cudaStream_t s,
                                 bool affine = false);

// DiT attention I/O (b2q_attn_io.cu).
cudaError_t launch_rows_to_heads(const float* src, int64_t B, int64_t T, int H, int D, int64_t ld_floats, int parts,
                                 unsigned norm_mask, const float* g0, const float* g1, float eps, void* o0, void* o1,
                                 void* o2, cudaStream_t s, bool f32_out = false);
cudaError_t launch_heads_q8(const void* o16, int64_t B, int64_t T, int H, int D, int64_t sb, int64_t sh,
                            int64_t st, int8_t* codes, float* scales, int64_t ld, int variant, cudaStream_t s);

// fp32 attention core, online softmax in IEEE fp32 (b2q_attention.cu): q [B][H][Tq][D],
// k, v [B][H][Tk][D] (+ optional k2, v2 [B][H][Tk2][D]), o rows [B*Tq][ldo] at column h*D.
cudaError_t launch_attention_f32(const float* q, const float* k, const float* v, const float* k2, const float* v2,
                                 int64_t B, int H, int64_t Tq, int64_t Tk, int64_t Tk2, int D, float scale, float* o,
                                 int64_t ldo_floats, cudaStream_t s);

// Tensor-core attention, D = 64, fp16 q / k / v / o (b2q_attention.cu): q [B][H][Tq][64],
// k, v [B][H][Tk][64] (+ k2, v2 [B][H][Tk2][64]), o rows [B*Tq][ldo halves] at column h*64.
cudaError_t launch_attention_f16(const void* q, const void* k, const void* v, const void* k2, const void* v2,
                                 int64_t B, int H, int64_t Tq, int64_t Tk, int64_t Tk2, float scale, void* o,
                                 int64_t ldo_halves, cudaStream_t s);
// The same with the output as the output projection's Q8_0 prepared activations
// (rows b*Tq + t, K = H*64; codes [rows][K], fp32 split scales [K/32][ld]),
// byte-equal to launch_attention_f16 followed by launch_heads_q8.
cudaError_t launch_attention_f16_q8(const void* q, const void* k, const void* v, const void* k2, const void* v2,
                                    int64_t B, int H, int64_t Tq, int64_t Tk, int64_t Tk2, float scale,
                                    int8_t* codes, float* scales, int64_t ld, int variant, cudaStream_t s);
// Status word of the attention kernels' bounded waits (its own translation unit).
cudaError_t read_attention_status(unsigned int* value, bool clear);

// Dequantize-to-float form (b2q_dense_f32.cu): GGUF rows -> fp32 / fp16 rows,
// and the strict fp32 mul_mat y = x . w^T (+ bias).
cudaError_t launch_dequantize(int wtype, const void* w, int64_t ldw_bytes, int64_t n, int64_t k, bool f16_out,
                              void* out, int64_t ldo_elems, cudaStream_t s);
cudaError_t launch_sgemm(const float* x, int64_t ldx, int64_t m, const float* w, int64_t ldw, int64_t n, int64_t k,
                         const float* bias, float* y, int64_t ldy, cudaStream_t s);

cudaError_t launch_gelu(const float* x, int64_t rows, int64_t cols, int64_t ldx_floats, float* y,
                        int64_t ldy_floats, cudaStream_t s);

constexpr int kMaxPeers = 8;  // ranks of one NVLink domain a column-parallel GEMM writes to

struct GemmArgs {
  SplitOperand w;     // weights: rows = N
  SplitOperand a;     // activations: rows = M
  int64_t M, N, K;
  float* y;           // [M][ldy]
  int64_t ldy;        // floats
  const float* bias;  // [N] or nullptr
  int32_t* dots;      // debug dump [M][N][K/32] or nullptr
  int n_peers = 0;    // > 0: write y_peer[q][m*ldy + y_col0 + n] for every q instead of y
  int64_t y_col0 = 0;
  float* y_peer[kMaxPeers] = {};
  int inject_stall = 0;  // self-test of the bounded waits (b2q_selftest_stalled_mul_mat)
  // Fused GELU + Q8_0 epilogue (q_codes != nullptr): instead of y, write
  // quantize_q8_0(gelu(y)) into the split layout of the next mul_mat's
  // activations (rows = M tokens, K_next = N): codes [M][N], scales [N/32][q_ld].
  int8_t* q_codes = nullptr;
  float* q_scales = nullptr;
  int64_t q_ld = 0;
  int q_variant = 0;
  // The same, column-parallel (q_peers): every one of the n_peers split
  // buffers at y_peer[q] (as bytes) receives this rank's columns; codes at
  // + q_code_off with row pitch q_k (the whole next-layer K), scales at
  // + q_scale_off with row stride q_ld.
  bool q_peers = false;
  int64_t q_k = 0, q_code_off = 0, q_scale_off = 0;
  // Gated residual epilogue (resid != nullptr): y = resid + gate[n] * (w.x + bias),
  // resid [M][ldr]; gate [N] or nullptr (no gate).
  const float* gate = nullptr;
  const float* resid = nullptr;
  int64_t ldr = 0;
  // Compact Q4_0 weights (q4c.nibbles != nullptr): w is unused; the kernel reads
  // the nibble blocks and fp16 scales and widens them on chip.
  Q4cWeight q4c = {nullptr, nullptr, 0};
  // Attention-head tile end (heads[0] != nullptr): instead of y, column
  // n = part*H*64 + h*64 + d of token m = b*heads_T + t goes, rounded to fp16,
  // to heads[part][((b*H + h)*heads_T + t)*64 + d] (N = parts*H*64).
  void* heads[2] = {nullptr, nullptr};
  int64_t heads_T = 0;
  int heads_H = 0;
};
cudaError_t launch_gemm_tc(const GemmArgs& args, int num_sms, cudaStream_t s);
// 2-D tensor map (cuTensorMapEncodeTiled through the runtime's driver entry point).
bool make_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                        uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swz);

// Q4_K x Q8_K GEMM (b2q_gemm_q4k.cuh):
//   weight: block_q4_K rows, ldw_bytes apart (16-byte aligned base and stride);
//   activations: int8 Q8_K codes [M][K], fp32 d [K/256][lda].
// y = w.x (+ bias), or resid + gate * (w.x + bias) when resid is set.
struct Q4kArgs {
  const uint8_t* w_raw;
  int64_t ldw_bytes;
  const int8_t* a_codes;
  const float* a_d;
  int64_t lda;
  int64_t M, N, K;
  float* y;
  int64_t ldy;
  const float* bias = nullptr;
  const float* gate = nullptr;
  const float* resid = nullptr;
  int64_t ldr = 0;
};
cudaError_t launch_gemm_q4k(const Q4kArgs& args, int num_sms, cudaStream_t s);

// F16 weights (b2q_gemm_f16.cuh): w fp16 [N][K] rows ldw_bytes apart, x16 fp16
// [M][K] rows ldx_bytes apart (both 16-byte aligned, K % 8 == 0);
// y[m][n] = sum_k w[n][k] x16[m][k] (+ bias[n]), fp32, ldy floats -- or, when
// y16 is not null, rounded to fp16 into y16 (ldy halves) instead of y.
cudaError_t launch_gemm_f16(const void* w, int64_t ldw_bytes, const void* x16, int64_t ldx_bytes, int64_t M,
                            int64_t N, int64_t K, float* y, int64_t ldy, const float* bias, int num_sms,
                            cudaStream_t s, void* y16 = nullptr);
// SLat sparse stages (b2q_sparse.cu).
// Submanifold-conv gather: g[t][o*C + c] = x16[idx[o*tokens + t]][c] for the
// 27 offsets o, zero where the index is < 0 or >= tokens.  C % 8 == 0.
cudaError_t launch_gather27(const void* x16, int64_t tokens, int64_t C, const int32_t* idx, void* g,
                            cudaStream_t s);
// fp16 -> fp32 of n values.
cudaError_t launch_half_to_float(const void* h, int64_t n, float* f, cudaStream_t s);
// Scatter-mean with fp16 partial sums in fine-row order (see b2q_sparse.cu);
// ws holds 3 * coarse + 1 + fine int32 (hist, cursor, offsets, child lists).
cudaError_t launch_scatter_mean_f16(const void* x16, int64_t fine, int64_t C, const int32_t* rows,
                                    const float* counts, int64_t coarse, void* out16, int32_t* ws,
                                    cudaStream_t s);
// The same in two parts: the child lists of every coarse row (a plan of
// 3 * coarse + 1 + fine int32, reusable while rows does not change), then the
// one-launch fp16 accumulation over a plan.
// Grouped F16 GEMM for the planned sparse convolution (b2q_gemm_f16.cuh):
// x16 [M_cap][K] in 256-row tiles, *m_tiles_dev of them valid; tile j uses the
// weight columns [k_group[j] * K, (k_group[j] + 1) * K) of w [N][Kw];
// fp32 y [M_cap][ldy].  K % 64 == 0.
cudaError_t launch_gemm_f16_grouped(const void* w, int64_t ldw_bytes, int64_t Kw, const void* x16, int64_t ldx_bytes,
                                    int64_t M_cap, int64_t N, int64_t K, float* y, int64_t ldy,
                                    const int32_t* m_tiles_dev, const int32_t* k_group, int64_t max_m_tiles,
                                    int num_sms, cudaStream_t s);
// Planned sparse convolution (b2q_sparse.cu): plan rows and size, plan build,
// and the run (pair gather into g [rows][C] fp16, grouped GEMM into part
// [rows][cout] fp32, ordered reduce into y16).  C % 64 == 0, cout % 8 == 0.
int64_t conv_plan_rows(int64_t tokens);
int64_t conv_plan_ints(int64_t tokens);
cudaError_t launch_conv_plan(const int32_t* idx, int64_t tokens, int32_t* plan, cudaStream_t s);
cudaError_t launch_conv_planned(const void* x16, int64_t tokens, int64_t C, const void* w16, int64_t cout,
                                const float* bias, const int32_t* plan, void* g, float* part, void* y16, int num_sms,
                                cudaStream_t s);
cudaError_t launch_scatter_plan(const int32_t* rows, int64_t fine, int64_t coarse, int32_t* plan, cudaStream_t s);
cudaError_t launch_scatter_mean_planned(const void* x16, int64_t C, const int32_t* plan, const float* counts,
                                        int64_t coarse, void* out16, cudaStream_t s);
// fp32 rows -> fp16 rows [m][ldy] (round to nearest even), k % 8 == 0.
cudaError_t launch_to_f16(const float* x, int64_t m, int64_t k, int64_t ldx_floats, void* y, int64_t ldy,
                          bool vec4, cudaStream_t s);

// CUDA-core kernel for M <= kGemvMaxM tokens (plain, bias, gate + residual);
// bit-identical to the tensor-core kernel (b2q_gemv.cu).
constexpr int64_t kGemvMaxM = 8;
cudaError_t launch_gemv(const GemmArgs& args, cudaStream_t s);
cudaError_t read_device_status(unsigned int* value, bool clear);

}  // namespace b2q
