// b2q_api.cu -- the extern "C" boundary (include/b2q.h): argument validation,
// workspace carving and kernel dispatch.  Host code only; never allocates,
// never synchronises inside a compute call, returns a status code for every
// failure instead of aborting.
#include "../../include/b2q.h"
#include "b2q_internal.h"

#include <atomic>
#include <climits>
#include <cmath>
#include <cstdint>

namespace {

using namespace b2q;

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Device check: the kernels are built for sm_100a only.
int check_device(int* sms) {
  const int n = current_device_sms();
  if (n < 0) return B2Q_ERR_CUDA;
  if (n == 0) return B2Q_ERR_UNSUPPORTED;
  if (sms) *sms = n;
  return B2Q_OK;
}

int from_cuda(cudaError_t e) { return e == cudaSuccess ? B2Q_OK : B2Q_ERR_CUDA; }

bool valid_wtype(int t) { return t == B2Q_TYPE_Q8_0 || t == B2Q_TYPE_Q4_0 || t == B2Q_TYPE_Q4_K; }
// Bytes of one raw row of k values.
int64_t raw_row_bytes(int t, int64_t k) {
  if (t == B2Q_TYPE_Q4_K) return (k / kQKK) * kQ4KBytes;
  return (k / kQK) * (t == B2Q_TYPE_Q8_0 ? kQ8Bytes : kQ4Bytes);
}

// Common checks of a weight operand in raw ggml block layout.
int check_raw_weight(int wtype, const void* w, int64_t ldw, int64_t n, int64_t k) {
  if (!valid_wtype(wtype)) return B2Q_ERR_UNSUPPORTED;
  if (n < 0 || k <= 0 || k % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX || k > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (n > 0 && !w) return B2Q_ERR_INVALID_ARG;
  if (wtype == B2Q_TYPE_Q4_K && k % kQKK != 0) return B2Q_ERR_INVALID_ARG;
  if (ldw < raw_row_bytes(wtype, k)) return B2Q_ERR_INVALID_ARG;
  if (!aligned(w, 2) || ldw % 2 != 0) return B2Q_ERR_MISALIGNED;
  return B2Q_OK;
}

struct Carve {
  uint8_t* p;
  size_t left;
  uint8_t* take(size_t bytes) {
    if (bytes > left) return nullptr;
    uint8_t* r = p;
    p += bytes;
    left -= bytes;
    return r;
  }
};

SplitOperand split_at(uint8_t* base, int64_t rows, int64_t k) {
  SplitOperand s;
  s.codes = reinterpret_cast<const int8_t*>(base);
  s.scales = reinterpret_cast<const float*>(base + round_up(rows * k, 256));
  s.rows = rows;
  s.ld = scale_ld(rows);
  return s;
}

// The compact Q4_0 entries' weight and activation operands.
int q4c_operands(const void* packed, int64_t n, int64_t k, const void* act, int64_t m, GemmArgs& g) {
  g.q4c = q4c_at(static_cast<const uint8_t*>(packed), n, k);
  g.a = split_at(static_cast<uint8_t*>(const_cast<void*>(act)), m, k);
  g.w = g.a;  // unused by the compact path
  g.M = m;
  g.N = n;
  g.K = k;
  g.dots = nullptr;
  return B2Q_OK;
}

int run_gemm(const SplitOperand& w, const SplitOperand& a, int64_t m, int64_t n, int64_t k,
             float* y, int64_t ldy_floats, const float* bias, int32_t* dots, int sms,
             cudaStream_t s) {
  GemmArgs g;
  g.w = w;
  g.a = a;
  g.M = m;
  g.N = n;
  g.K = k;
  g.y = y;
  g.ldy = ldy_floats;
  g.bias = bias;
  g.dots = dots;
  return from_cuda(launch_gemm_tc(g, sms, s));
}

// Activation quantize into the split layout + GEMM against a split weight.
int mul_mat_split(const SplitOperand& w, int64_t n, int64_t k, const float* x, int64_t m,
                  int64_t ldx, const float* bias, float* y, int64_t ldy, int variant, Carve& ws,
                  int sms, cudaStream_t s) {
  uint8_t* abuf = ws.take(split_bytes(m, k));
  if (!abuf) return B2Q_ERR_WORKSPACE;
  SplitOperand a = split_at(abuf, m, k);
  const bool vec4 = aligned(x, 16) && ldx % 16 == 0;
  cudaError_t e = launch_quantize_q8_0_split(x, m, k, ldx / 4, const_cast<int8_t*>(a.codes),
                                             const_cast<float*>(a.scales), a.ld, variant, vec4, s);
  if (e != cudaSuccess) return B2Q_ERR_CUDA;
  return run_gemm(w, a, m, n, k, y, ldy / 4, bias, nullptr, sms, s);
}

// The Q4_K GEMM on prepared operands (plain, bias, gate, residual).
int run_q4k(const Q4kWeight& w, const Q8kAct& a, int64_t m, int64_t n, int64_t k, const float* bias,
            const float* gate, const float* resid, int64_t ldr, float* y, int64_t ldy, int sms, cudaStream_t s) {
  Q4kArgs g;
  g.w_raw = w.raw;
  g.ldw_bytes = w.row_bytes;
  g.a_codes = a.codes;
  g.a_d = a.d;
  g.lda = a.ld;
  g.M = m;
  g.N = n;
  g.K = k;
  g.y = y;
  g.ldy = ldy;
  g.bias = bias;
  g.gate = gate;
  g.resid = resid;
  g.ldr = ldr;
  return from_cuda(launch_gemm_q4k(g, sms, s));
}

// Q8_K activation quantize + the Q4_K GEMM.
int mul_mat_q4k(const Q4kWeight& w, int64_t n, int64_t k, const float* x, int64_t m, int64_t ldx,
                const float* bias, float* y, int64_t ldy, Carve& ws, int sms, cudaStream_t s) {
  uint8_t* abuf = ws.take(q8k_bytes(m, k));
  if (!abuf) return B2Q_ERR_WORKSPACE;
  const Q8kAct a = q8k_at(abuf, m, k);
  const bool vec4 = aligned(x, 16) && ldx % 16 == 0;
  if (launch_quantize_q8_k(x, m, k, ldx / 4, a.codes, a.d, a.ld, vec4, s) != cudaSuccess) return B2Q_ERR_CUDA;
  return run_q4k(w, a, m, n, k, bias, nullptr, nullptr, 0, y, ldy / 4, sms, s);
}

int check_x_y(const float* x, int64_t m, int64_t k, int64_t ldx, float* y, int64_t n,
              int64_t ldy, int variant) {
  if (m < 0 || m > INT_MAX) return m < 0 ? B2Q_ERR_INVALID_ARG : B2Q_ERR_TOO_LARGE;
  if (variant != B2Q_ACT_X86 && variant != B2Q_ACT_REF && variant != B2Q_ACT_Q8_K) return B2Q_ERR_INVALID_ARG;
  if (variant == B2Q_ACT_Q8_K && k % kQKK != 0) return B2Q_ERR_INVALID_ARG;
  if (m > 0 && (!x || !y)) return B2Q_ERR_INVALID_ARG;
  if (ldx < k * 4 || ldy < n * 4) return B2Q_ERR_INVALID_ARG;
  if (!aligned(x, 4) || ldx % 4 != 0 || !aligned(y, 4) || ldy % 4 != 0) return B2Q_ERR_MISALIGNED;
  return B2Q_OK;
}

int check_norm(const float* x, int64_t m, int64_t c, int64_t x_rs, float eps, const float* ms, const float* sh) {
  if (m < 0 || c <= 0 || c % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (c > kNormMaxC || m > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (!(eps >= 0.0f)) return B2Q_ERR_INVALID_ARG;
  if (m > 0 && !x) return B2Q_ERR_INVALID_ARG;
  if (x_rs < c * 4) return B2Q_ERR_INVALID_ARG;
  if (!aligned(x, 16) || x_rs % 16 != 0 || (ms && !aligned(ms, 16)) || (sh && !aligned(sh, 16)))
    return B2Q_ERR_MISALIGNED;
  return B2Q_OK;
}

}  // namespace

namespace b2q {

int current_device_sms(int* device) {
  constexpr int kMaxDevices = 64;
  static std::atomic<int> cache[kMaxDevices];  // 0: not queried; -2: not sm_100; else SM count
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (device) *device = dev;
  int v = dev < kMaxDevices ? cache[dev].load(std::memory_order_relaxed) : 0;
  if (v == 0) {
    int major = 0, minor = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return -1;
    v = (major == 10 && minor == 0 && sms > 0) ? sms : -2;
    if (dev < kMaxDevices) cache[dev].store(v, std::memory_order_relaxed);
  }
  return v == -2 ? 0 : v;
}

}  // namespace b2q

extern "C" {

const char* b2q_status_string(int status) {
  switch (status) {
    case B2Q_OK: return "ok";
    case B2Q_ERR_INVALID_ARG: return "invalid argument";
    case B2Q_ERR_UNSUPPORTED: return "unsupported type or device (needs sm_100)";
    case B2Q_ERR_MISALIGNED: return "misaligned pointer or stride";
    case B2Q_ERR_WORKSPACE: return "workspace or packed buffer too small";
    case B2Q_ERR_CUDA: return "CUDA runtime error";
    case B2Q_ERR_DEVICE: return "device-side error (bounded wait gave up)";
    case B2Q_ERR_TOO_LARGE: return "size beyond the supported maximum";
    default: return "unknown status";
  }
}

const char* b2q_version(void) { return "b2q 0.1.0 sm_100a"; }

int b2q_quantize_q8_0(const float* x, int64_t nrows, int64_t k, int64_t x_row_stride_bytes,
                      void* y, int64_t y_row_stride_bytes, int variant, void* stream) {
  if (nrows < 0 || k <= 0 || k % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (variant != B2Q_ACT_X86 && variant != B2Q_ACT_REF) return B2Q_ERR_INVALID_ARG;
  if (nrows > 0 && (!x || !y)) return B2Q_ERR_INVALID_ARG;
  if (x_row_stride_bytes < k * 4 || y_row_stride_bytes < (k / kQK) * kQ8Bytes) return B2Q_ERR_INVALID_ARG;
  if (!aligned(x, 4) || x_row_stride_bytes % 4 != 0 || !aligned(y, 2) || y_row_stride_bytes % 2 != 0)
    return B2Q_ERR_MISALIGNED;
  if (int rc = check_device(nullptr)) return rc;
  const bool vec4 = aligned(x, 16) && x_row_stride_bytes % 16 == 0;
  return from_cuda(launch_quantize_q8_0_blocks(x, nrows, k, x_row_stride_bytes / 4,
                                               static_cast<uint8_t*>(y), y_row_stride_bytes,
                                               variant, vec4, static_cast<cudaStream_t>(stream)));
}

size_t b2q_weight_packed_bytes(int wtype, int64_t n, int64_t k) {
  if (!valid_wtype(wtype) || n < 0 || k <= 0 || k % (wtype == B2Q_TYPE_Q4_K ? kQKK : kQK) != 0) return 0;
  return wtype == B2Q_TYPE_Q4_K ? q4k_bytes(n, k) : split_bytes(n, k);
}

size_t b2q_act_prepared_bytes(int variant, int64_t m, int64_t k) {
  if (m < 0 || k <= 0 || k % kQK != 0) return 0;
  if (variant == B2Q_ACT_Q8_K) return k % kQKK == 0 ? q8k_bytes(m, k) : 0;
  return variant == B2Q_ACT_X86 || variant == B2Q_ACT_REF ? split_bytes(m, k) : 0;
}

// fp16 copy of the activations for F16 weights.
size_t f16_act_bytes(int64_t m, int64_t k) { return round_up(m * k * 2, 256); }

// ggml_mul_mat with F16 weights: x -> fp16 (round to nearest even) in the
// workspace, then the kind::f16 GEMM on the weight rows in place.
int mul_mat_f16(const void* w, int64_t ldw, int64_t n, int64_t k, const float* x, int64_t m, int64_t ldx,
                const float* bias, float* y, int64_t ldy, int variant, void* workspace, size_t workspace_bytes,
                void* stream) {
  if (n < 0 || k <= 0 || k % 8 != 0) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX || k > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (n > 0 && !w) return B2Q_ERR_INVALID_ARG;
  if (ldw < 2 * k) return B2Q_ERR_INVALID_ARG;
  if (variant != B2Q_ACT_X86 && variant != B2Q_ACT_REF) return B2Q_ERR_INVALID_ARG;
  if (int rc = check_x_y(x, m, k, ldx, y, n, ldy, variant)) return rc;
  if (!aligned(w, 16) || ldw % 16 != 0 || !aligned(workspace, 256) || (bias && !aligned(bias, 4)))
    return B2Q_ERR_MISALIGNED;
  if (m == 0 || n == 0) return B2Q_OK;
  if (!workspace || workspace_bytes < f16_act_bytes(m, k)) return B2Q_ERR_WORKSPACE;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec4 = aligned(x, 16) && ldx % 16 == 0;
  if (launch_to_f16(x, m, k, ldx / 4, workspace, k, vec4, s) != cudaSuccess) return B2Q_ERR_CUDA;
  return from_cuda(launch_gemm_f16(w, ldw, workspace, k * 2, m, n, k, y, ldy / 4, bias, sms, s));
}

// ------------------------------------------------------------ sparse stages
size_t b2q_sparse_conv_f16_workspace_bytes(int64_t tokens, int64_t channels, int64_t out_channels) {
  if (tokens < 0 || channels <= 0 || channels % 8 != 0 || out_channels <= 0) return 0;
  return round_up(tokens * 27 * channels * 2, 256) + round_up(out_channels * 4, 256);
}

int b2q_sparse_conv_f16(const void* x16, int64_t tokens, int64_t channels, const void* w16, int64_t out_channels,
                        const void* bias16, const int32_t* indices, void* y16, void* workspace,
                        size_t workspace_bytes, void* stream) {
  if (tokens < 0 || channels <= 0 || channels % 8 != 0 || out_channels <= 0) return B2Q_ERR_INVALID_ARG;
  if (tokens > INT_MAX || 27 * channels > INT_MAX || out_channels > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (tokens > 0 && (!x16 || !w16 || !indices || !y16)) return B2Q_ERR_INVALID_ARG;
  if (!aligned(x16, 16) || !aligned(w16, 16) || !aligned(y16, 2) || !aligned(bias16, 2) || !aligned(indices, 4) ||
      !aligned(workspace, 256))
    return B2Q_ERR_MISALIGNED;
  if (tokens == 0) return B2Q_OK;
  if (!workspace || workspace_bytes < b2q_sparse_conv_f16_workspace_bytes(tokens, channels, out_channels))
    return B2Q_ERR_WORKSPACE;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* g = static_cast<uint8_t*>(workspace);
  float* bias = reinterpret_cast<float*>(g + round_up(tokens * 27 * channels * 2, 256));
  const int64_t K = 27 * channels;
  if (launch_gather27(x16, tokens, channels, indices, g, s) != cudaSuccess) return B2Q_ERR_CUDA;
  if (bias16 && launch_half_to_float(bias16, out_channels, bias, s) != cudaSuccess) return B2Q_ERR_CUDA;
  return from_cuda(launch_gemm_f16(w16, K * 2, g, K * 2, tokens, out_channels, K, nullptr, out_channels,
                                   bias16 ? bias : nullptr, sms, s, y16));
}

size_t b2q_sparse_conv_plan_bytes(int64_t tokens) {
  if (tokens < 0 || tokens > INT_MAX / 32) return 0;
  return round_up(conv_plan_ints(tokens) * 4, 256);
}

int b2q_sparse_conv_plan(const int32_t* indices, int64_t tokens, void* plan, size_t plan_bytes, void* stream) {
  if (tokens < 0) return B2Q_ERR_INVALID_ARG;
  if (tokens > INT_MAX / 32) return B2Q_ERR_TOO_LARGE;
  if (!plan || (tokens > 0 && !indices)) return B2Q_ERR_INVALID_ARG;
  if (!aligned(indices, 4) || !aligned(plan, 16)) return B2Q_ERR_MISALIGNED;
  if (plan_bytes < b2q_sparse_conv_plan_bytes(tokens)) return B2Q_ERR_WORKSPACE;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_conv_plan(indices, tokens, static_cast<int32_t*>(plan), static_cast<cudaStream_t>(stream)));
}

size_t b2q_sparse_conv_f16_planned_workspace_bytes(int64_t tokens, int64_t channels, int64_t out_channels) {
  if (tokens < 0 || tokens > INT_MAX / 32 || channels <= 0 || channels % 64 != 0 || out_channels <= 0 ||
      out_channels % 8 != 0)
    return 0;
  const int64_t P = conv_plan_rows(tokens);
  return round_up(P * channels * 2, 256) + round_up(P * out_channels * 4, 256) + round_up(out_channels * 4, 256);
}

int b2q_sparse_conv_f16_planned(const void* x16, int64_t tokens, int64_t channels, const void* w16,
                                int64_t out_channels, const void* bias16, const void* plan, void* y16,
                                void* workspace, size_t workspace_bytes, void* stream) {
  if (tokens < 0 || channels <= 0 || channels % 64 != 0 || out_channels <= 0 || out_channels % 8 != 0)
    return B2Q_ERR_INVALID_ARG;
  if (tokens > INT_MAX / 32 || 27 * channels > INT_MAX || out_channels > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (tokens > 0 && (!x16 || !w16 || !plan || !y16)) return B2Q_ERR_INVALID_ARG;
  if (!aligned(x16, 16) || !aligned(w16, 16) || !aligned(y16, 16) || !aligned(bias16, 2) || !aligned(plan, 16) ||
      !aligned(workspace, 256))
    return B2Q_ERR_MISALIGNED;
  if (tokens == 0) return B2Q_OK;
  if (!workspace || workspace_bytes < b2q_sparse_conv_f16_planned_workspace_bytes(tokens, channels, out_channels))
    return B2Q_ERR_WORKSPACE;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t P = conv_plan_rows(tokens);
  uint8_t* g = static_cast<uint8_t*>(workspace);
  float* part = reinterpret_cast<float*>(g + round_up(P * channels * 2, 256));
  float* bias = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(part) + round_up(P * out_channels * 4, 256));
  if (bias16 && launch_half_to_float(bias16, out_channels, bias, s) != cudaSuccess) return B2Q_ERR_CUDA;
  return from_cuda(launch_conv_planned(x16, tokens, channels, w16, out_channels, bias16 ? bias : nullptr,
                                       static_cast<const int32_t*>(plan), g, part, y16, sms, s));
}

size_t b2q_sparse_scatter_mean_workspace_bytes(int64_t fine_rows, int64_t coarse_rows) {
  if (fine_rows < 0 || coarse_rows < 0) return 0;
  return round_up((3 * coarse_rows + 1 + fine_rows) * 4, 256);
}

int b2q_sparse_scatter_mean_f16(const void* features16, int64_t fine_rows, int64_t channels,
                                const int32_t* row_indices, const float* counts, int64_t coarse_rows, void* out16,
                                void* workspace, size_t workspace_bytes, void* stream) {
  if (fine_rows < 0 || coarse_rows < 0 || channels <= 0 || channels % 8 != 0) return B2Q_ERR_INVALID_ARG;
  if (fine_rows > INT_MAX || coarse_rows > INT_MAX / 4 || channels > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (coarse_rows > 0 && (!counts || !out16 || (fine_rows > 0 && (!features16 || !row_indices))))
    return B2Q_ERR_INVALID_ARG;
  if (!aligned(features16, 16) || !aligned(out16, 16) || !aligned(row_indices, 4) || !aligned(counts, 4) ||
      !aligned(workspace, 4))
    return B2Q_ERR_MISALIGNED;
  if (coarse_rows == 0) return B2Q_OK;
  if (!workspace || workspace_bytes < b2q_sparse_scatter_mean_workspace_bytes(fine_rows, coarse_rows))
    return B2Q_ERR_WORKSPACE;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_scatter_mean_f16(features16, fine_rows, channels, row_indices, counts, coarse_rows, out16,
                                           static_cast<int32_t*>(workspace), static_cast<cudaStream_t>(stream)));
}

int b2q_sparse_scatter_plan(const int32_t* row_indices, int64_t fine_rows, int64_t coarse_rows, void* plan,
                            size_t plan_bytes, void* stream) {
  if (fine_rows < 0 || coarse_rows < 0) return B2Q_ERR_INVALID_ARG;
  if (fine_rows > INT_MAX || coarse_rows > INT_MAX / 4) return B2Q_ERR_TOO_LARGE;
  if (coarse_rows > 0 && (!plan || (fine_rows > 0 && !row_indices))) return B2Q_ERR_INVALID_ARG;
  if (!aligned(row_indices, 4) || !aligned(plan, 4)) return B2Q_ERR_MISALIGNED;
  if (coarse_rows == 0) return B2Q_OK;
  if (plan_bytes < b2q_sparse_scatter_mean_workspace_bytes(fine_rows, coarse_rows)) return B2Q_ERR_WORKSPACE;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_scatter_plan(row_indices, fine_rows, coarse_rows, static_cast<int32_t*>(plan),
                                       static_cast<cudaStream_t>(stream)));
}

int b2q_sparse_scatter_mean_f16_planned(const void* features16, int64_t fine_rows, int64_t channels,
                                        const void* plan, const float* counts, int64_t coarse_rows, void* out16,
                                        void* stream) {
  if (fine_rows < 0 || coarse_rows < 0 || channels <= 0 || channels % 8 != 0) return B2Q_ERR_INVALID_ARG;
  if (fine_rows > INT_MAX || coarse_rows > INT_MAX / 4 || channels > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (coarse_rows > 0 && (!counts || !out16 || !plan || (fine_rows > 0 && !features16)))
    return B2Q_ERR_INVALID_ARG;
  if (!aligned(features16, 16) || !aligned(out16, 16) || !aligned(plan, 4) || !aligned(counts, 4))
    return B2Q_ERR_MISALIGNED;
  if (coarse_rows == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_scatter_mean_planned(features16, channels, static_cast<const int32_t*>(plan), counts,
                                               coarse_rows, out16, static_cast<cudaStream_t>(stream)));
}

size_t b2q_mul_mat_workspace_bytes(int wtype, int64_t m, int64_t n, int64_t k, int packed_weight) {
  if (wtype == B2Q_TYPE_F16) return (m < 0 || n < 0 || k <= 0 || k % 8 != 0) ? 0 : f16_act_bytes(m, k);
  if (wtype != B2Q_TYPE_Q4_K) return valid_wtype(wtype) ? b2q_mul_mat_workspace_size(m, n, k, packed_weight) : 0;
  if (m < 0 || n < 0 || k <= 0 || k % kQKK != 0) return 0;
  return q8k_bytes(m, k) + (packed_weight ? 0 : q4k_bytes(n, k));
}

int b2q_mul_mat_prepared_q4_k(const void* packed, int64_t n, int64_t k, const void* act, int64_t m,
                              const float* bias, const float* gate, const float* resid,
                              int64_t resid_row_stride_bytes, float* y, int64_t y_row_stride_bytes, void* stream) {
  if (n < 0 || m < 0 || k <= 0 || k % kQKK != 0) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX / 3 || m > INT_MAX || k > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (m > 0 && n > 0 && (!packed || !act || !y)) return B2Q_ERR_INVALID_ARG;
  if (y_row_stride_bytes < n * 4 || (resid && resid_row_stride_bytes < n * 4)) return B2Q_ERR_INVALID_ARG;
  if (resid == y && resid && resid_row_stride_bytes != y_row_stride_bytes) return B2Q_ERR_INVALID_ARG;
  if (!aligned(packed, 256) || !aligned(act, 256) || !aligned(y, 4) || y_row_stride_bytes % 4 != 0 ||
      (resid && (!aligned(resid, 4) || resid_row_stride_bytes % 4 != 0)) || (bias && !aligned(bias, 4)) ||
      (gate && !aligned(gate, 4)))
    return B2Q_ERR_MISALIGNED;
  if (m == 0 || n == 0) return B2Q_OK;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  return run_q4k(q4k_at(static_cast<uint8_t*>(const_cast<void*>(packed)), n, k),
                 q8k_at(static_cast<uint8_t*>(const_cast<void*>(act)), m, k), m, n, k, bias, gate, resid,
                 resid_row_stride_bytes / 4, y, y_row_stride_bytes / 4, sms, static_cast<cudaStream_t>(stream));
}

size_t b2q_weight_packed_size(int64_t n, int64_t k) {
  if (n < 0 || k <= 0 || k % kQK != 0) return 0;
  return split_bytes(n, k);
}

int b2q_weight_pack(int wtype, const void* w, int64_t n, int64_t k, int64_t w_row_stride_bytes,
                    void* packed, size_t packed_bytes, void* stream) {
  if (int rc = check_raw_weight(wtype, w, w_row_stride_bytes, n, k)) return rc;
  if (n > 0 && !packed) return B2Q_ERR_INVALID_ARG;
  if (packed_bytes < (wtype == B2Q_TYPE_Q4_K ? q4k_bytes(n, k) : split_bytes(n, k))) return B2Q_ERR_WORKSPACE;
  if (!aligned(packed, 256)) return B2Q_ERR_MISALIGNED;
  if (int rc = check_device(nullptr)) return rc;
  if (wtype == B2Q_TYPE_Q4_K) {  // the packed form is the rows themselves, contiguous and aligned
    const int64_t rb = raw_row_bytes(wtype, k);
    return from_cuda(cudaMemcpy2DAsync(packed, rb, w, w_row_stride_bytes, rb, n, cudaMemcpyDeviceToDevice,
                                       static_cast<cudaStream_t>(stream)));
  }
  SplitOperand s = split_at(static_cast<uint8_t*>(packed), n, k);
  return from_cuda(launch_pack_weights(wtype, static_cast<const uint8_t*>(w), n, k, w_row_stride_bytes,
                                       const_cast<int8_t*>(s.codes), const_cast<float*>(s.scales),
                                       s.ld, static_cast<cudaStream_t>(stream)));
}

int b2q_weight_upload(int wtype, const void* host_w, int64_t n, int64_t k, int64_t w_row_stride_bytes,
                      void* staging, size_t staging_bytes, void* packed, size_t packed_bytes, void* stream) {
  if (int rc = check_raw_weight(wtype, host_w, w_row_stride_bytes, n, k)) return rc;
  if (n > 0 && (!packed || !staging)) return B2Q_ERR_INVALID_ARG;
  const bool kq = wtype == B2Q_TYPE_Q4_K;
  if (packed_bytes < (kq ? q4k_bytes(n, k) : split_bytes(n, k))) return B2Q_ERR_WORKSPACE;
  const int64_t row_bytes = raw_row_bytes(wtype, k);
  if (n > 0 && staging_bytes < static_cast<size_t>(row_bytes)) return B2Q_ERR_WORKSPACE;
  if (!aligned(packed, 256) || !aligned(staging, 2)) return B2Q_ERR_MISALIGNED;
  if (n == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const SplitOperand out = split_at(static_cast<uint8_t*>(packed), n, k);
  const uint8_t* src = static_cast<const uint8_t*>(host_w);
  if (kq)  // the packed form is the rows themselves: straight into place, no staging needed
    return from_cuda(cudaMemcpy2DAsync(packed, row_bytes, src, w_row_stride_bytes, row_bytes, n,
                                       cudaMemcpyHostToDevice, s));
  const int64_t chunk = static_cast<int64_t>(staging_bytes / static_cast<size_t>(row_bytes));
  for (int64_t r0 = 0; r0 < n; r0 += chunk) {
    const int64_t rows = n - r0 < chunk ? n - r0 : chunk;
    if (cudaMemcpy2DAsync(staging, row_bytes, src + r0 * w_row_stride_bytes, w_row_stride_bytes, row_bytes, rows,
                          cudaMemcpyHostToDevice, s) != cudaSuccess)
      return B2Q_ERR_CUDA;
    if (launch_pack_weights(wtype, static_cast<const uint8_t*>(staging), rows, k, row_bytes,
                            const_cast<int8_t*>(out.codes) + r0 * k, const_cast<float*>(out.scales) + r0, out.ld,
                            s) != cudaSuccess)
      return B2Q_ERR_CUDA;
  }
  return B2Q_OK;
}

size_t b2q_mul_mat_workspace_size(int64_t m, int64_t n, int64_t k, int packed_weight) {
  if (m < 0 || n < 0 || k <= 0 || k % kQK != 0) return 0;
  return split_bytes(m, k) + (packed_weight ? 0 : split_bytes(n, k));
}

int b2q_mul_mat_packed(const void* packed, int64_t n, int64_t k, const float* x, int64_t m,
                       int64_t x_row_stride_bytes, const float* bias, float* y,
                       int64_t y_row_stride_bytes, int variant, void* workspace,
                       size_t workspace_bytes, void* stream) {
  if (n < 0 || k <= 0 || k % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX || k > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (int rc = check_x_y(x, m, k, x_row_stride_bytes, y, n, y_row_stride_bytes, variant)) return rc;
  if (n > 0 && !packed) return B2Q_ERR_INVALID_ARG;
  if (!aligned(packed, 256) || !aligned(workspace, 256) || (bias && !aligned(bias, 4)))
    return B2Q_ERR_MISALIGNED;
  if (m == 0 || n == 0) return B2Q_OK;
  if (!workspace) return B2Q_ERR_WORKSPACE;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  Carve ws{static_cast<uint8_t*>(workspace), workspace_bytes};
  if (variant == B2Q_ACT_Q8_K)  // Q8_K activations <=> a Q4_K-packed weight
    return mul_mat_q4k(q4k_at(static_cast<uint8_t*>(const_cast<void*>(packed)), n, k), n, k, x, m,
                       x_row_stride_bytes, bias, y, y_row_stride_bytes, ws, sms, static_cast<cudaStream_t>(stream));
  const SplitOperand w = split_at(static_cast<uint8_t*>(const_cast<void*>(packed)), n, k);
  return mul_mat_split(w, n, k, x, m, x_row_stride_bytes, bias, y, y_row_stride_bytes, variant, ws,
                       sms, static_cast<cudaStream_t>(stream));
}

int b2q_mul_mat(int wtype, const void* w, int64_t w_row_stride_bytes, int64_t n, int64_t k,
                const float* x, int64_t m, int64_t x_row_stride_bytes, const float* bias,
                float* y, int64_t y_row_stride_bytes, int variant, void* workspace,
                size_t workspace_bytes, void* stream) {
  if (wtype == B2Q_TYPE_F16)
    return mul_mat_f16(w, w_row_stride_bytes, n, k, x, m, x_row_stride_bytes, bias, y, y_row_stride_bytes, variant,
                       workspace, workspace_bytes, stream);
  if (int rc = check_raw_weight(wtype, w, w_row_stride_bytes, n, k)) return rc;
  if (int rc = check_x_y(x, m, k, x_row_stride_bytes, y, n, y_row_stride_bytes, variant)) return rc;
  if ((wtype == B2Q_TYPE_Q4_K) != (variant == B2Q_ACT_Q8_K)) return B2Q_ERR_INVALID_ARG;
  if (!aligned(workspace, 256) || (bias && !aligned(bias, 4))) return B2Q_ERR_MISALIGNED;
  if (m == 0 || n == 0) return B2Q_OK;
  if (!workspace) return B2Q_ERR_WORKSPACE;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Carve ws{static_cast<uint8_t*>(workspace), workspace_bytes};
  if (wtype == B2Q_TYPE_Q4_K) {
    // The GEMM reads the rows with the TMA: in place when 16-byte aligned,
    // else from a contiguous copy in the workspace.
    uint8_t* qbuf = ws.take(q4k_bytes(n, k));
    if (!qbuf) return B2Q_ERR_WORKSPACE;
    Q4kWeight q = q4k_at(qbuf, n, k);
    if (aligned(w, 16) && w_row_stride_bytes % 16 == 0) {
      q.raw = static_cast<const uint8_t*>(w);
      q.row_bytes = w_row_stride_bytes;
    } else if (cudaMemcpy2DAsync(qbuf, q.row_bytes, w, w_row_stride_bytes, q.row_bytes, n, cudaMemcpyDeviceToDevice,
                                 s) != cudaSuccess) {
      return B2Q_ERR_CUDA;
    }
    return mul_mat_q4k(q, n, k, x, m, x_row_stride_bytes, bias, y, y_row_stride_bytes, ws, sms, s);
  }
  uint8_t* wbuf = ws.take(split_bytes(n, k));
  if (!wbuf) return B2Q_ERR_WORKSPACE;
  const SplitOperand wsplit = split_at(wbuf, n, k);
  if (launch_pack_weights(wtype, static_cast<const uint8_t*>(w), n, k, w_row_stride_bytes,
                          const_cast<int8_t*>(wsplit.codes), const_cast<float*>(wsplit.scales),
                          wsplit.ld, s) != cudaSuccess)
    return B2Q_ERR_CUDA;
  return mul_mat_split(wsplit, n, k, x, m, x_row_stride_bytes, bias, y, y_row_stride_bytes, variant,
                       ws, sms, s);
}

size_t b2q_act_prepared_size(int64_t m, int64_t k) {
  if (m < 0 || k <= 0 || k % kQK != 0) return 0;
  return split_bytes(m, k);
}

int b2q_act_prepare(const float* x, int64_t m, int64_t k, int64_t x_row_stride_bytes, int variant,
                    void* act, size_t act_bytes, void* stream) {
  if (k <= 0 || k % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (k > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (m < 0 || m > INT_MAX) return m < 0 ? B2Q_ERR_INVALID_ARG : B2Q_ERR_TOO_LARGE;
  if (variant != B2Q_ACT_X86 && variant != B2Q_ACT_REF && variant != B2Q_ACT_Q8_K) return B2Q_ERR_INVALID_ARG;
  if (variant == B2Q_ACT_Q8_K && k % kQKK != 0) return B2Q_ERR_INVALID_ARG;
  if (m > 0 && (!x || !act)) return B2Q_ERR_INVALID_ARG;
  if (x_row_stride_bytes < k * 4) return B2Q_ERR_INVALID_ARG;
  if (!aligned(x, 4) || x_row_stride_bytes % 4 != 0 || !aligned(act, 256)) return B2Q_ERR_MISALIGNED;
  const bool kq = variant == B2Q_ACT_Q8_K;
  if (act_bytes < (kq ? q8k_bytes(m, k) : split_bytes(m, k))) return B2Q_ERR_WORKSPACE;
  if (m == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  const bool vec4 = aligned(x, 16) && x_row_stride_bytes % 16 == 0;
  if (kq) {
    const Q8kAct q = q8k_at(static_cast<uint8_t*>(act), m, k);
    return from_cuda(launch_quantize_q8_k(x, m, k, x_row_stride_bytes / 4, q.codes, q.d, q.ld, vec4,
                                          static_cast<cudaStream_t>(stream)));
  }
  const SplitOperand a = split_at(static_cast<uint8_t*>(act), m, k);
  return from_cuda(launch_quantize_q8_0_split(x, m, k, x_row_stride_bytes / 4,
                                              const_cast<int8_t*>(a.codes),
                                              const_cast<float*>(a.scales), a.ld, variant, vec4,
                                              static_cast<cudaStream_t>(stream)));
}

int b2q_mul_mat_prepared(const void* packed, int64_t n, int64_t k, const void* act, int64_t m,
                         const float* bias, float* y, int64_t y_row_stride_bytes, void* stream) {
  if (n < 0 || m < 0 || k <= 0 || k % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX || m > INT_MAX || k > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (m > 0 && n > 0 && (!packed || !act || !y)) return B2Q_ERR_INVALID_ARG;
  if (y_row_stride_bytes < n * 4) return B2Q_ERR_INVALID_ARG;
  if (!aligned(packed, 256) || !aligned(act, 256) || !aligned(y, 4) || y_row_stride_bytes % 4 != 0 ||
      (bias && !aligned(bias, 4)))
    return B2Q_ERR_MISALIGNED;
  if (m == 0 || n == 0) return B2Q_OK;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  const SplitOperand w = split_at(static_cast<uint8_t*>(const_cast<void*>(packed)), n, k);
  const SplitOperand a = split_at(static_cast<uint8_t*>(const_cast<void*>(act)), m, k);
  return run_gemm(w, a, m, n, k, y, y_row_stride_bytes / 4, bias, nullptr, sms,
                  static_cast<cudaStream_t>(stream));
}

int b2q_mul_mat_prepared_gelu_q8(const void* packed, int64_t n, int64_t k, const void* act, int64_t m,
                                 const float* bias, void* act_out, size_t act_out_bytes, int variant,
                                 void* stream) {
  if (n < 0 || m < 0 || k <= 0 || k % kQK != 0 || n % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX || m > INT_MAX || k > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (variant != B2Q_ACT_X86 && variant != B2Q_ACT_REF) return B2Q_ERR_INVALID_ARG;
  if (m > 0 && n > 0 && (!packed || !act || !act_out)) return B2Q_ERR_INVALID_ARG;
  if (!aligned(packed, 256) || !aligned(act, 256) || !aligned(act_out, 256) || (bias && !aligned(bias, 4)))
    return B2Q_ERR_MISALIGNED;
  if (n > 0 && act_out_bytes < split_bytes(m, n)) return B2Q_ERR_WORKSPACE;
  if (m == 0 || n == 0) return B2Q_OK;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  const SplitOperand out = split_at(static_cast<uint8_t*>(act_out), m, n);
  GemmArgs g;
  g.w = split_at(static_cast<uint8_t*>(const_cast<void*>(packed)), n, k);
  g.a = split_at(static_cast<uint8_t*>(const_cast<void*>(act)), m, k);
  g.M = m;
  g.N = n;
  g.K = k;
  g.y = nullptr;
  g.ldy = 0;
  g.bias = bias;
  g.dots = nullptr;
  g.q_codes = const_cast<int8_t*>(out.codes);
  g.q_scales = const_cast<float*>(out.scales);
  g.q_ld = out.ld;
  g.q_variant = variant;
  return from_cuda(launch_gemm_tc(g, sms, static_cast<cudaStream_t>(stream)));
}

int b2q_mul_mat_prepared_gate_residual(const void* packed, int64_t n, int64_t k, const void* act, int64_t m,
                                       const float* bias, const float* gate, const float* resid,
                                       int64_t resid_row_stride_bytes, float* y, int64_t y_row_stride_bytes,
                                       void* stream) {
  if (n < 0 || m < 0 || k <= 0 || k % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX || m > INT_MAX || k > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (m > 0 && n > 0 && (!packed || !act || !y || !resid)) return B2Q_ERR_INVALID_ARG;
  if (y_row_stride_bytes < n * 4 || resid_row_stride_bytes < n * 4) return B2Q_ERR_INVALID_ARG;
  if (resid == y && resid_row_stride_bytes != y_row_stride_bytes) return B2Q_ERR_INVALID_ARG;
  if (!aligned(packed, 256) || !aligned(act, 256) || !aligned(y, 4) || y_row_stride_bytes % 4 != 0 ||
      !aligned(resid, 4) || resid_row_stride_bytes % 4 != 0 || (bias && !aligned(bias, 4)) ||
      (gate && !aligned(gate, 4)))
    return B2Q_ERR_MISALIGNED;
  if (m == 0 || n == 0) return B2Q_OK;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  GemmArgs g;
  g.w = split_at(static_cast<uint8_t*>(const_cast<void*>(packed)), n, k);
  g.a = split_at(static_cast<uint8_t*>(const_cast<void*>(act)), m, k);
  g.M = m;
  g.N = n;
  g.K = k;
  g.y = y;
  g.ldy = y_row_stride_bytes / 4;
  g.bias = bias;
  g.dots = nullptr;
  g.gate = gate;
  g.resid = resid;
  g.ldr = resid_row_stride_bytes / 4;
  return from_cuda(launch_gemm_tc(g, sms, static_cast<cudaStream_t>(stream)));
}

int b2q_mul_mat_prepared_heads_f16(const void* packed, int64_t n, int64_t k, const void* act, int64_t m,
                                   const float* bias, int64_t B, int64_t T, int64_t H, int64_t D, int parts,
                                   void* out0, void* out1, void* stream) {
  if (n < 0 || m < 0 || k <= 0 || k % kQK != 0 || B < 0 || T < 0 || H <= 0) return B2Q_ERR_INVALID_ARG;
  if (parts != 1 && parts != 2) return B2Q_ERR_INVALID_ARG;
  if (D != 64) return B2Q_ERR_UNSUPPORTED;
  if (n != parts * H * D || m != B * T) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX || m > INT_MAX || k > INT_MAX || H > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (m > 0 && (!packed || !act || !out0 || (parts == 2 && !out1))) return B2Q_ERR_INVALID_ARG;
  if (m > 0 && m <= kGemvMaxM) return B2Q_ERR_UNSUPPORTED;  // few tokens: b2q_mul_mat_prepared + b2q_rows_to_heads
  if (!aligned(packed, 256) || !aligned(act, 256) || !aligned(out0, 2) || (out1 && !aligned(out1, 2)) ||
      (bias && !aligned(bias, 4)))
    return B2Q_ERR_MISALIGNED;
  if (m == 0) return B2Q_OK;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  GemmArgs g;
  g.w = split_at(static_cast<uint8_t*>(const_cast<void*>(packed)), n, k);
  g.a = split_at(static_cast<uint8_t*>(const_cast<void*>(act)), m, k);
  g.M = m;
  g.N = n;
  g.K = k;
  g.y = nullptr;
  g.ldy = n;
  g.bias = bias;
  g.dots = nullptr;
  g.heads[0] = out0;
  g.heads[1] = parts == 2 ? out1 : nullptr;
  g.heads_T = T;
  g.heads_H = static_cast<int>(H);
  return from_cuda(launch_gemm_tc(g, sms, static_cast<cudaStream_t>(stream)));
}

int b2q_gelu(const float* x, int64_t rows, int64_t cols, int64_t x_row_stride_bytes, float* y,
             int64_t y_row_stride_bytes, void* stream) {
  if (rows < 0 || cols < 0) return B2Q_ERR_INVALID_ARG;
  if (rows > 0 && cols > 0 && (!x || !y)) return B2Q_ERR_INVALID_ARG;
  if (x_row_stride_bytes < cols * 4 || y_row_stride_bytes < cols * 4) return B2Q_ERR_INVALID_ARG;
  if (!aligned(x, 4) || !aligned(y, 4) || x_row_stride_bytes % 4 != 0 || y_row_stride_bytes % 4 != 0)
    return B2Q_ERR_MISALIGNED;
  if (rows == 0 || cols == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_gelu(x, rows, cols, x_row_stride_bytes / 4, y, y_row_stride_bytes / 4,
                               static_cast<cudaStream_t>(stream)));
}

int b2q_norm_modulate(const float* x, int64_t m, int64_t c, int64_t x_row_stride_bytes, float eps,
                      const float* mod_scale, const float* mod_shift, float* y, int64_t y_row_stride_bytes,
                      void* stream) {
  if (int rc = check_norm(x, m, c, x_row_stride_bytes, eps, mod_scale, mod_shift)) return rc;
  if (m > 0 && !y) return B2Q_ERR_INVALID_ARG;
  if (y_row_stride_bytes < c * 4) return B2Q_ERR_INVALID_ARG;
  if (!aligned(y, 16) || y_row_stride_bytes % 16 != 0) return B2Q_ERR_MISALIGNED;
  if (m == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_norm_modulate(x, m, c, x_row_stride_bytes / 4, eps, mod_scale, mod_shift, y,
                                        y_row_stride_bytes / 4, nullptr, nullptr, 0, 0,
                                        static_cast<cudaStream_t>(stream)));
}

int b2q_norm_modulate_q8(const float* x, int64_t m, int64_t c, int64_t x_row_stride_bytes, float eps,
                         const float* mod_scale, const float* mod_shift, int variant, void* act, size_t act_bytes,
                         void* stream) {
  if (int rc = check_norm(x, m, c, x_row_stride_bytes, eps, mod_scale, mod_shift)) return rc;
  if (variant != B2Q_ACT_X86 && variant != B2Q_ACT_REF) return B2Q_ERR_INVALID_ARG;
  if (m > 0 && !act) return B2Q_ERR_INVALID_ARG;
  if (!aligned(act, 256)) return B2Q_ERR_MISALIGNED;
  if (act_bytes < split_bytes(m, c)) return B2Q_ERR_WORKSPACE;
  if (m == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  const SplitOperand a = split_at(static_cast<uint8_t*>(act), m, c);
  return from_cuda(launch_norm_modulate(x, m, c, x_row_stride_bytes / 4, eps, mod_scale, mod_shift, nullptr, 0,
                                        const_cast<int8_t*>(a.codes), const_cast<float*>(a.scales), a.ld,
                                        variant, static_cast<cudaStream_t>(stream)));
}

size_t b2q_weight_packed_q4_0_bytes(int64_t n, int64_t k) {
  if (n < 0 || k <= 0 || k % kQK != 0) return 0;
  return q4c_bytes(n, k);
}

int b2q_weight_pack_q4_0(const void* w, int64_t n, int64_t k, int64_t w_row_stride_bytes, void* packed,
                         size_t packed_bytes, void* stream) {
  if (n < 0 || k <= 0 || k % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX || k > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (n > 0 && (!w || !packed)) return B2Q_ERR_INVALID_ARG;
  if (w_row_stride_bytes < (k / kQK) * kQ4Bytes) return B2Q_ERR_INVALID_ARG;
  if (!aligned(w, 2) || w_row_stride_bytes % 2 != 0 || !aligned(packed, 256)) return B2Q_ERR_MISALIGNED;
  if (packed_bytes < q4c_bytes(n, k)) return B2Q_ERR_WORKSPACE;
  if (n == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  const Q4cWeight c = q4c_at(static_cast<const uint8_t*>(packed), n, k);
  return from_cuda(launch_pack_q4c(static_cast<const uint8_t*>(w), n, k, w_row_stride_bytes,
                                   const_cast<uint8_t*>(c.nibbles), const_cast<uint16_t*>(c.scales), c.ld,
                                   static_cast<cudaStream_t>(stream)));
}

int b2q_mul_mat_prepared_q4_0(const void* packed, int64_t n, int64_t k, const void* act, int64_t m,
                              const float* bias, const float* gate, const float* resid,
                              int64_t resid_row_stride_bytes, float* y, int64_t y_row_stride_bytes, void* stream) {
  if (n < 0 || m < 0 || k <= 0 || k % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX || m > INT_MAX || k > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (m > 0 && n > 0 && (!packed || !act || !y)) return B2Q_ERR_INVALID_ARG;
  if (y_row_stride_bytes < n * 4 || (resid && resid_row_stride_bytes < n * 4)) return B2Q_ERR_INVALID_ARG;
  if (resid == y && resid && resid_row_stride_bytes != y_row_stride_bytes) return B2Q_ERR_INVALID_ARG;
  if (!aligned(packed, 256) || !aligned(act, 256) || !aligned(y, 4) || y_row_stride_bytes % 4 != 0 ||
      (resid && (!aligned(resid, 4) || resid_row_stride_bytes % 4 != 0)) || (bias && !aligned(bias, 4)) ||
      (gate && !aligned(gate, 4)))
    return B2Q_ERR_MISALIGNED;
  if (m == 0 || n == 0) return B2Q_OK;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  GemmArgs g;
  q4c_operands(packed, n, k, act, m, g);
  g.y = y;
  g.ldy = y_row_stride_bytes / 4;
  g.bias = bias;
  g.gate = gate;
  g.resid = resid;
  g.ldr = resid ? resid_row_stride_bytes / 4 : 0;
  return from_cuda(launch_gemm_tc(g, sms, static_cast<cudaStream_t>(stream)));
}

int b2q_mul_mat_prepared_q4_0_gelu_q8(const void* packed, int64_t n, int64_t k, const void* act, int64_t m,
                                      const float* bias, void* act_out, size_t act_out_bytes, int variant,
                                      void* stream) {
  if (n < 0 || m < 0 || k <= 0 || k % kQK != 0 || n % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX || m > INT_MAX || k > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (variant != B2Q_ACT_X86 && variant != B2Q_ACT_REF) return B2Q_ERR_INVALID_ARG;
  if (m > 0 && n > 0 && (!packed || !act || !act_out)) return B2Q_ERR_INVALID_ARG;
  if (!aligned(packed, 256) || !aligned(act, 256) || !aligned(act_out, 256) || (bias && !aligned(bias, 4)))
    return B2Q_ERR_MISALIGNED;
  if (n > 0 && act_out_bytes < split_bytes(m, n)) return B2Q_ERR_WORKSPACE;
  if (m == 0 || n == 0) return B2Q_OK;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  const SplitOperand out = split_at(static_cast<uint8_t*>(act_out), m, n);
  GemmArgs g;
  q4c_operands(packed, n, k, act, m, g);
  g.y = nullptr;
  g.ldy = 0;
  g.bias = bias;
  g.q_codes = const_cast<int8_t*>(out.codes);
  g.q_scales = const_cast<float*>(out.scales);
  g.q_ld = out.ld;
  g.q_variant = variant;
  return from_cuda(launch_gemm_tc(g, sms, static_cast<cudaStream_t>(stream)));
}

int b2q_qkv_heads(const float* qkv, int64_t B, int64_t T, int64_t H, int64_t D, int64_t qkv_row_stride_bytes,
                  const float* gamma_q, const float* gamma_k, float eps, void* q16, void* k16, void* v16,
                  void* stream) {
  if (B < 0 || T < 0 || H <= 0 || (D != 32 && D != 64 && D != 128) || !(eps >= 0.0f)) return B2Q_ERR_INVALID_ARG;
  if (B * T > INT_MAX || H > 4096) return B2Q_ERR_TOO_LARGE;
  if (B * T > 0 && (!qkv || !q16 || !k16 || !v16)) return B2Q_ERR_INVALID_ARG;
  if (qkv_row_stride_bytes < 3 * H * D * 4) return B2Q_ERR_INVALID_ARG;
  if (!aligned(qkv, 4) || qkv_row_stride_bytes % 4 != 0 || !aligned(q16, 2) || !aligned(k16, 2) ||
      !aligned(v16, 2) || (gamma_q && !aligned(gamma_q, 4)) || (gamma_k && !aligned(gamma_k, 4)))
    return B2Q_ERR_MISALIGNED;
  if (B * T == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_rows_to_heads(qkv, B, T, static_cast<int>(H), static_cast<int>(D), qkv_row_stride_bytes / 4,
                                        3, 3u, gamma_q, gamma_k, eps, q16, k16, v16, static_cast<cudaStream_t>(stream)));
}

int b2q_rows_to_heads(const float* src, int64_t B, int64_t T, int64_t H, int64_t D, int parts,
                      int64_t src_row_stride_bytes, void* out0, void* out1, void* stream) {
  if (B < 0 || T < 0 || H <= 0 || (D != 32 && D != 64 && D != 128) || parts < 1 || parts > 2)
    return B2Q_ERR_INVALID_ARG;
  if (B * T > INT_MAX || H > 4096) return B2Q_ERR_TOO_LARGE;
  if (B * T > 0 && (!src || !out0 || (parts == 2 && !out1))) return B2Q_ERR_INVALID_ARG;
  if (src_row_stride_bytes < parts * H * D * 4) return B2Q_ERR_INVALID_ARG;
  if (!aligned(src, 4) || src_row_stride_bytes % 4 != 0 || !aligned(out0, 2) || (out1 && !aligned(out1, 2)))
    return B2Q_ERR_MISALIGNED;
  if (B * T == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_rows_to_heads(src, B, T, static_cast<int>(H), static_cast<int>(D), src_row_stride_bytes / 4,
                                        parts, 0u, nullptr, nullptr, 0.0f, out0, out1, nullptr,
                                        static_cast<cudaStream_t>(stream)));
}

int b2q_qkv_heads_f32(const float* qkv, int64_t B, int64_t T, int64_t H, int64_t D, int64_t qkv_row_stride_bytes,
                      const float* gamma_q, const float* gamma_k, float eps, float* q, float* k, float* v,
                      void* stream) {
  if (B < 0 || T < 0 || H <= 0 || (D != 32 && D != 64 && D != 128) || !(eps >= 0.0f)) return B2Q_ERR_INVALID_ARG;
  if (B * T > INT_MAX || H > 4096) return B2Q_ERR_TOO_LARGE;
  if (B * T > 0 && (!qkv || !q || !k || !v)) return B2Q_ERR_INVALID_ARG;
  if (qkv_row_stride_bytes < 3 * H * D * 4) return B2Q_ERR_INVALID_ARG;
  if (!aligned(qkv, 4) || qkv_row_stride_bytes % 4 != 0 || !aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) ||
      (gamma_q && !aligned(gamma_q, 4)) || (gamma_k && !aligned(gamma_k, 4)))
    return B2Q_ERR_MISALIGNED;
  if (B * T == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_rows_to_heads(qkv, B, T, static_cast<int>(H), static_cast<int>(D), qkv_row_stride_bytes / 4,
                                        3, 3u, gamma_q, gamma_k, eps, q, k, v, static_cast<cudaStream_t>(stream), true));
}

int b2q_rows_to_heads_f32(const float* src, int64_t B, int64_t T, int64_t H, int64_t D, int parts,
                          int64_t src_row_stride_bytes, float* out0, float* out1, void* stream) {
  if (B < 0 || T < 0 || H <= 0 || (D != 32 && D != 64 && D != 128) || parts < 1 || parts > 2)
    return B2Q_ERR_INVALID_ARG;
  if (B * T > INT_MAX || H > 4096) return B2Q_ERR_TOO_LARGE;
  if (B * T > 0 && (!src || !out0 || (parts == 2 && !out1))) return B2Q_ERR_INVALID_ARG;
  if (src_row_stride_bytes < parts * H * D * 4) return B2Q_ERR_INVALID_ARG;
  if (!aligned(src, 4) || src_row_stride_bytes % 4 != 0 || !aligned(out0, 16) || (out1 && !aligned(out1, 16)))
    return B2Q_ERR_MISALIGNED;
  if (B * T == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_rows_to_heads(src, B, T, static_cast<int>(H), static_cast<int>(D), src_row_stride_bytes / 4,
                                        parts, 0u, nullptr, nullptr, 0.0f, out0, out1, nullptr,
                                        static_cast<cudaStream_t>(stream), true));
}

int b2q_attention_f32(const float* q, const float* k, const float* v, int64_t B, int64_t H, int64_t Tq, int64_t Tk,
                      int64_t D, const float* k2, const float* v2, int64_t Tk2, float scale, float* o,
                      int64_t o_row_stride_bytes, void* stream) {
  if (B < 0 || Tq < 0 || Tk < 0 || H <= 0 || (D != 32 && D != 64 && D != 128) || !std::isfinite(scale))
    return B2Q_ERR_INVALID_ARG;
  if ((k2 == nullptr) != (v2 == nullptr) || (k2 && Tk2 < 0)) return B2Q_ERR_INVALID_ARG;
  const int64_t tk_all = Tk + (k2 ? Tk2 : 0);
  if (B * Tq > 0 && (!q || !o || tk_all <= 0 || (Tk > 0 && (!k || !v)))) return B2Q_ERR_INVALID_ARG;
  if (o_row_stride_bytes < H * D * 4 || o_row_stride_bytes % 4 != 0) return B2Q_ERR_INVALID_ARG;
  if (B > 65535 || H > 65535 || (Tq + 63) / 64 > INT_MAX || B * H * (tk_all > Tq ? tk_all : Tq) * D > (int64_t{1} << 40))
    return B2Q_ERR_TOO_LARGE;
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(k2, 16) || !aligned(v2, 16) || !aligned(o, 4))
    return B2Q_ERR_MISALIGNED;
  if (B * Tq == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_attention_f32(q, k, v, k2, v2, B, static_cast<int>(H), Tq, Tk, k2 ? Tk2 : 0,
                                        static_cast<int>(D), scale, o, o_row_stride_bytes / 4,
                                        static_cast<cudaStream_t>(stream)));
}

int b2q_attention_f16(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t Tq, int64_t Tk,
                      int64_t D, const void* k2, const void* v2, int64_t Tk2, float scale, void* o,
                      int64_t o_row_stride_bytes, void* stream) {
  if (B < 0 || Tq < 0 || Tk < 0 || H <= 0 || !std::isfinite(scale)) return B2Q_ERR_INVALID_ARG;
  if (D != 64) return B2Q_ERR_UNSUPPORTED;
  if ((k2 == nullptr) != (v2 == nullptr) || (k2 && Tk2 < 0)) return B2Q_ERR_INVALID_ARG;
  const int64_t tk_all = Tk + (k2 ? Tk2 : 0);
  if (B * Tq > 0 && (!q || !o || tk_all <= 0 || (Tk > 0 && (!k || !v)))) return B2Q_ERR_INVALID_ARG;
  if (o_row_stride_bytes < H * D * 2) return B2Q_ERR_INVALID_ARG;
  const int64_t rows = B * H * (Tq > tk_all ? Tq : tk_all);
  if (B > 65535 || H > 65535 || rows + 128 > INT_MAX || (Tq + 127) / 128 > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(k2, 16) || !aligned(v2, 16) || !aligned(o, 16) ||
      o_row_stride_bytes % 16 != 0)
    return B2Q_ERR_MISALIGNED;
  if (B * Tq == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_attention_f16(q, k, v, k2, v2, B, static_cast<int>(H), Tq, Tk, k2 ? Tk2 : 0, scale, o,
                                        o_row_stride_bytes / 2, static_cast<cudaStream_t>(stream)));
}

int b2q_attention_f16_q8(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t Tq, int64_t Tk,
                         int64_t D, const void* k2, const void* v2, int64_t Tk2, float scale, int variant, void* act,
                         size_t act_bytes, void* stream) {
  if (B < 0 || Tq < 0 || Tk < 0 || H <= 0 || !std::isfinite(scale)) return B2Q_ERR_INVALID_ARG;
  if (D != 64) return B2Q_ERR_UNSUPPORTED;
  if (variant != B2Q_ACT_X86 && variant != B2Q_ACT_REF) return B2Q_ERR_INVALID_ARG;
  if ((k2 == nullptr) != (v2 == nullptr) || (k2 && Tk2 < 0)) return B2Q_ERR_INVALID_ARG;
  const int64_t tk_all = Tk + (k2 ? Tk2 : 0);
  if (B * Tq > 0 && (!q || !act || tk_all <= 0 || (Tk > 0 && (!k || !v)))) return B2Q_ERR_INVALID_ARG;
  const int64_t rows = B * H * (Tq > tk_all ? Tq : tk_all);
  if (B > 65535 || H > 65535 || rows + 128 > INT_MAX || (Tq + 127) / 128 > INT_MAX || B * Tq > INT_MAX ||
      H * D > INT_MAX)
    return B2Q_ERR_TOO_LARGE;
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(k2, 16) || !aligned(v2, 16) ||
      !aligned(act, 256))
    return B2Q_ERR_MISALIGNED;
  if (act_bytes < split_bytes(B * Tq, H * D)) return B2Q_ERR_WORKSPACE;
  if (B * Tq == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  const SplitOperand a = split_at(static_cast<uint8_t*>(act), B * Tq, H * D);
  return from_cuda(launch_attention_f16_q8(q, k, v, k2, v2, B, static_cast<int>(H), Tq, Tk, k2 ? Tk2 : 0, scale,
                                           const_cast<int8_t*>(a.codes), const_cast<float*>(a.scales), a.ld, variant,
                                           static_cast<cudaStream_t>(stream)));
}

int b2q_layer_norm_q8(const float* x, int64_t m, int64_t c, int64_t x_row_stride_bytes, float eps, const float* weight,
                      const float* bias, int variant, void* act, size_t act_bytes, void* stream) {
  if (int rc = check_norm(x, m, c, x_row_stride_bytes, eps, weight, bias)) return rc;
  if (variant != B2Q_ACT_X86 && variant != B2Q_ACT_REF) return B2Q_ERR_INVALID_ARG;
  if (m > 0 && !act) return B2Q_ERR_INVALID_ARG;
  if (!aligned(act, 256)) return B2Q_ERR_MISALIGNED;
  if (act_bytes < split_bytes(m, c)) return B2Q_ERR_WORKSPACE;
  if (m == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  const SplitOperand a = split_at(static_cast<uint8_t*>(act), m, c);
  return from_cuda(launch_norm_modulate(x, m, c, x_row_stride_bytes / 4, eps, weight, bias, nullptr, 0,
                                        const_cast<int8_t*>(a.codes), const_cast<float*>(a.scales), a.ld, variant,
                                        static_cast<cudaStream_t>(stream), true));
}

int b2q_heads_act_prepare(const void* o16, int64_t B, int64_t T, int64_t H, int64_t D, int64_t stride_b,
                          int64_t stride_h, int64_t stride_t, int variant, void* act, size_t act_bytes,
                          void* stream) {
  if (B < 0 || T < 0 || H <= 0 || D <= 0 || D % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (variant != B2Q_ACT_X86 && variant != B2Q_ACT_REF) return B2Q_ERR_INVALID_ARG;
  if (B * T > INT_MAX || H * D > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (B * T > 0 && (!o16 || !act)) return B2Q_ERR_INVALID_ARG;
  if (stride_b < 0 || stride_h < 0 || stride_t < 0) return B2Q_ERR_INVALID_ARG;
  if (!aligned(o16, 2) || !aligned(act, 256)) return B2Q_ERR_MISALIGNED;
  if (act_bytes < split_bytes(B * T, H * D)) return B2Q_ERR_WORKSPACE;
  if (B * T == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  const SplitOperand a = split_at(static_cast<uint8_t*>(act), B * T, H * D);
  return from_cuda(launch_heads_q8(o16, B, T, static_cast<int>(H), static_cast<int>(D), stride_b, stride_h, stride_t,
                                   const_cast<int8_t*>(a.codes), const_cast<float*>(a.scales), a.ld, variant,
                                   static_cast<cudaStream_t>(stream)));
}

int b2q_mul_mat_prepared_peers(const void* packed, int64_t n, int64_t k, const void* act, int64_t m,
                               const float* bias, float* const* y_peers, int n_peers, int64_t y_col0,
                               int64_t y_row_stride_bytes, void* stream) {
  if (n < 0 || m < 0 || k <= 0 || k % kQK != 0 || y_col0 < 0) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX || m > INT_MAX || k > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (n_peers < 1 || n_peers > kMaxPeers || !y_peers) return B2Q_ERR_INVALID_ARG;
  if (m > 0 && n > 0 && (!packed || !act)) return B2Q_ERR_INVALID_ARG;
  if (y_row_stride_bytes < (y_col0 + n) * 4) return B2Q_ERR_INVALID_ARG;
  if (!aligned(packed, 256) || !aligned(act, 256) || y_row_stride_bytes % 4 != 0 ||
      (bias && !aligned(bias, 4)))
    return B2Q_ERR_MISALIGNED;
  for (int q = 0; q < n_peers; ++q) {
    if (!y_peers[q]) return B2Q_ERR_INVALID_ARG;
    if (!aligned(y_peers[q], 4)) return B2Q_ERR_MISALIGNED;
  }
  if (m == 0 || n == 0) return B2Q_OK;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  GemmArgs g;
  g.w = split_at(static_cast<uint8_t*>(const_cast<void*>(packed)), n, k);
  g.a = split_at(static_cast<uint8_t*>(const_cast<void*>(act)), m, k);
  g.M = m;
  g.N = n;
  g.K = k;
  g.y = y_peers[0];
  g.ldy = y_row_stride_bytes / 4;
  g.bias = bias;
  g.dots = nullptr;
  g.n_peers = n_peers;
  g.y_col0 = y_col0;
  for (int q = 0; q < n_peers; ++q) g.y_peer[q] = y_peers[q];
  return from_cuda(launch_gemm_tc(g, sms, static_cast<cudaStream_t>(stream)));
}

int b2q_mul_mat_prepared_gelu_q8_peers(const void* packed, int64_t n, int64_t k, const void* act, int64_t m,
                                       const float* bias, void* const* act_peers, int n_peers, int64_t n_total,
                                       int64_t col0, size_t act_bytes, int variant, void* stream) {
  if (n < 0 || m < 0 || k <= 0 || k % kQK != 0 || n % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (col0 < 0 || col0 % kQK != 0 || n_total % kQK != 0 || col0 + n > n_total) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX || m > INT_MAX || k > INT_MAX || n_total > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (variant != B2Q_ACT_X86 && variant != B2Q_ACT_REF) return B2Q_ERR_INVALID_ARG;
  if (n_peers < 1 || n_peers > kMaxPeers || !act_peers) return B2Q_ERR_INVALID_ARG;
  if (m > 0 && n > 0 && (!packed || !act)) return B2Q_ERR_INVALID_ARG;
  if (!aligned(packed, 256) || !aligned(act, 256) || (bias && !aligned(bias, 4))) return B2Q_ERR_MISALIGNED;
  for (int q = 0; q < n_peers; ++q) {
    if (!act_peers[q]) return B2Q_ERR_INVALID_ARG;
    if (!aligned(act_peers[q], 256)) return B2Q_ERR_MISALIGNED;
  }
  if (n > 0 && act_bytes < split_bytes(m, n_total)) return B2Q_ERR_WORKSPACE;
  if (m == 0 || n == 0) return B2Q_OK;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  // Every rank's buffer has the same split layout [m][n_total]: one pair of
  // offsets from the buffer base serves them all.
  uint8_t* base0 = static_cast<uint8_t*>(act_peers[0]);
  const SplitOperand out = split_at(base0, m, n_total);
  GemmArgs g;
  g.w = split_at(static_cast<uint8_t*>(const_cast<void*>(packed)), n, k);
  g.a = split_at(static_cast<uint8_t*>(const_cast<void*>(act)), m, k);
  g.M = m;
  g.N = n;
  g.K = k;
  g.y = nullptr;
  g.ldy = 0;
  g.bias = bias;
  g.dots = nullptr;
  g.n_peers = n_peers;
  for (int q = 0; q < n_peers; ++q) g.y_peer[q] = static_cast<float*>(act_peers[q]);
  g.q_peers = true;
  g.q_k = n_total;
  g.q_ld = out.ld;
  g.q_code_off = reinterpret_cast<const uint8_t*>(out.codes) - base0 + col0;
  g.q_scale_off = reinterpret_cast<const uint8_t*>(out.scales + (col0 / kQK) * out.ld) - base0;
  g.q_variant = variant;
  return from_cuda(launch_gemm_tc(g, sms, static_cast<cudaStream_t>(stream)));
}

int b2q_dequantize(int wtype, const void* w, int64_t w_row_stride_bytes, int64_t n, int64_t k, int out_type,
                   void* out, int64_t out_row_stride_bytes, void* stream) {
  if (wtype != B2Q_TYPE_Q8_0 && wtype != B2Q_TYPE_Q4_0 && wtype != B2Q_TYPE_Q4_K) return B2Q_ERR_UNSUPPORTED;
  if (out_type != B2Q_TYPE_F32 && out_type != B2Q_TYPE_F16) return B2Q_ERR_UNSUPPORTED;
  const int64_t unit = wtype == B2Q_TYPE_Q4_K ? kQKK : kQK;
  const int64_t esz = out_type == B2Q_TYPE_F32 ? 4 : 2;
  if (n < 0 || k <= 0 || k % unit != 0) return B2Q_ERR_INVALID_ARG;
  if (w_row_stride_bytes < raw_row_bytes(wtype, k) || out_row_stride_bytes < k * esz) return B2Q_ERR_INVALID_ARG;
  if (n > 0 && (!w || !out)) return B2Q_ERR_INVALID_ARG;
  if (!aligned(w, 2) || w_row_stride_bytes % 2 != 0 || !aligned(out, 16) || out_row_stride_bytes % 16 != 0)
    return B2Q_ERR_MISALIGNED;
  if (n == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_dequantize(wtype, w, w_row_stride_bytes, n, k, out_type == B2Q_TYPE_F16, out,
                                     out_row_stride_bytes / esz, static_cast<cudaStream_t>(stream)));
}

int b2q_mul_mat_f32(const float* w, int64_t w_row_stride_bytes, int64_t n, int64_t k, const float* x,
                    int64_t x_row_stride_bytes, int64_t m, const float* bias, float* y, int64_t y_row_stride_bytes,
                    void* stream) {
  if (n < 0 || m < 0 || k <= 0 || k % 4 != 0) return B2Q_ERR_INVALID_ARG;
  if (w_row_stride_bytes < k * 4 || x_row_stride_bytes < k * 4 || y_row_stride_bytes < n * 4)
    return B2Q_ERR_INVALID_ARG;
  if (m > 0 && n > 0 && (!w || !x || !y)) return B2Q_ERR_INVALID_ARG;
  if (!aligned(w, 16) || !aligned(x, 16) || w_row_stride_bytes % 16 != 0 || x_row_stride_bytes % 16 != 0 ||
      !aligned(y, 4) || y_row_stride_bytes % 4 != 0 || (bias && !aligned(bias, 4)))
    return B2Q_ERR_MISALIGNED;
  if (m == 0 || n == 0) return B2Q_OK;
  if ((m + 127) / 128 > 65535) return B2Q_ERR_TOO_LARGE;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_sgemm(x, x_row_stride_bytes / 4, m, w, w_row_stride_bytes / 4, n, k, bias, y,
                                y_row_stride_bytes / 4, static_cast<cudaStream_t>(stream)));
}

size_t b2q_block_dots_workspace_size(int64_t m, int64_t n, int64_t k) {
  if (m < 0 || n < 0 || k <= 0 || k % kQK != 0) return 0;
  return split_bytes(m, k) + split_bytes(n, k);
}

int b2q_block_dots(int wtype, const void* w, int64_t w_row_stride_bytes, int64_t n, int64_t k,
                   const void* a, int64_t m, int64_t a_row_stride_bytes, int32_t* dots,
                   void* workspace, size_t workspace_bytes, void* stream) {
  if (wtype == B2Q_TYPE_Q4_K) return B2Q_ERR_UNSUPPORTED;  // check path for the 32-value block types
  if (int rc = check_raw_weight(wtype, w, w_row_stride_bytes, n, k)) return rc;
  if (int rc = check_raw_weight(B2Q_TYPE_Q8_0, a, a_row_stride_bytes, m, k)) return rc;
  if (m > 0 && n > 0 && !dots) return B2Q_ERR_INVALID_ARG;
  if (m * n * (k / kQK) > (int64_t(1) << 28)) return B2Q_ERR_TOO_LARGE;
  if (!aligned(workspace, 256) || !aligned(dots, 4)) return B2Q_ERR_MISALIGNED;
  if (m == 0 || n == 0) return B2Q_OK;
  if (!workspace) return B2Q_ERR_WORKSPACE;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Carve ws{static_cast<uint8_t*>(workspace), workspace_bytes};
  uint8_t* wbuf = ws.take(split_bytes(n, k));
  uint8_t* abuf = ws.take(split_bytes(m, k));
  if (!wbuf || !abuf) return B2Q_ERR_WORKSPACE;
  const SplitOperand ws_ = split_at(wbuf, n, k), as_ = split_at(abuf, m, k);
  if (launch_pack_weights(wtype, static_cast<const uint8_t*>(w), n, k, w_row_stride_bytes,
                          const_cast<int8_t*>(ws_.codes), const_cast<float*>(ws_.scales), ws_.ld,
                          s) != cudaSuccess ||
      launch_pack_weights(B2Q_TYPE_Q8_0, static_cast<const uint8_t*>(a), m, k, a_row_stride_bytes,
                          const_cast<int8_t*>(as_.codes), const_cast<float*>(as_.scales), as_.ld,
                          s) != cudaSuccess)
    return B2Q_ERR_CUDA;
  return run_gemm(ws_, as_, m, n, k, nullptr, 0, nullptr, dots, sms, s);
}

int b2q_mul_mat_q_simt(int wtype, const void* w, int64_t w_row_stride_bytes, int64_t n,
                       int64_t k, const void* a, int64_t m, int64_t a_row_stride_bytes,
                       float* y, int64_t y_row_stride_bytes, void* stream) {
  if (wtype == B2Q_TYPE_Q4_K) return B2Q_ERR_UNSUPPORTED;  // check path for the 32-value block types
  if (int rc = check_raw_weight(wtype, w, w_row_stride_bytes, n, k)) return rc;
  if (int rc = check_raw_weight(B2Q_TYPE_Q8_0, a, a_row_stride_bytes, m, k)) return rc;
  if (m > 0 && n > 0 && !y) return B2Q_ERR_INVALID_ARG;
  if (y_row_stride_bytes < n * 4) return B2Q_ERR_INVALID_ARG;
  if (!aligned(y, 4) || y_row_stride_bytes % 4 != 0) return B2Q_ERR_MISALIGNED;
  if ((m + 7) / 8 > 65535) return B2Q_ERR_TOO_LARGE;
  if (m == 0 || n == 0) return B2Q_OK;
  if (int rc = check_device(nullptr)) return rc;
  return from_cuda(launch_gemm_simt(wtype, static_cast<const uint8_t*>(w), w_row_stride_bytes, n, k,
                                    static_cast<const uint8_t*>(a), a_row_stride_bytes, m, y,
                                    y_row_stride_bytes / 4, static_cast<cudaStream_t>(stream)));
}

int b2q_selftest_stalled_mul_mat(const void* packed, int64_t n, int64_t k, const void* act, int64_t m,
                                 float* y, int64_t y_row_stride_bytes, void* stream) {
  if (n <= 0 || m <= 0 || k <= 0 || k % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX || m > INT_MAX || k > INT_MAX) return B2Q_ERR_TOO_LARGE;
  if (!packed || !act || !y || y_row_stride_bytes < n * 4) return B2Q_ERR_INVALID_ARG;
  if (!aligned(packed, 256) || !aligned(act, 256) || !aligned(y, 4) || y_row_stride_bytes % 4 != 0)
    return B2Q_ERR_MISALIGNED;
  int sms = 0;
  if (int rc = check_device(&sms)) return rc;
  GemmArgs g;
  g.w = split_at(static_cast<uint8_t*>(const_cast<void*>(packed)), n, k);
  g.a = split_at(static_cast<uint8_t*>(const_cast<void*>(act)), m, k);
  g.M = m;
  g.N = n;
  g.K = k;
  g.y = y;
  g.ldy = y_row_stride_bytes / 4;
  g.bias = nullptr;
  g.dots = nullptr;
  g.inject_stall = 1;
  return from_cuda(launch_gemm_tc(g, sms, static_cast<cudaStream_t>(stream)));
}

int b2q_device_status(unsigned int* code, int clear) {
  if (!code) return B2Q_ERR_INVALID_ARG;
  if (int rc = check_device(nullptr)) return rc;
  if (cudaDeviceSynchronize() != cudaSuccess) return B2Q_ERR_CUDA;
  if (read_device_status(code, clear != 0) != cudaSuccess) return B2Q_ERR_CUDA;
  unsigned int attn = 0;
  if (read_attention_status(&attn, clear != 0) != cudaSuccess) return B2Q_ERR_CUDA;
  if (!*code) *code = attn;
  return *code ? B2Q_ERR_DEVICE : B2Q_OK;
}

}  // extern "C"
