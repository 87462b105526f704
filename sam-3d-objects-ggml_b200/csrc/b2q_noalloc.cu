// b2q_noalloc.cu -- b2q_mul_mat_packed_noalloc: the packed-weight mul_mat for
// callers that may not allocate device memory and have no workspace to lend.
// The prepared activations (the one scratch buffer b2q_mul_mat_packed carves
// from its caller's workspace) live instead in one file-scope device array of
// B2Q_NOALLOC_SCRATCH_BYTES, and the call then runs exactly the kernels of
// b2q_mul_mat_packed on it.
//
// Set-up: the first call on each device, with that device current, looks up
// the array's device address with cudaGetSymbolAddress (which also makes the
// CUDA runtime load this module, so the array is reserved on that device no
// later than that call) and caches it together with the CUDA context it
// belongs to.  Later calls on that device compare the current context with the
// cached one (one driver query) and reuse the address; if the context has
// changed -- after cudaDeviceReset, or a release and re-creation of the primary
// context, which reloads the module at a new address -- they redo the set-up.
// Make the first call on a device before any stream capture begins.
//
// Sharing: every call on a device uses the same array, which keeps the last
// call's contents.  Calls that can overlap on one device (several streams,
// several host threads without ordering) race on it; serialise them.
//
// Nothing in the array needs clearing: the quantize kernel writes every code
// and scale of the m rows before the GEMM reads them, and the GEMM's tensor
// copies stop at row m (rows past it read as zero fill, never from the array).
#include "../../include/b2q.h"
#include "b2q_internal.h"

#include <climits>
#include <cstdint>
#include <mutex>

namespace {

using namespace b2q;

constexpr size_t kScratchBytes = B2Q_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

__device__ __align__(256) static uint8_t g_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mu;
uint8_t* g_scratch_addr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// cuCtxGetCurrent through the runtime's driver entry point (the library links
// the static runtime only); nullptr when the driver does not provide it.
CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<CtxGetCurrentFn>(nullptr);
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  return fn;
}

CUcontext current_ctx() {
  CUcontext ctx = nullptr;
  if (CtxGetCurrentFn fn = ctx_get_current_fn()) fn(&ctx);
  return ctx;
}

// Device address of g_noalloc_scratch on the current device: looked up once per
// device and context, then read from the cache.
int scratch_on_current_device(uint8_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return B2Q_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return B2Q_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  const CUcontext ctx = current_ctx();
  if (!g_scratch_addr[dev] || !ctx || ctx != g_scratch_ctx[dev]) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return B2Q_ERR_CUDA;
    if (major != 10 || minor != 0) return B2Q_ERR_UNSUPPORTED;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return B2Q_ERR_CUDA;
    if (reinterpret_cast<uintptr_t>(p) % 256 != 0) return B2Q_ERR_MISALIGNED;
    g_scratch_addr[dev] = static_cast<uint8_t*>(p);
    g_scratch_ctx[dev] = current_ctx();  // the runtime call above made the context current
  }
  *out = g_scratch_addr[dev];
  return B2Q_OK;
}

}  // namespace

extern "C" int b2q_mul_mat_packed_noalloc(const void* packed, int64_t n, int64_t k, const float* x,
                                          int64_t m, int64_t x_row_stride_bytes, const float* bias,
                                          float* y, int64_t y_row_stride_bytes, int variant,
                                          void* stream) {
  if (n < 0 || m < 0 || k <= 0 || k % kQK != 0) return B2Q_ERR_INVALID_ARG;
  if (variant != B2Q_ACT_X86 && variant != B2Q_ACT_REF && variant != B2Q_ACT_Q8_K) return B2Q_ERR_INVALID_ARG;
  if (variant == B2Q_ACT_Q8_K && k % kQKK != 0) return B2Q_ERR_INVALID_ARG;
  if (n > INT_MAX || m > INT_MAX || k > INT_MAX) return B2Q_ERR_TOO_LARGE;
  // The same bound as b2q_act_prepared_bytes(variant, m, k).
  if ((variant == B2Q_ACT_Q8_K ? q8k_bytes(m, k) : split_bytes(m, k)) > kScratchBytes) return B2Q_ERR_TOO_LARGE;
  uint8_t* scratch = nullptr;
  if (m > 0 && n > 0) {
    if (int rc = scratch_on_current_device(&scratch)) return rc;
  }
  return b2q_mul_mat_packed(packed, n, k, x, m, x_row_stride_bytes, bias, y, y_row_stride_bytes,
                            variant, scratch, scratch ? kScratchBytes : 0, stream);
}
