// probe_int8_peak.cu -- measured dense int8 tensor-core rate of this GPU, the
// roofline denominator of the block GEMM (its tensor work is kind::i8 MMAs).
//
// One CTA per SM; one thread issues back-to-back tcgen05.mma kind::i8
// (M = 128, N = 256, K = 32, s8 x s8 -> s32) on operands resident in shared
// memory, rotating over two TMEM accumulators.  Timed with CUDA events:
//   burst      one launch of ~2 ms (the clock a short kernel sees)
//   sustained  launches back to back for ~2 s (the clock under the power cap)
// Prints one JSON line.  Build: make -C sam-3d-objects-ggml_b200 probe
#include <cuda_runtime.h>

#include <chrono>
#include <cstdint>
#include <cstdio>

#include "b2q_ptx.cuh"

namespace {

constexpr int kN = 256;
constexpr int kThreads = 128;
constexpr int kSmem = (128 + kN) * 128 + 1024;  // A 128 x 128 B, B 256 x 128 B (128B swizzle)

__device__ unsigned int g_probe_status = 0;

__global__ void __launch_bounds__(kThreads, 1) mma_loop(int iters) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (b2q::smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint32_t holder;
  __shared__ uint64_t done;
  for (int i = threadIdx.x; i < (128 + kN) * 128 / 4; i += kThreads)
    reinterpret_cast<uint32_t*>(sm)[i] = 0x01010101u * static_cast<uint32_t>(i & 7);
  b2q::fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    b2q::mbar_init(&done, 1);
    b2q::fence_mbarrier_init();
  }
  if (threadIdx.x < 32) {
    b2q::tmem_alloc(&holder, 512);
    b2q::tmem_relinquish();
  }
  b2q::tc_fence_before();
  __syncthreads();
  b2q::tc_fence_after();
  const uint32_t tmem = holder;
  if (threadIdx.x == 0) {
    const uint32_t a = b2q::smem_u32(sm), b = a + 128 * 128;
    constexpr uint32_t idesc = b2q::idesc_i8(128, kN);
    for (int it = 0; it < iters; ++it) {
      const uint32_t d = tmem + static_cast<uint32_t>(it & 1) * kN;
      const uint32_t k = static_cast<uint32_t>(it & 3) * 32;
      b2q::mma_i8(d, b2q::smem_desc_k_sw128(a + k), b2q::smem_desc_k_sw128(b + k), idesc, 0u);
    }
    b2q::mma_commit(&done);
    b2q::mbar_wait(&done, 0, &g_probe_status, 1u, nullptr);
  }
  b2q::tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    b2q::tc_fence_after();
    b2q::tmem_dealloc(tmem, 512);
  }
}

int fail(const char* what, cudaError_t e) {
  std::printf("{\"error\": \"%s: %s\"}\n", what, cudaGetErrorString(e));
  return 1;
}

}  // namespace

int main() {
  int dev = 0, sms = 0, major = 0, minor = 0, clk_khz = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) {
    std::printf("{\"error\": \"needs sm_100\"}\n");
    return 1;
  }
  cudaError_t e = cudaFuncSetAttribute(mma_loop, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e != cudaSuccess) return fail("attribute", e);
  const double macs_per_iter = 128.0 * kN * 32.0;
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);

  // burst: calibrate one launch to ~2 ms
  int iters = 4096;
  mma_loop<<<sms, kThreads, kSmem>>>(iters);  // warm-up
  if ((e = cudaDeviceSynchronize()) != cudaSuccess) return fail("warm-up", e);
  float ms = 0.f;
  for (int round = 0; round < 8; ++round) {
    cudaEventRecord(e0);
    mma_loop<<<sms, kThreads, kSmem>>>(iters);
    cudaEventRecord(e1);
    if ((e = cudaEventSynchronize(e1)) != cudaSuccess) return fail("burst", e);
    cudaEventElapsedTime(&ms, e0, e1);
    if (ms >= 1.5f) break;
    iters *= 2;
  }
  const double burst = 2.0 * macs_per_iter * iters * sms / (ms * 1e-3) / 1e12;

  // sustained: back-to-back launches for ~2 s
  const int launches = static_cast<int>(2000.0f / (ms > 0.01f ? ms : 0.01f)) + 1;
  cudaEventRecord(e0);
  for (int l = 0; l < launches; ++l) mma_loop<<<sms, kThreads, kSmem>>>(iters);
  cudaEventRecord(e1);
  if ((e = cudaEventSynchronize(e1)) != cudaSuccess) return fail("sustained", e);
  float ms_all = 0.f;
  cudaEventElapsedTime(&ms_all, e0, e1);
  const double sustained = 2.0 * macs_per_iter * iters * sms * launches / (ms_all * 1e-3) / 1e12;

  unsigned int status = 0;
  cudaMemcpyFromSymbol(&status, g_probe_status, sizeof(status));
  cudaDeviceGetAttribute(&clk_khz, cudaDevAttrClockRate, dev);
  std::printf(
      "{\"int8_dense_tops_burst\": %.1f, \"int8_dense_tops_sustained\": %.1f, \"mma\": \"tcgen05 kind::i8 "
      "128x%dx32, one issuing thread per SM\", \"sms\": %d, \"iters_per_launch\": %d, \"burst_ms\": %.3f, "
      "\"sustained_launches\": %d, \"sustained_ms\": %.1f, \"status\": %u}\n",
      burst, sustained, kN, sms, iters, ms, launches, ms_all, status);
  return status ? 1 : 0;
}
