// b2q_sparse.cu -- the sparse stages of the SLat flow transformer around its
// linears (cpp_ggml/src/slat_flow_graph.cpp:161-236; ggml patch
// 0001-sam3d-ggml-combined.patch:151-272 for the CPU semantics):
//
//   submanifold convolution, F16: y[t] = bias + sum_o W_o . x[idx[o][t]] over the
//     27 neighbour offsets o (missing neighbours: index < 0, contribute
//     nothing), fp32 accumulation, fp16 result.  Built as gather27 (the 27
//     neighbour rows of every token side by side, zero rows for missing ones:
//     exactly the reference's get_rows + reshape of slat_flow_graph.cpp:
//     185-191) followed by the tcgen05 kind::f16 GEMM with K = 27 * C, whose
//     weight layout [Cout][27][C] is the converter's row format.
//   scatter-mean, F16 (the 2x downsample): out[c] = (0 + sum of the fine rows
//     mapped to c) / counts[c], every partial sum rounded to fp16 in fine-row
//     order, then an fp32 division (the divisor counts the initial zero).
//     The order is what makes it bit-exact with the reference's CPU path, so
//     the fine rows of each coarse row are first listed in ascending order
//     (count, scan, fill, per-row sort of the short lists) and then summed by
//     one thread per (coarse row, 8 channels) in that order: no float atomics.
#include <cuda_fp16.h>

#include "b2q_internal.h"

namespace b2q {

namespace {

int grid_cap(int64_t units, int per_block, int per_sm) {
  int sms = current_device_sms();
  if (sms <= 0) sms = 148;
  const int64_t blocks = (units + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(sms) * per_sm;
  return static_cast<int>(blocks < cap ? blocks : cap);
}

// One thread per (token, offset, 8 channels): 16-byte load, 16-byte store;
// consecutive threads write consecutive 16 bytes of g.
__global__ void __launch_bounds__(256) gather27_kernel(const uint4* __restrict__ x, int64_t tokens, int64_t c8,
                                                       const int32_t* __restrict__ idx, uint4* __restrict__ g) {
  const int64_t per_token = 27 * c8;
  const int64_t units = tokens * per_token;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < units;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = u / per_token, r = u - t * per_token;
    const int64_t o = r / c8, ch = r - o * c8;
    const int32_t src = __ldg(idx + o * tokens + t);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (src >= 0 && src < tokens) v = __ldg(x + src * c8 + ch);
    g[u] = v;
  }
}

__global__ void half_to_float_kernel(const __half* __restrict__ h, int64_t n, float* __restrict__ f) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    f[i] = __half2float(h[i]);
}

// ---------------------------------------------------------------- scatter-mean
// Rows outside [0, coarse) are skipped, as the reference's CPU loop skips them.
__global__ void count_children_kernel(const int32_t* __restrict__ rows, int64_t fine, int64_t coarse,
                                      int32_t* __restrict__ hist) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < fine;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t c = rows[i];
    if (c >= 0 && c < coarse) atomicAdd(hist + c, 1);
  }
}

// Exclusive scan of hist[0, n) into off[0, n], one block of 1024 threads:
// each thread scans a contiguous chunk, the chunk totals are scanned in
// shared memory.
constexpr int kScanThreads = 1024;
__global__ void __launch_bounds__(kScanThreads) scan_kernel(const int32_t* __restrict__ hist, int64_t n,
                                                            int32_t* __restrict__ off) {
  __shared__ int32_t part[kScanThreads];
  const int64_t chunk = (n + kScanThreads - 1) / kScanThreads;
  const int64_t b = threadIdx.x * chunk, e = b + chunk < n ? b + chunk : n;
  int32_t s = 0;
  for (int64_t i = b; i < e; ++i) s += hist[i];
  part[threadIdx.x] = s;
  __syncthreads();
  for (int d = 1; d < kScanThreads; d <<= 1) {  // inclusive Hillis-Steele scan of the totals
    const int32_t v = threadIdx.x >= d ? part[threadIdx.x - d] : 0;
    __syncthreads();
    part[threadIdx.x] += v;
    __syncthreads();
  }
  int32_t run = part[threadIdx.x] - s;  // exclusive prefix of this chunk
  for (int64_t i = b; i < e; ++i) {
    off[i] = run;
    run += hist[i];
  }
  if (threadIdx.x == kScanThreads - 1) off[n] = part[kScanThreads - 1];
}

__global__ void fill_children_kernel(const int32_t* __restrict__ rows, int64_t fine, int64_t coarse,
                                     const int32_t* __restrict__ off, int32_t* __restrict__ cursor,
                                     int32_t* __restrict__ list) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < fine;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t c = rows[i];
    if (c >= 0 && c < coarse) list[off[c] + atomicAdd(cursor + c, 1)] = static_cast<int32_t>(i);
  }
}

// Each coarse row's list into ascending fine-row order (insertion sort: the
// lists are short -- at most 8 children in a 2x downsample).
__global__ void sort_children_kernel(const int32_t* __restrict__ off, int64_t coarse, int32_t* __restrict__ list) {
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < coarse;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t b = off[c], e = off[c + 1];
    for (int32_t i = b + 1; i < e; ++i) {
      const int32_t v = list[i];
      int32_t j = i - 1;
      while (j >= b && list[j] > v) {
        list[j + 1] = list[j];
        --j;
      }
      list[j + 1] = v;
    }
  }
}

// One thread per (coarse row, 8 channels): fp16 partial sums in list order,
// each one fp16(fp32(acc) + fp32(x)), then fp16(fp32(acc) / counts[c]).
__global__ void __launch_bounds__(256) scatter_mean_kernel(const uint4* __restrict__ x, int64_t c8,
                                                           const int32_t* __restrict__ off,
                                                           const int32_t* __restrict__ list,
                                                           const float* __restrict__ counts, int64_t coarse,
                                                           uint4* __restrict__ out) {
  const int64_t units = coarse * c8;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < units;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = u / c8, ch = u - c * c8;
    __half acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = __float2half_rn(0.0f);
    const int32_t b = off[c], e = off[c + 1];
    for (int32_t j = b; j < e; ++j) {
      const uint4 v = __ldg(x + static_cast<int64_t>(list[j]) * c8 + ch);
      const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __float2half_rn(__fadd_rn(__half2float(acc[i]), __half2float(h[i])));
    }
    const float d = counts[c];
    uint4 o;
    __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
    for (int i = 0; i < 8; ++i) oh[i] = __float2half_rn(__fdiv_rn(__half2float(acc[i]), d));
    out[u] = o;
  }
}

}  // namespace

cudaError_t launch_gather27(const void* x16, int64_t tokens, int64_t C, const int32_t* idx, void* g,
                            cudaStream_t s) {
  const int64_t c8 = C / 8;
  const int64_t units = tokens * 27 * c8;
  if (units == 0) return cudaSuccess;
  gather27_kernel<<<grid_cap(units, 256, 16), 256, 0, s>>>(static_cast<const uint4*>(x16), tokens, c8, idx,
                                                           static_cast<uint4*>(g));
  return cudaGetLastError();
}

cudaError_t launch_half_to_float(const void* h, int64_t n, float* f, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  half_to_float_kernel<<<grid_cap(n, 256, 8), 256, 0, s>>>(static_cast<const __half*>(h), n, f);
  return cudaGetLastError();
}

// Plan layout (int32): hist[coarse], cursor[coarse], off[coarse + 1], list[fine].
cudaError_t launch_scatter_plan(const int32_t* rows, int64_t fine, int64_t coarse, int32_t* plan, cudaStream_t s) {
  if (coarse == 0) return cudaSuccess;
  int32_t* hist = plan;
  int32_t* cursor = plan + coarse;
  int32_t* off = plan + 2 * coarse;
  int32_t* list = plan + 3 * coarse + 1;
  cudaError_t e = cudaMemsetAsync(hist, 0, 2 * coarse * sizeof(int32_t), s);
  if (e != cudaSuccess) return e;
  if (fine > 0) count_children_kernel<<<grid_cap(fine, 256, 8), 256, 0, s>>>(rows, fine, coarse, hist);
  scan_kernel<<<1, kScanThreads, 0, s>>>(hist, coarse, off);
  if (fine > 0)
    fill_children_kernel<<<grid_cap(fine, 256, 8), 256, 0, s>>>(rows, fine, coarse, off, cursor, list);
  sort_children_kernel<<<grid_cap(coarse, 256, 8), 256, 0, s>>>(off, coarse, list);
  return cudaGetLastError();
}

cudaError_t launch_scatter_mean_planned(const void* x16, int64_t C, const int32_t* plan, const float* counts,
                                        int64_t coarse, void* out16, cudaStream_t s) {
  if (coarse == 0) return cudaSuccess;
  const int32_t* off = plan + 2 * coarse;
  const int32_t* list = plan + 3 * coarse + 1;
  const int64_t c8 = C / 8;
  scatter_mean_kernel<<<grid_cap(coarse * c8, 256, 16), 256, 0, s>>>(
      static_cast<const uint4*>(x16), c8, off, list, counts, coarse, static_cast<uint4*>(out16));
  return cudaGetLastError();
}

cudaError_t launch_scatter_mean_f16(const void* x16, int64_t fine, int64_t C, const int32_t* rows,
                                    const float* counts, int64_t coarse, void* out16, int32_t* ws,
                                    cudaStream_t s) {
  cudaError_t e = launch_scatter_plan(rows, fine, coarse, ws, s);
  if (e != cudaSuccess) return e;
  return launch_scatter_mean_planned(x16, C, ws, counts, coarse, out16, s);
}

}  // namespace b2q
