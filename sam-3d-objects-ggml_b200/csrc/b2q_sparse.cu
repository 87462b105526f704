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

// ------------------------------------------------- planned sparse convolution
// Plan (int32), built once per neighbour table:
//   cnt[27] valid pairs per offset | goff[28] row start of each offset's group,
//   groups padded to 256-row tiles | m_tiles[1] | pair_src[P] source token of
//   each padded row (-1: padding) | pair_of[27][tokens] row of (offset, token)
//   or -1 | tile_off[P / 256] offset of each tile.
// P = plan_rows(tokens) bounds the padded row count of any table.
constexpr int kPlanHead = 27 + 28 + 1;

__global__ void __launch_bounds__(256) conv_count_kernel(const int32_t* __restrict__ idx, int64_t tokens,
                                                         int32_t* __restrict__ cnt) {
  __shared__ int32_t local[27];
  if (threadIdx.x < 27) local[threadIdx.x] = 0;
  __syncthreads();
  const int64_t units = 27 * tokens;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < units;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t s = idx[u];
    if (s >= 0 && s < tokens) atomicAdd(local + u / tokens, 1);
  }
  __syncthreads();
  if (threadIdx.x < 27 && local[threadIdx.x]) atomicAdd(cnt + threadIdx.x, local[threadIdx.x]);
}

// One block: group starts (each group rounded up to whole 256-row tiles), the
// tile count and every tile's offset.
__global__ void __launch_bounds__(256) conv_layout_kernel(int32_t* __restrict__ plan, int64_t max_tiles,
                                                          int32_t* __restrict__ tile_off) {
  const int32_t* cnt = plan;
  int32_t* goff = plan + 27;
  __shared__ int32_t g[28];
  if (threadIdx.x == 0) {
    g[0] = 0;
    for (int o = 0; o < 27; ++o) g[o + 1] = g[o] + (cnt[o] + 255) / 256 * 256;
    plan[27 + 28] = g[27] / 256;
  }
  __syncthreads();
  if (threadIdx.x < 28) goff[threadIdx.x] = g[threadIdx.x];
  for (int o = 0; o < 27; ++o)
    for (int32_t j = g[o] / 256 + threadIdx.x; j < g[o + 1] / 256 && j < max_tiles; j += blockDim.x) tile_off[j] = o;
}

// One block per offset: a block-wide scan of the valid flags over the tokens
// (in token order, so the layout is deterministic) places every pair.
__global__ void __launch_bounds__(1024) conv_fill_kernel(const int32_t* __restrict__ idx, int64_t tokens,
                                                         const int32_t* __restrict__ plan,
                                                         int32_t* __restrict__ pair_src,
                                                         int32_t* __restrict__ pair_of) {
  __shared__ int32_t warp_sums[32];
  __shared__ int32_t base_s;
  const int o = blockIdx.x;
  const int32_t g0 = plan[27 + o], g1 = plan[27 + o + 1], n_valid = plan[o];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (threadIdx.x == 0) base_s = 0;
  __syncthreads();
  for (int64_t t0 = 0; t0 < tokens; t0 += blockDim.x) {
    const int64_t t = t0 + threadIdx.x;
    const int32_t s = t < tokens ? idx[o * tokens + t] : -1;
    const bool v = s >= 0 && s < tokens;
    const unsigned bal = __ballot_sync(0xffffffffu, v);
    if (lane == 0) warp_sums[wid] = __popc(bal);
    __syncthreads();
    if (wid == 0) {
      int32_t x = warp_sums[lane];
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int32_t y = __shfl_up_sync(0xffffffffu, x, d);
        if (lane >= d) x += y;
      }
      warp_sums[lane] = x;  // inclusive
    }
    __syncthreads();
    const int32_t before = (wid ? warp_sums[wid - 1] : 0) + __popc(bal & ((1u << lane) - 1u));
    const int32_t base = base_s;
    if (t < tokens) {
      const int32_t r = g0 + base + before;
      pair_of[o * tokens + t] = v ? r : -1;
      if (v) pair_src[r] = s;
    }
    __syncthreads();
    if (threadIdx.x == 0) base_s = base + warp_sums[31];
    __syncthreads();
  }
  for (int32_t r = g0 + n_valid + threadIdx.x; r < g1; r += blockDim.x) pair_src[r] = -1;  // padding rows
}

// Rows of the padded pair matrix: g[r] = x[pair_src[r]] (zero for padding),
// for r below the plan's row count.
__global__ void __launch_bounds__(256) gather_pairs_kernel(const uint4* __restrict__ x, int64_t tokens, int64_t c8,
                                                           const int32_t* __restrict__ plan, int64_t max_rows,
                                                           const int32_t* __restrict__ pair_src,
                                                           uint4* __restrict__ g) {
  int64_t rows = static_cast<int64_t>(plan[27 + 28]) * 256;
  rows = rows < 0 ? 0 : (rows > max_rows ? max_rows : rows);  // a plan never exceeds its own capacity
  const int64_t units = rows * c8;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < units;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = u / c8, ch = u - r * c8;
    const int32_t s = pair_src[r];
    g[u] = (s >= 0 && s < tokens) ? __ldg(x + s * c8 + ch) : make_uint4(0u, 0u, 0u, 0u);
  }
}

// y16[t][8 outputs] = fp16(bias + sum over offsets o = 0..26 of the pair
// partials), fp32, offsets in ascending order.
__global__ void __launch_bounds__(256) conv_reduce_kernel(const float4* __restrict__ part, int64_t cout8,
                                                          int64_t part_rows, const int32_t* __restrict__ pair_of,
                                                          int64_t tokens, const float* __restrict__ bias,
                                                          uint4* __restrict__ y) {
  const int64_t units = tokens * cout8;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < units;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = u / cout8, c = u - t * cout8;
    float a[8];
    if (bias) {
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(bias) + 2 * c);
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(bias) + 2 * c + 1);
      a[0] = b0.x, a[1] = b0.y, a[2] = b0.z, a[3] = b0.w, a[4] = b1.x, a[5] = b1.y, a[6] = b1.z, a[7] = b1.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = 0.0f;
    }
    // All 27 pair rows first (independent loads), then the partials; the adds
    // stay in offset order.
    int32_t rr[27];
#pragma unroll
    for (int o = 0; o < 27; ++o) rr[o] = __ldg(pair_of + o * tokens + t);
#pragma unroll
    for (int o = 0; o < 27; ++o) {
      const int32_t r = rr[o];
      if (r < 0 || r >= part_rows) continue;
      const float4 p0 = __ldg(part + (static_cast<int64_t>(r) * cout8 + c) * 2);
      const float4 p1 = __ldg(part + (static_cast<int64_t>(r) * cout8 + c) * 2 + 1);
      a[0] = __fadd_rn(a[0], p0.x), a[1] = __fadd_rn(a[1], p0.y), a[2] = __fadd_rn(a[2], p0.z);
      a[3] = __fadd_rn(a[3], p0.w), a[4] = __fadd_rn(a[4], p1.x), a[5] = __fadd_rn(a[5], p1.y);
      a[6] = __fadd_rn(a[6], p1.z), a[7] = __fadd_rn(a[7], p1.w);
    }
    uint4 o16;
    __half* h = reinterpret_cast<__half*>(&o16);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = __float2half_rn(a[i]);
    y[u] = o16;
  }
}

}  // namespace

int64_t conv_plan_rows(int64_t tokens) { return round_up(27 * tokens + 27 * 255, 256); }
int64_t conv_plan_ints(int64_t tokens) {
  return kPlanHead + conv_plan_rows(tokens) + 27 * tokens + conv_plan_rows(tokens) / 256;
}

cudaError_t launch_conv_plan(const int32_t* idx, int64_t tokens, int32_t* plan, cudaStream_t s) {
  const int64_t P = conv_plan_rows(tokens);
  int32_t* pair_src = plan + kPlanHead;
  int32_t* pair_of = pair_src + P;
  int32_t* tile_off = pair_of + 27 * tokens;
  cudaError_t e = cudaMemsetAsync(plan, 0, kPlanHead * sizeof(int32_t), s);
  if (e != cudaSuccess) return e;
  if (tokens > 0) conv_count_kernel<<<grid_cap(27 * tokens, 256, 8), 256, 0, s>>>(idx, tokens, plan);
  conv_layout_kernel<<<1, 256, 0, s>>>(plan, P / 256, tile_off);
  if (tokens > 0) conv_fill_kernel<<<27, 1024, 0, s>>>(idx, tokens, plan, pair_src, pair_of);
  return cudaGetLastError();
}

cudaError_t launch_conv_planned(const void* x16, int64_t tokens, int64_t C, const void* w16, int64_t cout,
                                const float* bias, const int32_t* plan, void* g, float* part, void* y16, int num_sms,
                                cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  const int64_t P = conv_plan_rows(tokens);
  const int32_t* pair_src = plan + kPlanHead;
  const int32_t* pair_of = pair_src + P;
  const int32_t* tile_off = pair_of + 27 * tokens;
  const int64_t c8 = C / 8;
  gather_pairs_kernel<<<grid_cap(P * c8, 256, 16), 256, 0, s>>>(static_cast<const uint4*>(x16), tokens, c8, plan, P,
                                                                pair_src, static_cast<uint4*>(g));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  e = launch_gemm_f16_grouped(w16, 27 * C * 2, 27 * C, g, C * 2, P, cout, C, part, cout, plan + 27 + 28, tile_off,
                              P / 256, num_sms, s);
  if (e != cudaSuccess) return e;
  const int64_t cout8 = cout / 8;
  conv_reduce_kernel<<<grid_cap(tokens * cout8, 256, 16), 256, 0, s>>>(
      reinterpret_cast<const float4*>(part), cout8, P, pair_of, tokens, bias, static_cast<uint4*>(y16));
  return cudaGetLastError();
}

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
