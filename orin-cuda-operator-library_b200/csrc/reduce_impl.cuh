// Internal interface of the reduce kernels, shared by the entry points.
#pragma once

#include "opl_common.cuh"

namespace opl {

constexpr int kReduceThreads = 256;
// Upper bound on partial-sum CTAs (and so on FP64 partials per call).
constexpr int kReduceMaxCtas = 4096;

// Launches reduce_partials_kernel with `blocks` CTAs on `stream`.
cudaError_t reduce_partials_launch(const float* input, std::size_t n, double* partials,
                                   int blocks, cudaStream_t stream);

// Fixed-order sum over a CTA of kReduceThreads threads (warp xor-trees, then
// the warp totals in warp order); the result is valid in thread 0.
__device__ __forceinline__ double block_sum_fixed(double v) {
  __shared__ double warp_totals[kReduceThreads / 32];
  v = warp_sum(v);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (lane == 0) warp_totals[warp] = v;
  __syncthreads();
  double total = 0.0;
  if (threadIdx.x == 0)
    for (int w = 0; w < kReduceThreads / 32; ++w) total += warp_totals[w];
  return total;
}

// Sum of partials t, t + kReduceThreads, ... (in that order) for thread t,
// count <= kReduceMaxCtas: all loads issued before the adds, so the thread
// waits for one memory latency instead of one per partial.
__device__ __forceinline__ double sum_partials_strided(const double* __restrict__ partials,
                                                       int count) {
  constexpr int kPer = kReduceMaxCtas / kReduceThreads;
  double vals[kPer];
#pragma unroll
  for (int u = 0; u < kPer; ++u) {
    const int i = static_cast<int>(threadIdx.x) + u * kReduceThreads;
    vals[u] = i < count ? ld_coherent(partials + i) : 0.0;  // after griddepcontrol.wait
  }
  double v = 0.0;
#pragma unroll
  for (int u = 0; u < kPer; ++u) v += vals[u];
  return v;
}

// Number of partial-sum CTAs for n elements starting at input (at most
// kReduceMaxCtas).
int reduce_grid(const float* input, std::size_t n);

// Enqueues the partial kernel (blocks CTAs, one FP64 partial each written to
// partials[0..blocks)) and the fixed-order finalize kernel, which writes the
// total to *out_f32 and/or *out_f64 (either may be nullptr).
cudaError_t reduce_enqueue(const float* input, std::size_t n, double* partials,
                           int blocks, float* out_f32, double* out_f64,
                           cudaStream_t stream);

}  // namespace opl
