// Internal interface of the reduce kernels, shared by the entry points.
#pragma once

#include "opl_common.cuh"

namespace opl {

constexpr int kReduceThreads = 512;
constexpr int kReduceCtasPerSm = 4;

// Per-CTA FP64 partial sums of input[0..n) into partials[blockIdx.x]
// (kReduceThreads threads; triggers programmatic dependent launch).
__global__ void reduce_partials_kernel(const float* __restrict__ input, std::size_t n,
                                       double* __restrict__ partials);

// Number of partial-sum CTAs used for n elements on the current device
// (at most sm_count() * kReduceCtasPerSm).
int reduce_grid(std::size_t n);

// Enqueues the partial kernel (blocks CTAs, one FP64 partial each written to
// partials[0..blocks)) and the fixed-order finalize kernel, which writes the
// total to *out_f32 and/or *out_f64 (either may be nullptr).
cudaError_t reduce_enqueue(const float* input, std::size_t n, double* partials,
                           int blocks, float* out_f32, double* out_f64,
                           cudaStream_t stream);

}  // namespace opl
