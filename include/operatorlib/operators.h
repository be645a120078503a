#pragma once

// Public C++ API of the B200 operator library.
//
// Drop-in for the reference header include/operatorlib/operators.h:8-46
// (same namespace, names, argument order, defaults and cudaError_t returns).
// Every function here is a thin forwarder onto the C-ABI declared in
// operatorlib/opl_capi.h; the forwarders are compiled into libopl_b200.so.
//
// Conventions (reference docs/launcher_extraction.md:9-15):
//   * all pointers are caller-owned device memory, outputs pre-allocated;
//   * work is enqueued on `stream` (nullptr = legacy default stream) and the
//     device is never synchronised;
//   * bad arguments return cudaErrorInvalidValue, otherwise the launch error
//     (asynchronous faults surface at the caller's next synchronisation);
//   * the current CUDA device is the device the work runs on.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>

namespace operatorlib {

// Sum of n floats into *output (a single float). Reference src/reduce.cu:54-69.
// Deterministic: the same n on the same device gives bit-identical results.
cudaError_t reduce_sum_f32(const float* input, float* output, std::size_t n,
                           cudaStream_t stream = nullptr);

// Numerically stable softmax over the last dimension of a rows x cols matrix.
// Reference src/softmax.cu:182-202.
cudaError_t softmax_f32(const float* input, float* output, int rows, int cols,
                        cudaStream_t stream = nullptr);

// Out-of-place transpose: output[c][r] = input[r][c]. Reference
// src/transpose.cu:38-47.
cudaError_t transpose_f32(const float* input, float* output, int rows, int cols,
                          cudaStream_t stream = nullptr);

// y = x * rsqrt(mean(x^2) + epsilon) * weight per token row. Reference
// src/rmsnorm.cu:77-95.
cudaError_t rmsnorm_f32(const float* input, const float* weight, float* output,
                        int tokens, int hidden, float epsilon,
                        cudaStream_t stream = nullptr);

// Row-major C[M,N] = A[M,K] * B[K,N], FP32 FFMA (no TF32). Reference
// src/gemm.cu:440-453.
cudaError_t gemm_f32(const float* a, const float* b, float* c, int m, int n,
                     int k, cudaStream_t stream = nullptr);

// FP16 inputs, FP32 tensor-core accumulation and FP32 output. Reference
// src/gemm.cu:455-479.
cudaError_t gemm_f16(const __half* a, const __half* b, float* c, int m, int n,
                     int k, cudaStream_t stream = nullptr);

// Q/K/V and output use contiguous [B,H,S,D] row-major storage, D <= 128.
// Reference src/attention.cu:445-484.
cudaError_t attention_f32(const float* q, const float* k, const float* v,
                          float* output, int batch, int heads, int sequence,
                          int head_dim, bool causal,
                          cudaStream_t stream = nullptr);

// FP16 Q/K/V, FP32 online-softmax state and FP32 output. Reference
// src/attention.cu:486-507.
cudaError_t attention_f16(const __half* q, const __half* k, const __half* v,
                          float* output, int batch, int heads, int sequence,
                          int head_dim, bool causal,
                          cudaStream_t stream = nullptr);

}  // namespace operatorlib
