// Internal interface of the SIMT (FFMA) GEMM.
#pragma once

#include "opl_common.cuh"

namespace opl {

// Row-major C[M,N] = A[M,K] * B[K,N] with FP32 FFMA accumulation; T is float
// or __half (converted to FP32 on load).  Any shape and alignment.
template <typename T>
cudaError_t gemm_simt(const T* a, const T* b, float* c, int m, int n, int k,
                      cudaStream_t stream);

// Tensor-core (tcgen05) FP16 GEMM with FP32 accumulation and output; any
// shape (unaligned strides are staged through padded copies).
cudaError_t gemm_f16_tc(const __half* a, const __half* b, float* c, int m, int n,
                        int k, cudaStream_t stream);

// Skinny FP16 GEMM for M <= 16 (bandwidth-bound on B): split-K SIMT kernel
// with a fixed-order reduction; gemv_f16_supported says whether it applies
// (N % 8 == 0, 16-byte aligned B and C).
bool gemv_f16_supported(const void* b, const void* c, int m, int n);
cudaError_t gemv_f16(const __half* a, const __half* b, float* c, int m, int n, int k,
                     cudaStream_t stream);

// Skinny FP16 GEMM for M <= 128 on the tensor cores with swapped operands
// (C^T = B^T A^T), K split across a thread-block cluster and summed through
// distributed shared memory; needs N % 8 == 0, K % 8 == 0 and 16-byte
// aligned A and B (TMA row strides and bases).
bool gemv_tc_supported(const void* a, const void* b, int m, int n, int k);
cudaError_t gemv_tc(const __half* a, const __half* b, float* c, int m, int n, int k,
                    cudaStream_t stream);

// Skinny-N FP16 product on the same kernel: C[i][j] (row stride ldc) =
// sum_k A[i][k] * bt[j][k] for i < m, j < ns <= 128; A row stride lda and
// bt ([ns][k], row stride ldbt) -- strides multiples of 8 halves, 16-byte
// aligned bases.
cudaError_t gemm_small_n_tc(const __half* a, int lda, const __half* bt, int ldbt, float* c,
                            int ldc, int m, int ns, int k, cudaStream_t stream);

}  // namespace opl
