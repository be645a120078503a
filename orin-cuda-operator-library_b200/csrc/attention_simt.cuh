// Internal interface of the SIMT (FFMA) attention forward.
#pragma once

#include "opl_common.cuh"

namespace opl {

// O = softmax(Q K^T / sqrt(d) [causal]) V over contiguous [B,H,S,D] tensors,
// D <= 128, FP32 accumulation; T is float or __half.
template <typename T>
cudaError_t attention_simt(const T* q, const T* k, const T* v, float* out,
                           int batch, int heads, int seq, int d, bool causal,
                           cudaStream_t stream);

}  // namespace opl
