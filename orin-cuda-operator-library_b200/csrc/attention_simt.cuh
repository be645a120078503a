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

// tcgen05 FP16 attention (FP32 state and output) for head_dim <= 128 with
// head_dim % 8 == 0 (computed as 64 or 128 with zero padding) and 16-byte
// aligned tensors; attention_tc_supported says whether it applies.
bool attention_tc_supported(int head_dim, const void* q, const void* k, const void* v,
                            const void* out);
cudaError_t attention_f16_tc(const __half* q, const __half* k, const __half* v, float* out,
                             int batch, int heads, int seq, int head_dim, bool causal,
                             cudaStream_t stream);

// Tiled FP32 FFMA attention for head_dim <= 128 with head_dim % 4 == 0
// (computed as 64 or 128 with zero padding) and 16-byte aligned tensors
// (attention_f32_tiled_supported); other shapes use attention_simt.
bool attention_f32_tiled_supported(int head_dim, const void* q, const void* k, const void* v,
                                   const void* out);
cudaError_t attention_f32_tiled(const float* q, const float* k, const float* v, float* out,
                                int batch, int heads, int seq, int head_dim, bool causal,
                                cudaStream_t stream);

}  // namespace opl
