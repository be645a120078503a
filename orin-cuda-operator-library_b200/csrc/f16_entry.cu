// FP16 entry points: route each call to the tensor-core kernel when the shape
// fits it, else to the SIMT kernel (same FP32 accumulation contract).
#include "attention_simt.cuh"
#include "gemm_simt.cuh"

extern "C" int opl_gemm_f16(const opl_half_t* a, const opl_half_t* b, float* c,
                            int m, int n, int k, opl_stream_t stream) {
  if (a == nullptr || b == nullptr || c == nullptr || m <= 0 || n <= 0 || k <= 0)
    return cudaErrorInvalidValue;
  if (opl::gemv_tc_supported(a, b, m, n, k))
    return opl::gemv_tc(reinterpret_cast<const __half*>(a),
                        reinterpret_cast<const __half*>(b), c, m, n, k, stream);
  if (opl::gemv_f16_supported(b, c, m, n))
    return opl::gemv_f16(reinterpret_cast<const __half*>(a),
                         reinterpret_cast<const __half*>(b), c, m, n, k, stream);
  return opl::gemm_f16_tc(reinterpret_cast<const __half*>(a),
                          reinterpret_cast<const __half*>(b), c, m, n, k, stream);
}

extern "C" int opl_attention_f16(const opl_half_t* q, const opl_half_t* k,
                                 const opl_half_t* v, float* output, int batch,
                                 int heads, int sequence, int head_dim,
                                 int causal, opl_stream_t stream) {
  if (q == nullptr || k == nullptr || v == nullptr || output == nullptr ||
      batch <= 0 || heads <= 0 || sequence <= 0 || head_dim <= 0 ||
      head_dim > 128)
    return cudaErrorInvalidValue;
  const __half* qh = reinterpret_cast<const __half*>(q);
  const __half* kh = reinterpret_cast<const __half*>(k);
  const __half* vh = reinterpret_cast<const __half*>(v);
  if (opl::attention_tc_supported(head_dim, q, k, v, output))
    return opl::attention_f16_tc(qh, kh, vh, output, batch, heads, sequence, head_dim,
                                 causal != 0, stream);
  return opl::attention_simt<__half>(
      reinterpret_cast<const __half*>(q), reinterpret_cast<const __half*>(k),
      reinterpret_cast<const __half*>(v), output, batch, heads, sequence,
      head_dim, causal != 0, stream);
}
