// C entry points onto the REFERENCE launchers (operatorlib::* of the
// reference's include/operatorlib/operators.h, implemented by its src/*.cu,
// compiled unmodified for sm_100a into oracle/_ref/).  Test/bench
// infrastructure only: lets the GPU tests compare against the reference's own
// kernels on the same B200 and lets bench.py time them side by side.
#include "operatorlib/operators.h"

extern "C" {

int ref_reduce_sum_f32(const float* x, float* y, size_t n, cudaStream_t s) {
  return operatorlib::reduce_sum_f32(x, y, n, s);
}
int ref_softmax_f32(const float* x, float* y, int r, int c, cudaStream_t s) {
  return operatorlib::softmax_f32(x, y, r, c, s);
}
int ref_transpose_f32(const float* x, float* y, int r, int c, cudaStream_t s) {
  return operatorlib::transpose_f32(x, y, r, c, s);
}
int ref_rmsnorm_f32(const float* x, const float* w, float* y, int t, int h,
                    float eps, cudaStream_t s) {
  return operatorlib::rmsnorm_f32(x, w, y, t, h, eps, s);
}
int ref_gemm_f32(const float* a, const float* b, float* c, int m, int n, int k,
                 cudaStream_t s) {
  return operatorlib::gemm_f32(a, b, c, m, n, k, s);
}
int ref_gemm_f16(const __half* a, const __half* b, float* c, int m, int n,
                 int k, cudaStream_t s) {
  return operatorlib::gemm_f16(a, b, c, m, n, k, s);
}
int ref_attention_f32(const float* q, const float* k, const float* v, float* o,
                      int b, int h, int sq, int d, int causal, cudaStream_t s) {
  return operatorlib::attention_f32(q, k, v, o, b, h, sq, d, causal != 0, s);
}
int ref_attention_f16(const __half* q, const __half* k, const __half* v,
                      float* o, int b, int h, int sq, int d, int causal,
                      cudaStream_t s) {
  return operatorlib::attention_f16(q, k, v, o, b, h, sq, d, causal != 0, s);
}

}  // extern "C"
