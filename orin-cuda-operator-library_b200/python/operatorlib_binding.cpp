// TORCH_LIBRARY(operatorlib, ...) binding of the B200 operator library.
//
// Drop-in for the reference binding python/operatorlib_binding.cpp:190-206:
// the six schemas are identical; the CUDA dispatch key runs the kernels (and,
// beyond the reference, a Meta key gives shapes for FakeTensor tracing);
// inputs must be contiguous CUDA tensors (no implicit copies), outputs are
// allocated here, work goes on the input device's current stream under a
// device guard, and the user-facing error texts match the reference's
// (python/test_extension.py:124-168 checks them).  Every launch goes through
// the C++ API of operatorlib/operators.h, which forwards to the C-ABI.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cmath>
#include <cstdint>
#include <limits>

#include "operatorlib/operators.h"

namespace {

using at::Tensor;

// Meta (shape-only) calls run the same checks minus the device check.
thread_local bool g_meta_call = false;

struct MetaCall {
  MetaCall() { g_meta_call = true; }
  ~MetaCall() { g_meta_call = false; }
};

void require_cuda_contiguous(const Tensor& t, const char* name) {
  if (!g_meta_call) TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

void require_matching(const Tensor& x, const Tensor& y, const char* xn,
                      const char* yn) {
  TORCH_CHECK(x.device() == y.device(), xn, " and ", yn,
              " must be on the same CUDA device");
  TORCH_CHECK(x.scalar_type() == y.scalar_type(), xn, " and ", yn,
              " must have the same dtype");
}

int as_positive_int(int64_t value, const char* what) {
  TORCH_CHECK(value > 0 && value <= std::numeric_limits<int>::max(), what,
              " must be in the positive int32 range");
  return static_cast<int>(value);
}

void raise_on_error(cudaError_t status, const char* op) {
  TORCH_CHECK(status == cudaSuccess, op, " launch failed: ",
              cudaGetErrorString(status));
}

cudaStream_t stream_of(const Tensor& t) {
  return at::cuda::getCurrentCUDAStream(t.get_device()).stream();
}

const __half* half_ptr(const Tensor& t) {
  return reinterpret_cast<const __half*>(t.data_ptr<at::Half>());
}

Tensor op_reduce_sum(const Tensor& input) {
  require_cuda_contiguous(input, "input");
  TORCH_CHECK(input.scalar_type() == at::kFloat,
              "reduce_sum supports float32 input only");
  TORCH_CHECK(input.numel() > 0, "input must be non-empty");
  if (g_meta_call) return at::empty({}, input.options());
  c10::cuda::CUDAGuard guard(input.device());
  Tensor out = at::empty({}, input.options());
  raise_on_error(operatorlib::reduce_sum_f32(
                     input.data_ptr<float>(), out.data_ptr<float>(),
                     static_cast<std::size_t>(input.numel()), stream_of(input)),
                 "reduce_sum");
  return out;
}

Tensor op_softmax(const Tensor& input) {
  require_cuda_contiguous(input, "input");
  TORCH_CHECK(input.scalar_type() == at::kFloat,
              "softmax supports float32 input only");
  TORCH_CHECK(input.dim() >= 1, "input must have at least one dimension");
  const int cols = as_positive_int(input.size(-1), "last dimension");
  const int rows = as_positive_int(input.numel() / input.size(-1), "row count");
  if (g_meta_call) return at::empty_like(input);
  c10::cuda::CUDAGuard guard(input.device());
  Tensor out = at::empty_like(input);
  raise_on_error(operatorlib::softmax_f32(input.data_ptr<float>(),
                                          out.data_ptr<float>(), rows, cols,
                                          stream_of(input)),
                 "softmax");
  return out;
}

Tensor op_transpose(const Tensor& input) {
  require_cuda_contiguous(input, "input");
  TORCH_CHECK(input.scalar_type() == at::kFloat,
              "transpose supports float32 input only");
  TORCH_CHECK(input.dim() == 2, "input must be a 2D matrix");
  const int rows = as_positive_int(input.size(0), "rows");
  const int cols = as_positive_int(input.size(1), "cols");
  if (g_meta_call) return at::empty({cols, rows}, input.options());
  c10::cuda::CUDAGuard guard(input.device());
  Tensor out = at::empty({cols, rows}, input.options());
  raise_on_error(operatorlib::transpose_f32(input.data_ptr<float>(),
                                            out.data_ptr<float>(), rows, cols,
                                            stream_of(input)),
                 "transpose");
  return out;
}

Tensor op_rmsnorm(const Tensor& input, const Tensor& weight, double epsilon) {
  require_cuda_contiguous(input, "input");
  require_cuda_contiguous(weight, "weight");
  require_matching(input, weight, "input", "weight");
  TORCH_CHECK(input.scalar_type() == at::kFloat,
              "rmsnorm supports float32 input only");
  TORCH_CHECK(input.dim() >= 1, "input must have at least one dimension");
  TORCH_CHECK(weight.dim() == 1, "weight must be 1D");
  TORCH_CHECK(std::isfinite(epsilon) && epsilon > 0.0,
              "epsilon must be finite and positive");
  const int hidden = as_positive_int(input.size(-1), "hidden size");
  TORCH_CHECK(weight.numel() == hidden,
              "weight length must equal the input hidden size");
  const int tokens =
      as_positive_int(input.numel() / input.size(-1), "token count");
  if (g_meta_call) return at::empty_like(input);
  c10::cuda::CUDAGuard guard(input.device());
  Tensor out = at::empty_like(input);
  raise_on_error(operatorlib::rmsnorm_f32(
                     input.data_ptr<float>(), weight.data_ptr<float>(),
                     out.data_ptr<float>(), tokens, hidden,
                     static_cast<float>(epsilon), stream_of(input)),
                 "rmsnorm");
  return out;
}

Tensor op_gemm(const Tensor& a, const Tensor& b) {
  require_cuda_contiguous(a, "a");
  require_cuda_contiguous(b, "b");
  require_matching(a, b, "a", "b");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2, "a and b must be 2D matrices");
  TORCH_CHECK(a.size(1) == b.size(0), "a.size(1) must equal b.size(0)");
  TORCH_CHECK(a.scalar_type() == at::kFloat || a.scalar_type() == at::kHalf,
              "gemm supports float32 or float16 inputs only");
  const int m = as_positive_int(a.size(0), "M");
  const int k = as_positive_int(a.size(1), "K");
  const int n = as_positive_int(b.size(1), "N");
  if (g_meta_call) return at::empty({m, n}, a.options().dtype(at::kFloat));
  c10::cuda::CUDAGuard guard(a.device());
  Tensor c = at::empty({m, n}, a.options().dtype(at::kFloat));
  const cudaError_t status =
      a.scalar_type() == at::kFloat
          ? operatorlib::gemm_f32(a.data_ptr<float>(), b.data_ptr<float>(),
                                  c.data_ptr<float>(), m, n, k, stream_of(a))
          : operatorlib::gemm_f16(half_ptr(a), half_ptr(b), c.data_ptr<float>(),
                                  m, n, k, stream_of(a));
  raise_on_error(status, "gemm");
  return c;
}

Tensor op_attention(const Tensor& q, const Tensor& k, const Tensor& v,
                    bool causal) {
  require_cuda_contiguous(q, "q");
  require_cuda_contiguous(k, "k");
  require_cuda_contiguous(v, "v");
  require_matching(q, k, "q", "k");
  require_matching(q, v, "q", "v");
  TORCH_CHECK(q.dim() == 4, "q, k and v must use [B,H,S,D] layout");
  TORCH_CHECK(q.sizes() == k.sizes() && q.sizes() == v.sizes(),
              "q, k and v must have identical shapes");
  TORCH_CHECK(q.scalar_type() == at::kFloat || q.scalar_type() == at::kHalf,
              "attention supports float32 or float16 inputs only");
  const int batch = as_positive_int(q.size(0), "batch");
  const int heads = as_positive_int(q.size(1), "heads");
  const int sequence = as_positive_int(q.size(2), "sequence");
  const int head_dim = as_positive_int(q.size(3), "head dimension");
  TORCH_CHECK(head_dim <= 128, "head dimension must be at most 128");
  TORCH_CHECK(static_cast<int64_t>(batch) * heads <=
                  std::numeric_limits<int>::max(),
              "batch * heads exceeds the supported int32 range");
  if (g_meta_call) return at::empty(q.sizes(), q.options().dtype(at::kFloat));
  c10::cuda::CUDAGuard guard(q.device());
  Tensor out = at::empty(q.sizes(), q.options().dtype(at::kFloat));
  const cudaError_t status =
      q.scalar_type() == at::kFloat
          ? operatorlib::attention_f32(q.data_ptr<float>(), k.data_ptr<float>(),
                                       v.data_ptr<float>(), out.data_ptr<float>(),
                                       batch, heads, sequence, head_dim, causal,
                                       stream_of(q))
          : operatorlib::attention_f16(half_ptr(q), half_ptr(k), half_ptr(v),
                                       out.data_ptr<float>(), batch, heads,
                                       sequence, head_dim, causal, stream_of(q));
  raise_on_error(status, "attention");
  return out;
}

// Meta kernels: output shape/dtype only, after the same argument checks, so
// FakeTensor tracing (torch.compile, torch.export) sees the ops.  The
// reference registers the CUDA key only.
Tensor meta_reduce_sum(const Tensor& input) {
  MetaCall meta;
  return op_reduce_sum(input);
}
Tensor meta_softmax(const Tensor& input) {
  MetaCall meta;
  return op_softmax(input);
}
Tensor meta_transpose(const Tensor& input) {
  MetaCall meta;
  return op_transpose(input);
}
Tensor meta_rmsnorm(const Tensor& input, const Tensor& weight, double epsilon) {
  MetaCall meta;
  return op_rmsnorm(input, weight, epsilon);
}
Tensor meta_gemm(const Tensor& a, const Tensor& b) {
  MetaCall meta;
  return op_gemm(a, b);
}
Tensor meta_attention(const Tensor& q, const Tensor& k, const Tensor& v, bool causal) {
  MetaCall meta;
  return op_attention(q, k, v, causal);
}

}  // namespace

TORCH_LIBRARY(operatorlib, m) {
  m.def("reduce_sum(Tensor input) -> Tensor");
  m.def("softmax(Tensor input) -> Tensor");
  m.def("transpose(Tensor input) -> Tensor");
  m.def("rmsnorm(Tensor input, Tensor weight, float epsilon=1e-5) -> Tensor");
  m.def("gemm(Tensor a, Tensor b) -> Tensor");
  m.def("attention(Tensor q, Tensor k, Tensor v, bool causal=False) -> Tensor");
}

TORCH_LIBRARY_IMPL(operatorlib, CUDA, m) {
  m.impl("reduce_sum", &op_reduce_sum);
  m.impl("softmax", &op_softmax);
  m.impl("transpose", &op_transpose);
  m.impl("rmsnorm", &op_rmsnorm);
  m.impl("gemm", &op_gemm);
  m.impl("attention", &op_attention);
}

TORCH_LIBRARY_IMPL(operatorlib, Meta, m) {
  m.impl("reduce_sum", &meta_reduce_sum);
  m.impl("softmax", &meta_softmax);
  m.impl("transpose", &meta_transpose);
  m.impl("rmsnorm", &meta_rmsnorm);
  m.impl("gemm", &meta_gemm);
  m.impl("attention", &meta_attention);
}
