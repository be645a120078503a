// Launcher smoke test of the C++ API (include/operatorlib/operators.h),
// linked against the static library target `operatorlib`.
//
// Every launcher runs once on a small ragged shape on a non-default stream
// and is checked against a double-precision loop on the host, with the gates
// the library is held to: FP32 row ops 1e-5 relative, reduce 1e-6 relative,
// transpose bit-exact, FP16 GEMM / attention 2e-2 absolute, FP32 GEMM and
// attention 1e-3 / 1e-4.  Argument errors must come back as
// cudaErrorInvalidValue without touching the GPU.  Prints one PASS line per
// launcher; exits non-zero on the first failure.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <vector>

#include "operatorlib/operators.h"

namespace {

void check_cuda(cudaError_t e, const char* what, int line) {
  if (e != cudaSuccess) {
    std::fprintf(stderr, "line %d: %s: %s\n", line, what, cudaGetErrorString(e));
    std::exit(1);
  }
}
#define CK(x) check_cuda((x), #x, __LINE__)

void require(bool ok, const char* what, double err) {
  if (!ok) {
    std::fprintf(stderr, "%s FAILED (error %.3g)\n", what, err);
    std::exit(1);
  }
}

template <typename T>
struct DeviceBuffer {
  T* ptr = nullptr;
  std::size_t count = 0;
  explicit DeviceBuffer(std::size_t n) : count(n) { CK(cudaMalloc(&ptr, n * sizeof(T))); }
  DeviceBuffer(const std::vector<T>& host, cudaStream_t s) : DeviceBuffer(host.size()) {
    CK(cudaMemcpyAsync(ptr, host.data(), host.size() * sizeof(T), cudaMemcpyHostToDevice, s));
  }
  ~DeviceBuffer() { cudaFree(ptr); }
  std::vector<T> read(cudaStream_t s) const {
    std::vector<T> host(count);
    CK(cudaMemcpyAsync(host.data(), ptr, count * sizeof(T), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    return host;
  }
};

std::vector<float> uniform(std::size_t n, unsigned seed, float lo, float hi) {
  std::mt19937 gen(seed);
  std::uniform_real_distribution<float> dist(lo, hi);
  std::vector<float> v(n);
  for (float& x : v) x = dist(gen);
  return v;
}

std::vector<__half> to_half(const std::vector<float>& v) {
  std::vector<__half> h(v.size());
  for (std::size_t i = 0; i < v.size(); ++i) h[i] = __float2half_rn(v[i]);
  return h;
}

std::vector<float> from_half(const std::vector<__half>& h) {
  std::vector<float> v(h.size());
  for (std::size_t i = 0; i < h.size(); ++i) v[i] = __half2float(h[i]);
  return v;
}

void test_reduce(cudaStream_t s) {
  const std::size_t n = 1000003;
  const auto x = uniform(n, 1, -1.f, 1.f);
  double want = 0.0;
  for (float v : x) want += v;
  DeviceBuffer<float> dx(x, s), out(1);
  CK(operatorlib::reduce_sum_f32(dx.ptr, out.ptr, n, s));
  const double got = out.read(s)[0];
  const double err = std::fabs(got - want);
  require(err <= 1e-6 * std::fabs(want) + 1e-6, "reduce_sum_f32", err);
  std::printf("reduce_sum_f32=PASS\n");
}

void test_softmax(cudaStream_t s) {
  const int rows = 37, cols = 1003;
  const auto x = uniform(std::size_t(rows) * cols, 2, -8.f, 8.f);
  DeviceBuffer<float> dx(x, s), dy(x.size());
  CK(operatorlib::softmax_f32(dx.ptr, dy.ptr, rows, cols, s));
  const auto y = dy.read(s);
  double worst = 0.0;
  for (int r = 0; r < rows; ++r) {
    const float* row = &x[std::size_t(r) * cols];
    double m = row[0], sum = 0.0;
    for (int c = 1; c < cols; ++c) m = std::fmax(m, row[c]);
    for (int c = 0; c < cols; ++c) sum += std::exp(row[c] - m);
    for (int c = 0; c < cols; ++c) {
      const double want = std::exp(row[c] - m) / sum;
      const double err = std::fabs(y[std::size_t(r) * cols + c] - want);
      require(err <= 1e-5 * want + 1e-9, "softmax_f32", err);
      worst = std::fmax(worst, err);
    }
  }
  std::printf("softmax_f32=PASS\n");
}

void test_transpose(cudaStream_t s) {
  for (const auto& shape : {std::pair<int, int>{65, 37}, std::pair<int, int>{64, 96}}) {
    const int rows = shape.first, cols = shape.second;
    const auto x = uniform(std::size_t(rows) * cols, 3, -1.f, 1.f);
    DeviceBuffer<float> dx(x, s), dy(x.size());
    CK(operatorlib::transpose_f32(dx.ptr, dy.ptr, rows, cols, s));
    const auto y = dy.read(s);
    for (int r = 0; r < rows; ++r)
      for (int c = 0; c < cols; ++c)
        require(std::memcmp(&y[std::size_t(c) * rows + r], &x[std::size_t(r) * cols + c],
                            sizeof(float)) == 0,
                "transpose_f32", 1.0);
  }
  std::printf("transpose_f32=PASS\n");
}

void test_rmsnorm(cudaStream_t s) {
  const int tokens = 9, hidden = 1023;
  const float eps = 1e-6f;
  const auto x = uniform(std::size_t(tokens) * hidden, 4, -2.f, 2.f);
  const auto w = uniform(hidden, 5, 0.5f, 1.5f);
  DeviceBuffer<float> dx(x, s), dw(w, s), dy(x.size());
  CK(operatorlib::rmsnorm_f32(dx.ptr, dw.ptr, dy.ptr, tokens, hidden, eps, s));
  const auto y = dy.read(s);
  for (int t = 0; t < tokens; ++t) {
    double ss = 0.0;
    for (int h = 0; h < hidden; ++h) ss += double(x[t * hidden + h]) * x[t * hidden + h];
    const double inv = 1.0 / std::sqrt(ss / hidden + eps);
    for (int h = 0; h < hidden; ++h) {
      const double want = x[t * hidden + h] * inv * w[h];
      const double err = std::fabs(y[t * hidden + h] - want);
      require(err <= 1e-5 * std::fabs(want) + 1e-6, "rmsnorm_f32", err);
    }
  }
  std::printf("rmsnorm_f32=PASS\n");
}

std::vector<double> gemm_ref(const std::vector<float>& a, const std::vector<float>& b, int m,
                             int n, int k) {
  std::vector<double> c(std::size_t(m) * n, 0.0);
  for (int i = 0; i < m; ++i)
    for (int p = 0; p < k; ++p)
      for (int j = 0; j < n; ++j) c[std::size_t(i) * n + j] += double(a[i * k + p]) * b[p * n + j];
  return c;
}

void test_gemm(cudaStream_t s) {
  const int m = 129, n = 257, k = 72;
  const float scale = 1.f / std::sqrt(float(k));
  const auto a = uniform(std::size_t(m) * k, 6, -scale, scale);
  const auto b = uniform(std::size_t(k) * n, 7, -scale, scale);
  const auto want = gemm_ref(a, b, m, n, k);
  {
    DeviceBuffer<float> da(a, s), db(b, s), dc(std::size_t(m) * n);
    CK(operatorlib::gemm_f32(da.ptr, db.ptr, dc.ptr, m, n, k, s));
    const auto c = dc.read(s);
    for (std::size_t i = 0; i < c.size(); ++i) {
      const double err = std::fabs(c[i] - want[i]);
      require(err <= 1e-3 + 1e-3 * std::fabs(want[i]), "gemm_f32", err);
    }
    std::printf("gemm_f32=PASS\n");
  }
  {
    const auto ah = to_half(a), bh = to_half(b);
    const auto want16 = gemm_ref(from_half(ah), from_half(bh), m, n, k);
    DeviceBuffer<__half> da(ah, s), db(bh, s);
    DeviceBuffer<float> dc(std::size_t(m) * n);
    CK(operatorlib::gemm_f16(da.ptr, db.ptr, dc.ptr, m, n, k, s));
    const auto c = dc.read(s);
    for (std::size_t i = 0; i < c.size(); ++i) {
      const double err = std::fabs(c[i] - want16[i]);
      require(err <= 2e-2, "gemm_f16", err);
    }
    std::printf("gemm_f16=PASS\n");
  }
}

// Double-precision attention of one [S, D] head.
void attention_ref(const float* q, const float* k, const float* v, double* o, int s, int d,
                   bool causal) {
  std::vector<double> p(s);
  for (int i = 0; i < s; ++i) {
    const int visible = causal ? i + 1 : s;
    double m = -INFINITY;
    for (int j = 0; j < visible; ++j) {
      double dot = 0.0;
      for (int x = 0; x < d; ++x) dot += double(q[i * d + x]) * k[j * d + x];
      p[j] = dot / std::sqrt(double(d));
      m = std::fmax(m, p[j]);
    }
    double den = 0.0;
    for (int j = 0; j < visible; ++j) den += (p[j] = std::exp(p[j] - m));
    for (int x = 0; x < d; ++x) {
      double acc = 0.0;
      for (int j = 0; j < visible; ++j) acc += p[j] * v[j * d + x];
      o[i * d + x] = acc / den;
    }
  }
}

void test_attention(cudaStream_t s) {
  const int batch = 1, heads = 2, seq = 200, dim = 128;
  const std::size_t count = std::size_t(batch) * heads * seq * dim;
  const auto q = uniform(count, 8, -1.f, 1.f), k = uniform(count, 9, -1.f, 1.f),
             v = uniform(count, 10, -1.f, 1.f);
  std::vector<double> want(count);
  for (bool causal : {false, true}) {
    {
      for (int h = 0; h < batch * heads; ++h) {
        const std::size_t off = std::size_t(h) * seq * dim;
        attention_ref(&q[off], &k[off], &v[off], &want[off], seq, dim, causal);
      }
      DeviceBuffer<float> dq(q, s), dk(k, s), dv(v, s), dout(count);
      CK(operatorlib::attention_f32(dq.ptr, dk.ptr, dv.ptr, dout.ptr, batch, heads, seq, dim,
                                    causal, s));
      const auto o = dout.read(s);
      for (std::size_t i = 0; i < count; ++i) {
        const double err = std::fabs(o[i] - want[i]);
        require(err <= 1e-4 + 1e-4 * std::fabs(want[i]), "attention_f32", err);
      }
    }
    {
      const auto qh = to_half(q), kh = to_half(k), vh = to_half(v);
      const auto qf = from_half(qh), kf = from_half(kh), vf = from_half(vh);
      for (int h = 0; h < batch * heads; ++h) {
        const std::size_t off = std::size_t(h) * seq * dim;
        attention_ref(&qf[off], &kf[off], &vf[off], &want[off], seq, dim, causal);
      }
      DeviceBuffer<__half> dq(qh, s), dk(kh, s), dv(vh, s);
      DeviceBuffer<float> dout(count);
      CK(operatorlib::attention_f16(dq.ptr, dk.ptr, dv.ptr, dout.ptr, batch, heads, seq, dim,
                                    causal, s));
      const auto o = dout.read(s);
      for (std::size_t i = 0; i < count; ++i) {
        const double err = std::fabs(o[i] - want[i]);
        require(err <= 2e-2, "attention_f16", err);
      }
    }
  }
  std::printf("attention_f32=PASS\nattention_f16=PASS\n");
}

void test_argument_errors(cudaStream_t s) {
  float* f = reinterpret_cast<float*>(0x1000);
  const cudaError_t bad = cudaErrorInvalidValue;
  require(operatorlib::reduce_sum_f32(nullptr, f, 10, s) == bad, "reduce null", 1);
  require(operatorlib::softmax_f32(f, f, 0, 4, s) == bad, "softmax rows 0", 1);
  require(operatorlib::transpose_f32(f, f, 4, -1, s) == bad, "transpose cols < 0", 1);
  require(operatorlib::rmsnorm_f32(f, f, f, 4, 4, 0.f, s) == bad, "rmsnorm eps 0", 1);
  require(operatorlib::gemm_f32(f, f, nullptr, 4, 4, 4, s) == bad, "gemm null", 1);
  require(operatorlib::attention_f32(f, f, f, f, 1, 1, 4, 129, false, s) == bad,
          "attention head_dim 129", 1);
  CK(cudaGetLastError());
  std::printf("argument_errors=PASS\n");
}

}  // namespace

int main() {
  cudaStream_t s;
  CK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  test_argument_errors(s);
  test_reduce(s);
  test_softmax(s);
  test_transpose(s);
  test_rmsnorm(s);
  test_gemm(s);
  test_attention(s);
  CK(cudaStreamDestroy(s));
  std::printf("operatorlib_b200_smoke=PASS\n");
  return 0;
}
