// Exposes the reference's CPU RMSNorm loop (rmsnorm/rmsnorm_v3.cu:154-172) by
// compiling that source in this translation unit (its main() renamed).
// Test/bench infrastructure only.
#define main opl_ref_unused_main_rmsnorm
#include REF_SOURCE
#undef main

extern "C" void ref_cpu_rmsnorm(const float* x, const float* w, float* y,
                                int tokens, int hidden, float eps) {
  const std::vector<float> input(x, x + static_cast<size_t>(tokens) * hidden);
  const std::vector<float> weight(w, w + hidden);
  std::vector<float> output;
  cpu_rmsnorm(input, weight, &output, tokens, hidden, eps);
  std::copy(output.begin(), output.end(), y);
}
