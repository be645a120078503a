// Exposes the reference's CPU softmax loop (softmax/softmax_v4.cu:253-268) by
// compiling that source in this translation unit (its main() renamed).
// Test/bench infrastructure only.
#define main opl_ref_unused_main_softmax
#include REF_SOURCE
#undef main

extern "C" void ref_cpu_softmax(const float* x, float* y, int rows, int cols) {
  const std::vector<float> input(x, x + static_cast<size_t>(rows) * cols);
  std::vector<float> output;
  cpu_softmax(input, &output, rows, cols);
  std::copy(output.begin(), output.end(), y);
}
