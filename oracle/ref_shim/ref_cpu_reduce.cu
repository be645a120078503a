// Exposes the reference's own CPU verification loop for reduce-sum
// (reduce/reduce_v3.cu:125-128) by compiling that source file in this
// translation unit (its main() renamed).  REF_SOURCE is set by
// oracle/build_oracle.py.  Test/bench infrastructure only.
#define main opl_ref_unused_main_reduce
#include REF_SOURCE
#undef main

extern "C" float ref_cpu_reduce_sum(const float* x, size_t n) {
  const std::vector<float> input(x, x + n);
  return cpu_reference(input);
}
