// Reduce-sum FP32 -> one float (reference src/reduce.cu:14-69).
//
// B200 design: every thread issues eight 128-bit streaming loads at once and
// the grid is sized so that, for inputs up to kReduceMaxCtas * 8 KB x 4
// (134 M floats), each thread makes a single pass -- about two waves of
// 256-thread CTAs, eight resident per SM, 256 KB of loads in flight per SM,
// with retiring CTAs replaced at once by the block scheduler (measured on
// B200: faster than grid-stride loops, contiguous chunks per CTA or a
// bulk-copy ring of 16 KB stages).  Larger inputs loop grid-stride.  Each
// float4 is summed in FP32 and accumulated in FP64; each CTA writes one FP64
// partial and a finalize kernel sums the partials in a fixed order.  No
// atomics, so the result is deterministic (the reference combines block
// partials with a float atomicAdd, src/reduce.cu:46, whose order varies run
// to run).  The finalize kernel is launched with programmatic dependent
// launch so its launch latency overlaps the partial kernel.  The partials
// live in a stream-ordered workspace (cudaMallocAsync / cudaFreeAsync on the
// caller's stream).
#include "opl_common.cuh"
#include "reduce_impl.cuh"

namespace opl {

namespace {
constexpr int kUnroll = 8;
}  // namespace

// The input split into its float4 body and the (at most three) scalars
// before the first 16-byte boundary and after the last whole float4; the
// host computes it so the hot loop carries no edge arithmetic (the edge
// checks in every thread cost ~0.5 us at 16M floats).
struct ReduceSplit {
  const float4* body;
  std::size_t vectors;
  const float* head;
  const float* tail;
  int n_head, n_tail;
};

ReduceSplit reduce_split(const float* input, std::size_t n) {
  const std::uintptr_t address = reinterpret_cast<std::uintptr_t>(input);
  std::size_t head = ((16u - (address & 15u)) & 15u) / 4u;
  if (head > n) head = n;
  const std::size_t vectors = (n - head) / 4;
  const std::size_t tail_start = head + vectors * 4;
  return ReduceSplit{reinterpret_cast<const float4*>(input + head), vectors, input,
                     input + tail_start, static_cast<int>(head),
                     static_cast<int>(n - tail_start)};
}

__global__ void __launch_bounds__(kReduceThreads)
    reduce_partials_kernel(ReduceSplit in, double* __restrict__ partials) {
  // Launched with programmatic dependent launch: scheduled while the
  // previous kernel on the stream drains, global reads only after it is done.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // CTA b covers kUnroll consecutive CTA-widths of float4 per pass.
  const std::size_t span = static_cast<std::size_t>(kReduceThreads) * kUnroll;
  const std::size_t stride = static_cast<std::size_t>(gridDim.x) * span;
  double acc = 0.0;
  std::size_t i = static_cast<std::size_t>(blockIdx.x) * span + threadIdx.x;
  for (; i + (kUnroll - 1) * kReduceThreads < in.vectors; i += stride) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = ld_stream(in.body + i + u * kReduceThreads);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      acc += static_cast<double>((v[u].x + v[u].y) + (v[u].z + v[u].w));
  }
  // The ragged last span (only the CTA that reaches it).
  for (; i < in.vectors; i += kReduceThreads) {
    const float4 a = ld_stream(in.body + i);
    acc += static_cast<double>((a.x + a.y) + (a.z + a.w));
  }
  if (blockIdx.x == 0) {  // the edge scalars, on CTA 0's first threads
    if (static_cast<int>(threadIdx.x) < in.n_head) acc += static_cast<double>(in.head[threadIdx.x]);
    if (static_cast<int>(threadIdx.x) < in.n_tail) acc += static_cast<double>(in.tail[threadIdx.x]);
  }

  // Let the dependent finalize grid start launching while partials drain.
  asm volatile("griddepcontrol.launch_dependents;");
  acc = block_sum_fixed(acc);
  if (threadIdx.x == 0) partials[blockIdx.x] = acc;
}

// kReduceThreads threads; thread t sums partials t, t + kReduceThreads, ...
// then a fixed tree.
__global__ void __launch_bounds__(kReduceThreads)
    reduce_finalize_kernel(const double* __restrict__ partials, int count,
                           float* __restrict__ output_f32,
                           double* __restrict__ output_f64) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  double v = sum_partials_strided(partials, count);
  v = block_sum_fixed(v);
  if (threadIdx.x == 0) {
    if (output_f32 != nullptr) *output_f32 = static_cast<float>(v);
    if (output_f64 != nullptr) *output_f64 = v;
  }
}

int reduce_grid(const float* input, std::size_t n) {
  // Exactly the CTAs the aligned float4 body needs (the scalar head and tail
  // ride along on the first threads), at least one.
  const std::uintptr_t address = reinterpret_cast<std::uintptr_t>(input);
  std::size_t head = ((16u - (address & 15u)) & 15u) / 4u;
  if (head > n) head = n;
  const std::size_t vectors = (n - head) / 4;
  const std::size_t span = static_cast<std::size_t>(kReduceThreads) * kUnroll;
  std::size_t blocks = (vectors + span - 1) / span;
  if (blocks > static_cast<std::size_t>(kReduceMaxCtas)) blocks = kReduceMaxCtas;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

cudaError_t reduce_partials_launch(const float* input, std::size_t n, double* partials,
                                   int blocks, cudaStream_t stream) {
  return launch_pdl(reduce_partials_kernel, dim3(blocks), dim3(kReduceThreads), stream,
                    reduce_split(input, n), partials);
}

cudaError_t reduce_enqueue(const float* input, std::size_t n, double* partials,
                           int blocks, float* out_f32, double* out_f64,
                           cudaStream_t stream) {
  cudaError_t error = reduce_partials_launch(input, n, partials, blocks, stream);
  if (error != cudaSuccess) return error;

  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(1);
  config.blockDim = dim3(kReduceThreads);
  config.dynamicSmemBytes = 0;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  const double* partials_const = partials;
  return cudaLaunchKernelEx(&config, reduce_finalize_kernel, partials_const,
                            blocks, out_f32, out_f64);
}

static int reduce_with_workspace(const float* input, std::size_t n,
                                 float* out_f32, double* out_f64,
                                 cudaStream_t stream) {
  const int blocks = reduce_grid(input, n);
  void* workspace = nullptr;
  cudaError_t error = cudaMallocAsync(&workspace, blocks * sizeof(double), stream);
  if (error != cudaSuccess) return error;
  error = reduce_enqueue(input, n, static_cast<double*>(workspace), blocks,
                         out_f32, out_f64, stream);
  const cudaError_t free_error = cudaFreeAsync(workspace, stream);
  if (error != cudaSuccess) return error;
  return free_error;
}

}  // namespace opl

extern "C" int opl_reduce_sum_f32(const float* input, float* output, size_t n,
                                  opl_stream_t stream) {
  if (input == nullptr || output == nullptr || n == 0) return cudaErrorInvalidValue;
  return opl::reduce_with_workspace(input, n, output, nullptr, stream);
}

extern "C" int opl_reduce_sum_partial_f64(const float* input, double* output,
                                          size_t n, opl_stream_t stream) {
  if (input == nullptr || output == nullptr || n == 0) return cudaErrorInvalidValue;
  return opl::reduce_with_workspace(input, n, nullptr, output, stream);
}
