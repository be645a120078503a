// Reduce-sum FP32 -> one float (reference src/reduce.cu:14-69).
//
// B200 design: a grid sized to the SM count (4 x 512-thread CTAs per SM) in
// which every thread keeps four 128-bit streaming loads in flight, sums each
// float4 in FP32 and accumulates in FP64.  Each CTA writes one FP64 partial;
// a one-warp finalize kernel sums the partials in a fixed order.  No atomics,
// so the result is deterministic (the reference combines block partials with
// a float atomicAdd, src/reduce.cu:46, whose order varies run to run).  The
// finalize kernel is launched with programmatic dependent launch so its launch
// latency overlaps the partial kernel.  The partials live in a stream-ordered
// workspace (cudaMallocAsync / cudaFreeAsync on the caller's stream).
#include "opl_common.cuh"
#include "reduce_impl.cuh"

namespace opl {

__global__ void __launch_bounds__(kReduceThreads)
    reduce_partials_kernel(const float* __restrict__ input, std::size_t n,
                           double* __restrict__ partials) {
  __shared__ double warp_partials[kReduceThreads / 32];
  // Scalars before the first 16-byte boundary, then float4 body, then tail.
  const std::uintptr_t address = reinterpret_cast<std::uintptr_t>(input);
  std::size_t head = ((16u - (address & 15u)) & 15u) / 4u;
  if (head > n) head = n;
  const std::size_t vectors = (n - head) / 4;
  const std::size_t tail_start = head + vectors * 4;
  const float4* body = reinterpret_cast<const float4*>(input + head);

  const std::size_t tid =
      static_cast<std::size_t>(blockIdx.x) * kReduceThreads + threadIdx.x;
  const std::size_t stride = static_cast<std::size_t>(gridDim.x) * kReduceThreads;

  double acc = 0.0;
  std::size_t i = tid;
  for (; i + 3 * stride < vectors; i += 4 * stride) {
    const float4 a = ld_stream(body + i);
    const float4 b = ld_stream(body + i + stride);
    const float4 c = ld_stream(body + i + 2 * stride);
    const float4 d = ld_stream(body + i + 3 * stride);
    acc += static_cast<double>((a.x + a.y) + (a.z + a.w));
    acc += static_cast<double>((b.x + b.y) + (b.z + b.w));
    acc += static_cast<double>((c.x + c.y) + (c.z + c.w));
    acc += static_cast<double>((d.x + d.y) + (d.z + d.w));
  }
  for (; i < vectors; i += stride) {
    const float4 a = ld_stream(body + i);
    acc += static_cast<double>((a.x + a.y) + (a.z + a.w));
  }
  if (tid < head) acc += static_cast<double>(input[tid]);
  if (tid < n - tail_start) acc += static_cast<double>(input[tail_start + tid]);

  acc = warp_sum(acc);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (lane == 0) warp_partials[warp] = acc;
  __syncthreads();
  // Let the dependent finalize grid start launching while partials drain.
  asm volatile("griddepcontrol.launch_dependents;");
  if (warp == 0) {
    double v = lane < kReduceThreads / 32 ? warp_partials[lane] : 0.0;
    v = warp_sum(v);
    if (lane == 0) partials[blockIdx.x] = v;
  }
}

// One warp; lane l sums partials l, l+32, ... then a fixed xor-tree.
__global__ void __launch_bounds__(32)
    reduce_finalize_kernel(const double* __restrict__ partials, int count,
                           float* __restrict__ output_f32,
                           double* __restrict__ output_f64) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  double v = 0.0;
  for (int i = threadIdx.x; i < count; i += 32) v += partials[i];
  v = warp_sum(v);
  if (threadIdx.x == 0) {
    if (output_f32 != nullptr) *output_f32 = static_cast<float>(v);
    if (output_f64 != nullptr) *output_f64 = v;
  }
}

int reduce_grid(std::size_t n) {
  const std::size_t vectors = n / 4 + 1;
  std::size_t blocks = (vectors + kReduceThreads * 4 - 1) / (kReduceThreads * 4);
  const std::size_t cap = static_cast<std::size_t>(sm_count()) * kReduceCtasPerSm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

cudaError_t reduce_enqueue(const float* input, std::size_t n, double* partials,
                           int blocks, float* out_f32, double* out_f64,
                           cudaStream_t stream) {
  reduce_partials_kernel<<<blocks, kReduceThreads, 0, stream>>>(input, n,
                                                                 partials);
  cudaError_t error = cudaGetLastError();
  if (error != cudaSuccess) return error;

  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(1);
  config.blockDim = dim3(32);
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
  const int blocks = reduce_grid(n);
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
