// Row softmax over the last dimension (reference src/softmax.cu:52-202).
//
// Every row length up to 32768 floats runs single-pass from registers
// (row_cache.cuh): one HBM read and one HBM write per element, for aligned
// and ragged rows alike (the reference's general kernel reads twice and
// writes twice, src/softmax.cu:119-176).  Longer rows use a two-read
// streaming kernel with an online (max, sum) first pass.
//
// Arithmetic per row, the reference's steps: m = max(x); e = e^(x - m);
// s = sum(e); y = e * (1 / s).  e^(x - m) is 2^((x - m) log2 e) on the MUFU
// ex2 unit: with x - m formed first, its relative error is at most about
// 2.4e-7 + 6e-8 |x - m| (the instruction's ~2 ulp plus the rounding of the
// scaled argument), inside the 1e-5 gate for every |x - m| before the result
// underflows, where CUDA's expf spends several FP32-pipe instructions per
// element.
#include "row_cache.cuh"

namespace opl {

namespace {
__device__ __forceinline__ float exp_ex2(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
  return y;
}
}  // namespace

template <int kGroup, int kBlock, int kItems, bool kVec>
__global__ void __launch_bounds__(kBlock)
    softmax_cached_kernel(const float* __restrict__ input,
                          float* __restrict__ output, int rows, int cols) {
  pdl_begin();
  constexpr int kWidth = RowElems<kVec>::kWidth;
  constexpr int kRowsPerBlock = kBlock / kGroup;
  __shared__ float scratch_max[kBlock / 32];
  __shared__ float scratch_sum[kBlock / 32];
  const int t = threadIdx.x % kGroup;
  const int row = blockIdx.x * kRowsPerBlock + threadIdx.x / kGroup;
  if (kGroup == 32 && row >= rows) return;  // whole warp leaves together
  const std::size_t offset = static_cast<std::size_t>(row) * cols;

  float v[kItems * kWidth];
  load_row<kGroup, kItems, kVec>(input + offset, cols, t, -FLT_MAX, v);
  float m = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < kItems * kWidth; ++i) m = fmaxf(m, v[i]);
  m = group_reduce<kGroup, kBlock, true>(m, scratch_max);

  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < kItems * kWidth; ++i) {
    v[i] = exp_ex2(v[i] - m);  // padding slots: e^(-FLT_MAX - m) == 0
    s += v[i];
  }
  s = group_reduce<kGroup, kBlock, false>(s, scratch_sum);
  const float inverse = 1.0f / s;
#pragma unroll
  for (int i = 0; i < kItems * kWidth; ++i) v[i] *= inverse;
  store_row<kGroup, kItems, kVec>(output + offset, cols, t, v);
}

// Rows longer than the register cache: pass 1 reads the row once keeping an
// online (max, sum of exp) per thread, merged across the CTA; pass 2 reads it
// again and writes e^(x - m) / s.
constexpr int kLongThreads = 1024;

__global__ void __launch_bounds__(kLongThreads)
    softmax_long_kernel(const float* __restrict__ input, float* __restrict__ output,
                        int cols) {
  __shared__ float sm[kLongThreads / 32];
  __shared__ float ss[kLongThreads / 32];
  const std::size_t offset = static_cast<std::size_t>(blockIdx.x) * cols;
  const float* row = input + offset;
  float m = -FLT_MAX;
  float s = 0.0f;
  for (int c = threadIdx.x; c < cols; c += kLongThreads) {
    const float x = row[c];
    if (x > m) {
      s = s * exp_ex2(m - x) + 1.0f;
      m = x;
    } else {
      s += exp_ex2(x - m);
    }
  }
  // Merge (m, s) pairs: first the CTA maximum, then rescaled sums.
  const float block_max = group_reduce<kLongThreads, kLongThreads, true>(m, sm);
  s = s * exp_ex2(m - block_max);
  const float block_sum = group_reduce<kLongThreads, kLongThreads, false>(s, ss);
  const float inverse = 1.0f / block_sum;
  float* out = output + offset;
  for (int c = threadIdx.x; c < cols; c += kLongThreads)
    st_stream(out + c, exp_ex2(row[c] - block_max) * inverse);
}

}  // namespace opl

extern "C" int opl_softmax_f32(const float* input, float* output, int rows,
                               int cols, opl_stream_t stream) {
  using namespace opl;
  if (input == nullptr || output == nullptr || rows <= 0 || cols <= 0)
    return cudaErrorInvalidValue;
  const bool vec = (cols % 4 == 0) && aligned16(input) && aligned16(output);
  RowShape shape;
  if (!pick_row_shape(vec ? cols / 4 : cols, vec, &shape)) {
    softmax_long_kernel<<<rows, kLongThreads, 0, stream>>>(input, output, cols);
    return cudaGetLastError();
  }
#define OPL_SOFTMAX_LAUNCH(G, B, I, V)                                          \
  {                                                                             \
    const int rows_per_block = (B) / (G);                                       \
    const int blocks = (rows + rows_per_block - 1) / rows_per_block;            \
    const cudaError_t e = launch_pdl(softmax_cached_kernel<G, B, I, V>,         \
                                     dim3(blocks), dim3(B), stream, input,      \
                                     output, rows, cols);                       \
    if (e != cudaSuccess) return e;                                             \
  }
  OPL_ROW_DISPATCH(shape, vec, OPL_SOFTMAX_LAUNCH);
#undef OPL_SOFTMAX_LAUNCH
  return cudaGetLastError();
}
