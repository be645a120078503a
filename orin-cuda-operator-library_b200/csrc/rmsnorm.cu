// RMSNorm: y = x * rsqrt(sum(x^2) / hidden + eps) * w per token row
// (reference src/rmsnorm.cu:27-95).
//
// Rows up to 32768 elements are read once into registers (row_cache.cuh), so
// x crosses HBM once (the reference re-reads x in its second pass,
// src/rmsnorm.cu:43-51); w (one row) stays L2-resident across rows.  Longer
// rows use a two-read streaming kernel.  Per element the product is formed as
// (x * inv_rms) * w, the reference's order.
#include "row_cache.cuh"

namespace opl {

template <int kGroup, int kBlock, int kItems, bool kVec>
__global__ void __launch_bounds__(kBlock)
    rmsnorm_cached_kernel(const float* __restrict__ input,
                          const float* __restrict__ weight,
                          float* __restrict__ output, int tokens, int hidden,
                          float epsilon) {
  constexpr int kWidth = RowElems<kVec>::kWidth;
  constexpr int kRowsPerBlock = kBlock / kGroup;
  __shared__ float scratch[kBlock / 32];
  const int t = threadIdx.x % kGroup;
  const int row = blockIdx.x * kRowsPerBlock + threadIdx.x / kGroup;
  if (kGroup == 32 && row >= tokens) return;
  const std::size_t offset = static_cast<std::size_t>(row) * hidden;

  float v[kItems * kWidth];
  load_row<kGroup, kItems, kVec>(input + offset, hidden, t, 0.0f, v);
  float sq = 0.0f;
#pragma unroll
  for (int i = 0; i < kItems * kWidth; ++i) sq = fmaf(v[i], v[i], sq);
  sq = group_reduce<kGroup, kBlock, false>(sq, scratch);
  const float inverse_rms = rsqrtf(sq / static_cast<float>(hidden) + epsilon);

  if constexpr (kVec) {
    const float4* w4 = reinterpret_cast<const float4*>(weight);
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const int idx = t + j * kGroup;
      if (idx < (hidden >> 2)) {
        const float4 w = __ldg(w4 + idx);
        v[4 * j + 0] = v[4 * j + 0] * inverse_rms * w.x;
        v[4 * j + 1] = v[4 * j + 1] * inverse_rms * w.y;
        v[4 * j + 2] = v[4 * j + 2] * inverse_rms * w.z;
        v[4 * j + 3] = v[4 * j + 3] * inverse_rms * w.w;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const int col = t + j * kGroup;
      if (col < hidden) v[j] = v[j] * inverse_rms * __ldg(weight + col);
    }
  }
  store_row<kGroup, kItems, kVec>(output + offset, hidden, t, v);
}

constexpr int kRmsLongThreads = 1024;

__global__ void __launch_bounds__(kRmsLongThreads)
    rmsnorm_long_kernel(const float* __restrict__ input,
                        const float* __restrict__ weight,
                        float* __restrict__ output, int hidden, float epsilon) {
  __shared__ float scratch[kRmsLongThreads / 32];
  const std::size_t offset = static_cast<std::size_t>(blockIdx.x) * hidden;
  const float* row = input + offset;
  float sq = 0.0f;
  for (int c = threadIdx.x; c < hidden; c += kRmsLongThreads)
    sq = fmaf(row[c], row[c], sq);
  sq = group_reduce<kRmsLongThreads, kRmsLongThreads, false>(sq, scratch);
  const float inverse_rms = rsqrtf(sq / static_cast<float>(hidden) + epsilon);
  float* out = output + offset;
  for (int c = threadIdx.x; c < hidden; c += kRmsLongThreads)
    st_stream(out + c, row[c] * inverse_rms * __ldg(weight + c));
}

}  // namespace opl

extern "C" int opl_rmsnorm_f32(const float* input, const float* weight,
                               float* output, int tokens, int hidden,
                               float epsilon, opl_stream_t stream) {
  using namespace opl;
  // `!(epsilon > 0)` also rejects NaN.
  if (input == nullptr || weight == nullptr || output == nullptr ||
      tokens <= 0 || hidden <= 0 || !(epsilon > 0.0f))
    return cudaErrorInvalidValue;
  const bool vec = (hidden % 4 == 0) && aligned16(input) && aligned16(output) &&
                   aligned16(weight);
  RowShape shape;
  if (!pick_row_shape(vec ? hidden / 4 : hidden, vec, &shape)) {
    rmsnorm_long_kernel<<<tokens, kRmsLongThreads, 0, stream>>>(
        input, weight, output, hidden, epsilon);
    return cudaGetLastError();
  }
#define OPL_RMSNORM_LAUNCH(G, B, I, V)                                          \
  {                                                                             \
    const int rows_per_block = (B) / (G);                                       \
    const int blocks = (tokens + rows_per_block - 1) / rows_per_block;          \
    rmsnorm_cached_kernel<G, B, I, V><<<blocks, B, 0, stream>>>(                \
        input, weight, output, tokens, hidden, epsilon);                        \
  }
  OPL_ROW_DISPATCH(shape, vec, OPL_RMSNORM_LAUNCH);
#undef OPL_RMSNORM_LAUNCH
  return cudaGetLastError();
}
