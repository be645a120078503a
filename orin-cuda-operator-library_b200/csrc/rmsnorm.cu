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

// At most 64 registers (1024 threads per SM), as the softmax kernel of the
// same shape: 4097 x 1023 is 1,025 CTAs of 128 threads, one wave at 8 CTAs
// per SM but 1.15 waves at the 6 that 80 registers allowed.
template <int kGroup, int kBlock, int kItems, bool kVec>
__global__ void __launch_bounds__(kBlock, 1024 / kBlock)
    rmsnorm_cached_kernel(const float* __restrict__ input,
                          const float* __restrict__ weight,
                          float* __restrict__ output, int tokens, int hidden,
                          float epsilon) {
  pdl_begin();
  constexpr int kWidth = RowElems<kVec>::kWidth;
  constexpr int kRowsPerBlock = kBlock / kGroup;
  __shared__ float scratch[kBlock / 32];
  // Scalar warp-per-row shapes: w (at most 32 kItems floats) staged in shared
  // memory once per CTA, after the row's own loads are issued.
  constexpr bool kStageW = !kVec && kGroup == 32;
  __shared__ float w_s[kStageW ? kItems * 32 : 1];
  const int t = threadIdx.x % kGroup;
  const int row = blockIdx.x * kRowsPerBlock + threadIdx.x / kGroup;
  const bool active = !(kGroup == 32 && row >= tokens);
  const std::size_t offset = static_cast<std::size_t>(active ? row : 0) * hidden;

  float v[kItems * kWidth];
  if (active) load_row<kGroup, kItems, kVec>(input + offset, hidden, t, 0.0f, v);
  if constexpr (kStageW) {
    for (int c = threadIdx.x; c < hidden; c += kBlock) w_s[c] = ld_ro(weight + c);
    __syncthreads();
  }
  if (!active) return;
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
        const float4 w = ld_ro(w4 + idx);
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
      if constexpr (kStageW) {
        if (col < hidden) v[j] = v[j] * inverse_rms * w_s[col];
      } else {
        if (col < hidden) v[j] = v[j] * inverse_rms * ld_ro(weight + col);
      }
    }
  }
  store_row<kGroup, kItems, kVec>(output + offset, hidden, t, v);
}

// Rows of 2049..4096 floats (16-byte aligned): one 128-thread CTA per row;
// each thread keeps 4 of its 8 float4 in registers and streams the other 4
// into shared memory with cp.async (16-byte copies that hold no registers
// while in flight).  At <= 32 registers and 8 KB of shared memory, 16 CTAs
// fit per SM, so every row of 2048 x 4096 is in flight at once; caching the
// whole row in registers (64 per thread) allows only 8 CTAs per SM and the
// grid runs in 1.73 waves.
constexpr int kRmsSplitThreads = 128;

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gmem_src)
               : "memory");
}

__global__ void __launch_bounds__(kRmsSplitThreads, 16)
    rmsnorm_split_kernel(const float* __restrict__ input, const float* __restrict__ weight,
                         float* __restrict__ output, int hidden, float epsilon) {
  __shared__ __align__(16) float4 half_row[4 * kRmsSplitThreads];
  __shared__ float scratch[kRmsSplitThreads / 32];
  const int t = threadIdx.x;
  const int vectors = hidden >> 2;  // 513 .. 1024
  const float4* x4 = reinterpret_cast<const float4*>(input + static_cast<size_t>(blockIdx.x) * hidden);
  // Slots t + 128*j: j = 0..3 in registers, j = 4..7 through shared memory.
#pragma unroll
  for (int j = 4; j < 8; ++j) {
    const int idx = t + j * kRmsSplitThreads;
    if (idx < vectors) cp_async16(&half_row[t + (j - 4) * kRmsSplitThreads], x4 + idx);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  float4 v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = ld_stream(x4 + t + j * kRmsSplitThreads);  // 4*128 < 513
  float sq = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sq = fmaf(v[j].x, v[j].x, sq);
    sq = fmaf(v[j].y, v[j].y, sq);
    sq = fmaf(v[j].z, v[j].z, sq);
    sq = fmaf(v[j].w, v[j].w, sq);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");  // each thread reads only its own copies
#pragma unroll
  for (int j = 4; j < 8; ++j) {
    if (t + j * kRmsSplitThreads < vectors) {
      const float4 u = half_row[t + (j - 4) * kRmsSplitThreads];
      sq = fmaf(u.x, u.x, sq);
      sq = fmaf(u.y, u.y, sq);
      sq = fmaf(u.z, u.z, sq);
      sq = fmaf(u.w, u.w, sq);
    }
  }
  sq = group_reduce<kRmsSplitThreads, kRmsSplitThreads, false>(sq, scratch);
  const float inverse_rms = rsqrtf(sq / static_cast<float>(hidden) + epsilon);
  const float4* w4 = reinterpret_cast<const float4*>(weight);
  float4* y4 = reinterpret_cast<float4*>(output + static_cast<size_t>(blockIdx.x) * hidden);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int idx = t + j * kRmsSplitThreads;
    if (idx < vectors) {
      const float4 u = j < 4 ? v[j] : half_row[t + (j - 4) * kRmsSplitThreads];
      const float4 w = ld_ro(w4 + idx);
      st_stream(y4 + idx, make_float4(u.x * inverse_rms * w.x, u.y * inverse_rms * w.y,
                                      u.z * inverse_rms * w.z, u.w * inverse_rms * w.w));
    }
  }
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
    st_stream(out + c, row[c] * inverse_rms * ld_ro(weight + c));
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
  if (vec && hidden > 2048 && hidden <= 4096) {
    rmsnorm_split_kernel<<<tokens, kRmsSplitThreads, 0, stream>>>(input, weight, output,
                                                                  hidden, epsilon);
    return cudaGetLastError();
  }
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
    const cudaError_t e = launch_pdl(rmsnorm_cached_kernel<G, B, I, V>,         \
                                     dim3(blocks), dim3(B), stream, input,      \
                                     weight, output, tokens, hidden, epsilon);  \
    if (e != cudaSuccess) return e;                                             \
  }
  OPL_ROW_DISPATCH(shape, vec, OPL_RMSNORM_LAUNCH);
#undef OPL_RMSNORM_LAUNCH
  return cudaGetLastError();
}
