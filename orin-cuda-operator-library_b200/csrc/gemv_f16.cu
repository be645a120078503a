// Skinny FP16 GEMM, M <= 16 (decode-style calls; reference src/gemm.cu:
// 455-479 sends these to wmma_small_m_kernel / hgemm_scalar_kernel, the path
// its report calls the "final weak point").
//
// With so few rows the product is bound by streaming B (K x N FP16) from
// HBM, not by math, and a 128-row tensor-core tile would give only N/256
// CTAs.  Here each warp owns a 256-column slab of B and one K chunk: lane l
// loads the 16 bytes (8 columns) at columns 8l..8l+7 of every row of its
// chunk -- 512 contiguous bytes per warp per row, eight rows in flight per
// lane -- and accumulates all M rows in FP32 registers, reading A (converted
// to FP32 once into shared memory) as broadcasts.  K is split across CTAs to
// fill the GPU; the per-split partial sums land in a stream-ordered
// workspace and a second kernel adds them in a fixed order, so results are
// deterministic.  Products of two FP16 values are exact in FP32.
#include "gemm_simt.cuh"

namespace opl {

namespace {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kSlab = 256;  // columns per warp (32 lanes x 8)
constexpr int kRowsInFlight = 8;

template <int M>
__global__ void __launch_bounds__(kGemvThreads)
    gemv_f16_partial_kernel(const __half* __restrict__ a, const __half* __restrict__ b,
                            float* __restrict__ partial, int m, int n, int k,
                            int k_chunk) {
  extern __shared__ float a_s[];  // [M][k_chunk]
  const int split = blockIdx.y;
  const int k0 = split * k_chunk;
  const int kc = min(k_chunk, k - k0);
  for (int i = threadIdx.x; i < M * kc; i += kGemvThreads) {
    const int r = i / kc;
    const int kk = i - r * kc;
    a_s[r * k_chunk + kk] =
        r < m ? __half2float(a[static_cast<size_t>(r) * k + k0 + kk]) : 0.0f;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int col = (blockIdx.x * kGemvWarps + warp) * kSlab + lane * 8;
  if (col >= n) return;  // n % 8 == 0 on this path: a group is all in or out
  float acc[M][8];
#pragma unroll
  for (int r = 0; r < M; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[r][c] = 0.0f;

  const uint4* bp = reinterpret_cast<const uint4*>(b + static_cast<size_t>(k0) * n + col);
  const size_t row_stride = static_cast<size_t>(n) / 8;  // in uint4
  for (int kk = 0; kk < kc; kk += kRowsInFlight) {
    uint4 raw[kRowsInFlight];
#pragma unroll
    for (int u = 0; u < kRowsInFlight; ++u)
      raw[u] = kk + u < kc ? __ldg(bp + (kk + u) * row_stride) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int u = 0; u < kRowsInFlight; ++u) {
      if (kk + u >= kc) break;
      const __half2* h = reinterpret_cast<const __half2*>(&raw[u]);
      float bv[8];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float2 f = __half22float2(h[c]);
        bv[2 * c] = f.x;
        bv[2 * c + 1] = f.y;
      }
#pragma unroll
      for (int r = 0; r < M; ++r) {
        const float av = a_s[r * k_chunk + kk + u];
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[r][c] = fmaf(av, bv[c], acc[r][c]);
      }
    }
  }
  float* out = partial + static_cast<size_t>(split) * m * n + col;
#pragma unroll
  for (int r = 0; r < M; ++r) {
    if (r >= m) break;
    float4* o = reinterpret_cast<float4*>(out + static_cast<size_t>(r) * n);
    o[0] = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    o[1] = make_float4(acc[r][4], acc[r][5], acc[r][6], acc[r][7]);
  }
}

// C[i] = sum over splits s = 0, 1, ... of partial[s][i], in that order.
__global__ void __launch_bounds__(256)
    gemv_reduce_kernel(const float* __restrict__ partial, float* __restrict__ c,
                       size_t count, int splits) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float s = 0.0f;
    for (int p = 0; p < splits; ++p) s += partial[static_cast<size_t>(p) * count + i];
    c[i] = s;
  }
}

template <int M>
cudaError_t launch_gemv(const __half* a, const __half* b, float* c, int m, int n, int k,
                        cudaStream_t stream) {
  const int col_blocks = (n + kGemvWarps * kSlab - 1) / (kGemvWarps * kSlab);
  // About 3 CTAs per SM (enough bytes in flight to stream B at full HBM
  // rate), K chunks of at least 16 rows, and partial sums no larger than
  // half of B (splits * M * N * 4 <= K * N * 2 / 2).
  int splits = (3 * sm_count() + col_blocks - 1) / col_blocks;
  splits = max(1, min(splits, min((k + 15) / 16, max(1, k / (4 * M)))));
  int k_chunk = (k + splits - 1) / splits;
  k_chunk = (k_chunk + kRowsInFlight - 1) / kRowsInFlight * kRowsInFlight;
  splits = (k + k_chunk - 1) / k_chunk;
  const size_t smem = sizeof(float) * M * k_chunk;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(gemv_f16_partial_kernel<M>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const size_t count = static_cast<size_t>(m) * n;
  void* ws = nullptr;
  cudaError_t e = cudaMallocAsync(&ws, count * splits * sizeof(float), stream);
  if (e != cudaSuccess) return e;
  float* partial = static_cast<float*>(ws);
  gemv_f16_partial_kernel<M><<<dim3(col_blocks, splits), kGemvThreads, smem, stream>>>(
      a, b, partial, m, n, k, k_chunk);
  e = cudaGetLastError();
  if (e == cudaSuccess) {
    const size_t want = (count + 255) / 256;
    const int blocks = static_cast<int>(want < static_cast<size_t>(8 * sm_count()) ? want : 8 * sm_count());
    gemv_reduce_kernel<<<blocks, 256, 0, stream>>>(partial, c, count, splits);
    e = cudaGetLastError();
  }
  const cudaError_t f = cudaFreeAsync(ws, stream);
  return e != cudaSuccess ? e : f;
}

}  // namespace

bool gemv_f16_supported(const void* b, const void* c, int m, int n) {
  return m >= 1 && m <= 16 && n % 8 == 0 && aligned16(b) && aligned16(c);
}

cudaError_t gemv_f16(const __half* a, const __half* b, float* c, int m, int n, int k,
                     cudaStream_t stream) {
  if (m <= 1) return launch_gemv<1>(a, b, c, m, n, k, stream);
  if (m <= 2) return launch_gemv<2>(a, b, c, m, n, k, stream);
  if (m <= 4) return launch_gemv<4>(a, b, c, m, n, k, stream);
  if (m <= 8) return launch_gemv<8>(a, b, c, m, n, k, stream);
  return launch_gemv<16>(a, b, c, m, n, k, stream);
}

}  // namespace opl
