// FP32-FFMA GEMM, row-major C[M,N] = A[M,K] * B[K,N]
// (reference src/gemm.cu:59-216 and :440-453).
//
// 128x128 CTA tile, K step 8, 256 threads each owning an 8x8 register tile
// (updated with packed FP32x2 FMAs, two independent FP32 FMAs per instruction)
// (two 4-row by two 4-column quads, so shared-memory fragment reads are
// conflict-free 128-bit loads).  A is stored k-major in shared memory so both
// operands are read as float4.  Global tiles are prefetched into registers
// while the current shared tile is consumed (double-buffered shared memory),
// one __syncthreads per K step.  Every FMA is a plain FP32 FFMA: no TF32.
//
// Work units are tiles in a 1-D grid (row-major over tiles).  When the last
// wave of resident CTAs (2 per SM) would run at most half full, its tiles
// are split into two K halves that add into a zeroed C -- 0 + a + b is
// order-independent, so results stay deterministic -- and the last wave runs
// two half-length passes instead of one mostly idle full one (4096^3: 1024
// tiles = 3 x 296 + 136).
//
// The same kernel, instantiated for __half inputs (converted to FP32 on the
// way into shared memory), is the FP16 path for shapes the tensor-core kernel
// does not take; products of two FP16 values are exact in FP32.
#include "gemm_simt.cuh"

namespace opl {

namespace {

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kBK = 8;
constexpr int kThreads = 256;

// Packed FP32 pair arithmetic (sm_100a f32x2): one instruction performs two
// independent IEEE FP32 FMAs, so the 8x8 register tile needs 32 issue slots
// per K step instead of 64 -- same per-element rounding as fmaf.
__device__ __forceinline__ uint64_t dup2(float a) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(a));
  return r;
}
__device__ __forceinline__ void fma2(uint64_t& acc, uint64_t a, uint64_t b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

template <typename T>
struct Quad {
  static __device__ __forceinline__ void load(const T* __restrict__ p, int valid,
                                              bool vec_ok, float (&out)[4]);
};

template <>
__device__ __forceinline__ void Quad<float>::load(const float* __restrict__ p,
                                                  int valid, bool vec_ok,
                                                  float (&out)[4]) {
  if (vec_ok && valid >= 4) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p));
    out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = i < valid ? __ldg(p + i) : 0.0f;
  }
}

template <>
__device__ __forceinline__ void Quad<__half>::load(const __half* __restrict__ p,
                                                   int valid, bool vec_ok,
                                                   float (&out)[4]) {
  if (vec_ok && valid >= 4) {
    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
    const __half2 lo = *reinterpret_cast<const __half2*>(&raw.x);
    const __half2 hi = *reinterpret_cast<const __half2*>(&raw.y);
    const float2 a = __half22float2(lo);
    const float2 b = __half22float2(hi);
    out[0] = a.x; out[1] = a.y; out[2] = b.x; out[3] = b.y;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = i < valid ? __half2float(p[i]) : 0.0f;
  }
}

// Zeroes the C tiles [tiles_full, tiles) (row-major over n_tiles columns of
// tiles); blockIdx.y picks an 8-row slice of the 128-row tile.
__global__ void __launch_bounds__(kBN)
    zero_simt_tiles_kernel(float* __restrict__ c, int m, int n, int n_tiles, int tiles_full) {
  const int t = tiles_full + static_cast<int>(blockIdx.x);
  const int col = (t % n_tiles) * kBN + static_cast<int>(threadIdx.x);
  if (col >= n) return;
  const int row0 = (t / n_tiles) * kBM + static_cast<int>(blockIdx.y) * 8;
  const int row_end = min(m, row0 + 8);
  for (int row = row0; row < row_end; ++row) c[static_cast<std::size_t>(row) * n + col] = 0.0f;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
    gemm_simt_kernel(const T* __restrict__ a, const T* __restrict__ b,
                     float* __restrict__ c, int m, int n, int k, bool a_vec,
                     bool b_vec, bool c_vec, int n_tiles, int tiles_full) {
  __shared__ __align__(16) float as[2][kBK][kBM];
  __shared__ __align__(16) float bs[2][kBK][kBN];

  const int tid = threadIdx.x;
  const int k_tiles_all = (k + kBK - 1) / kBK;
  // Unit -> tile and K-tile range (a split unit covers one K half).
  const int u = static_cast<int>(blockIdx.x);
  const bool split = u >= tiles_full;
  const int tile = split ? tiles_full + ((u - tiles_full) >> 1) : u;
  const int k_half = k_tiles_all / 2;
  const int kt_begin = split && ((u - tiles_full) & 1) ? k_half : 0;
  const int kt_end = split && !((u - tiles_full) & 1) ? k_half : k_tiles_all;
  const int block_m = (tile / n_tiles) * kBM;
  const int block_n = (tile % n_tiles) * kBN;

  // Global-load assignment: A quad = row tid/2, k offset 4*(tid%2);
  // B quad = k row tid/32, n offset 4*(tid%32).
  const int a_row = block_m + (tid >> 1);
  const int a_k = (tid & 1) * 4;
  const int b_k = tid >> 5;
  const int b_col = block_n + (tid & 31) * 4;

  float a_reg[4], b_reg[4];
  auto fetch = [&](int k0) {
    const int ak = k0 + a_k;
    if (a_row < m && ak < k)
      Quad<T>::load(a + static_cast<std::size_t>(a_row) * k + ak, k - ak, a_vec,
                    a_reg);
    else
      a_reg[0] = a_reg[1] = a_reg[2] = a_reg[3] = 0.0f;
    const int bk = k0 + b_k;
    if (bk < k && b_col < n)
      Quad<T>::load(b + static_cast<std::size_t>(bk) * n + b_col, n - b_col,
                    b_vec, b_reg);
    else
      b_reg[0] = b_reg[1] = b_reg[2] = b_reg[3] = 0.0f;
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) as[buf][a_k + i][tid >> 1] = a_reg[i];
    *reinterpret_cast<float4*>(&bs[buf][b_k][(tid & 31) * 4]) =
        make_float4(b_reg[0], b_reg[1], b_reg[2], b_reg[3]);
  };

  const int tx = tid & 15;  // column quads tx*4 and 64 + tx*4
  const int ty = tid >> 4;  // row quads ty*4 and 64 + ty*4
  uint64_t acc2[8][4];  // acc2[i][p] = columns (2p, 2p+1) of row i
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int p = 0; p < 4; ++p) acc2[i][p] = 0;  // (+0.0f, +0.0f)

  fetch(kt_begin * kBK);
  stash(0);
  __syncthreads();
  for (int t = kt_begin; t < kt_end; ++t) {
    const int buf = (t - kt_begin) & 1;
    if (t + 1 < kt_end) fetch((t + 1) * kBK);
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      float af[8];
      const float4 a0 = *reinterpret_cast<const float4*>(&as[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&as[buf][kk][64 + ty * 4]);
      const ulonglong2 b0 = *reinterpret_cast<const ulonglong2*>(&bs[buf][kk][tx * 4]);
      const ulonglong2 b1 = *reinterpret_cast<const ulonglong2*>(&bs[buf][kk][64 + tx * 4]);
      af[0] = a0.x; af[1] = a0.y; af[2] = a0.z; af[3] = a0.w;
      af[4] = a1.x; af[5] = a1.y; af[6] = a1.z; af[7] = a1.w;
      const uint64_t bp[4] = {b0.x, b0.y, b1.x, b1.y};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint64_t a2 = dup2(af[i]);
#pragma unroll
        for (int p = 0; p < 4; ++p) fma2(acc2[i][p], a2, bp[p]);
      }
    }
    if (t + 1 < kt_end) stash(buf ^ 1);
    __syncthreads();
  }

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int p = 0; p < 4; ++p) unpack2(acc2[i][p], acc[i][2 * p], acc[i][2 * p + 1]);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = block_m + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (row >= m) continue;
    float* crow = c + static_cast<std::size_t>(row) * n;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int col = block_n + half * 64 + tx * 4;
      const float* v = &acc[i][half * 4];
      if (split) {  // half of a tail tile: add into the zeroed C
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (col + j < n) atomicAdd(crow + col + j, v[j]);
      } else if (c_vec && col + 3 < n) {
        *reinterpret_cast<float4*>(crow + col) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (col + j < n) crow[col + j] = v[j];
      }
    }
  }
}

}  // namespace

template <typename T>
cudaError_t gemm_simt(const T* a, const T* b, float* c, int m, int n, int k,
                      cudaStream_t stream) {
  const std::size_t elem = sizeof(T);
  const bool a_vec = (k % 4 == 0) && ((reinterpret_cast<std::uintptr_t>(a) % (4 * elem)) == 0);
  const bool b_vec = (n % 4 == 0) && ((reinterpret_cast<std::uintptr_t>(b) % (4 * elem)) == 0);
  const bool c_vec = (n % 4 == 0) && aligned16(c);
  const long long n_tiles = (n + kBN - 1) / kBN;
  const long long tiles = n_tiles * ((m + kBM - 1) / kBM);
  const long long slots = 2LL * sm_count();  // resident CTAs (launch bounds: 2 per SM)
  const long long tail = tiles % slots;
  const bool split = tiles > slots && tail != 0 && 2 * tail <= slots && k >= 16 * kBK;
  const long long tiles_full = split ? tiles - tail : tiles;
  const long long units = tiles_full + (split ? 2 * tail : 0);
  if (units > 0x7fffffffLL) return cudaErrorInvalidValue;
  if (split) {
    zero_simt_tiles_kernel<<<dim3(static_cast<unsigned>(tail), kBM / 8), kBN, 0, stream>>>(
        c, m, n, static_cast<int>(n_tiles), static_cast<int>(tiles_full));
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  gemm_simt_kernel<T><<<static_cast<unsigned>(units), kThreads, 0, stream>>>(
      a, b, c, m, n, k, a_vec, b_vec, c_vec, static_cast<int>(n_tiles),
      static_cast<int>(tiles_full));
  return cudaGetLastError();
}

template cudaError_t gemm_simt<float>(const float*, const float*, float*, int,
                                      int, int, cudaStream_t);
template cudaError_t gemm_simt<__half>(const __half*, const __half*, float*,
                                       int, int, int, cudaStream_t);

}  // namespace opl

extern "C" int opl_gemm_f32(const float* a, const float* b, float* c, int m,
                            int n, int k, opl_stream_t stream) {
  if (a == nullptr || b == nullptr || c == nullptr || m <= 0 || n <= 0 || k <= 0)
    return cudaErrorInvalidValue;
  return opl::gemm_simt<float>(a, b, c, m, n, k, stream);
}
