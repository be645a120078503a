// FP16 / BF16 input-output variants of softmax and RMSNorm (arithmetic in
// FP32, results rounded to the storage type once).  The reference's launchers
// are FP32-only and defer 16-bit I/O to a later "library interface stage"
// (docs/standalone_benchmark.md:14-16); these halve the HBM bytes per element.
//
// Same structure as the FP32 row kernels (row_cache.cuh): a warp or a CTA owns
// a row, caches it in registers (8 elements per 128-bit load when rows are
// 16-byte aligned, else one element per load), reduces across the group and
// writes once.  Rows too long for the register cache use a two-read kernel.
#include <cuda_bf16.h>

#include "row_cache.cuh"

namespace opl {

namespace {

template <typename T>
struct Io16;
template <>
struct Io16<__half> {
  static __device__ __forceinline__ float load(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_bits(unsigned short b) { return __ushort_as_half(b); }
  static __device__ __forceinline__ __half store(float f) { return __float2half_rn(f); }
};
template <>
struct Io16<__nv_bfloat16> {
  static __device__ __forceinline__ float load(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_bits(unsigned short b) {
    return __ushort_as_bfloat16(b);
  }
  static __device__ __forceinline__ __nv_bfloat16 store(float f) { return __float2bfloat16_rn(f); }
};

// One 16-bit element by a volatile-asm load (kept after griddepcontrol.wait;
// see ld_ro), as FP32.
template <typename T>
__device__ __forceinline__ float ld_ro16(const T* p) {
  unsigned short b;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(b) : "l"(p));
  return Io16<T>::load(Io16<T>::from_bits(b));
}

// e^x as 2^(x log2 e) on the MUFU ex2 unit (ex2.approx.f32, relative error
// about 2^-22; subnormal results kept).  With x = v - m formed first, the
// argument's rounding adds at most ~1e-5 relative for |x| < 88, far below the
// rounding of the 16-bit output (2^-11 for FP16, 2^-8 for BF16), where
// CUDA's expf spends several FMA and ALU instructions per element.
__device__ __forceinline__ float exp_mufu(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
  return y;
}

template <typename T, int kGroup, int kItems, bool kVec>
__device__ __forceinline__ void load16(const T* __restrict__ row, int cols, int t, float fill,
                                       float (&v)[kItems * (kVec ? 8 : 1)]) {
  if constexpr (kVec) {
    const uint4* row8 = reinterpret_cast<const uint4*>(row);
    const int vectors = cols >> 3;
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const int idx = t + j * kGroup;
      if (idx < vectors) {
        uint4 raw = ld_ro(row8 + idx);
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[8 * j + i] = Io16<T>::load(e[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[8 * j + i] = fill;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const int col = t + j * kGroup;
      v[j] = col < cols ? ld_ro16(row + col) : fill;
    }
  }
}

template <typename T, int kGroup, int kItems, bool kVec>
__device__ __forceinline__ void store16(T* __restrict__ row, int cols, int t,
                                        const float (&v)[kItems * (kVec ? 8 : 1)]) {
  if constexpr (kVec) {
    uint4* row8 = reinterpret_cast<uint4*>(row);
    const int vectors = cols >> 3;
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const int idx = t + j * kGroup;
      if (idx < vectors) {
        uint4 raw;
        T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i) e[i] = Io16<T>::store(v[8 * j + i]);
        row8[idx] = raw;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const int col = t + j * kGroup;
      if (col < cols) row[col] = Io16<T>::store(v[j]);
    }
  }
}

template <typename T, int kGroup, int kBlock, int kItems, bool kVec>
__global__ void __launch_bounds__(kBlock)
    softmax16_kernel(const T* __restrict__ input, T* __restrict__ output, int rows, int cols) {
  constexpr int kW = kVec ? 8 : 1;
  pdl_begin();
  __shared__ float scratch_max[kBlock / 32];
  __shared__ float scratch_sum[kBlock / 32];
  const int t = threadIdx.x % kGroup;
  const int row = blockIdx.x * (kBlock / kGroup) + threadIdx.x / kGroup;
  if (kGroup == 32 && row >= rows) return;
  const size_t offset = static_cast<size_t>(row) * cols;
  float v[kItems * kW];
  load16<T, kGroup, kItems, kVec>(input + offset, cols, t, -FLT_MAX, v);
  float m = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < kItems * kW; ++i) m = fmaxf(m, v[i]);
  m = group_reduce<kGroup, kBlock, true>(m, scratch_max);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < kItems * kW; ++i) {
    v[i] = exp_mufu(v[i] - m);  // padding slots (-FLT_MAX) underflow to 0
    s += v[i];
  }
  s = group_reduce<kGroup, kBlock, false>(s, scratch_sum);
  const float inverse = 1.0f / s;
#pragma unroll
  for (int i = 0; i < kItems * kW; ++i) v[i] *= inverse;
  store16<T, kGroup, kItems, kVec>(output + offset, cols, t, v);
}

template <typename T, int kGroup, int kBlock, int kItems, bool kVec>
__global__ void __launch_bounds__(kBlock)
    rmsnorm16_kernel(const T* __restrict__ input, const T* __restrict__ weight,
                     T* __restrict__ output, int tokens, int hidden, float epsilon) {
  constexpr int kW = kVec ? 8 : 1;
  pdl_begin();
  __shared__ float scratch[kBlock / 32];
  const int t = threadIdx.x % kGroup;
  const int row = blockIdx.x * (kBlock / kGroup) + threadIdx.x / kGroup;
  if (kGroup == 32 && row >= tokens) return;
  const size_t offset = static_cast<size_t>(row) * hidden;
  float v[kItems * kW];
  load16<T, kGroup, kItems, kVec>(input + offset, hidden, t, 0.0f, v);
  float sq = 0.0f;
#pragma unroll
  for (int i = 0; i < kItems * kW; ++i) sq = fmaf(v[i], v[i], sq);
  sq = group_reduce<kGroup, kBlock, false>(sq, scratch);
  const float inverse_rms = rsqrtf(sq / static_cast<float>(hidden) + epsilon);
  // The weight row is read chunk by chunk (it stays in L2 across rows).
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    float w[kW];
    if constexpr (kVec) {
      const int idx = t + j * kGroup;
      if (idx < (hidden >> 3)) {
        uint4 raw = ld_ro(reinterpret_cast<const uint4*>(weight) + idx);
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = Io16<T>::load(e[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = 0.0f;
      }
    } else {
      const int col = t + j * kGroup;
      w[0] = col < hidden ? ld_ro16(weight + col) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < kW; ++i) v[kW * j + i] = v[kW * j + i] * inverse_rms * w[i];
  }
  store16<T, kGroup, kItems, kVec>(output + offset, hidden, t, v);
}

// Rows beyond the register cache: two reads of the row.
constexpr int kLong16 = 1024;

template <typename T>
__global__ void __launch_bounds__(kLong16)
    softmax16_long_kernel(const T* __restrict__ input, T* __restrict__ output, int cols) {
  __shared__ float sm[kLong16 / 32];
  __shared__ float ss[kLong16 / 32];
  const size_t offset = static_cast<size_t>(blockIdx.x) * cols;
  float m = -FLT_MAX, s = 0.0f;
  for (int c = threadIdx.x; c < cols; c += kLong16) {
    const float x = Io16<T>::load(input[offset + c]);
    if (x > m) {
      s = s * expf(m - x) + 1.0f;
      m = x;
    } else {
      s += expf(x - m);
    }
  }
  const float bm = group_reduce<kLong16, kLong16, true>(m, sm);
  s *= expf(m - bm);
  const float inverse = 1.0f / group_reduce<kLong16, kLong16, false>(s, ss);
  for (int c = threadIdx.x; c < cols; c += kLong16)
    output[offset + c] = Io16<T>::store(expf(Io16<T>::load(input[offset + c]) - bm) * inverse);
}

template <typename T>
__global__ void __launch_bounds__(kLong16)
    rmsnorm16_long_kernel(const T* __restrict__ input, const T* __restrict__ weight,
                          T* __restrict__ output, int hidden, float epsilon) {
  __shared__ float scratch[kLong16 / 32];
  const size_t offset = static_cast<size_t>(blockIdx.x) * hidden;
  float sq = 0.0f;
  for (int c = threadIdx.x; c < hidden; c += kLong16) {
    const float x = Io16<T>::load(input[offset + c]);
    sq = fmaf(x, x, sq);
  }
  sq = group_reduce<kLong16, kLong16, false>(sq, scratch);
  const float inverse_rms = rsqrtf(sq / static_cast<float>(hidden) + epsilon);
  for (int c = threadIdx.x; c < hidden; c += kLong16)
    output[offset + c] = Io16<T>::store(Io16<T>::load(input[offset + c]) * inverse_rms *
                                        Io16<T>::load(weight[c]));
}

struct Shape16 {
  int group, block, items;
};

// Smallest register-cached shape holding `count` slots (uint4 of 8 elements
// when vec, single elements otherwise); false when the row is too long.
bool pick16(int count, bool vec, Shape16* s) {
  // {128, 128, 4}: one 4096-wide row per 128-thread CTA, 32 floats per
  // thread -- small enough for 16 CTAs per SM, so a 2048-row call is in
  // flight in one wave.
  static const Shape16 kVec[] = {{32, 128, 1},  {32, 128, 2},   {32, 128, 4},    {128, 128, 4},
                                 {256, 256, 4}, {256, 256, 8}, {1024, 1024, 4}};
  static const Shape16 kScalar[] = {{32, 128, 1}, {32, 128, 4}, {32, 128, 16}, {32, 128, 32},
                                    {256, 256, 32}, {1024, 1024, 32}};
  const Shape16* table = vec ? kVec : kScalar;
  const int entries = vec ? static_cast<int>(sizeof(kVec) / sizeof(kVec[0]))
                          : static_cast<int>(sizeof(kScalar) / sizeof(kScalar[0]));
  for (int i = 0; i < entries; ++i)
    if (static_cast<long long>(table[i].group) * table[i].items >= count) {
      *s = table[i];
      return true;
    }
  return false;
}

#define OPL_ROW16_DISPATCH(s, vec, BODY)                                         \
  do {                                                                           \
    if (vec) {                                                                   \
      if (s.group == 32 && s.items == 1) BODY(32, 128, 1, true)                  \
      else if (s.group == 32 && s.items == 2) BODY(32, 128, 2, true)             \
      else if (s.group == 32) BODY(32, 128, 4, true)                             \
      else if (s.group == 128) BODY(128, 128, 4, true)                           \
      else if (s.group == 256 && s.items == 4) BODY(256, 256, 4, true)           \
      else if (s.group == 256) BODY(256, 256, 8, true)                           \
      else BODY(1024, 1024, 4, true)                                             \
    } else {                                                                     \
      if (s.group == 32 && s.items == 1) BODY(32, 128, 1, false)                 \
      else if (s.group == 32 && s.items == 4) BODY(32, 128, 4, false)            \
      else if (s.group == 32 && s.items == 16) BODY(32, 128, 16, false)          \
      else if (s.group == 32) BODY(32, 128, 32, false)                           \
      else if (s.group == 256) BODY(256, 256, 32, false)                         \
      else BODY(1024, 1024, 32, false)                                           \
    }                                                                            \
  } while (0)

template <typename T>
int softmax16(const T* input, T* output, int rows, int cols, cudaStream_t stream) {
  if (input == nullptr || output == nullptr || rows <= 0 || cols <= 0)
    return cudaErrorInvalidValue;
  const bool vec = cols % 8 == 0 && aligned16(input) && aligned16(output);
  Shape16 s;
  if (!pick16(vec ? cols / 8 : cols, vec, &s)) {
    softmax16_long_kernel<T><<<rows, kLong16, 0, stream>>>(input, output, cols);
    return cudaGetLastError();
  }
#define OPL_SOFTMAX16(G, B, I, V)                                                         \
  {                                                                                       \
    const int per = (B) / (G);                                                            \
    const cudaError_t e = launch_pdl(softmax16_kernel<T, G, B, I, V>,                   \
                                     dim3((rows + per - 1) / per), dim3(B), stream, input,  \
                                     output, rows, cols);                                   \
    if (e != cudaSuccess) return e;                                                       \
  }
  OPL_ROW16_DISPATCH(s, vec, OPL_SOFTMAX16);
#undef OPL_SOFTMAX16
  return cudaGetLastError();
}

template <typename T>
int rmsnorm16(const T* input, const T* weight, T* output, int tokens, int hidden, float eps,
              cudaStream_t stream) {
  if (input == nullptr || weight == nullptr || output == nullptr || tokens <= 0 ||
      hidden <= 0 || !(eps > 0.0f))
    return cudaErrorInvalidValue;
  const bool vec = hidden % 8 == 0 && aligned16(input) && aligned16(output) && aligned16(weight);
  Shape16 s;
  if (!pick16(vec ? hidden / 8 : hidden, vec, &s)) {
    rmsnorm16_long_kernel<T><<<tokens, kLong16, 0, stream>>>(input, weight, output, hidden, eps);
    return cudaGetLastError();
  }
#define OPL_RMSNORM16(G, B, I, V)                                                         \
  {                                                                                       \
    const int per = (B) / (G);                                                            \
    const cudaError_t e = launch_pdl(rmsnorm16_kernel<T, G, B, I, V>,                   \
                                     dim3((tokens + per - 1) / per), dim3(B), stream,       \
                                     input, weight, output, tokens, hidden, eps);           \
    if (e != cudaSuccess) return e;                                                       \
  }
  OPL_ROW16_DISPATCH(s, vec, OPL_RMSNORM16);
#undef OPL_RMSNORM16
  return cudaGetLastError();
}

}  // namespace

}  // namespace opl

extern "C" {

int opl_softmax_f16(const opl_half_t* input, opl_half_t* output, int rows, int cols,
                    opl_stream_t stream) {
  return opl::softmax16(reinterpret_cast<const __half*>(input), reinterpret_cast<__half*>(output),
                        rows, cols, stream);
}

int opl_softmax_bf16(const opl_bf16_t* input, opl_bf16_t* output, int rows, int cols,
                     opl_stream_t stream) {
  return opl::softmax16(reinterpret_cast<const __nv_bfloat16*>(input),
                        reinterpret_cast<__nv_bfloat16*>(output), rows, cols, stream);
}

int opl_rmsnorm_f16(const opl_half_t* input, const opl_half_t* weight, opl_half_t* output,
                    int tokens, int hidden, float epsilon, opl_stream_t stream) {
  return opl::rmsnorm16(reinterpret_cast<const __half*>(input),
                        reinterpret_cast<const __half*>(weight), reinterpret_cast<__half*>(output),
                        tokens, hidden, epsilon, stream);
}

int opl_rmsnorm_bf16(const opl_bf16_t* input, const opl_bf16_t* weight, opl_bf16_t* output,
                     int tokens, int hidden, float epsilon, opl_stream_t stream) {
  return opl::rmsnorm16(reinterpret_cast<const __nv_bfloat16*>(input),
                        reinterpret_cast<const __nv_bfloat16*>(weight),
                        reinterpret_cast<__nv_bfloat16*>(output), tokens, hidden, epsilon, stream);
}

}  // extern "C"
