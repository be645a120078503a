// FlashAttention-style forward on FP32 FFMA (reference src/attention.cu:51-214
// and :445-484): O = softmax(Q K^T / sqrt(D) [+ causal mask]) V over
// contiguous [B,H,S,D] tensors, D <= 128, with an online softmax so the SxS
// score matrix never exists.
//
// One CTA = one (batch*head, 64-query tile), 256 threads.  Thread (tr, tc)
// owns query rows 4*tr..4*tr+3 in BOTH phases, so its running row maximum and
// denominator stay in registers:
//   S phase:  S[4x4] over keys tc*4..tc*4+3 of the 64-key tile, from Q (rows
//             in shared memory) and K^T (shared, key-contiguous);
//   softmax:  row max / sum across the 16 lanes sharing tr (xor shuffles);
//   PV phase: O[4 rows x 8 cols] (cols 4*tc.. and 64+4*tc..) += P V.
// Causal tiles beyond the diagonal are skipped; the diagonal tile is masked.
// T = float is the FP32 path; T = __half is the FP16 path for shapes the
// tensor-core kernel does not take (inputs converted to FP32 on load).
#include "attention_simt.cuh"

namespace opl {

namespace {

constexpr int kRows = 64;
constexpr int kKeys = 64;
constexpr int kThreads = 256;
constexpr int kKtPitch = kKeys + 4;

__device__ __forceinline__ float to_float(float x) { return x; }
__device__ __forceinline__ float to_float(__half x) { return __half2float(x); }

template <typename T>
__global__ void __launch_bounds__(kThreads)
    attention_simt_kernel(const T* __restrict__ q, const T* __restrict__ k,
                          const T* __restrict__ v, float* __restrict__ out,
                          int seq, int d, int dp, bool causal, float scale) {
  extern __shared__ __align__(16) float smem[];
  const int pitch = dp + 4;
  float* qs = smem;                     // [kRows][pitch]
  float* kt = qs + kRows * pitch;       // [dp][kKtPitch]
  float* vs = kt + dp * kKtPitch;       // [kKeys][pitch]
  float* ps = vs + kKeys * pitch;       // [kRows][kKtPitch]

  const int q_tiles = (seq + kRows - 1) / kRows;
  const int bh = blockIdx.x / q_tiles;
  const int q0 = (blockIdx.x - bh * q_tiles) * kRows;
  const std::size_t base = static_cast<std::size_t>(bh) * seq * d;
  const int tid = threadIdx.x;
  const int tr = tid >> 4;
  const int tc = tid & 15;

  // Q tile -> shared (zero-padded rows and columns).
  for (int idx = tid; idx < kRows * dp; idx += kThreads) {
    const int r = idx / dp;
    const int c = idx - r * dp;
    float x = 0.0f;
    if (q0 + r < seq && c < d) x = to_float(q[base + static_cast<std::size_t>(q0 + r) * d + c]);
    qs[r * pitch + c] = x;
  }

  float m_run[4], l_run[4], o[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) o[i][j] = 0.0f;
  }

  const int q_last = min(q0 + kRows, seq) - 1;
  const int key_end = causal ? q_last + 1 : seq;
  for (int k0 = 0; k0 < key_end; k0 += kKeys) {
    __syncthreads();  // previous tile fully consumed
    // K tile transposed (lanes walk keys so shared stores are conflict-free),
    // V tile row-major.
    for (int idx = tid; idx < kKeys * dp; idx += kThreads) {
      const int c = idx / kKeys;
      const int key = idx - c * kKeys;
      float x = 0.0f;
      if (k0 + key < seq && c < d) x = to_float(k[base + static_cast<std::size_t>(k0 + key) * d + c]);
      kt[c * kKtPitch + key] = x;
    }
    for (int idx = tid; idx < kKeys * dp; idx += kThreads) {
      const int key = idx / dp;
      const int c = idx - key * dp;
      float x = 0.0f;
      if (k0 + key < seq && c < d) x = to_float(v[base + static_cast<std::size_t>(k0 + key) * d + c]);
      vs[key * pitch + c] = x;
    }
    __syncthreads();

    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
    for (int c = 0; c < dp; ++c) {
      const float4 kv = *reinterpret_cast<const float4*>(&kt[c * kKtPitch + tc * 4]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float qv = qs[(tr * 4 + i) * pitch + c];
        s[i][0] = fmaf(qv, kv.x, s[i][0]);
        s[i][1] = fmaf(qv, kv.y, s[i][1]);
        s[i][2] = fmaf(qv, kv.z, s[i][2]);
        s[i][3] = fmaf(qv, kv.w, s[i][3]);
      }
    }

    // Online softmax for the thread's 4 rows; the 16 lanes sharing tr hold
    // the 64 keys of those rows.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = q0 + tr * 4 + i;
      float tile_max = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = k0 + tc * 4 + j;
        const bool valid = key < seq && (!causal || key <= row);
        s[i][j] = valid ? s[i][j] * scale : -INFINITY;
        tile_max = fmaxf(tile_max, s[i][j]);
      }
#pragma unroll
      for (int o2 = 8; o2 > 0; o2 >>= 1)
        tile_max = fmaxf(tile_max, __shfl_xor_sync(kFullMask, tile_max, o2));
      const float m_new = fmaxf(m_run[i], tile_max);
      // Rows with nothing visible yet keep m = -inf; guard the rescale.
      const float alpha = (m_new == -INFINITY) ? 1.0f : expf(m_run[i] - m_new);
      float tile_sum = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = (s[i][j] == -INFINITY) ? 0.0f : expf(s[i][j] - m_new);
        s[i][j] = p;
        tile_sum += p;
      }
#pragma unroll
      for (int o2 = 8; o2 > 0; o2 >>= 1)
        tile_sum += __shfl_xor_sync(kFullMask, tile_sum, o2);
      l_run[i] = l_run[i] * alpha + tile_sum;
      m_run[i] = m_new;
#pragma unroll
      for (int j = 0; j < 8; ++j) o[i][j] *= alpha;
      *reinterpret_cast<float4*>(&ps[(tr * 4 + i) * kKtPitch + tc * 4]) =
          make_float4(s[i][0], s[i][1], s[i][2], s[i][3]);
    }
    __syncwarp();
    // The 16 lanes of a row group wrote that group's P rows; a half-warp
    // reads only its own rows, so a warp-level barrier suffices.

    const bool hi = 64 + tc * 4 < dp;
    const int key_count = min(kKeys, seq - k0);
    for (int j = 0; j < key_count; ++j) {
      const float4 v0 = *reinterpret_cast<const float4*>(&vs[j * pitch + tc * 4]);
      float4 v1 = make_float4(0.f, 0.f, 0.f, 0.f);
      if (hi) v1 = *reinterpret_cast<const float4*>(&vs[j * pitch + 64 + tc * 4]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float p = ps[(tr * 4 + i) * kKtPitch + j];
        o[i][0] = fmaf(p, v0.x, o[i][0]);
        o[i][1] = fmaf(p, v0.y, o[i][1]);
        o[i][2] = fmaf(p, v0.z, o[i][2]);
        o[i][3] = fmaf(p, v0.w, o[i][3]);
        o[i][4] = fmaf(p, v1.x, o[i][4]);
        o[i][5] = fmaf(p, v1.y, o[i][5]);
        o[i][6] = fmaf(p, v1.z, o[i][6]);
        o[i][7] = fmaf(p, v1.w, o[i][7]);
      }
    }
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = q0 + tr * 4 + i;
    if (row >= seq) continue;
    const float inv = 1.0f / l_run[i];
    float* orow = out + base + static_cast<std::size_t>(row) * d;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = (j < 4 ? tc * 4 + j : 64 + tc * 4 + (j - 4));
      if (col < d) orow[col] = o[i][j] * inv;
    }
  }
}

}  // namespace

template <typename T>
cudaError_t attention_simt(const T* q, const T* k, const T* v, float* out,
                           int batch, int heads, int seq, int d, bool causal,
                           cudaStream_t stream) {
  const long long total = static_cast<long long>(batch) * heads;
  const long long tiles = total * ((seq + kRows - 1) / kRows);
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidValue;
  const int dp = (d + 3) & ~3;
  const std::size_t smem =
      sizeof(float) * (static_cast<std::size_t>(kRows) * (dp + 4) +
                       static_cast<std::size_t>(dp) * kKtPitch +
                       static_cast<std::size_t>(kKeys) * (dp + 4) +
                       static_cast<std::size_t>(kRows) * kKtPitch);
  cudaError_t error = cudaFuncSetAttribute(
      attention_simt_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
      static_cast<int>(smem));
  if (error != cudaSuccess) return error;
  const dim3 grid(static_cast<unsigned>(tiles));
  const float scale = 1.0f / sqrtf(static_cast<float>(d));
  attention_simt_kernel<T><<<grid, kThreads, smem, stream>>>(q, k, v, out, seq,
                                                             d, dp, causal, scale);
  return cudaGetLastError();
}

template cudaError_t attention_simt<float>(const float*, const float*,
                                           const float*, float*, int, int, int,
                                           int, bool, cudaStream_t);
template cudaError_t attention_simt<__half>(const __half*, const __half*,
                                            const __half*, float*, int, int,
                                            int, int, bool, cudaStream_t);

}  // namespace opl

extern "C" int opl_attention_f32(const float* q, const float* k, const float* v,
                                 float* output, int batch, int heads,
                                 int sequence, int head_dim, int causal,
                                 opl_stream_t stream) {
  if (q == nullptr || k == nullptr || v == nullptr || output == nullptr ||
      batch <= 0 || heads <= 0 || sequence <= 0 || head_dim <= 0 ||
      head_dim > 128)
    return cudaErrorInvalidValue;
  if (opl::attention_f32_tiled_supported(head_dim, q, k, v, output))
    return opl::attention_f32_tiled(q, k, v, output, batch, heads, sequence, head_dim,
                                    causal != 0, stream);
  return opl::attention_simt<float>(q, k, v, output, batch, heads, sequence,
                                    head_dim, causal != 0, stream);
}
