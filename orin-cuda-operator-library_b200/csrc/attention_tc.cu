// FlashAttention-style forward on tcgen05 tensor cores: FP16 Q/K/V, FP32
// softmax state and FP32 output (reference src/attention.cu:222-360 and
// :486-507 -- there a 16x16 WMMA kernel with QK^T on one warp).
//
// One CTA = one (batch*head, 128-query tile); causal grids start with the
// longest (bottom) tiles.  384 threads:
//   warp 0    TMA producer: Q once; K_j and V_j (128 keys each) into two
//             2-slot rings with separate barriers (K_{j+1} streams in as soon
//             as QK_{j-1} is done, independent of PV), all 128-byte swizzled boxes of 64 columns from a
//             3-D [B*H, S, D] tensor map (rows past S read as zero);
//   warp 1    MMA issuer (one thread):
//               S_j = Q K_j^T   M128 N128 K=D  (both K-major)   -> TMEM S[j%2]
//               O  += P_j V_j   M128 N=D K128  (P K-major, V N-major) -> TMEM O
//             QK_{j+1} is issued before PV_j, so the next scores are computed
//             while the softmax warps work on tile j;
//   warps 4-11 softmax, two warpgroups, each owning half the keys of every
//             row (thread = query row = TMEM lane; 64 fp32 scores in
//             registers): mask only on edge tiles (keys >= S, causal), row
//             max exchanged between the groups in shared memory, running max
//             in the log2 domain, P = exp2(s - m) rounded to FP16 into a
//             swizzled shared tile (the A operand of PV), row sum in FP32
//             (per group, added at the end).  The running max
//             used for P is only moved when a row's maximum grows by more
//             than 8 (a factor 256), so O in TMEM is rescaled rarely; P then
//             stays <= 256, well inside FP16.  At the end O / l is stored.
//   warps 2-3 idle after set-up.
// TMEM: S double buffer (2 x 128 columns) + O (D columns) within 512.
//
// All waits are bounded (tc_common.cuh); on giving up the CTA drains its
// TMA loads and MMAs, frees TMEM and exits, recording the watchdog word.
#include "attention_simt.cuh"
#include "tc_common.cuh"
#include "tmap.cuh"

namespace opl {

namespace {

constexpr int kRowsQ = 128;
constexpr int kKeys = 128;
constexpr int kThreads = 384;
constexpr int kSoftmaxWarp0 = 4;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int D>
struct AttnCfg {
  static constexpr int kBoxes = D / 64;                    // 64-column boxes per row
  static constexpr int kTileBytes = kRowsQ * D * 2;        // Q, K or V tile
  static constexpr int kBoxBytes = kRowsQ * 64 * 2;        // 16 KB
  static constexpr int kPBytes = kRowsQ * kKeys * 2;       // 32 KB
  static constexpr int kStageBytes = 2 * kTileBytes;       // K + V
  static constexpr int kQOff = 0;
  static constexpr int kStageOff = kTileBytes;
  static constexpr int kPOff = kStageOff + 2 * kStageBytes;
  static constexpr int kXchgOff = kPOff + kPBytes;             // 3 x 256 floats
  static constexpr int kBarOff = kXchgOff + 3 * 256 * 4;
  static constexpr size_t kSmem = kBarOff + 256 + 1024;
  static constexpr uint32_t kIdescQK = tc::idesc_f16_f32(kRowsQ, kKeys, false, false);
  static constexpr uint32_t kIdescPV = tc::idesc_f16_f32(kRowsQ, D, false, true);
};

struct AttnBars {
  uint64_t q_full;
  uint64_t k_full[2];
  uint64_t k_empty[2];
  uint64_t v_full[2];
  uint64_t v_empty[2];
  uint64_t s_full[2];
  uint64_t p_ready;
  uint64_t pv_done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// K-major SW128 operand made of 64-column boxes of 128 rows: the 16-wide K
// step kk lives in box kk/4 at byte offset 32*(kk%4).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk, int box_bytes) {
  return tc::smem_desc_sw128(base + (kk >> 2) * box_bytes + (kk & 3) * 32, 16, 1024);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap map_q,
                        const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, float* __restrict__ out,
                        int heads_total, int seq, int causal, float scale_log2,
                        int* watchdog) {
  using Cfg = AttnCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  AttnBars* bars = reinterpret_cast<AttnBars*>(smem + Cfg::kBarOff);
  volatile int* abort = &bars->abort;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int q_tiles = (seq + kRowsQ - 1) / kRowsQ;
  const int bh = blockIdx.x % heads_total;
  const int qb = q_tiles - 1 - static_cast<int>(blockIdx.x / heads_total);
  const int q0 = qb * kRowsQ;
  const int kv_tiles_all = (seq + kKeys - 1) / kKeys;
  const int n_tiles = causal ? min(kv_tiles_all, (q0 + kRowsQ - 1) / kKeys + 1) : kv_tiles_all;

  if (threadIdx.x == 0) {
    tc::mbar_init(&bars->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&bars->k_full[i], 1);
      tc::mbar_init(&bars->k_empty[i], 1);
      tc::mbar_init(&bars->v_full[i], 1);
      tc::mbar_init(&bars->v_empty[i], 1);
      tc::mbar_init(&bars->s_full[i], 1);
    }
    tc::mbar_init(&bars->p_ready, 256);
    tc::mbar_init(&bars->pv_done, 1);
    tc::mbar_init(&bars->drain, 1);
    bars->abort = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&map_q);
    tc::prefetch_tmap(&map_k);
    tc::prefetch_tmap(&map_v);
  }
  if (warp == 1) tc::tmem_alloc(&bars->tmem_base, kTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t tmem_o = tmem + 2 * kKeys;

  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------- producer
    // K and V have separate slots and barriers: K_{j+1} only waits for
    // QK_{j-1} to finish with its slot, V_{j+1} for PV_{j-1}.
    uint32_t issued_mask = 0, issued_parity = 0;  // bit s: K slot s, bit 2+s: V slot s
    tc::mbar_expect_tx(&bars->q_full, Cfg::kTileBytes);
#pragma unroll
    for (int b = 0; b < Cfg::kBoxes; ++b)
      tc::tma_load_3d(smem + Cfg::kQOff + b * Cfg::kBoxBytes, &map_q, b * 64, q0, bh,
                      &bars->q_full);
    for (int j = 0; j < n_tiles && !*abort; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      uint8_t* ks = smem + Cfg::kStageOff + st * Cfg::kStageBytes;
      uint8_t* vs = ks + Cfg::kTileBytes;
      if (!tc::mbar_wait(&bars->k_empty[st], ph ^ 1, abort, watchdog, tc::kWatchdogAttention))
        break;
      tc::mbar_expect_tx(&bars->k_full[st], Cfg::kTileBytes);
#pragma unroll
      for (int b = 0; b < Cfg::kBoxes; ++b)
        tc::tma_load_3d(ks + b * Cfg::kBoxBytes, &map_k, b * 64, j * kKeys, bh,
                        &bars->k_full[st]);
      issued_mask |= 1u << st;
      issued_parity = (issued_parity & ~(1u << st)) | (ph << st);
      if (!tc::mbar_wait(&bars->v_empty[st], ph ^ 1, abort, watchdog, tc::kWatchdogAttention))
        break;
      tc::mbar_expect_tx(&bars->v_full[st], Cfg::kTileBytes);
#pragma unroll
      for (int b = 0; b < Cfg::kBoxes; ++b)
        tc::tma_load_3d(vs + b * Cfg::kBoxBytes, &map_v, b * 64, j * kKeys, bh,
                        &bars->v_full[st]);
      issued_mask |= 4u << st;
      issued_parity = (issued_parity & ~(4u << st)) | (ph << (st + 2));
    }
    if (*abort) {
      const uint32_t qa = tc::smem_u32(&bars->q_full);
      for (uint32_t i = 0; i < tc::kMaxPolls && !tc::mbar_try_wait(qa, 0); ++i) {
      }
      for (int b = 0; b < 4; ++b)
        if (issued_mask & (1u << b)) {
          const uint32_t a = tc::smem_u32(b < 2 ? &bars->k_full[b] : &bars->v_full[b - 2]);
          for (uint32_t i = 0; i < tc::kMaxPolls; ++i)
            if (tc::mbar_try_wait(a, (issued_parity >> b) & 1u)) break;
        }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------- MMA issuer
    bool issued_any = false;
    const uint32_t q_addr = tc::smem_u32(smem + Cfg::kQOff);
    const uint32_t p_addr = tc::smem_u32(smem + Cfg::kPOff);
    auto issue_qk = [&](int j) -> bool {
      const int st = j & 1;
      if (!tc::mbar_wait(&bars->k_full[st], (j >> 1) & 1, abort, watchdog,
                         tc::kWatchdogAttention))
        return false;
      tc::tc_fence_after();
      const uint32_t k_addr = tc::smem_u32(smem + Cfg::kStageOff + st * Cfg::kStageBytes);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        tc::umma_f16(tmem + st * kKeys, kmajor_desc(q_addr, kk, Cfg::kBoxBytes),
                     kmajor_desc(k_addr, kk, Cfg::kBoxBytes), Cfg::kIdescQK, kk != 0);
      tc::umma_commit(&bars->s_full[st]);
      tc::umma_commit(&bars->k_empty[st]);
      issued_any = true;
      return true;
    };
    bool ok = tc::mbar_wait(&bars->q_full, 0, abort, watchdog, tc::kWatchdogAttention);
    if (ok) {
      tc::tc_fence_after();
      ok = issue_qk(0);
    }
    for (int j = 0; ok && j < n_tiles; ++j) {
      if (j + 1 < n_tiles && !issue_qk(j + 1)) break;
      if (!tc::mbar_wait(&bars->p_ready, j & 1, abort, watchdog, tc::kWatchdogAttention))
        break;
      const int st = j & 1;
      if (!tc::mbar_wait(&bars->v_full[st], (j >> 1) & 1, abort, watchdog,
                         tc::kWatchdogAttention))
        break;
      tc::tc_fence_after();
      const uint32_t v_addr =
          tc::smem_u32(smem + Cfg::kStageOff + st * Cfg::kStageBytes + Cfg::kTileBytes);
#pragma unroll
      for (int kk = 0; kk < kKeys / 16; ++kk)
        // V: N-major (D contiguous), 64-column boxes of 128 keys (16 KB
        // apart); a 16-key step is two 8-row groups (2 KB).
        tc::umma_f16(tmem_o, kmajor_desc(p_addr, kk, Cfg::kBoxBytes),
                     tc::smem_desc_sw128(v_addr + kk * 2048, Cfg::kBoxBytes, 1024),
                     Cfg::kIdescPV, (j | kk) != 0);
      tc::umma_commit(&bars->pv_done);
      tc::umma_commit(&bars->v_empty[st]);
    }
    if (*abort && issued_any) {
      tc::umma_commit(&bars->drain);
      const uint32_t a = tc::smem_u32(&bars->drain);
      for (uint32_t i = 0; i < tc::kMaxPolls && !tc::mbar_try_wait(a, 0); ++i) {
      }
    }
  } else if (warp >= kSoftmaxWarp0) {
    // ---------------------------------------------------------- softmax
    // Two warpgroups share each S tile: group g owns keys [64g, 64g+64) of
    // every row, O columns [g*D/2, (g+1)*D/2) for rescaling and output, and
    // its own partial row sum.  Row maxima are exchanged through shared
    // memory (double-buffered by tile parity) behind a 256-thread barrier.
    const int g = (warp - kSoftmaxWarp0) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row in tile == TMEM lane
    const int row = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    float* xchg = reinterpret_cast<float*>(smem + Cfg::kXchgOff);  // [2][2][128]
    uint8_t* p_tile = smem + Cfg::kPOff + g * Cfg::kBoxBytes;
    constexpr int kHalfKeys = kKeys / 2;
    constexpr int kHalfD = D / 2;
    const int limit = causal ? min(seq - 1, row) : seq - 1;  // last visible key
    float m_used = -INFINITY;
    float l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      if (!tc::mbar_wait_warp(&bars->s_full[st], (j >> 1) & 1, abort, watchdog,
                              tc::kWatchdogAttention)) {
        ok = false;
        break;
      }
      tc::tc_fence_after();
      float s[kHalfKeys];
#pragma unroll
      for (int c = 0; c < kHalfKeys / 32; ++c) {
        float chunk[32];
        tc::tmem_ld32(tmem + lane_off + st * kKeys + g * kHalfKeys + c * 32, chunk);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = chunk[i];
      }
      const int key0 = j * kKeys + g * kHalfKeys;
      float mx = -INFINITY;
      if (key0 + kHalfKeys - 1 <= limit) {  // interior: nothing masked
#pragma unroll
        for (int i = 0; i < kHalfKeys; ++i) {
          s[i] *= scale_log2;
          mx = fmaxf(mx, s[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < kHalfKeys; ++i) {
          s[i] = (key0 + i <= limit) ? s[i] * scale_log2 : -INFINITY;
          mx = fmaxf(mx, s[i]);
        }
      }
      float* xm = xchg + st * 256;
      xm[g * 128 + r] = mx;
      named_barrier_sync(1, 256);
      mx = fmaxf(xm[r], xm[128 + r]);
      float alpha = 1.0f;
      if (mx > m_used + kRescaleThreshold) {
        alpha = (m_used == -INFINITY) ? 0.0f : exp2f(m_used - mx);
        m_used = mx;
        l *= alpha;
      }
      float sum = 0.0f;
#pragma unroll
      for (int i = 0; i < kHalfKeys; ++i) {
        s[i] = exp2f(s[i] - m_used);  // -inf -> 0
        sum += s[i];
      }
      l += sum;
      // P_{j-1} must be consumed (PV_{j-1} done) before P and O are touched.
      if (j > 0) {
        if (!tc::mbar_wait_warp(&bars->pv_done, (j - 1) & 1, abort, watchdog,
                                tc::kWatchdogAttention)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        if (__any_sync(kFullMask, alpha != 1.0f)) {
#pragma unroll 1
          for (int c = 0; c < kHalfD / 32; ++c) {
            float o[32];
            const uint32_t col = tmem_o + lane_off + g * kHalfD + c * 32;
            tc::tmem_ld32(col, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tc::tmem_st32(col, o);
          }
        }
      }
      // P row r, keys [64g, 64g+64) -> box g of the K-major SW128 tile: 128 B
      // per row, 16-byte chunk c stored at chunk (c ^ (r & 7)).
#pragma unroll
      for (int c = 0; c < kHalfKeys / 8; ++c) {
        __align__(16) __half2 h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          h[i] = __floats2half2_rn(s[c * 8 + 2 * i], s[c * 8 + 2 * i + 1]);
        *reinterpret_cast<uint4*>(p_tile + r * 128 + ((c ^ (r & 7)) * 16)) =
            *reinterpret_cast<const uint4*>(h);
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->p_ready);
    }
    if (ok && tc::mbar_wait_warp(&bars->pv_done, (n_tiles - 1) & 1, abort, watchdog,
                                 tc::kWatchdogAttention)) {
      tc::tc_fence_after();
      float* xs = xchg + 512;
      xs[g * 128 + r] = l;
      named_barrier_sync(1, 256);
      const float inv = 1.0f / (xs[r] + xs[128 + r]);
      float* orow = out + (static_cast<size_t>(bh) * seq + row) * D + g * kHalfD;
#pragma unroll 1
      for (int c = 0; c < kHalfD / 32; ++c) {
        float o[32];
        tc::tmem_ld32(tmem_o + lane_off + g * kHalfD + c * 32, o);
        if (row < seq) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            st_stream(reinterpret_cast<float4*>(orow + c * 32 + i),
                      make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv));
        }
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

template <int D>
cudaError_t launch_attention_tc(const __half* q, const __half* k, const __half* v,
                                float* out, int heads_total, int seq, bool causal,
                                cudaStream_t stream) {
  using Cfg = AttnCfg<D>;
  CUtensorMap maps[3];
  const __half* ptrs[3] = {q, k, v};
  const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(seq),
                            static_cast<uint64_t>(heads_total)};
  const uint64_t strides[2] = {static_cast<uint64_t>(D) * 2,
                               static_cast<uint64_t>(D) * 2 * seq};
  const uint32_t box[3] = {64, 128, 1};
  for (int i = 0; i < 3; ++i) {
    const cudaError_t e = encode_tmap(&maps[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, ptrs[i],
                                      dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e != cudaSuccess) return e;
  }
  cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel<D>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(Cfg::kSmem));
  if (e != cudaSuccess) return e;
  const long long ctas = static_cast<long long>(heads_total) * ((seq + kRowsQ - 1) / kRowsQ);
  if (ctas > 0x7fffffffLL) return cudaErrorInvalidValue;
  const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
  attention_tc_kernel<D><<<static_cast<unsigned>(ctas), kThreads, Cfg::kSmem, stream>>>(
      maps[0], maps[1], maps[2], out, heads_total, seq, causal ? 1 : 0, scale_log2,
      watchdog_word());
  return cudaGetLastError();
}

}  // namespace

bool attention_tc_supported(int head_dim, const void* q, const void* k, const void* v,
                            const void* out) {
  return (head_dim == 64 || head_dim == 128) && aligned16(q) && aligned16(k) &&
         aligned16(v) && aligned16(out);
}

cudaError_t attention_f16_tc(const __half* q, const __half* k, const __half* v, float* out,
                             int batch, int heads, int seq, int head_dim, bool causal,
                             cudaStream_t stream) {
  const long long total = static_cast<long long>(batch) * heads;
  if (total > 0x7fffffffLL) return cudaErrorInvalidValue;
  if (head_dim == 128)
    return launch_attention_tc<128>(q, k, v, out, static_cast<int>(total), seq, causal, stream);
  return launch_attention_tc<64>(q, k, v, out, static_cast<int>(total), seq, causal, stream);
}

}  // namespace opl
