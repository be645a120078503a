// FP32 flash-attention forward on FFMA, tiled like an SGEMM, for head_dim 64
// or 128 (reference src/attention.cu:51-150 and :445-484, there one warp per
// query row with a shuffle-reduced dot product per key).
//
// CTA = (batch*head, 128 query rows), 256 threads; thread (tr, tc) with
// tr = tid / 16 (0..15), tc = tid % 16 owns query rows 8*tr .. 8*tr+7 in both
// phases, so its running max / denominator stay in registers:
//   S phase   S[8 rows][4 keys] (keys 4*tc..) over D: per d one 8-row Q
//             fragment (Q stored d-major in shared memory, two 128-bit loads)
//             and one 4-key K fragment (K stored d-major, one 128-bit load);
//   softmax   row max / sum across the 16 lanes of a row group (xor
//             shuffles), online rescaling of O; scores in the log2 domain,
//             exponentials by the MUFU ex2 instruction;
//   PV phase  O[8 rows][D/16 columns] += P V over the 64 keys: P stored
//             key-major (8-row fragment = two 128-bit loads), V row-major.
// Register-tile updates use packed fma.rn.f32x2 (two independent FP32 FMAs
// per instruction, same rounding as fmaf).  Causal tiles past the diagonal
// are skipped; the grid starts with the longest (bottom) query blocks.  When
// (head, query block) units would leave SMs idle, one CTA per SM runs an
// equal share of all KV tiles (balanced schedule) and
// attention_combine_ranges_kernel merges the units split between CTAs.
#include <algorithm>

#include "attention_simt.cuh"

namespace opl {

namespace {

constexpr int kBM = 128;
constexpr int kBN = 64;
constexpr int kThreads = 256;

__device__ __forceinline__ uint64_t dup2f(float a) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(a));
  return r;
}
__device__ __forceinline__ uint64_t pack2f(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void fma2f(uint64_t& acc, uint64_t a, uint64_t b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}
// 2^x on the MUFU unit (ex2.approx, relative error ~2^-22; 2^-inf = 0).
__device__ __forceinline__ float exp2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void unpack2f(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

template <int D>
struct F32Cfg {
  static constexpr int kQPitch = kBM + 4;   // Qt[d][row]
  static constexpr int kKPitch = kBN + 4;   // Kt[d][key]
  static constexpr int kVPitch = D + 4;     // V[key][d]
  static constexpr int kPPitch = kBM + 4;   // Pt[key][row]
  static constexpr int kCols = D / 16;      // output columns per thread
  static constexpr size_t kSmemFloats = static_cast<size_t>(D) * kQPitch +
                                        static_cast<size_t>(D) * kKPitch +
                                        static_cast<size_t>(kBN) * kVPitch +
                                        static_cast<size_t>(kBN) * kPPitch;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attention_f32_tiled_kernel(const float* __restrict__ q, const float* __restrict__ k,
                               const float* __restrict__ v, float* __restrict__ out,
                               int heads_total, int seq, int hd, int causal, float scale_log2,
                               int balanced, float* __restrict__ part_o,
                               float2* __restrict__ part_ml) {
  using Cfg = F32Cfg<D>;
  extern __shared__ __align__(16) float smem[];
  float* qt = smem;                              // [D][kQPitch]
  float* kt = qt + D * Cfg::kQPitch;             // [D][kKPitch]
  float* vs = kt + D * Cfg::kKPitch;             // [kBN][kVPitch]
  float* pt = vs + kBN * Cfg::kVPitch;           // [kBN][kPPitch]

  const int q_blocks = (seq + kBM - 1) / kBM;
  const int tid = threadIdx.x;
  const int tr = tid >> 4;
  const int tc = tid & 15;
  // Work units: unit u = (head u % heads_total, query block q_blocks - 1 -
  // u / heads_total), longest (bottom) blocks first; a unit's work is its KV
  // tiles.  balanced == 0: CTA = unit, all of its KV tiles.  balanced == 1:
  // the units' KV tiles laid end to end are cut into gridDim.x
  // equal ranges, one per CTA; a CTA runs every (unit, KV range) segment of
  // its range, writing a unit it covers whole straight to `out` and a unit
  // it covers in part (at most its first and last segments) to partial slot
  // 2 blockIdx.x (first) or 2 blockIdx.x + 1 (last), which
  // attention_combine_ranges_kernel merges.
  auto unit_tiles = [&](long long u) {
    const int qb_u = q_blocks - 1 - static_cast<int>(u / heads_total);
    const int last = min(qb_u * kBM + kBM, seq) - 1;
    return ((causal ? last + 1 : seq) + kBN - 1) / kBN;
  };
  long long unit, pos, range_end, unit_start = 0;
  if (!balanced) {
    unit = blockIdx.x;
    pos = 0;
    range_end = 0;  // unused
  } else {
    // Units come in groups of heads_total with equal tile counts (one query
    // block each), so the prefix sums walk q_blocks groups, not all units.
    long long total = 0;
    for (int g = 0; g < q_blocks; ++g) total += static_cast<long long>(heads_total) *
                                                unit_tiles(static_cast<long long>(g) * heads_total);
    pos = total * blockIdx.x / gridDim.x;
    range_end = total * (blockIdx.x + 1) / gridDim.x;
    unit = 0;
    for (int g = 0; g < q_blocks; ++g) {
      const long long t = unit_tiles(static_cast<long long>(g) * heads_total);
      if (unit_start + t * heads_total <= pos) {
        unit_start += t * heads_total;
        unit += heads_total;
        continue;
      }
      const long long in_group = (pos - unit_start) / t;
      unit += in_group;
      unit_start += in_group * t;
      break;
    }
  }
  bool first_segment = true;
  for (;;) {
  if (balanced && pos >= range_end) break;
  const int rest = static_cast<int>(unit);
  const int bh = rest % heads_total;
  const int qb = q_blocks - 1 - rest / heads_total;
  const int q0 = qb * kBM;
  // hd <= D: the caller's head_dim; columns hd .. D-1 are zero padding.
  const size_t base = static_cast<size_t>(bh) * seq * hd;
  __syncthreads();  // the previous segment is done with the shared tiles

  // Q tile -> d-major shared copy (rows past S are zero).
  for (int idx = tid; idx < kBM * (D / 4); idx += kThreads) {
    const int row = idx % kBM;
    const int c4 = idx / kBM;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + row < seq && 4 * c4 < hd)
      x = __ldg(reinterpret_cast<const float4*>(q + base + static_cast<size_t>(q0 + row) * hd) + c4);
    qt[(4 * c4 + 0) * Cfg::kQPitch + row] = x.x;
    qt[(4 * c4 + 1) * Cfg::kQPitch + row] = x.y;
    qt[(4 * c4 + 2) * Cfg::kQPitch + row] = x.z;
    qt[(4 * c4 + 3) * Cfg::kQPitch + row] = x.w;
  }

  float m_run[8], l_run[8];
  uint64_t o2[8][Cfg::kCols / 2];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.0f;
#pragma unroll
    for (int c = 0; c < Cfg::kCols / 2; ++c) o2[i][c] = 0;
  }

  const int q_last = min(q0 + kBM, seq) - 1;
  const int key_total = causal ? q_last + 1 : seq;
  // This CTA's share of the unit's KV tiles (all of them when not balanced).
  const int kv_tiles = (key_total + kBN - 1) / kBN;
  int tile_lo = 0, tile_hi = kv_tiles;
  if (balanced) {
    tile_lo = static_cast<int>(pos - unit_start);
    tile_hi = static_cast<int>(min(range_end - unit_start, static_cast<long long>(kv_tiles)));
  }
  const int key_begin = tile_lo * kBN;
  const int key_end = min(tile_hi * kBN, key_total);
  // Partial result slot of this CTA's first / last segment when it covers the
  // unit in part; -1: the whole unit, written to out.
  long long part_slot = -1;
  if (balanced && (tile_lo > 0 || tile_hi < kv_tiles))
    part_slot = 2LL * blockIdx.x + (first_segment ? 0 : 1);
  for (int k0 = key_begin; k0 < key_end; k0 += kBN) {
    __syncthreads();  // previous tile consumed (and Q written on the first pass)
    for (int idx = tid; idx < kBN * (D / 4); idx += kThreads) {
      const int key = idx % kBN;
      const int c4 = idx / kBN;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 + key < seq && 4 * c4 < hd)
        x = __ldg(reinterpret_cast<const float4*>(k + base + static_cast<size_t>(k0 + key) * hd) + c4);
      kt[(4 * c4 + 0) * Cfg::kKPitch + key] = x.x;
      kt[(4 * c4 + 1) * Cfg::kKPitch + key] = x.y;
      kt[(4 * c4 + 2) * Cfg::kKPitch + key] = x.z;
      kt[(4 * c4 + 3) * Cfg::kKPitch + key] = x.w;
    }
    // V by 16-byte cp.async: it lands while the S phase and the softmax run
    // (waited for before the PV phase); out-of-range pieces are zeroed.
    for (int idx = tid; idx < kBN * (D / 4); idx += kThreads) {
      const int key = idx / (D / 4);
      const int c4 = idx % (D / 4);
      float* dst = &vs[key * Cfg::kVPitch + 4 * c4];
      if (k0 + key < seq && 4 * c4 < hd) {
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                         static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                     "l"(v + base + static_cast<size_t>(k0 + key) * hd + 4 * c4)
                     : "memory");
      } else {
        *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    __syncthreads();

    // S = Q K^T for rows 8tr.., keys 4tc..: s2[r][j] holds rows (2r, 2r + 1)
    // of key j, so the Q operand pairs come straight from the 128-bit loads
    // and only the four K values are duplicated.
    uint64_t s2[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int j = 0; j < 4; ++j) s2[r][j] = 0;
    // Causal: a warp whose 16 rows (8tr.. for its two tr) all precede this
    // tile's first key sees none of it -- its S and PV loops are skipped
    // (warp-uniform); the mask below then gives P = 0 and an unchanged max.
    const bool warp_masked = causal && q0 + 16 * (tid >> 5) + 15 < k0;
    if (!warp_masked)
#pragma unroll 8
    for (int d = 0; d < D; ++d) {
      const ulonglong2 qa = *reinterpret_cast<const ulonglong2*>(&qt[d * Cfg::kQPitch + tr * 8]);
      const ulonglong2 qb = *reinterpret_cast<const ulonglong2*>(&qt[d * Cfg::kQPitch + tr * 8 + 4]);
      const float4 kk = *reinterpret_cast<const float4*>(&kt[d * Cfg::kKPitch + tc * 4]);
      const uint64_t qp[4] = {qa.x, qa.y, qb.x, qb.y};
      const float kv[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint64_t b = dup2f(kv[j]);
#pragma unroll
        for (int r = 0; r < 4; ++r) fma2f(s2[r][j], qp[r], b);
      }
    }

    // Online softmax per row; the 16 lanes sharing tr hold the row's 64 keys.
    // P goes to shared memory after the loop, rows 8tr .. 8tr + 7 of each key
    // as two 128-bit stores.
    float pr[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = q0 + tr * 8 + i;
      float s[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float lo, hi;
        unpack2f(s2[i >> 1][j], lo, hi);
        s[j] = (i & 1) ? hi : lo;
      }
      float tile_max = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = k0 + tc * 4 + j;
        const bool valid = key < seq && (!causal || key <= row);
        s[j] = valid ? s[j] * scale_log2 : -INFINITY;  // log2 domain
        tile_max = fmaxf(tile_max, s[j]);
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1)
        tile_max = fmaxf(tile_max, __shfl_xor_sync(kFullMask, tile_max, o));
      const float m_new = fmaxf(m_run[i], tile_max);
      const float alpha = (m_new == -INFINITY) ? 1.0f : exp2_mufu(m_run[i] - m_new);
      float tile_sum = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[j] = (s[j] == -INFINITY) ? 0.0f : exp2_mufu(s[j] - m_new);
        tile_sum += s[j];
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) tile_sum += __shfl_xor_sync(kFullMask, tile_sum, o);
      l_run[i] = l_run[i] * alpha + tile_sum;
      m_run[i] = m_new;
      const uint64_t a2 = dup2f(alpha);
#pragma unroll
      for (int c = 0; c < Cfg::kCols / 2; ++c) {
        uint64_t scaled = 0;
        fma2f(scaled, o2[i][c], a2);
        o2[i][c] = scaled;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) pr[i][j] = s[j];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float* dst = &pt[(tc * 4 + j) * Cfg::kPPitch + tr * 8];
      *reinterpret_cast<float4*>(dst) = make_float4(pr[0][j], pr[1][j], pr[2][j], pr[3][j]);
      *reinterpret_cast<float4*>(dst + 4) = make_float4(pr[4][j], pr[5][j], pr[6][j], pr[7][j]);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // this thread's V pieces landed
    __syncthreads();

    // O += P V over this tile's keys.
    const int key_count = warp_masked ? 0 : min(kBN, seq - k0);
#pragma unroll 4
    for (int j = 0; j < key_count; ++j) {
      const float4 pa = *reinterpret_cast<const float4*>(&pt[j * Cfg::kPPitch + tr * 8]);
      const float4 pb = *reinterpret_cast<const float4*>(&pt[j * Cfg::kPPitch + tr * 8 + 4]);
      const float pv[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
      uint64_t vv[Cfg::kCols / 2];
      if constexpr (Cfg::kCols == 8) {
        const ulonglong2 v0 = *reinterpret_cast<const ulonglong2*>(&vs[j * Cfg::kVPitch + tc * 8]);
        const ulonglong2 v1 = *reinterpret_cast<const ulonglong2*>(&vs[j * Cfg::kVPitch + tc * 8 + 4]);
        vv[0] = v0.x; vv[1] = v0.y; vv[2] = v1.x; vv[3] = v1.y;
      } else {
        const ulonglong2 v0 = *reinterpret_cast<const ulonglong2*>(&vs[j * Cfg::kVPitch + tc * 4]);
        vv[0] = v0.x; vv[1] = v0.y;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint64_t a = dup2f(pv[i]);
#pragma unroll
        for (int c = 0; c < Cfg::kCols / 2; ++c) fma2f(o2[i][c], a, vv[c]);
      }
    }
  }

  if (part_slot >= 0) {
    // Partial result of this KV range: unnormalised O with its (m, l);
    // attention_combine_ranges_kernel merges the parts.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = q0 + tr * 8 + i;
      if (row >= seq) continue;
      const size_t r_index = static_cast<size_t>(part_slot) * kBM + (row - q0);
      if (tc == 0) part_ml[r_index] = make_float2(m_run[i], l_run[i]);
      float* orow = part_o + r_index * hd + tc * Cfg::kCols;
#pragma unroll
      for (int c = 0; c < Cfg::kCols / 2; c += 2) {
        float a0, a1, b0, b1;
        unpack2f(o2[i][c], a0, a1);
        unpack2f(o2[i][c + 1], b0, b1);
        if (tc * Cfg::kCols + 2 * c < hd)
          *reinterpret_cast<float4*>(orow + 2 * c) = make_float4(a0, a1, b0, b1);
      }
    }
  } else {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = q0 + tr * 8 + i;
    if (row >= seq) continue;
    const float inv = 1.0f / l_run[i];
    float* orow = out + base + static_cast<size_t>(row) * hd + tc * Cfg::kCols;
#pragma unroll
    for (int c = 0; c < Cfg::kCols / 2; c += 2) {
      float a0, a1, b0, b1;
      unpack2f(o2[i][c], a0, a1);
      unpack2f(o2[i][c + 1], b0, b1);
      if (tc * Cfg::kCols + 2 * c < hd)
        *reinterpret_cast<float4*>(orow + 2 * c) =
            make_float4(a0 * inv, a1 * inv, b0 * inv, b1 * inv);
    }
  }
  }
  if (!balanced) break;
  pos = unit_start + tile_hi;
  unit_start += kv_tiles;
  ++unit;
  first_segment = false;
  }
}

}  // namespace

// Merges the partial results of the balanced schedule: for every unit that
// more than one CTA covered, per row, m = max over its parts, O = sum of the
// parts' O 2^(m_p - m) / sum of l_p 2^(m_p - m) (log2 domain), parts in CTA order
// (deterministic).  A unit's parts sit in slot 2c (its CTA c started inside
// the unit) or 2c + 1 (CTA c started before it).  One CTA per 8 rows of a
// unit: thread 0 finds the covering CTAs, then each warp merges one row with
// all of its loads issued before the arithmetic.
constexpr int kMaxParts = 8;

__global__ void __launch_bounds__(256)
    attention_combine_ranges_kernel(const float* __restrict__ part_o,
                                    const float2* __restrict__ part_ml, float* __restrict__ out,
                                    int heads_total, int seq, int d, int causal, int ctas) {
  __shared__ int s_parts;
  __shared__ long long s_slot[kMaxParts];
  const int q_blocks = (seq + kBM - 1) / kBM;
  const long long u = blockIdx.x / (kBM / 8);
  auto group_tiles = [&](int g) {
    const int qb_g = q_blocks - 1 - g;
    const int last = min(qb_g * kBM + kBM, seq) - 1;
    return static_cast<long long>(((causal ? last + 1 : seq) + kBN - 1) / kBN);
  };
  if (threadIdx.x == 0) {
    long long total = 0, start = 0;
    const int group_u = static_cast<int>(u / heads_total);
    for (int g = 0; g < q_blocks; ++g) {
      const long long t = group_tiles(g);
      if (g == group_u) start = total + (u - static_cast<long long>(g) * heads_total) * t;
      total += t * heads_total;
    }
    const long long end = start + group_tiles(group_u);
    // CTAs whose ranges [c total / ctas, (c + 1) total / ctas) meet [start, end).
    long long c_lo = max(0LL, start * ctas / total - 1);
    while ((c_lo + 1) * total / ctas <= start) ++c_lo;
    int parts = 0;
    for (long long c = c_lo; c < ctas && c * total / ctas < end && parts < kMaxParts; ++c)
      s_slot[parts++] = 2 * c + ((c * total / ctas >= start) ? 0 : 1);
    s_parts = parts;
  }
  __syncthreads();
  const int parts = s_parts;
  if (parts <= 1) return;  // one CTA covered the unit whole and wrote it
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = static_cast<int>(u % heads_total);
  const int r = static_cast<int>(blockIdx.x % (kBM / 8)) * 8 + warp;
  const int row = (q_blocks - 1 - static_cast<int>(u / heads_total)) * kBM + r;
  if (row >= seq) return;
  float2 ml[kMaxParts];
  float ov[kMaxParts][4];
#pragma unroll
  for (int p = 0; p < kMaxParts; ++p) {
    const bool in = p < parts;
    ml[p] = in ? part_ml[s_slot[p] * kBM + r] : make_float2(-INFINITY, 0.0f);
    const float* o = part_o + ((in ? s_slot[p] : 0) * kBM + r) * d;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int col = lane + 32 * i;
      ov[p][i] = (in && col < d) ? o[col] : 0.0f;
    }
  }
  float m = -INFINITY;
#pragma unroll
  for (int p = 0; p < kMaxParts; ++p) m = fmaxf(m, ml[p].x);
  float l = 0.0f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int p = 0; p < kMaxParts; ++p) {
    if (ml[p].x == -INFINITY) continue;
    const float w = exp2f(ml[p].x - m);  // (m, l) are in the log2 domain
    l += ml[p].y * w;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] += ov[p][i] * w;
  }
  const float inv = 1.0f / l;
  float* orow = out + (static_cast<size_t>(bh) * seq + row) * d;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int col = lane + 32 * i;
    if (col < d) orow[col] = acc[i] * inv;
  }
}

namespace {

template <int D>
cudaError_t launch_f32_tiled(const float* q, const float* k, const float* v, float* out,
                             int heads_total, int seq, int hd, bool causal, cudaStream_t stream) {
  using Cfg = F32Cfg<D>;
  const size_t smem = Cfg::kSmemFloats * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(attention_f32_tiled_kernel<D>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const long long units = static_cast<long long>(heads_total) * ((seq + kBM - 1) / kBM);
  if (units > 0x7fffffffLL) return cudaErrorInvalidValue;
  // Scores are kept in the log2 domain: 2^(s log2(e) / sqrt(d) - m) = e^(s / sqrt(d) - m').
  const float scale = 1.4426950408889634f / sqrtf(static_cast<float>(hd));
  // A full grid (at least one unit per SM, and at least two KV tiles to
  // share out): one CTA per unit.
  const int kv_tiles = (seq + kBN - 1) / kBN;
  if (units >= sm_count() || kv_tiles < 4) {
    attention_f32_tiled_kernel<D><<<static_cast<unsigned>(units), kThreads, smem, stream>>>(
        q, k, v, out, heads_total, seq, hd, causal ? 1 : 0, scale, 0, nullptr, nullptr);
    return cudaGetLastError();
  }
  // Grids that would leave SMs idle: the balanced schedule, one CTA per SM
  // over equal ranges of all KV tiles (no partial last wave, and the long
  // bottom rows of causal grids spread over several CTAs), the units split
  // between CTAs merged afterwards.
  // At most kMaxParts CTAs may share one unit: with R = total / grid tiles
  // per CTA, a unit of T tiles meets at most T / R + 2 ranges.
  long long total_tiles = 0, max_tiles = 1;
  for (int qb = 0; qb < (seq + kBM - 1) / kBM; ++qb) {
    const int last = std::min(qb * kBM + kBM, seq) - 1;
    const long long t = ((causal ? last + 1 : seq) + kBN - 1) / kBN;
    total_tiles += t * heads_total;
    max_tiles = std::max(max_tiles, t);
  }
  const int grid = static_cast<int>(std::max<long long>(
      1, std::min<long long>({static_cast<long long>(sm_count()), total_tiles,
                              (kMaxParts - 2) * total_tiles / max_tiles})));
  const size_t slots = 2 * static_cast<size_t>(grid);
  void* ws = nullptr;
  e = cudaMallocAsync(&ws, slots * kBM * (hd * sizeof(float) + sizeof(float2)), stream);
  if (e != cudaSuccess) return e;
  float* part_o = static_cast<float*>(ws);
  float2* part_ml = reinterpret_cast<float2*>(part_o + slots * kBM * hd);
  attention_f32_tiled_kernel<D><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(
      q, k, v, out, heads_total, seq, hd, causal ? 1 : 0, scale, 1, part_o, part_ml);
  e = cudaGetLastError();
  if (e == cudaSuccess) {
    attention_combine_ranges_kernel<<<static_cast<unsigned>(units * (kBM / 8)), 256, 0, stream>>>(
        part_o, part_ml, out, heads_total, seq, hd, causal ? 1 : 0, grid);
    e = cudaGetLastError();
  }
  const cudaError_t f = cudaFreeAsync(ws, stream);
  return e != cudaSuccess ? e : f;
}

}  // namespace

bool attention_f32_tiled_supported(int head_dim, const void* q, const void* k, const void* v,
                                   const void* out) {
  // Any head_dim <= 128 with float4 rows, computed as 64 or 128 (zero padding).
  return head_dim >= 4 && head_dim <= 128 && head_dim % 4 == 0 && aligned16(q) &&
         aligned16(k) && aligned16(v) && aligned16(out);
}

cudaError_t attention_f32_tiled(const float* q, const float* k, const float* v, float* out,
                                int batch, int heads, int seq, int head_dim, bool causal,
                                cudaStream_t stream) {
  const long long total = static_cast<long long>(batch) * heads;
  if (total > 0x7fffffffLL) return cudaErrorInvalidValue;
  if (head_dim > 64)
    return launch_f32_tiled<128>(q, k, v, out, static_cast<int>(total), seq, head_dim, causal,
                                 stream);
  return launch_f32_tiled<64>(q, k, v, out, static_cast<int>(total), seq, head_dim, causal,
                              stream);
}

}  // namespace opl
