// FlashAttention-style forward on tcgen05 tensor cores: FP16 Q/K/V, FP32
// softmax state and FP32 output (reference src/attention.cu:222-360 and
// :486-507 -- there a 16x16 WMMA kernel with QK^T on one warp).
//
// One CTA = one (batch*head, pair of 128-query tiles A and B); causal grids
// start with the longest (bottom) pairs.  When pairs would leave SMs idle, a
// CTA takes one query tile split over the key axis instead ("split mode"):
// "tile" A handles the even key blocks and "tile" B the odd ones of the same
// queries (B reads Q_A), each with its own running max, row sum and O
// accumulator, merged in a fixed order at the end -- so both softmax
// warpgroups and the tensor-pipe ping-pong stay busy.  320 threads:
//   warp 0     TMA producer: Q_A, Q_B once; K_j and V_j (128 keys each)
//              into two 2-slot rings with separate barriers, all 128-byte
//              swizzled 64-column boxes of a 3-D [B*H, S, D] tensor map
//              (rows past S read as zero);
//   warp 1     MMA issuer (one thread), ping-pong over the two tiles:
//                PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1), ...
//              S_X = Q_X K^T: M128 N128 K=D, both operands K-major in smem;
//              O_X += P_X V:  M128 N=D K128, P_X read from TMEM, V N-major in
//              smem -- so while one tile's softmax runs, the tensor pipe
//              works on the other tile;
//   warps 2-5  softmax of tile A, warps 6-9 softmax of tile B (thread = query
//              row = TMEM lane, 128 fp32 scores in registers): mask only on
//              edge tiles, running max in the log2 domain, P = 2^(s - m) on
//              the MUFU unit, P packed to FP16 and stored back
//              into the first 64 columns of the tile's own S columns (the
//              TMEM A operand of PV), row sum in FP32.  The max used for P
//              only moves when a row's maximum grows by more than 8 (a factor
//              256), so O is rarely rescaled and P stays <= 256 (FP16-safe).
// TMEM: S_A, S_B (128 columns each), O_A, O_B (D columns each).
// Ordering: tcgen05.mma ops of one thread run in issue order, and the commit
// that signals S_X(j) follows PV_X(j-1); so when a softmax warp sees S_X(j),
// the previous P_X was consumed and O_X is stable for rescaling.
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
constexpr int kThreads = 320;
constexpr int kSoftmaxWarp0 = 2;  // warps 2-5: tile A, warps 6-9: tile B
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int D>
struct AttnCfg {
  static constexpr int kBoxes = D / 64;              // 64-column boxes per row
  static constexpr int kTileBytes = kRowsQ * D * 2;  // one Q, K or V tile
  static constexpr int kBoxBytes = kRowsQ * 64 * 2;  // 16 KB
  static constexpr int kQOff = 0;                    // Q_A, Q_B
  static constexpr int kKOff = 2 * kTileBytes;       // K slots 0, 1
  static constexpr int kVOff = 4 * kTileBytes;       // V slots 0, 1
  static constexpr int kBarOff = 6 * kTileBytes;
  static constexpr int kXchgOff = kBarOff + 256;  // split mode: (m, l) of both halves
  static constexpr size_t kSmem = kXchgOff + 2048 + 1024;
  static constexpr uint32_t kIdescQK = tc::idesc_f16_f32(kRowsQ, kKeys, false, false);
  static constexpr uint32_t kIdescPV = tc::idesc_f16_f32(kRowsQ, D, false, true);
  static constexpr uint32_t kColO0 = 2 * kKeys;  // O_A; O_B follows at +D
};

struct AttnBars {
  uint64_t q_full;
  uint64_t k_full[2];
  uint64_t k_empty[2];
  uint64_t v_full[2];
  uint64_t v_empty[2];
  uint64_t s_full[2];   // per tile X
  uint64_t p_ready[2];  // per tile X
  uint64_t o_done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// 2^x by the MUFU ex2 instruction (flushes subnormal results to zero;
// 2^-inf = 0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Named barrier 1 over `count` threads.
__device__ __forceinline__ void bar_sync_named(int count) {
  asm volatile("bar.sync 1, %0;" ::"r"(count) : "memory");
}

__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void split_f32x2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// 2^x for two values on the FMA pipe instead of MUFU, so that part of each
// block's exponentials run beside the MUFU ones (both units busy).  Range
// reduction: adding 1.5 * 2^23 rounds x to the nearest integer n, which then
// sits in the low mantissa bits of the sum; f = x - n lies in [-0.5, 0.5];
// 2^f is a degree-4 polynomial fitted for minimum relative error on that
// interval (Lawson-weighted least squares, fitted for this kernel; 2.7e-6
// relative, against 2^-11 for the FP16 rounding P gets next); 2^n is added
// to the exponent field (bits(sum) << 23 keeps exactly n << 23).  Inputs
// must lie in [-120, 120]: callers clamp at -120, where 2^x is far below
// FP16's smallest subnormal.
constexpr float kExpRound = 12582912.0f;  // 1.5 * 2^23
constexpr float kExpC0 = 0.9999992847442627f;
constexpr float kExpC1 = 0.6931218504905701f;
constexpr float kExpC2 = 0.240247443318367f;
constexpr float kExpC3 = 0.055917806923389435f;
constexpr float kExpC4 = 0.009570068679749966f;

__device__ __forceinline__ void exp2_poly_x2(uint64_t x, float& y0, float& y1) {
  const uint64_t t = add_f32x2(x, f32x2(kExpRound, kExpRound));
  const uint64_t n = add_f32x2(t, f32x2(-kExpRound, -kExpRound));
  const uint64_t f = fma_f32x2(n, f32x2(-1.0f, -1.0f), x);
  uint64_t p = fma_f32x2(f32x2(kExpC4, kExpC4), f, f32x2(kExpC3, kExpC3));
  p = fma_f32x2(p, f, f32x2(kExpC2, kExpC2));
  p = fma_f32x2(p, f, f32x2(kExpC1, kExpC1));
  p = fma_f32x2(p, f, f32x2(kExpC0, kExpC0));
  float p0, p1, t0, t1;
  split_f32x2(p, p0, p1);
  split_f32x2(t, t0, t1);
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

__device__ __forceinline__ float pack_half2_bits(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return __uint_as_float(*reinterpret_cast<const uint32_t*>(&h));
}

}  // namespace

namespace {

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap map_q,
                        const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v,
                        const __grid_constant__ CUtensorMap map_o,
                        int heads_total, int seq, int head_dim, int causal, float scale_log2,
                        int tiles_per_cta, int* watchdog) {
  using Cfg = AttnCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  AttnBars* bars = reinterpret_cast<AttnBars*>(smem + Cfg::kBarOff);
  volatile int* abort = &bars->abort;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int q_tiles = (seq + kRowsQ - 1) / kRowsQ;
  const int pairs = (q_tiles + tiles_per_cta - 1) / tiles_per_cta;
  const int bh = blockIdx.x % heads_total;
  const int pair = pairs - 1 - static_cast<int>(blockIdx.x / heads_total);
  const int qt0 = tiles_per_cta * pair;
  const bool split = tiles_per_cta == 1;
  const bool valid_b = tiles_per_cta == 2 && qt0 + 1 < q_tiles;  // a second Q tile
  const int kv_all = (seq + kKeys - 1) / kKeys;
  // n_tiles[x]: key blocks tile x processes; n_load: key blocks loaded.
  int n_tiles[2];
  int n_load;
  if (split) {
    n_load = causal ? min(kv_all, qt0 + 1) : kv_all;
    n_tiles[0] = (n_load + 1) / 2;  // blocks 0, 2, 4, ...
    n_tiles[1] = n_load / 2;        // blocks 1, 3, 5, ...
  } else {
    n_tiles[0] = causal ? min(kv_all, qt0 + 1) : kv_all;
    n_tiles[1] = valid_b ? (causal ? min(kv_all, qt0 + 2) : kv_all) : 0;
    n_load = max(n_tiles[0], n_tiles[1]);
  }

  if (threadIdx.x == 0) {
    tc::mbar_init(&bars->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&bars->k_full[i], 1);
      tc::mbar_init(&bars->k_empty[i], 1);
      tc::mbar_init(&bars->v_full[i], 1);
      tc::mbar_init(&bars->v_empty[i], 1);
      tc::mbar_init(&bars->s_full[i], 1);
      tc::mbar_init(&bars->p_ready[i], 128);
    }
    tc::mbar_init(&bars->o_done, 1);
    tc::mbar_init(&bars->drain, 1);
    bars->abort = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&map_q);
    tc::prefetch_tmap(&map_k);
    tc::prefetch_tmap(&map_v);
    tc::prefetch_tmap(&map_o);
  }
  if (warp == 1) tc::tmem_alloc(&bars->tmem_base, kTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  // Launched with programmatic dependent launch: the set-up above overlaps
  // the previous kernel on the stream; global memory is touched only after
  // it has completed.  The next kernel may start its own set-up at once.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------- producer
    uint32_t issued_mask = 0, issued_parity = 0;  // bit s: K slot s, bit 2+s: V slot s
    tc::mbar_expect_tx(&bars->q_full, (valid_b ? 2 : 1) * Cfg::kTileBytes);
    for (int x = 0; x < (valid_b ? 2 : 1); ++x)
#pragma unroll
      for (int b = 0; b < Cfg::kBoxes; ++b)
        tc::tma_load_3d(smem + Cfg::kQOff + x * Cfg::kTileBytes + b * Cfg::kBoxBytes, &map_q,
                        b * 64, (qt0 + x) * kRowsQ, bh, &bars->q_full);
    for (int j = 0; j < n_load && !*abort; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!tc::mbar_wait(&bars->k_empty[st], ph ^ 1, abort, watchdog, tc::kWatchdogAttention))
        break;
      tc::mbar_expect_tx(&bars->k_full[st], Cfg::kTileBytes);
#pragma unroll
      for (int b = 0; b < Cfg::kBoxes; ++b)
        tc::tma_load_3d(smem + Cfg::kKOff + st * Cfg::kTileBytes + b * Cfg::kBoxBytes, &map_k,
                        b * 64, j * kKeys, bh, &bars->k_full[st]);
      issued_mask |= 1u << st;
      issued_parity = (issued_parity & ~(1u << st)) | (ph << st);
      if (!tc::mbar_wait(&bars->v_empty[st], ph ^ 1, abort, watchdog, tc::kWatchdogAttention))
        break;
      tc::mbar_expect_tx(&bars->v_full[st], Cfg::kTileBytes);
#pragma unroll
      for (int b = 0; b < Cfg::kBoxes; ++b)
        tc::tma_load_3d(smem + Cfg::kVOff + st * Cfg::kTileBytes + b * Cfg::kBoxBytes, &map_v,
                        b * 64, j * kKeys, bh, &bars->v_full[st]);
      issued_mask |= 4u << st;
      issued_parity = (issued_parity & ~(4u << st)) | (ph << (st + 2));
    }
    if (*abort) {  // let in-flight TMA writes land before the CTA exits
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
    // Shared-memory descriptors are built once: a K step only moves the
    // start-address field (address / 16, bits 0-13), and smem addresses stay
    // below 256 KB, so adding the step's offset / 16 never carries out of the
    // field.  This keeps each MMA at a few instructions -- the issuing thread
    // shares its sub-partition with two softmax warps, and rebuilding two
    // 64-bit descriptors per MMA made issue, not the tensor pipe, the limit.
    const uint32_t q_addr = tc::smem_u32(smem + Cfg::kQOff);
    const uint64_t q_desc[2] = {tc::smem_desc_sw128(q_addr, 16, 1024),
                                tc::smem_desc_sw128(q_addr + Cfg::kTileBytes, 16, 1024)};
    const uint32_t k_addr0 = tc::smem_u32(smem + Cfg::kKOff);
    const uint64_t k_desc[2] = {tc::smem_desc_sw128(k_addr0, 16, 1024),
                                tc::smem_desc_sw128(k_addr0 + Cfg::kTileBytes, 16, 1024)};
    const uint32_t v_addr0 = tc::smem_u32(smem + Cfg::kVOff);
    const uint64_t v_desc[2] = {tc::smem_desc_sw128(v_addr0, Cfg::kBoxBytes, 1024),
                                tc::smem_desc_sw128(v_addr0 + Cfg::kTileBytes, Cfg::kBoxBytes,
                                                    1024)};
    // K-major step kk: box kk/4, 32 bytes per 16 columns inside the box.
    auto kstep = [](int kk) {
      return static_cast<uint64_t>(((kk >> 2) * Cfg::kBoxBytes + (kk & 3) * 32) >> 4);
    };
    // S block `buf` = Q_x K_j^T (K_j already landed); commit signals s_full[buf].
    auto qk_into = [&](int buf, int x, int j) {
      const uint64_t qd = q_desc[x], kd = k_desc[j & 1];
      const uint32_t d_tmem = tmem + buf * kKeys;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        tc::umma_f16(d_tmem, qd + kstep(kk), kd + kstep(kk), Cfg::kIdescQK, kk != 0);
      tc::umma_commit(&bars->s_full[buf]);
      issued_any = true;
    };
    auto qk = [&](int x, int j) { qk_into(x, x, j); };
    // In split mode tile x handles key block b = 2 j + x, which sits in
    // ring slot b & 1 == x with phase (b >> 1) & 1 == j & 1.
    // O_x += P (FP16 pairs in the first 64 columns of S block `buf`; 8
    // packed columns per 16 keys) * V_j.
    auto pv_from = [&](int buf, int x, int j, bool first) {
      const uint64_t vd = v_desc[j & 1];
      const uint32_t d_tmem = tmem + Cfg::kColO0 + x * D;
      const uint32_t p_tmem = tmem + buf * kKeys;
      // V: N-major (D contiguous), 64-column boxes of 128 keys (16 KB
      // apart); a 16-key step is two 8-row groups (2 KB).
      tc::umma_f16_tmem_a(d_tmem, p_tmem, vd, Cfg::kIdescPV, first ? 0u : 1u);
#pragma unroll
      for (int kk = 1; kk < kKeys / 16; ++kk)
        tc::umma_f16_tmem_a(d_tmem, p_tmem + kk * 8, vd + static_cast<uint64_t>(kk * 128),
                            Cfg::kIdescPV, 1u);
      issued_any = true;
    };
    auto pv = [&](int x, int j) { pv_from(x, x, j, j == 0); };
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      const bool ok = tc::mbar_wait(bar, parity, abort, watchdog, tc::kWatchdogAttention);
      if (ok) tc::tc_fence_after();
      return ok;
    };
    bool ok = wait(&bars->q_full, 0) && wait(&bars->k_full[0], 0);
    if (split) {
      // Per tile x: PV_x(j), then QK_x(j+1) -- S_x(j+1) is committed after
      // PV_x(j), so a softmax warp that sees it finds O_x stable.
      if (ok) {
        qk_into(0, 0, 0);
        tc::umma_commit(&bars->k_empty[0]);
        if (n_tiles[1] > 0) {
          ok = wait(&bars->k_full[1], 0);
          if (ok) {
            qk_into(1, 0, 1);
            tc::umma_commit(&bars->k_empty[1]);
          }
        }
      }
      for (int j = 0; ok && j < n_tiles[0]; ++j) {
        for (int x = 0; ok && x < 2; ++x) {
          if (j >= n_tiles[x]) continue;
          const int b = 2 * j + x;
          ok = wait(&bars->v_full[x], j & 1) && wait(&bars->p_ready[x], j & 1);
          if (!ok) break;
          pv_from(x, x, b, j == 0);
          tc::umma_commit(&bars->v_empty[x]);
          if (j + 1 < n_tiles[x]) {
            ok = wait(&bars->k_full[x], (j + 1) & 1);
            if (!ok) break;
            qk_into(x, 0, b + 2);
            tc::umma_commit(&bars->k_empty[x]);
          }
        }
      }
    } else {
      if (ok) {
        qk(0, 0);
        if (n_tiles[1] > 0) qk(1, 0);
        tc::umma_commit(&bars->k_empty[0]);
      }
      for (int j = 0; ok && j < n_load; ++j) {
        const bool do_a = j < n_tiles[0], do_b = j < n_tiles[1];
        const bool next_a = j + 1 < n_tiles[0], next_b = j + 1 < n_tiles[1];
        if (!wait(&bars->v_full[j & 1], (j >> 1) & 1)) break;
        if (do_a) {
          if (!wait(&bars->p_ready[0], j & 1)) break;
          pv(0, j);
        }
        if (next_a || next_b) {
          if (!wait(&bars->k_full[(j + 1) & 1], ((j + 1) >> 1) & 1)) break;
        }
        if (next_a) qk(0, j + 1);
        if (do_b) {
          if (!wait(&bars->p_ready[1], j & 1)) break;
          pv(1, j);
        }
        tc::umma_commit(&bars->v_empty[j & 1]);
        if (next_b) qk(1, j + 1);
        if (next_a || next_b) tc::umma_commit(&bars->k_empty[(j + 1) & 1]);
      }
    }
    if (!*abort) {
      tc::umma_commit(&bars->o_done);
    } else if (issued_any) {  // wait for issued MMAs before TMEM is freed
      tc::umma_commit(&bars->drain);
      const uint32_t a = tc::smem_u32(&bars->drain);
      for (uint32_t i = 0; i < tc::kMaxPolls && !tc::mbar_try_wait(a, 0); ++i) {
      }
    }
  } else if (warp >= kSoftmaxWarp0) {
    // ---------------------------------------------------------- softmax
    const int x = (warp - kSoftmaxWarp0) >> 2;  // tile A or B
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row in tile == TMEM lane
    const int row = (qt0 + (split ? 0 : x)) * kRowsQ + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t o_col = tmem + lane_off + Cfg::kColO0 + x * D;
    const int limit = causal ? min(seq - 1, row) : seq - 1;  // last visible key
    const int n = n_tiles[x];
    float m_used = -INFINITY;
    float l = 0.0f;
    bool ok = n > 0;
    for (int j = 0; ok && j < n; ++j) {
      const uint32_t s_col = tmem + lane_off + x * kKeys;
      if (!tc::mbar_wait_warp(&bars->s_full[x], j & 1, abort, watchdog,
                              tc::kWatchdogAttention)) {
        ok = false;
        break;
      }
      tc::tc_fence_after();
      float s[kKeys];
      {
        uint32_t raw[kKeys];
#pragma unroll
        for (int c = 0; c < kKeys / 32; ++c) tc::tmem_ld32_nowait(s_col + c * 32, raw + c * 32);
#pragma unroll
        for (int c = 0; c < kKeys / 32; ++c) tc::tmem_wait_ld32(raw + c * 32);
#pragma unroll
        for (int i = 0; i < kKeys; ++i) s[i] = __uint_as_float(raw[i]);
      }
      const int key0 = (split ? 2 * j + x : j) * kKeys;
      if (key0 + kKeys - 1 > limit) {  // edge tile: mask keys past the limit
#pragma unroll
        for (int i = 0; i < kKeys; ++i)
          if (key0 + i > limit) s[i] = -INFINITY;
      }
      // Raw-score maximum (scale > 0 commutes with max); eight independent
      // partial maxima / sums keep dependency chains short.
      // pm[a] = max of s[a], s[a + 8], ...: s[0 .. 7], then 16 scores per
      // step, then the last 8 when (kKeys - 8) is an odd multiple of 8.
      float pm[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) pm[a] = s[a];
#pragma unroll
      for (int i = 8; i + 16 <= kKeys; i += 16) {
#pragma unroll
        for (int a = 0; a < 8; ++a) pm[a] = fmax3(pm[a], s[i + a], s[i + 8 + a]);
      }
      if constexpr ((kKeys - 8) % 16 == 8) {
#pragma unroll
        for (int a = 0; a < 8; ++a) pm[a] = fmaxf(pm[a], s[kKeys - 8 + a]);
      }
      const float mx = scale_log2 * fmax3(fmax3(pm[0], pm[1], pm[2]), fmax3(pm[3], pm[4], pm[5]),
                                          fmaxf(pm[6], pm[7]));
      float alpha = 1.0f;
      if (mx > m_used + kRescaleThreshold) {
        alpha = (m_used == -INFINITY) ? 0.0f : exp2f(m_used - mx);
        m_used = mx;
        l *= alpha;
      }
      // 2^(s*scale - m) for the 128 keys: 80 on the MUFU unit (ex2.approx,
      // relative error ~2^-22) and 48 (pairs 0, 3 and 6 of every 8) as an
      // FMA-pipe polynomial (exp2_poly_x2), so that MUFU -- which two
      // softmax warps share per sub-partition -- is no longer the only unit
      // doing exponentials.  Both errors are far below the FP16 rounding of
      // P.  Eight independent partial sums.  Scale-and-shift, the polynomial
      // and the row sum run on packed FP32 pairs (fma.rn.f32x2 /
      // add.rn.f32x2: two IEEE FP32 operations per instruction).
      uint64_t ps2[4] = {0, 0, 0, 0};
      const uint64_t scale2 = f32x2(scale_log2, scale_log2);
      const uint64_t shift2 = f32x2(-m_used, -m_used);
#pragma unroll
      for (int i = 0; i < kKeys / 2; ++i) {
        float x0, x1;
        split_f32x2(fma_f32x2(f32x2(s[2 * i], s[2 * i + 1]), scale2, shift2), x0, x1);
        if ((i & 7) == 0 || (i & 7) == 3 || (i & 7) == 6) {
          exp2_poly_x2(f32x2(fmaxf(x0, -120.0f), fmaxf(x1, -120.0f)), s[2 * i], s[2 * i + 1]);
        } else {
          s[2 * i] = fast_exp2(x0);  // -inf -> 0
          s[2 * i + 1] = fast_exp2(x1);
        }
        ps2[i & 3] = add_f32x2(ps2[i & 3], f32x2(s[2 * i], s[2 * i + 1]));
      }
      float ps[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) split_f32x2(ps2[k], ps[2 * k], ps[2 * k + 1]);
      l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
      // P as packed FP16 pairs (packed in place, front to back) into the
      // first 64 columns of S_x.
#pragma unroll
      for (int i = 0; i < kKeys / 2; ++i) s[i] = pack_half2_bits(s[2 * i], s[2 * i + 1]);
      tc::tmem_st32(s_col, s);
      tc::tmem_st32(s_col + 32, s + 32);
      // O_x is stable here (S_x(j) was committed after PV_x(j-1), and
      // PV_x(j) waits for p_ready); rescaled after P is out of registers.
      if (j > 0 && __any_sync(kFullMask, alpha != 1.0f)) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tc::tmem_ld32(o_col + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tc::tmem_st32(o_col + c * 32, o);
        }
      }
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->p_ready[x]);
    }
    if (split) {
      // Merge the halves: m = max(m_A, m_B), O = (O_A 2^(m_A - m) +
      // O_B 2^(m_B - m)) / (l_A 2^(m_A - m) + l_B 2^(m_B - m)).  Every
      // softmax thread passes the named barrier exactly once.  Half x then
      // writes O columns [x D/2, (x + 1) D/2) through TMA stores.
      float* xch = reinterpret_cast<float*>(smem + Cfg::kXchgOff);  // [x][m, l][row]
      xch[(2 * x) * kRowsQ + r] = m_used;
      xch[(2 * x + 1) * kRowsQ + r] = l;
      const bool done = (ok || n == 0) && tc::mbar_wait_warp(&bars->o_done, 0, abort, watchdog,
                                                            tc::kWatchdogAttention);
      bar_sync_named(256);
      if (done) {
        tc::tc_fence_after();
        const bool has_b = n_tiles[1] > 0;
        const float ma = xch[r], la = xch[kRowsQ + r];
        const float mb = has_b ? xch[2 * kRowsQ + r] : -INFINITY;
        const float lb = has_b ? xch[3 * kRowsQ + r] : 0.0f;
        const float m = fmaxf(ma, mb);
        const float ca = exp2f(ma - m);
        const float cb = mb == -INFINITY ? 0.0f : exp2f(mb - m);
        const float inv = 1.0f / (la * ca + lb * cb);
        const float wa = ca * inv, wb = cb * inv;
        const uint32_t oa_col = tmem + lane_off + Cfg::kColO0;
        uint8_t* stage = smem + Cfg::kQOff + (warp - kSoftmaxWarp0) * 8192;
        const int y0 = qt0 * kRowsQ + quarter * 32;
        // All of this warp's TMEM loads are issued before one wait (each
        // load waited for alone costs its full latency).
        uint32_t oraw[2 * (D / 64)][32];
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tc::tmem_ld32_nowait(oa_col + x * (D / 2) + c * 32, oraw[2 * c]);
          tc::tmem_ld32_nowait(oa_col + D + x * (D / 2) + c * 32, oraw[2 * c + 1]);
        }
#pragma unroll
        for (int c = 0; c < 2 * (D / 64); ++c) tc::tmem_wait_ld32(oraw[c]);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          const int col = x * (D / 2) + c * 32;
          float o[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            o[i] = __uint_as_float(oraw[2 * c][i]) * wa;
            if (has_b) o[i] = fmaf(__uint_as_float(oraw[2 * c + 1][i]), wb, o[i]);
          }
          uint8_t* buf = stage + (c & 1) * 4096;
          if (lane == 0) tc::bulk_wait_read<1>();
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 8; ++k)
            *reinterpret_cast<float4*>(buf + lane * 128 + ((k ^ (lane & 7)) * 16)) =
                make_float4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
          tc::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && y0 < seq && col < head_dim) {  // columns >= head_dim: padding
            tc::tma_store_3d(&map_o, buf, col, y0, bh);
            tc::bulk_commit();
          }
        }
        if (lane == 0) tc::bulk_wait_read<0>();  // smem reads done; the grid end publishes the writes
      }
    } else if (ok &&
               tc::mbar_wait_warp(&bars->o_done, 0, abort, watchdog, tc::kWatchdogAttention)) {
      // Every MMA is done, so Q/K/V shared memory is free: each warp stages
      // 32 rows x 32 columns of O at a time (128-byte swizzle: thread = row
      // writes its eight 16-byte pieces at piece ^ (row % 8), conflict-free)
      // in two 4 KB buffers and writes them with TMA stores (rows past S
      // are clipped by the tensor map), instead of 32 separate row
      // segments per store instruction.
      tc::tc_fence_after();
      const float inv = 1.0f / l;
      // One 4 KB staging buffer per 32 columns (8 warps x D KB fits in the
      // Q and K regions), so no store waits for an earlier one; all TMEM
      // loads are issued before one wait.
      uint8_t* stage = smem + Cfg::kQOff + (warp - kSoftmaxWarp0) * (D / 32) * 4096;
      const int y0 = (qt0 + x) * kRowsQ + quarter * 32;
      uint32_t oraw[D / 32][32];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) tc::tmem_ld32_nowait(o_col + c * 32, oraw[c]);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) tc::tmem_wait_ld32(oraw[c]);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = __uint_as_float(oraw[c][i]);
        uint8_t* buf = stage + c * 4096;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<float4*>(buf + lane * 128 + ((k ^ (lane & 7)) * 16)) =
              make_float4(o[4 * k] * inv, o[4 * k + 1] * inv, o[4 * k + 2] * inv,
                          o[4 * k + 3] * inv);
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && y0 < seq && c * 32 < head_dim) {  // columns >= head_dim: padding
          tc::tma_store_3d(&map_o, buf, c * 32, y0, bh);
          tc::bulk_commit();
        }
      }
      if (lane == 0) tc::bulk_wait_read<0>();  // smem reads done; the grid end publishes the writes
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

// D is the padded head dimension the kernel computes with (64 or 128);
// head_dim <= D (a multiple of 8) is the caller's: the tensor maps have
// head_dim columns, so TMA fills columns head_dim .. D-1 of Q, K and V with
// zeros (they add nothing to Q K^T, and give O columns that are not stored).
template <int D>
cudaError_t launch_attention_tc(const __half* q, const __half* k, const __half* v,
                                float* out, int heads_total, int seq, int head_dim, bool causal,
                                cudaStream_t stream) {
  using Cfg = AttnCfg<D>;
  CUtensorMap maps[4];
  const __half* ptrs[3] = {q, k, v};
  const uint64_t dims[3] = {static_cast<uint64_t>(head_dim), static_cast<uint64_t>(seq),
                            static_cast<uint64_t>(heads_total)};
  const uint64_t strides[2] = {static_cast<uint64_t>(head_dim) * 2,
                               static_cast<uint64_t>(head_dim) * 2 * seq};
  const uint32_t box[3] = {64, 128, 1};
  for (int i = 0; i < 3; ++i) {
    const cudaError_t e = encode_tmap(&maps[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, ptrs[i],
                                      dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e != cudaSuccess) return e;
  }
  {  // O: FP32 [B*H, S, D], 32 x 32 store boxes
    const uint64_t o_strides[2] = {static_cast<uint64_t>(head_dim) * 4,
                                   static_cast<uint64_t>(head_dim) * 4 * seq};
    const uint32_t o_box[3] = {32, 32, 1};
    const cudaError_t e = encode_tmap(&maps[3], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, out, dims,
                                      o_strides, o_box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e != cudaSuccess) return e;
  }
  cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel<D>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(Cfg::kSmem));
  if (e != cudaSuccess) return e;
  // Two query tiles per CTA (tensor-pipe ping-pong) unless that would leave
  // SMs idle; then one tile per CTA for twice the CTAs.
  const long long q_tiles = (seq + kRowsQ - 1) / kRowsQ;
  const int tiles_per_cta =
      (static_cast<long long>(heads_total) * ((q_tiles + 1) / 2) >= 2LL * sm_count()) ? 2 : 1;
  const long long ctas =
      static_cast<long long>(heads_total) * ((q_tiles + tiles_per_cta - 1) / tiles_per_cta);
  if (ctas > 0x7fffffffLL) return cudaErrorInvalidValue;
  const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(head_dim));
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(static_cast<unsigned>(ctas));
  config.blockDim = dim3(kThreads);
  config.dynamicSmemBytes = Cfg::kSmem;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  return cudaLaunchKernelEx(&config, attention_tc_kernel<D>, maps[0], maps[1], maps[2], maps[3],
                            heads_total, seq, head_dim, causal ? 1 : 0, scale_log2, tiles_per_cta,
                            watchdog_word());
}

}  // namespace

bool attention_tc_supported(int head_dim, const void* q, const void* k, const void* v,
                            const void* out) {
  // Any head_dim <= 128 with 16-byte rows: computed as 64 or 128 (zero padding).
  return head_dim >= 8 && head_dim <= 128 && head_dim % 8 == 0 && aligned16(q) &&
         aligned16(k) && aligned16(v) && aligned16(out);
}

cudaError_t attention_f16_tc(const __half* q, const __half* k, const __half* v, float* out,
                             int batch, int heads, int seq, int head_dim, bool causal,
                             cudaStream_t stream) {
  const long long total = static_cast<long long>(batch) * heads;
  if (total > 0x7fffffffLL) return cudaErrorInvalidValue;
  if (head_dim > 64)
    return launch_attention_tc<128>(q, k, v, out, static_cast<int>(total), seq, head_dim, causal,
                                    stream);
  return launch_attention_tc<64>(q, k, v, out, static_cast<int>(total), seq, head_dim, causal,
                                 stream);
}

}  // namespace opl
