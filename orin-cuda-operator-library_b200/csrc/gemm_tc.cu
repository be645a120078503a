// FP16 x FP16 -> FP32 GEMM on the 5th-generation tensor cores (tcgen05),
// row-major C[M,N] = A[M,K] * B[K,N] (reference src/gemm.cu:230-336 and
// :455-479 -- there a 128x128 WMMA tile kernel with cp.async).
//
// Persistent, warp-specialised kernel, one CTA per SM (192 threads):
//   warp 0  TMA producer: per 64-wide K block, one 128x64 A box (K-major)
//           and four 64x64 B boxes (N-major) into a 4-stage ring of 48 KB
//           stages, 128-byte swizzled, completion on a "full" mbarrier;
//   warp 1  MMA issuer (one thread): 4 x tcgen05.mma kind::f16
//           M=128 N=256 K=16 per K block into a TMEM accumulator; commits
//           release the smem stage ("empty") and, after the last K block,
//           hand the accumulator to the epilogue ("tmem_full");
//   warps 2-5 epilogue: tcgen05.ld of their 32 TMEM lanes, a per-warp
//           transpose through shared memory, coalesced predicated FP32
//           row stores, then "tmem_empty".
// The 512 TMEM columns hold two 128x256 FP32 accumulators, so the epilogue of
// tile i overlaps the main loop of tile i+1.  Tiles are walked in groups of
// 16 M blocks so concurrently running CTAs share A and B panels in L2.
// B is consumed in its natural row-major (N-major) layout through the
// descriptor's MN-major mode: no transposed copy.  When M and N are both at
// least 256 the CTA-pair version of this kernel (gemm_tc_pair_kernel, 256 x
// 256 tiles on the two-SM MMA) runs instead.
//
// Every mbarrier wait is bounded (tc_common.cuh): a wait that gives up sets
// the CTA's abort flag and the device watchdog word; the CTA then drains its
// outstanding TMA loads and MMAs (again bounded), frees TMEM and exits.
#include <algorithm>

#include "gemm_simt.cuh"
#include "tc_common.cuh"
#include "tmap.cuh"

namespace opl {

namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK * 2;       // 16 KB
constexpr int kBBoxBytes = kBK * 64 * 2;     // 8 KB: 64 K rows x 64 N
constexpr int kBBytes = kBBoxBytes * (kBN / 64);
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr int kGroupM = 16;
constexpr uint32_t kIdesc = tc::idesc_f16_f32(kBM, kBN, false, true);
constexpr int kStagePitch = 33;                          // floats per staged row
constexpr int kEpiStageBytes = 4 * 32 * kStagePitch * 4;  // 4 warps x 32x33 floats
constexpr size_t kSmemBytes = kStages * kStageBytes + kEpiStageBytes + 1024 + 256;

struct Barriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

constexpr int kPairBM = 256;  // tile height of the CTA-pair kernel

// Work units: tiles [0, tiles_full) whole; each remaining tail tile as two
// K halves (2 units), so the last wave is two half-length passes instead of
// one mostly idle full one.  Split units add into C (zeroed beforehand).
// BM: tile height (128, or 256 for a CTA pair); grid_ctas counts CTAs or
// pairs, whichever runs one tile at a time.
template <int BM>
struct TileGridT {
  int m_blocks, n_blocks, tiles, tiles_full, units, k_blocks, group_m = kGroupM;
  __host__ __device__ void init(int m, int n, int k, int grid_ctas, bool split_tail) {
    m_blocks = (m + BM - 1) / BM;
    n_blocks = (n + kBN - 1) / kBN;
    tiles = m_blocks * n_blocks;
    k_blocks = (k + kBK - 1) / kBK;
    tiles_full = split_tail ? (tiles / grid_ctas) * grid_ctas : tiles;
    units = tiles_full + 2 * (tiles - tiles_full);
  }
  __device__ void unit(int u, int& mb, int& nb, int& kb0, int& kb1, bool& split) const {
    split = u >= tiles_full;
    const int t = split ? tiles_full + ((u - tiles_full) >> 1) : u;
    coords(t, mb, nb);
    const int half = k_blocks / 2;
    kb0 = split && ((u - tiles_full) & 1) ? half : 0;
    kb1 = split && !((u - tiles_full) & 1) ? half : k_blocks;
  }
  __host__ __device__ void coords(int t, int& mb, int& nb) const {
    const int per_group = group_m * n_blocks;
    const int group = t / per_group;
    const int first_m = group * group_m;
    const int rows = min(m_blocks - first_m, group_m);
    const int local = t - group * per_group;
    mb = first_m + local % rows;
    nb = local / rows;
  }
};
using TileGrid = TileGridT<kBM>;

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a,
                   const __grid_constant__ CUtensorMap map_b, float* __restrict__ c,
                   int m, int n, int k, int ldc, int split_tail, int* watchdog) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* epi_stage = reinterpret_cast<float*>(smem + kStages * kStageBytes);
  Barriers* bars = reinterpret_cast<Barriers*>(smem + kStages * kStageBytes + kEpiStageBytes);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  TileGrid grid;
  grid.init(m, n, k, gridDim.x, split_tail != 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&bars->full[s], 1);
      tc::mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&bars->tmem_full[b], 1);
      tc::mbar_init(&bars->tmem_empty[b], 128);
    }
    tc::mbar_init(&bars->drain, 1);
    bars->abort = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&map_a);
    tc::prefetch_tmap(&map_b);
  }
  if (warp == 1) tc::tmem_alloc(&bars->tmem_base, kTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_mask = 0, issued_parity = 0;
    for (int u = blockIdx.x; u < grid.units && !*abort; u += gridDim.x) {
      int mb, nb, kb0, kb1;
      bool split;
      grid.unit(u, mb, nb, kb0, kb1, split);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!tc::mbar_wait(&bars->empty[stage], phase ^ 1, abort, watchdog,
                           tc::kWatchdogGemm))
          break;
        uint8_t* sa = smem + stage * kStageBytes;
        uint8_t* sb = sa + kABytes;
        tc::mbar_expect_tx(&bars->full[stage], kStageBytes);
        tc::tma_load_2d(sa, &map_a, kb * kBK, mb * kBM, &bars->full[stage]);
#pragma unroll
        for (int j = 0; j < kBN / 64; ++j)
          tc::tma_load_2d(sb + j * kBBoxBytes, &map_b, nb * kBN + j * 64, kb * kBK,
                          &bars->full[stage]);
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if (*abort) {  // let in-flight TMA writes land before the CTA exits
      for (int s = 0; s < kStages; ++s)
        if (issued_mask & (1u << s)) {
          const uint32_t addr = tc::smem_u32(&bars->full[s]);
          for (uint32_t i = 0; i < tc::kMaxPolls; ++i)
            if (tc::mbar_try_wait(addr, (issued_parity >> s) & 1u)) break;
        }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool issued_any = false;
    for (int u = blockIdx.x; u < grid.units && !*abort; u += gridDim.x) {
      int mb, nb, kb0, kb1;
      bool split;
      grid.unit(u, mb, nb, kb0, kb1, split);
      if (!tc::mbar_wait(&bars->tmem_empty[acc], acc_phase ^ 1, abort, watchdog,
                         tc::kWatchdogGemm))
        break;
      tc::tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * kBN;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!tc::mbar_wait(&bars->full[stage], phase, abort, watchdog, tc::kWatchdogGemm))
          break;
        tc::tc_fence_after();
        const uint32_t a_addr = tc::smem_u32(smem + stage * kStageBytes);
        const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          // A: K-major rows of 128 B; a 16-wide K step is 32 B inside the
          // swizzle atom.  B: N-major, 64-column boxes 8 KB apart; a 16-row
          // K step is two 8-row groups (2 KB).
          const uint64_t a_desc = tc::smem_desc_sw128(a_addr + kk * 32, 16, 1024);
          const uint64_t b_desc = tc::smem_desc_sw128(b_addr + kk * 2048, kBBoxBytes, 1024);
          tc::umma_f16(d_tmem, a_desc, b_desc, kIdesc, (kb != kb0) || (kk != 0));
        }
        issued_any = true;
        tc::umma_commit(&bars->empty[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (*abort) break;
      tc::umma_commit(&bars->tmem_full[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (*abort && issued_any) {  // wait for issued MMAs before TMEM is freed
      tc::umma_commit(&bars->drain);
      const uint32_t addr = tc::smem_u32(&bars->drain);
      for (uint32_t i = 0; i < tc::kMaxPolls; ++i)
        if (tc::mbar_try_wait(addr, 0)) break;
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    // Each warp reads a 32x32 FP32 block (its 32 TMEM lanes = C rows, 32
    // columns) per chunk, transposes it through a padded shared buffer and
    // writes it row by row with lanes across columns: 128-byte coalesced
    // stores for any ldc (thread-per-row stores would touch 32 rows per
    // instruction).
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    float* stage = epi_stage + (warp - 2) * 32 * kStagePitch;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < grid.units; u += gridDim.x) {
      if (!tc::mbar_wait_warp(&bars->tmem_full[acc], acc_phase, abort, watchdog,
                              tc::kWatchdogGemm))
        break;
      tc::tc_fence_after();
      int mb, nb, kb0, kb1;
      bool split;
      grid.unit(u, mb, nb, kb0, kb1, split);
      const int row0 = mb * kBM + quarter * 32;
#pragma unroll 1
      for (int chunk = 0; chunk < kBN / 32; ++chunk) {
        float v[32];
        tc::tmem_ld32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                          acc * kBN + chunk * 32,
                      v);
#pragma unroll
        for (int i = 0; i < 32; ++i) stage[lane * kStagePitch + i] = v[i];
        __syncwarp();
        const int col = nb * kBN + chunk * 32 + lane;
        if (col < n) {
          const int rows = min(32, m - row0);
          if (split) {  // half of a tail tile: add into the zeroed C
#pragma unroll 4
            for (int rr = 0; rr < rows; ++rr)
              atomicAdd(c + static_cast<size_t>(row0 + rr) * ldc + col,
                        stage[rr * kStagePitch + lane]);
          } else {
#pragma unroll 4
            for (int rr = 0; rr < rows; ++rr)
              st_stream(c + static_cast<size_t>(row0 + rr) * ldc + col,
                        stage[rr * kStagePitch + lane]);
          }
        }
        __syncwarp();
      }
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->tmem_empty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc(tmem_base, kTmemCols);
}

// Zeroes the C tiles [tiles_full, tiles) that the GEMM will build from two
// K halves added together (0 + a + b is the same in either order, so the
// result stays deterministic).  One CTA per tile.
// Zeroes row slice `slice` (BM/16 rows, one column per thread, kBN threads)
// of tail tile `tail_index` of the tile grid (m, n, k, grid_ctas, group_m).
template <int BM>
__device__ __forceinline__ void zero_tail_slice(float* __restrict__ c, int m, int n, int k,
                                                int ldc, int grid_ctas, int group_m,
                                                int tail_index, int slice) {
  TileGridT<BM> grid;
  grid.group_m = group_m;
  grid.init(m, n, k, grid_ctas, true);
  int mb, nb;
  grid.coords(grid.tiles_full + tail_index, mb, nb);
  const int col = nb * kBN + threadIdx.x;
  if (col >= n) return;
  const int row0 = mb * BM + slice * (BM / 16);
  const int row_end = min(m, row0 + BM / 16);
#pragma unroll 8
  for (int row = row0; row < row_end; ++row) c[static_cast<size_t>(row) * ldc + col] = 0.0f;
}

template <int BM>
__global__ void __launch_bounds__(256)
    zero_tail_tiles_kernel(float* __restrict__ c, int m, int n, int k, int ldc,
                           int grid_ctas, int group_m) {
  // blockIdx.x: tail tile; blockIdx.y: its BM/16-row slice (16 per tile).
  zero_tail_slice<BM>(c, m, n, k, ldc, grid_ctas, group_m, blockIdx.x, blockIdx.y);
}

// The CTA-pair kernel's work split for C[m, n] over k: pairs in the grid
// and, when the last wave is split into K halves, how many tail tiles must be
// zeroed first (0 otherwise).  One place decides it, so a caller that zeroes
// the tail inside its own launch agrees with launch_gemm_tc.
struct PairPlan {
  bool use_pair = false;
  int pairs = 0, tail = 0, group_m = kGroupM;
  bool split_tail = false;
};

PairPlan pair_plan(int m, int n, int k) {
  PairPlan p;
  p.use_pair = m >= kPairBM && n >= kBN && sm_count() >= 2;
  if (!p.use_pair) return p;
  const int k_blocks = (k + kBK - 1) / kBK;
  const long long tiles =
      static_cast<long long>((m + kPairBM - 1) / kPairBM) * ((n + kBN - 1) / kBN);
  const int max_pairs = sm_count() / 2;
  p.pairs = static_cast<int>(tiles < max_pairs ? tiles : max_pairs);
  const int tail = static_cast<int>(tiles % p.pairs);
  p.split_tail = tiles > p.pairs && tail != 0 && 2 * tail <= p.pairs && k_blocks >= 8;
  p.tail = p.split_tail ? tail : 0;
  return p;
}

// Eight halves starting at half `o` (0..7) of the 16 halves in w[0..7]
// (little endian: half 2k is the low 16 bits of w[k]).
__device__ __forceinline__ uint4 halves_at(const uint32_t (&w)[8], int o) {
  uint32_t r[4];
  switch (o) {
#define OPL_EVEN(O)                                                   \
  case O:                                                             \
    r[0] = w[O / 2]; r[1] = w[O / 2 + 1]; r[2] = w[O / 2 + 2]; r[3] = w[O / 2 + 3]; \
    break;
#define OPL_ODD(O)                                                    \
  case O:                                                             \
    r[0] = __funnelshift_r(w[O / 2], w[O / 2 + 1], 16);               \
    r[1] = __funnelshift_r(w[O / 2 + 1], w[O / 2 + 2], 16);           \
    r[2] = __funnelshift_r(w[O / 2 + 2], w[O / 2 + 3], 16);           \
    r[3] = __funnelshift_r(w[O / 2 + 3], w[O / 2 + 4], 16);           \
    break;
    OPL_EVEN(0) OPL_ODD(1) OPL_EVEN(2) OPL_ODD(3) OPL_EVEN(4) OPL_ODD(5) OPL_EVEN(6)
    default: OPL_ODD(7)
#undef OPL_EVEN
#undef OPL_ODD
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// Widest N remainder whose product the A-padding pass computes itself.
constexpr int kPadDotMaxTail = 8;


// One zero-padded row-major FP16 matrix of the padding pass: src is rows x
// cols at any 2-byte-aligned base, dst is prow x pcol (pcol a multiple of 8).
struct PadJob {
  const __half* src;
  int rows, cols;
  __half* dst;
  int prow, pcol;
};

// Fallback for rows too long for pad_rows_bulk_kernel's shared-memory ring.
// Both operands' padded copies in ONE launch, one CTA per destination row
// (job 0's rows first, then job 1's).  Within a warp, lane l writes group
// g0 + l (8 halves = 16 bytes) of the row: it loads the one aligned 16-byte
// word under its group's start and takes the next word from lane l + 1 by
// shuffle (lane 31 loads one more), then shifts by the row's start offset --
// one 128-bit load and one 128-bit store per 16 bytes, no division (a
// thread-per-group grid with a 64-bit row division ran at 4.1 TB/s, this
// layout at 4.5 TB/s (5.1 TB/s with two CTAs per row, which the CTA-wide
// remainder dot below rules out; 512 threads per row: 4.0 TB/s); an aligned
// copy of the same bytes runs at 5.7 TB/s).
// With n_tail > 0, job 1's rows (A) also compute the narrow N remainder
// c[r][j] = sum over kk of A[r][kk] * bt[j][kk], j < n_tail <= kPadDotMaxTail,
// bt the K-major tail strip of B (row stride pcol, zero past cols; a few KB,
// served from L1): products of two halves are exact in FP32; each thread sums
// its groups in order, then warps (xor tree) and the CTA's warps in a fixed
// order, so results repeat bit for bit.
// The same launch also zeroes the CTA-pair GEMM's split tail tiles (16 CTAs
// per tile, before the rows), which would otherwise take a launch of its own.
constexpr int kPadThreads = 256;
static_assert(kPadThreads == kBN, "tail zeroing writes one column per thread");

struct TailZeroJob {
  float* c;
  int m, n, k, ldc, pairs, group_m, tail;  // tail == 0: nothing to zero
};

__global__ void __launch_bounds__(kPadThreads)
    pad_rows_kernel(PadJob j0, PadJob j1, const __half* __restrict__ bt, int n_tail,
                    float* __restrict__ c, int ldc, TailZeroJob zero) {
  __shared__ float part[kPadThreads / 32][kPadDotMaxTail];
  // The zeroing CTAs come first, so they run beside the rows rather than
  // as a tail after them.
  const int zero_ctas = 16 * zero.tail;
  if (static_cast<int>(blockIdx.x) < zero_ctas) {
    const int z = static_cast<int>(blockIdx.x);
    zero_tail_slice<kPairBM>(zero.c, zero.m, zero.n, zero.k, zero.ldc, zero.pairs,
                             zero.group_m, z >> 4, z & 15);
    return;
  }
  const int item = static_cast<int>(blockIdx.x) - zero_ctas;
  const bool second = item >= j0.prow;
  const PadJob& job = second ? j1 : j0;
  const int r = second ? item - j0.prow : item;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int groups = job.pcol / 8;
  const uintptr_t addr = reinterpret_cast<uintptr_t>(job.src);
  const uint4* src4 = reinterpret_cast<const uint4*>(addr & ~uintptr_t(15));
  const size_t lead = (addr & 15u) >> 1;
  const size_t total = (lead + static_cast<size_t>(job.rows) * job.cols + 7) / 8;
  const size_t row_h = lead + static_cast<size_t>(r) * job.cols;
  const int o = static_cast<int>(row_h & 7);
  const bool dot = second && n_tail > 0;
  float acc[kPadDotMaxTail];
#pragma unroll
  for (int t = 0; t < kPadDotMaxTail; ++t) acc[t] = 0.0f;
  uint4* drow = reinterpret_cast<uint4*>(job.dst + static_cast<size_t>(r) * job.pcol);
  for (int g0 = warp * 32; g0 < groups; g0 += kPadThreads) {
    const int g = g0 + lane;
    uint4 out = make_uint4(0, 0, 0, 0);
    if (r < job.rows && g0 * 8 < job.cols) {  // warp-uniform
      const size_t c0 = (row_h + static_cast<size_t>(g) * 8) >> 3;
      const uint4 lo = c0 < total ? __ldg(src4 + c0) : make_uint4(0, 0, 0, 0);
      uint4 extra = make_uint4(0, 0, 0, 0);
      if (lane == 31 && c0 + 1 < total) extra = __ldg(src4 + c0 + 1);
      uint4 hi;
      hi.x = __shfl_down_sync(kFullMask, lo.x, 1);
      hi.y = __shfl_down_sync(kFullMask, lo.y, 1);
      hi.z = __shfl_down_sync(kFullMask, lo.z, 1);
      hi.w = __shfl_down_sync(kFullMask, lo.w, 1);
      if (lane == 31) hi = extra;
      const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
      out = halves_at(w, o);
      const int valid = job.cols - g * 8;  // halves of this group inside the row
      if (valid < 8) {
        uint32_t* ow = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (2 * i >= valid) ow[i] = 0;
          else if (2 * i + 1 >= valid) ow[i] &= 0xffffu;
        }
      }
    }
    if (g < groups) {
      drow[g] = out;
      if (dot) {
        const __half2* a2 = reinterpret_cast<const __half2*>(&out);
#pragma unroll
        for (int t = 0; t < kPadDotMaxTail; ++t) {
          if (t < n_tail) {
            const uint4 bv =
                __ldg(reinterpret_cast<const uint4*>(bt + static_cast<size_t>(t) * job.pcol) + g);
            const __half2* b2 = reinterpret_cast<const __half2*>(&bv);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 af = __half22float2(a2[i]);
              const float2 bf = __half22float2(b2[i]);
              acc[t] = fmaf(af.x, bf.x, acc[t]);
              acc[t] = fmaf(af.y, bf.y, acc[t]);
            }
          }
        }
      }
    }
  }
  if (dot) {  // CTA-uniform
#pragma unroll
    for (int t = 0; t < kPadDotMaxTail; ++t) {
      if (t < n_tail) {
        const float v = warp_sum(acc[t]);
        if (lane == 0) part[warp][t] = v;
      }
    }
    __syncthreads();
    if (static_cast<int>(threadIdx.x) < n_tail) {
      float v = 0.0f;
#pragma unroll
      for (int w = 0; w < kPadThreads / 32; ++w) v += part[w][threadIdx.x];
      c[static_cast<size_t>(r) * ldc + threadIdx.x] = v;
    }
  }
}

// The padding pass with the source rows fetched by the copy engine: a
// persistent grid (kBulkCtasPerSm CTAs per SM) in which each CTA streams its
// rows (item w, w + P, ...) into
// a kBulkStages-deep shared-memory ring with one cp.async.bulk per row (the
// 16-byte-aligned words spanning the row: every word holds bytes of the row,
// so nothing outside the caller's matrix is read), completion on an mbarrier
// per stage; its threads then shift each staged row into place and write
// the padded row with coalesced 16-byte stores (and, for A's rows, the
// narrow remainder's dot: per-thread sums in group order, warp xor trees,
// then the warps in order, so results repeat bit for bit).  Up to
// kBulkStages rows per CTA are in flight without holding registers.  The
// dot's warp sums go to a ring of kDotRing rows and lanes of the last warp
// finish each row after the barrier that releases its stage, so the dot
// adds no barrier of its own; the CTAs zero the GEMM's split tail tiles
// while their first rows arrive.  Waits are bounded; a CTA that gives up
// trips the watchdog, waits (bounded) for its copies in flight and returns.
// 4095 x 4097 x 4093: 30 us against 38 us for pad_rows_kernel (one CTA per
// row, zeroing CTAs of their own), the copy alone ~23 us.
constexpr int kBulkStages = 4;
constexpr int kBulkCtasPerSm = 4;

__device__ __forceinline__ void bulk_load_1d(uint32_t dst, const void* src, uint32_t bytes,
                                             uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__global__ void __launch_bounds__(kPadThreads)
    pad_rows_bulk_kernel(PadJob j0, PadJob j1, const __half* __restrict__ bt, int n_tail,
                         float* __restrict__ c, int ldc, TailZeroJob zero, int stage_bytes,
                         int* watchdog) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ uint64_t full[kBulkStages];
  // Dot partials of the last kDotRing rows: part[row % kDotRing][warp][t].
  constexpr int kDotRing = 8;
  __shared__ float part[kDotRing][kPadThreads / 32][kPadDotMaxTail];
  __shared__ int abort_flag;
  const int w = static_cast<int>(blockIdx.x);
  const int workers = static_cast<int>(gridDim.x);
  const int rows_total = j0.prow + j1.prow;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBulkStages; ++s) tc::mbar_init(&full[s], 1);
    abort_flag = 0;
    tc::fence_barrier_init();
  }
  __syncthreads();
  const uint32_t ring_base = tc::smem_u32(ring);
  // Source range of item i's row: the aligned words holding it (bytes == 0:
  // a zero row past the source, nothing to load).
  auto source = [&](int item, const __half*& src, uint32_t& bytes, int& lead) {
    const bool second = item >= j0.prow;
    const PadJob& job = second ? j1 : j0;
    const int r = second ? item - j0.prow : item;
    bytes = 0;
    lead = 0;
    src = nullptr;
    if (r >= job.rows) return;
    const uintptr_t start = reinterpret_cast<uintptr_t>(job.src + static_cast<size_t>(r) * job.cols);
    const uintptr_t end = start + static_cast<uintptr_t>(job.cols) * 2;
    const uintptr_t a0 = start & ~uintptr_t(15), a1 = (end + 15) & ~uintptr_t(15);
    src = reinterpret_cast<const __half*>(a0);
    bytes = static_cast<uint32_t>(a1 - a0);
    lead = static_cast<int>((start & 15u) >> 1);
  };
  uint32_t pending = 0;  // thread 0: stages with a copy issued and not consumed
  auto issue = [&](int i) {  // thread 0
    const int item = w + i * workers;
    if (item >= rows_total) return;
    const __half* src;
    uint32_t bytes;
    int lead;
    source(item, src, bytes, lead);
    if (bytes == 0) return;
    const int st = i % kBulkStages;
    pending |= 1u << st;
    tc::mbar_expect_tx(&full[st], bytes);
    bulk_load_1d(ring_base + st * stage_bytes, src, bytes, tc::smem_u32(&full[st]));
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < kBulkStages; ++i) issue(i);
  // The GEMM's split tail tiles are zeroed while the first rows arrive.
  for (int z = w; z < 16 * zero.tail; z += workers)
    zero_tail_slice<kPairBM>(zero.c, zero.m, zero.n, zero.k, zero.ldc, zero.pairs,
                             zero.group_m, z >> 4, z & 15);
  // Lanes 0 .. n_tail - 1 of the last warp finish each row's dot.
  const int fin = static_cast<int>(threadIdx.x) - (kPadThreads - 32);
  uint32_t phases = 0;  // parity per stage (loaded rows only)
  bool ok = true;
  for (int i = 0;; ++i) {
    const int item = w + i * workers;
    if (item >= rows_total) break;
    const bool second = item >= j0.prow;
    const PadJob& job = second ? j1 : j0;
    const int r = second ? item - j0.prow : item;
    const int st = i % kBulkStages;
    const __half* src;
    uint32_t bytes;
    int lead;
    source(item, src, bytes, lead);
    if (bytes > 0) {
      const bool got = tc::mbar_wait(&full[st], (phases >> st) & 1u, &abort_flag, watchdog,
                                     tc::kWatchdogGemm);
      if (!__syncthreads_and(got)) {
        ok = false;
        break;
      }
      phases ^= 1u << st;
      pending &= ~(1u << st);
    }
    const uint4* staged = reinterpret_cast<const uint4*>(ring + st * stage_bytes);
    uint4* drow = reinterpret_cast<uint4*>(job.dst + static_cast<size_t>(r) * job.pcol);
    const int groups = job.pcol / 8;
    const bool dot = second && n_tail > 0;
    float acc[kPadDotMaxTail];
#pragma unroll
    for (int t = 0; t < kPadDotMaxTail; ++t) acc[t] = 0.0f;
    for (int g = threadIdx.x; g < groups; g += kPadThreads) {
      uint4 out = make_uint4(0, 0, 0, 0);
      const int valid = bytes > 0 ? job.cols - g * 8 : 0;  // halves of this group in the row
      if (valid > 0) {
        const uint4 lo = staged[g], hi = staged[g + 1];
        const uint32_t wv[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
        out = halves_at(wv, lead);
        if (valid < 8) {
          uint32_t* ow = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (2 * q >= valid) ow[q] = 0;
            else if (2 * q + 1 >= valid) ow[q] &= 0xffffu;
          }
        }
      }
      drow[g] = out;
      if (dot) {
        const __half2* a2 = reinterpret_cast<const __half2*>(&out);
#pragma unroll
        for (int t = 0; t < kPadDotMaxTail; ++t) {
          if (t < n_tail) {
            const uint4 bv =
                __ldg(reinterpret_cast<const uint4*>(bt + static_cast<size_t>(t) * job.pcol) + g);
            const __half2* b2 = reinterpret_cast<const __half2*>(&bv);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float2 af = __half22float2(a2[q]);
              const float2 bf = __half22float2(b2[q]);
              acc[t] = fmaf(af.x, bf.x, acc[t]);
              acc[t] = fmaf(af.y, bf.y, acc[t]);
            }
          }
        }
      }
    }
    if (dot) {  // CTA-uniform
#pragma unroll
      for (int t = 0; t < kPadDotMaxTail; ++t) {
        if (t < n_tail) {
          const float v = warp_sum(acc[t]);
          if (lane == 0) part[i % kDotRing][warp][t] = v;
        }
      }
    }
    __syncthreads();  // the stage is consumed (and the dot partials are in)
    if (threadIdx.x == 0) issue(i + kBulkStages);
    // Row i's slot is written again only at row i + kDotRing, after
    // kDotRing - 1 more barriers, so no barrier guards this read.
    if (dot && fin >= 0 && fin < n_tail) {
      float v = 0.0f;
#pragma unroll
      for (int q = 0; q < kPadThreads / 32; ++q) v += part[i % kDotRing][q][fin];
      c[static_cast<size_t>(r) * ldc + fin] = v;
    }
  }
  if (!ok && threadIdx.x == 0) {
    // Copies this CTA issued and did not consume: wait for them (bounded)
    // before the CTA's shared memory is released.
    for (int s = 0; s < kBulkStages; ++s) {
      if (!((pending >> s) & 1u)) continue;
      const uint32_t a = tc::smem_u32(&full[s]);
      const uint64_t t0 = globaltimer_ns();
      while (!tc::mbar_try_wait(a, (phases >> s) & 1u) && globaltimer_ns() - t0 < tc::kMaxWaitNs) {
      }
    }
  }
}

// ------------------------------------------------------------------ CTA pairs
// The same GEMM with the two-SM MMA (tcgen05.mma.cta_group::2, M=256): a
// cluster of two CTAs computes one 256 x 256 tile, each CTA holding 128 rows
// of A and 128 columns of B in its shared memory and 128 rows x 256 columns
// of the accumulator in its TMEM.  Per CTA and K block that is 32 KB of
// operands instead of 48 KB for the same MMA work, so shared-memory traffic
// (tensor-core reads plus TMA writes, ~192 B/clk in the one-SM kernel against
// ~128 B/clk available) no longer caps the tensor pipe.
//   warp 0 of each CTA  TMA producer for its own halves; completion is
//            counted on the leader CTA's "full" barrier (pair form of the
//            load, no multicast), the leader arming it with both CTAs' bytes;
//   warp 1 of the leader  issues the pair MMAs; its commits arrive on both
//            CTAs' "empty" / "tmem_full" barriers;
//   warps 2-5 of each CTA  epilogue of its 128 rows; each warp then arrives
//            on the leader's "tmem_empty" barrier.
// A cluster barrier after set-up and before exit keeps each CTA's barriers
// and TMEM alive while its partner may still use them.
constexpr int kPairStages = 6;
constexpr int kPairABytes = 128 * kBK * 2;   // 16 KB: this CTA's 128 rows of A
constexpr int kPairBBytes = 2 * kBBoxBytes;  // 16 KB: this CTA's 128 columns of B
constexpr int kPairStageBytes = kPairABytes + kPairBBytes;
constexpr uint32_t kPairIdesc = tc::idesc_f16_f32(kPairBM, kBN, false, true);
constexpr size_t kPairSmemBytes =
    kPairStages * kPairStageBytes + kEpiStageBytes + 1024 + 256;
constexpr uint16_t kPairMask = 0x3;  // both CTAs of the cluster

struct PairBarriers {
  uint64_t full[kPairStages];   // leader: both CTAs' loads of a stage
  uint64_t empty[kPairStages];  // each CTA: the pair MMAs released the stage
  uint64_t tmem_full[2];        // each CTA: accumulator complete
  uint64_t tmem_empty[2];       // leader: 8 epilogue warps (both CTAs) done
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap map_a,
                        const __grid_constant__ CUtensorMap map_b, float* __restrict__ c,
                        int m, int n, int k, int ldc, int split_tail, int group_m,
                        int* watchdog) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* epi_stage = reinterpret_cast<float*>(smem + kPairStages * kPairStageBytes);
  PairBarriers* bars =
      reinterpret_cast<PairBarriers*>(smem + kPairStages * kPairStageBytes + kEpiStageBytes);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int pairs = static_cast<int>(gridDim.x >> 1);
  TileGridT<kPairBM> grid;
  grid.group_m = group_m;
  grid.init(m, n, k, pairs, split_tail != 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      tc::mbar_init(&bars->full[s], 1);
      tc::mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&bars->tmem_full[b], 1);
      tc::mbar_init(&bars->tmem_empty[b], 8);
    }
    tc::mbar_init(&bars->drain, 1);
    bars->abort = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&map_a);
    tc::prefetch_tmap(&map_b);
  }
  if (warp == 1) tc::tmem_alloc_pair(&bars->tmem_base, kTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::cluster_sync();  // both CTAs' barriers exist before any cross-CTA use
  tc::tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    bool issued_any = false;
    for (int u = pair; u < grid.units && !*abort; u += pairs) {
      int mb, nb, kb0, kb1;
      bool split;
      grid.unit(u, mb, nb, kb0, kb1, split);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!tc::mbar_wait_cluster(&bars->empty[stage], phase ^ 1, abort, watchdog,
                                   tc::kWatchdogGemm))
          break;
        if (leader) tc::mbar_expect_tx(&bars->full[stage], 2 * kPairStageBytes);
        const uint32_t full_leader = tc::mapa_shared(&bars->full[stage], 0);
        uint8_t* sa = smem + stage * kPairStageBytes;
        uint8_t* sb = sa + kPairABytes;
        tc::tma_load_2d_pair(sa, &map_a, kb * kBK, mb * kPairBM + rank * 128, full_leader);
#pragma unroll
        for (int j = 0; j < 2; ++j)
          tc::tma_load_2d_pair(sb + j * kBBoxBytes, &map_b, nb * kBN + rank * 128 + j * 64,
                               kb * kBK, full_leader);
        issued_any = true;
        if (++stage == kPairStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if (*abort && issued_any) {
      // Completions of this CTA's loads are counted on the leader's
      // barriers; give the copies in flight time to land (bounded).
      for (int i = 0; i < (1 << 14); ++i) __nanosleep(64);
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool issued_any = false;
    for (int u = pair; u < grid.units && !*abort; u += pairs) {
      int mb, nb, kb0, kb1;
      bool split;
      grid.unit(u, mb, nb, kb0, kb1, split);
      if (!tc::mbar_wait_cluster(&bars->tmem_empty[acc], acc_phase ^ 1, abort, watchdog,
                                 tc::kWatchdogGemm))
        break;
      tc::tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * kBN;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!tc::mbar_wait_cluster(&bars->full[stage], phase, abort, watchdog,
                                   tc::kWatchdogGemm))
          break;
        tc::tc_fence_after();
        const uint32_t a_addr = tc::smem_u32(smem + stage * kPairStageBytes);
        const uint32_t b_addr = a_addr + kPairABytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          // Same operand layouts as the one-SM kernel, per CTA: A K-major
          // 128-byte rows (K step 32 B), B N-major 64-column boxes 8 KB
          // apart (K step two 8-row groups, 2 KB).
          const uint64_t a_desc = tc::smem_desc_sw128(a_addr + kk * 32, 16, 1024);
          const uint64_t b_desc = tc::smem_desc_sw128(b_addr + kk * 2048, kBBoxBytes, 1024);
          tc::umma_f16_pair(d_tmem, a_desc, b_desc, kPairIdesc, (kb != kb0) || (kk != 0));
        }
        issued_any = true;
        tc::umma_commit_pair(&bars->empty[stage], kPairMask);
        if (++stage == kPairStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (*abort) break;
      tc::umma_commit_pair(&bars->tmem_full[acc], kPairMask);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (*abort && issued_any) {  // wait for issued MMAs before TMEM is freed
      tc::umma_commit_pair(&bars->drain, 0x1);
      const uint32_t addr = tc::smem_u32(&bars->drain);
      for (uint32_t i = 0; i < tc::kMaxPolls; ++i)
        if (tc::mbar_try_wait(addr, 0)) break;
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    float* stage = epi_stage + (warp - 2) * 32 * kStagePitch;
    const uint32_t empty_leader0 = tc::mapa_shared(&bars->tmem_empty[0], 0);
    const uint32_t empty_leader1 = tc::mapa_shared(&bars->tmem_empty[1], 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = pair; u < grid.units; u += pairs) {
      if (!tc::mbar_wait_cluster_warp(&bars->tmem_full[acc], acc_phase, abort, watchdog,
                                      tc::kWatchdogGemm))
        break;
      tc::tc_fence_after();
      int mb, nb, kb0, kb1;
      bool split;
      grid.unit(u, mb, nb, kb0, kb1, split);
      const int row0 = mb * kPairBM + static_cast<int>(rank) * 128 + quarter * 32;
#pragma unroll 1
      for (int chunk = 0; chunk < kBN / 32; ++chunk) {
        float v[32];
        tc::tmem_ld32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kBN +
                          chunk * 32,
                      v);
#pragma unroll
        for (int i = 0; i < 32; ++i) stage[lane * kStagePitch + i] = v[i];
        __syncwarp();
        const int col = nb * kBN + chunk * 32 + lane;
        if (col < n) {
          const int rows = min(32, m - row0);
          if (split) {  // half of a tail tile: add into the zeroed C
#pragma unroll 4
            for (int rr = 0; rr < rows; ++rr)
              atomicAdd(c + static_cast<size_t>(row0 + rr) * ldc + col,
                        stage[rr * kStagePitch + lane]);
          } else {
#pragma unroll 4
            for (int rr = 0; rr < rows; ++rr)
              st_stream(c + static_cast<size_t>(row0 + rr) * ldc + col,
                        stage[rr * kStagePitch + lane]);
          }
        }
        __syncwarp();
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cluster(acc == 0 ? empty_leader0 : empty_leader1);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::cluster_sync();  // the partner is done with this CTA's barriers and TMEM
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc_pair(tmem_base, kTmemCols);
}

// tail_prezeroed: the caller already zeroed the pair plan's tail tiles.
cudaError_t launch_gemm_tc(const __half* a, const __half* b, float* c, int m, int n,
                           int k, int lda, int ldb, int ldc, cudaStream_t stream,
                           bool tail_prezeroed = false) {
  CUtensorMap map_a, map_b;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(lda) * 2};
    const uint32_t box[2] = {kBK, kBM};
    cudaError_t e = encode_tmap(&map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a, dims,
                                strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e != cudaSuccess) return e;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(ldb), static_cast<uint64_t>(k)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldb) * 2};
    const uint32_t box[2] = {64, kBK};
    cudaError_t e = encode_tmap(&map_b, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, b, dims,
                                strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e != cudaSuccess) return e;
  }
  const int k_blocks = (k + kBK - 1) / kBK;
  const PairPlan plan = pair_plan(m, n, k);
  if (plan.use_pair) {
    // CTA pairs: 256 x 256 tiles, one pair per two SMs.
    const int group_m = plan.group_m;
    const int pairs = plan.pairs;
    const bool split_tail = plan.split_tail;
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_pair_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kPairSmemBytes));
    if (e != cudaSuccess) return e;
    if (split_tail && !tail_prezeroed) {
      zero_tail_tiles_kernel<kPairBM><<<dim3(plan.tail, 16), kBN, 0, stream>>>(
          c, m, n, k, ldc, pairs, group_m);
      e = cudaGetLastError();
      if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(static_cast<unsigned>(2 * pairs));
    config.blockDim = dim3(kThreads);
    config.dynamicSmemBytes = kPairSmemBytes;
    config.stream = stream;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeClusterDimension;
    attribute[0].val.clusterDim.x = 2;
    attribute[0].val.clusterDim.y = 1;
    attribute[0].val.clusterDim.z = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelEx(&config, gemm_tc_pair_kernel, map_a, map_b, c, m, n, k, ldc,
                              split_tail ? 1 : 0, group_m, watchdog_word());
  }
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kSmemBytes));
  if (e != cudaSuccess) return e;
  const long long tiles =
      static_cast<long long>((m + kBM - 1) / kBM) * ((n + kBN - 1) / kBN);
  const int grid = static_cast<int>(tiles < sm_count() ? tiles : sm_count());
  // Split the tail tiles in K when the last wave would run at most half full
  // (two halves per CTA then still fit in one wave) and K is deep enough.
  const int tail = static_cast<int>(tiles % grid);
  const bool split_tail = tiles > grid && tail != 0 && 2 * tail <= grid && k_blocks >= 8;
  if (split_tail) {
    zero_tail_tiles_kernel<kBM><<<dim3(tail, 16), kBN, 0, stream>>>(c, m, n, k, ldc, grid,
                                                                   kGroupM);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  gemm_tc_kernel<<<grid, kThreads, kSmemBytes, stream>>>(map_a, map_b, c, m, n, k, ldc,
                                                         split_tail ? 1 : 0, watchdog_word());
  return cudaGetLastError();
}

// The n_tail columns [n_main, n_main + n_tail) of B (row stride ldb, k rows)
// as a K-major strip bt[j][kk] (row stride kp; zero for kk >= k).
__global__ void __launch_bounds__(256)
    tail_columns_kernel(const __half* __restrict__ b, int k, int ldb, int n_main, int n_tail,
                        __half* __restrict__ bt, int kp) {
  const int kk = blockIdx.x * 256 + threadIdx.x;
  if (kk >= kp) return;
  for (int j = 0; j < n_tail; ++j)
    bt[static_cast<size_t>(j) * kp + kk] =
        kk < k ? b[static_cast<size_t>(kk) * ldb + n_main + j] : __float2half(0.0f);
}

}  // namespace

// Tensor-core GEMM for any shape: strides that TMA cannot address (rows not
// a multiple of 16 bytes, or unaligned bases) go through zero-padded copies
// in a stream-ordered workspace.  When N ends in a narrow remainder (at most
// 64 columns past a multiple of the 256-wide tile), the 256-wide kernel
// covers the first n_main columns and the remainder runs as a skinny-N
// product (gemm_small_n_tc, or, for at most 8 columns when A needs a padded
// copy anyway, inside that copy's pass) -- instead of one extra, almost empty
// tile per 128 rows (4095 x 4097 x 4093: 544 tiles and a fourth wave vs 512).
cudaError_t gemm_f16_tc(const __half* a, const __half* b, float* c, int m, int n, int k,
                        cudaStream_t stream) {
  const bool a_ok = (k % 8 == 0) && aligned16(a);
  const bool b_ok = (n % 8 == 0) && (k % 8 == 0) && aligned16(b);
  const int n_tail = n % kBN;
  const bool split_n = n > kBN && n_tail != 0 && n_tail <= 64 && m > 128;
  if (a_ok && b_ok && !split_n) return launch_gemm_tc(a, b, c, m, n, k, k, n, n, stream);

  const int kp = (k + 7) & ~7;
  const int n_main = split_n ? n - n_tail : n;
  // B as the big kernel reads it: the caller's (b_ok) or a padded copy of
  // its first n_main columns (n_main rounded up to 8 without a split).
  const int ldb_copy = split_n ? n_main : ((n + 7) & ~7);
  const size_t a_elems = a_ok ? 0 : static_cast<size_t>(m) * kp;
  const size_t b_elems = b_ok ? 0 : static_cast<size_t>(kp) * ldb_copy;
  const size_t t_elems = split_n ? static_cast<size_t>(n_tail) * kp : 0;
  const size_t a_bytes = (a_elems * 2 + 255) & ~size_t(255);
  const size_t b_bytes = (b_elems * 2 + 255) & ~size_t(255);
  void* ws = nullptr;
  cudaError_t e = cudaMallocAsync(&ws, a_bytes + b_bytes + t_elems * 2 + 16, stream);
  if (e != cudaSuccess) return e;
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  const __half* a_use = a;
  const __half* b_use = b;
  __half* bt = reinterpret_cast<__half*>(wsb + a_bytes + b_bytes);
  // The remainder's K-major strip of B first (the A rows' dot reads it).
  if (split_n)
    tail_columns_kernel<<<(kp + 255) / 256, 256, 0, stream>>>(b, k, n, n_main, n_tail, bt, kp);
  // A narrow remainder is computed by the padding pass when A is padded.
  const bool tail_in_pad = split_n && !a_ok && n_tail <= kPadDotMaxTail;
  // Padded copies (B's rows first, then A's) in one launch.
  PadJob jobs[2];
  int n_jobs = 0;
  if (!b_ok) {
    __half* dst = reinterpret_cast<__half*>(wsb + a_bytes);
    jobs[n_jobs++] = PadJob{b, k, n, dst, kp, ldb_copy};
    b_use = dst;
  }
  if (!a_ok) {
    __half* dst = reinterpret_cast<__half*>(wsb);
    jobs[n_jobs++] = PadJob{a, m, k, dst, m, kp};
    a_use = dst;
  }
  if (n_jobs == 1) jobs[1] = jobs[0], jobs[0].prow = 0;  // the single job runs as job 1
  // The GEMM's split tail tiles are zeroed by the same launch.
  const PairPlan plan = pair_plan(m, n_main, kp);
  const TailZeroJob zero{c, m, n_main, kp, n, plan.pairs, plan.group_m, plan.tail};
  bool tail_zeroed = false;
  if (n_jobs > 0) {
    // (a block count beyond grid.x's limit fails to launch; the error is returned)
    const long long blocks =
        static_cast<long long>(jobs[0].prow) + jobs[1].prow + 16LL * zero.tail;
    // Ring stage: the widest staged row plus the one word the shift reads past
    // the last group.
    int words = 0;
    for (int j = 0; j < 2; ++j)
      if (jobs[j].prow > 0)
        words = std::max({words, jobs[j].pcol / 8, (jobs[j].cols + 7 + 7) / 8});
    const int stage_bytes = ((words + 1) * 16 + 127) & ~127;
    const int ring = kBulkStages * stage_bytes;
    const int per_sm = std::min(kBulkCtasPerSm, (200 * 1024) / ring);
    if (per_sm >= 1) {
      e = cudaFuncSetAttribute(pad_rows_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               ring);
      if (e == cudaSuccess) {
        const int bulk_blocks = per_sm * sm_count();
        pad_rows_bulk_kernel<<<bulk_blocks, kPadThreads, ring, stream>>>(
            jobs[0], jobs[1], bt, tail_in_pad ? n_tail : 0, c + n_main, n, zero, stage_bytes,
            watchdog_word());
      }
    } else {
      pad_rows_kernel<<<static_cast<unsigned>(blocks), kPadThreads, 0, stream>>>(
          jobs[0], jobs[1], bt, tail_in_pad ? n_tail : 0, c + n_main, n, zero);
    }
    tail_zeroed = true;
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  const int lda = a_ok ? k : kp;
  const int ldb = b_ok ? n : ldb_copy;
  if (e == cudaSuccess)
    e = launch_gemm_tc(a_use, b_use, c, m, n_main, kp, lda, ldb, n, stream, tail_zeroed);
  if (e == cudaSuccess && split_n && !tail_in_pad)
    e = gemm_small_n_tc(a_use, lda, bt, kp, c + n_main, n, m, n_tail, kp, stream);
  const cudaError_t f = cudaFreeAsync(ws, stream);
  return e != cudaSuccess ? e : f;
}

}  // namespace opl
