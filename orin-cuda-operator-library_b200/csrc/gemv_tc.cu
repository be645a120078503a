// Skinny FP16 GEMM (M <= 128) on the tensor cores with swapped operands
// (reference src/gemm.cu:455-479 sends small M to wmma_small_m_kernel /
// hgemm_scalar_kernel).
//
// With few rows of A the product is bound by streaming B (K x N FP16) from
// HBM, and a 128-row output tile would leave most of the GPU idle (N / 256
// tiles).  So the kernel computes the transposed product
//     C^T[N, M] = B^T[N, K] * A^T[K, M]
// with tcgen05.mma M=128 (128 columns of C per CTA) and N = M padded to
// 16/32/64/128: B is the MN-major "A" operand read straight from its
// row-major layout (two 64x64 TMA boxes per 64-deep K block, 128-byte
// swizzle), A the K-major "B" operand (one box of Mp rows, rows >= M filled
// with zeros by TMA).  The tensor cores do the arithmetic; the kernel's job is
// keeping HBM busy, so every CTA runs a deep TMA ring (6-11 stages, up to
// ~200 KB in flight per SM) with a single MMA-issuing thread draining it.
//
// K is split across the CTAs of a thread-block cluster (up to 8) so that
// ceil(N/128) column tiles still fill the SMs.  Each CTA leaves its FP32
// partial tile in its own shared memory; after a cluster barrier, CTA q sums
// output rows r = q, q + cs, ... over the cluster's partials in rank order
// through distributed shared memory and stores them.  One launch, no
// workspace, and a fixed summation order: results are deterministic.
//
// The same kernel serves skinny-N products (kSmallN): C[M, n] = A[M,K] B[K,n]
// for n <= 128 (the tail columns of a GEMM whose N is not a multiple of the
// big kernel's 256-wide tiles), with A as the big K-major operand (one
// 128 x 64 box per K block) and the n columns of B, transposed into a
// K-major [Np, K] strip, as the small one.
//
// No cluster multicast is used (each CTA loads its own tiles).  Every
// mbarrier wait is bounded; a wait that gives up sets the watchdog word,
// the CTA drains its outstanding copies and MMAs and still reaches both
// cluster barriers, so no CTA of the cluster is left waiting.
#include "gemm_simt.cuh"
#include "tc_common.cuh"
#include "tmap.cuh"

namespace opl {

namespace {

constexpr int kTile = 128;  // columns of C (rows of the MMA) per CTA
constexpr int kBK = 64;
constexpr int kBoxBytes = kBK * 64 * 2;  // 64 K rows x 64 columns of B
constexpr int kBtBytes = 2 * kBoxBytes;  // 16 KB per K block
constexpr int kThreads = 128;
constexpr int kMaxCluster = 8;
constexpr size_t kRingBudget = 200 * 1024;
constexpr int kWatchdogGemv = 0x6e05;

template <int MP, bool kSmallN>
struct GemvCfg {
  static constexpr int kABytes = MP * kBK * 2;  // Mp rows x 128 B
  static constexpr int kStageBytes = kBtBytes + kABytes;
  static constexpr int kStages = static_cast<int>(kRingBudget / kStageBytes);
  static constexpr uint32_t kTmemCols = MP < 32 ? 32 : MP;
  static constexpr uint32_t kIdesc = tc::idesc_f16_f32(kTile, MP, !kSmallN, false);
  static constexpr int kRedBytes = MP * kTile * 4;  // partial tile, aliases the ring
  static_assert(kRedBytes <= kStages * kStageBytes, "partial tile must fit in the ring");
  static constexpr size_t kSmem = static_cast<size_t>(kStages) * kStageBytes + 1024 + 512;
};

template <int S>
struct GemvBars {
  uint64_t full[S];
  uint64_t empty[S];
  uint64_t done;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}

// Reads a float from the shared memory of cluster CTA `rank` at the address
// that `local` has in this CTA.
__device__ __forceinline__ float ld_cluster_f32(const float* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(remote)
               : "r"(tc::smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// map_b: the big operand (B, or A when kSmallN); map_a: the small one.  n is
// the big extent (columns of C, or rows when kSmallN), m the small one.
template <int MP, bool kSmallN>
__global__ void __launch_bounds__(kThreads, 1)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_a, float* __restrict__ c, int m,
                   int n, int ldc, int k_blocks, int kb_per, int* watchdog) {
  using Cfg = GemvCfg<MP, kSmallN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto* bars = reinterpret_cast<GemvBars<S>*>(smem + S * Cfg::kStageBytes);
  float* red = reinterpret_cast<float*>(smem);  // [MP][kTile], after the last MMA
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  uint32_t cluster_n;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(cluster_n));
  const int tile = static_cast<int>(blockIdx.x / cluster_n);
  const int n0 = tile * kTile;
  const int kb0 = static_cast<int>(rank) * kb_per;
  const int kb1 = min(k_blocks, kb0 + kb_per);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      tc::mbar_init(&bars->full[s], 1);
      tc::mbar_init(&bars->empty[s], 1);
    }
    tc::mbar_init(&bars->done, 1);
    bars->abort = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&map_b);
    tc::prefetch_tmap(&map_a);
  }
  if (warp == 2) tc::tmem_alloc(&bars->tmem_base, Cfg::kTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  // Programmatic dependent launch: the set-up above overlaps the previous
  // kernel on the stream; global memory is touched only after it completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_mask = 0, issued_parity = 0;
    for (int kb = kb0; kb < kb1 && !*abort; ++kb) {
      if (!tc::mbar_wait(&bars->empty[stage], phase ^ 1, abort, watchdog, kWatchdogGemv))
        break;
      uint8_t* sb = smem + stage * Cfg::kStageBytes;
      tc::mbar_expect_tx(&bars->full[stage], Cfg::kStageBytes);
      if (kSmallN) {
        tc::tma_load_2d(sb, &map_b, kb * kBK, n0, &bars->full[stage]);  // 128 rows x 64 K
      } else {
        tc::tma_load_2d(sb, &map_b, n0, kb * kBK, &bars->full[stage]);
        tc::tma_load_2d(sb + kBoxBytes, &map_b, n0 + 64, kb * kBK, &bars->full[stage]);
      }
      tc::tma_load_2d(sb + kBtBytes, &map_a, kb * kBK, 0, &bars->full[stage]);
      issued_mask |= 1u << stage;
      issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
      if (++stage == S) {
        stage = 0;
        phase ^= 1;
      }
    }
    if (*abort) {  // let in-flight TMA writes land before the CTA moves on
      for (int s = 0; s < S; ++s)
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
    for (int kb = kb0; kb < kb1; ++kb) {
      if (!tc::mbar_wait(&bars->full[stage], phase, abort, watchdog, kWatchdogGemv)) break;
      tc::tc_fence_after();
      const uint32_t bt = tc::smem_u32(smem + stage * Cfg::kStageBytes);
      const uint32_t at = bt + kBtBytes;
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) {
        // B^T: MN-major, two 64-column boxes 8 KB apart, a 16-deep K step is
        // two 8-row groups (2 KB).  A^T: K-major 128-byte rows, a K step is
        // 32 B inside the swizzle atom.
        // (kSmallN: the big operand is K-major like A^T.)
        const uint64_t bt_desc = kSmallN ? tc::smem_desc_sw128(bt + kk * 32, 16, 1024)
                                         : tc::smem_desc_sw128(bt + kk * 2048, kBoxBytes, 1024);
        const uint64_t at_desc = tc::smem_desc_sw128(at + kk * 32, 16, 1024);
        tc::umma_f16(tmem, bt_desc, at_desc, Cfg::kIdesc, (kb != kb0) || (kk != 0));
      }
      tc::umma_commit(&bars->empty[stage]);
      if (++stage == S) {
        stage = 0;
        phase ^= 1;
      }
    }
    // Arrives when every MMA issued above has completed (at once if none).
    tc::umma_commit(&bars->done);
  }
  __syncwarp();

  // ------------------------------------------------------------ epilogue
  // Thread t owns TMEM lane t = column n0 + t of C; its MP accumulator
  // columns are the rows of C.
  const bool have = kb1 > kb0;
  bool ok = tc::mbar_wait_warp(&bars->done, 0, abort, watchdog, kWatchdogGemv);
  tc::tc_fence_after();
  const int t = threadIdx.x;
  const int col = n0 + t;
#pragma unroll 1
  for (int c0 = 0; c0 < MP; c0 += 32) {
    float v[32];
    if (ok && have) {
      tc::tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c0, v);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = ok ? 0.0f : __int_as_float(0x7fffffff);
    }
    const int rows = min(32, MP - c0);
    if (cluster_n == 1) {
#pragma unroll
      for (int r = 0; r < 32; ++r)
        if (col < n && r < rows && c0 + r < m)
          c[kSmallN ? static_cast<size_t>(col) * ldc + c0 + r
                    : static_cast<size_t>(c0 + r) * ldc + col] = v[r];
    } else {
#pragma unroll
      for (int r = 0; r < 32; ++r)
        if (r < rows) red[(c0 + r) * kTile + t] = v[r];
    }
  }

  if (cluster_n > 1) {
    cluster_sync_all();  // every CTA's partial tile is in its shared memory
    if (col < n)
      for (int r = static_cast<int>(rank); r < m; r += static_cast<int>(cluster_n)) {
        float s = 0.0f;
        for (uint32_t p = 0; p < cluster_n; ++p) s += ld_cluster_f32(red + r * kTile + t, p);
        c[kSmallN ? static_cast<size_t>(col) * ldc + r : static_cast<size_t>(r) * ldc + col] = s;
      }
    cluster_sync_all();  // peers keep their shared memory until all reads are done
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 2) tc::tmem_dealloc(tmem, Cfg::kTmemCols);
}

// Encodes the maps and launches.  Skinny-M: big = B [k][n] (row stride ldb),
// small = A [m][k].  Skinny-N: big = A [m_big][k] (row stride lda), small =
// the K-major strip [Np][k] (row stride ld_small); `n` is then m_big and `m`
// the number of tail columns.
template <int MP, bool kSmallN>
cudaError_t launch_gemv_tc(const __half* big, int ld_big, const __half* small, int ld_small,
                           float* c, int ldc, int m, int n, int k, cudaStream_t stream) {
  using Cfg = GemvCfg<MP, kSmallN>;
  CUtensorMap map_b, map_a;
  {
    const uint64_t dims[2] = {kSmallN ? static_cast<uint64_t>(k) : static_cast<uint64_t>(n),
                              kSmallN ? static_cast<uint64_t>(n) : static_cast<uint64_t>(k)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ld_big) * 2};
    const uint32_t box[2] = {64, kSmallN ? static_cast<uint32_t>(kTile) : kBK};
    cudaError_t e = encode_tmap(&map_b, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, big, dims, strides,
                                box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e != cudaSuccess) return e;
  }
  {
    // Rows past m (the small extent) read as zero.
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ld_small) * 2};
    const uint32_t box[2] = {kBK, MP};
    cudaError_t e = encode_tmap(&map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, small, dims,
                                strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e != cudaSuccess) return e;
  }
  cudaError_t e = cudaFuncSetAttribute(gemv_tc_kernel<MP, kSmallN>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(Cfg::kSmem));
  if (e != cudaSuccess) return e;

  // Tiles of 128 along the big extent x K splits: as many splits (one per
  // cluster CTA, at most 8) as keep tiles * splits within the SM count,
  // every split non-empty.
  const int tiles = (n + kTile - 1) / kTile;
  const int k_blocks = (k + kBK - 1) / kBK;
  int cs = sm_count() / tiles;
  cs = cs < 1 ? 1 : (cs > kMaxCluster ? kMaxCluster : cs);
  if (cs > k_blocks) cs = k_blocks;
  const int kb_per = (k_blocks + cs - 1) / cs;
  cs = (k_blocks + kb_per - 1) / kb_per;

  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(static_cast<unsigned>(tiles * cs));
  config.blockDim = dim3(kThreads);
  config.dynamicSmemBytes = Cfg::kSmem;
  config.stream = stream;
  cudaLaunchAttribute attribute[2];
  attribute[0].id = cudaLaunchAttributeClusterDimension;
  attribute[0].val.clusterDim.x = static_cast<unsigned>(cs);
  attribute[0].val.clusterDim.y = 1;
  attribute[0].val.clusterDim.z = 1;
  attribute[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[1].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attribute;
  config.numAttrs = 2;
  return cudaLaunchKernelEx(&config, gemv_tc_kernel<MP, kSmallN>, map_b, map_a, c, m, n, ldc,
                            k_blocks, kb_per, watchdog_word());
}

}  // namespace

bool gemv_tc_supported(const void* a, const void* b, int m, int n, int k) {
  return m >= 1 && m <= 128 && n % 8 == 0 && k % 8 == 0 && aligned16(a) && aligned16(b);
}

cudaError_t gemv_tc(const __half* a, const __half* b, float* c, int m, int n, int k,
                    cudaStream_t stream) {
  if (m <= 16) return launch_gemv_tc<16, false>(b, n, a, k, c, n, m, n, k, stream);
  if (m <= 32) return launch_gemv_tc<32, false>(b, n, a, k, c, n, m, n, k, stream);
  if (m <= 64) return launch_gemv_tc<64, false>(b, n, a, k, c, n, m, n, k, stream);
  return launch_gemv_tc<128, false>(b, n, a, k, c, n, m, n, k, stream);
}

cudaError_t gemm_small_n_tc(const __half* a, int lda, const __half* bt, int ldbt, float* c,
                            int ldc, int m, int ns, int k, cudaStream_t stream) {
  if (ns <= 16) return launch_gemv_tc<16, true>(a, lda, bt, ldbt, c, ldc, ns, m, k, stream);
  if (ns <= 32) return launch_gemv_tc<32, true>(a, lda, bt, ldbt, c, ldc, ns, m, k, stream);
  if (ns <= 64) return launch_gemv_tc<64, true>(a, lda, bt, ldbt, c, ldc, ns, m, k, stream);
  return launch_gemv_tc<128, true>(a, lda, bt, ldbt, c, ldc, ns, m, k, stream);
}

}  // namespace opl
