// Multi-GPU reduce-sum fused with its all-reduce over NVLink peer memory.
//
// The reference's reduce is single-GPU (src/reduce.cu:54-69).  Sharded across
// G GPUs, each GPU sums its chunk and the G partial sums must be combined:
// the one real exchange on this operator path.  Instead of a separate NCCL
// all-reduce launch, the finalize kernel of the reduce does the exchange
// itself: it writes this GPU's FP64 partial into a slot of every peer's team
// buffer with peer stores, publishes a flag with a system-scope release
// store, waits (bounded) for every peer's flag, and adds the G slots in rank
// order -- so all GPUs compute the bit-identical total.
//
// Team buffer (one cudaMalloc per GPU, opened by the peers through CUDA IPC):
//   uint64 seq                       local call counter (device side, so the
//                                    launch is replayable in a CUDA graph)
//   uint64 flags[kMaxTeam]           flags[r] = last call number rank r posted
//   double slots[2][kMaxTeam]        slots[call parity][r] = rank r's partial
//   uint64 failed                    set (locally, never by a peer) when this
//                                    rank's wait for a peer timed out
// A rank can post call c+1 only after it saw every flag of call c, which each
// peer raises only after it finished reading its slots for call c-1 (same
// parity as c+1): double-buffered slots never overwrite unread values.
//
// A rank whose wait timed out has not seen every flag of that call, so it may
// never post again: its `failed` word stays set and every later call on it
// returns NaN at once without touching the peers.  A peer still waiting for
// it times out in turn (its own wait is bounded too) and fails the same way,
// so after a timeout the whole team answers NaN until it is destroyed and
// created again.
//
// Plain peer loads/stores only (no multimem, no TMA, no cluster multicast).
#include <cstring>
#include <new>

#include "reduce_impl.cuh"

namespace opl {

namespace {

constexpr int kMaxTeam = 8;
constexpr uint32_t kTeamMaxPolls = 1u << 24;              // backstop
constexpr uint64_t kTeamMaxWaitNs = 2000ull * 1000ull * 1000ull;  // 2 s
constexpr int kWatchdogTeam = 0x6e04;

struct TeamBuffer {
  unsigned long long seq;
  unsigned long long flags[kMaxTeam];
  double slots[2][kMaxTeam];
  unsigned long long failed;
};

struct TeamPeers {
  TeamBuffer* peer[kMaxTeam];  // peer[r] = rank r's buffer, mapped here
};

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// One CTA: fixed-order sum of this GPU's CTA partials; then its first warp
// exchanges with the team and sums the team's partials in rank order.
__global__ void __launch_bounds__(kReduceThreads)
    reduce_team_finalize_kernel(const double* __restrict__ partials, int count,
                                TeamPeers peers, int rank, int world,
                                float* __restrict__ output, int* watchdog) {
  __shared__ double local_total;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  double v = sum_partials_strided(partials, count);
  v = block_sum_fixed(v);
  if (threadIdx.x == 0) local_total = v;
  __syncthreads();
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  v = local_total;

  TeamBuffer* mine = peers.peer[rank];
  if (mine->failed != 0) {  // an earlier call timed out: never post again
    if (lane == 0) *output = __int_as_float(0x7fffffff);
    return;
  }
  const unsigned long long call = mine->seq + 1;  // same on every rank
  const int parity = static_cast<int>(call & 1);
  if (lane < world) {
    TeamBuffer* dst = peers.peer[lane];
    dst->slots[parity][rank] = v;
    st_release_sys(&dst->flags[rank], call);
  }
  bool ok = true;
  if (lane < world) {
    const uint64_t start = globaltimer_ns();
    uint32_t polls = 0;
    while (ld_acquire_sys(&mine->flags[lane]) < call) {
      if (++polls == kTeamMaxPolls ||
          ((polls & 63u) == 0u && globaltimer_ns() - start > kTeamMaxWaitNs)) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  ok = __all_sync(kFullMask, ok);
  if (lane == 0) {
    if (!ok) {
      watchdog_trip(watchdog, kWatchdogTeam);
      mine->failed = 1;
      *output = __int_as_float(0x7fffffff);  // NaN marks the failed exchange
    } else {
      double total = 0.0;
      for (int r = 0; r < world; ++r) {
        (void)ld_acquire_sys(&mine->flags[r]);  // orders this lane's slot reads
        total += mine->slots[parity][r];
      }
      *output = static_cast<float>(total);
    }
    mine->seq = call;
  }
}

}  // namespace

struct Team {
  int rank = 0;
  int world = 0;
  int device = -1;
  TeamBuffer* local = nullptr;
  TeamPeers peers{};
  bool opened[kMaxTeam] = {};
};

}  // namespace opl

extern "C" {

int opl_team_create(int rank, int world, void** team_out, void* ipc_handle_out) {
  using namespace opl;
  if (team_out == nullptr || ipc_handle_out == nullptr || world < 1 || world > kMaxTeam ||
      rank < 0 || rank >= world)
    return cudaErrorInvalidValue;
  Team* team = new (std::nothrow) Team;
  if (team == nullptr) return cudaErrorMemoryAllocation;
  team->rank = rank;
  team->world = world;
  team->device = current_device();
  cudaError_t e = cudaMalloc(&team->local, sizeof(TeamBuffer));
  if (e == cudaSuccess) e = cudaMemset(team->local, 0, sizeof(TeamBuffer));
  cudaIpcMemHandle_t handle;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&handle, team->local);
  if (e != cudaSuccess) {
    if (team->local != nullptr) cudaFree(team->local);
    delete team;
    return e;
  }
  std::memcpy(ipc_handle_out, &handle, sizeof(handle));
  team->peers.peer[rank] = team->local;
  *team_out = team;
  return cudaSuccess;
}

int opl_team_connect(void* team_ptr, const void* all_handles) {
  using namespace opl;
  Team* team = static_cast<Team*>(team_ptr);
  if (team == nullptr || all_handles == nullptr) return cudaErrorInvalidValue;
  const auto* handles = static_cast<const cudaIpcMemHandle_t*>(all_handles);
  for (int r = 0; r < team->world; ++r) {
    if (r == team->rank || team->opened[r]) continue;
    void* ptr = nullptr;
    const cudaError_t e =
        cudaIpcOpenMemHandle(&ptr, handles[r], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return e;
    team->peers.peer[r] = static_cast<TeamBuffer*>(ptr);
    team->opened[r] = true;
  }
  return cudaSuccess;
}

int opl_team_reduce_sum_f32(void* team_ptr, const float* input, float* output, size_t n,
                            opl_stream_t stream) {
  using namespace opl;
  Team* team = static_cast<Team*>(team_ptr);
  if (team == nullptr || input == nullptr || output == nullptr || n == 0)
    return cudaErrorInvalidValue;
  for (int r = 0; r < team->world; ++r)
    if (team->peers.peer[r] == nullptr) return cudaErrorInvalidValue;  // not connected
  const int blocks = reduce_grid(input, n);
  void* workspace = nullptr;
  cudaError_t e = cudaMallocAsync(&workspace, blocks * sizeof(double), stream);
  if (e != cudaSuccess) return e;
  double* partials = static_cast<double*>(workspace);
  e = reduce_partials_launch(input, n, partials, blocks, stream);
  if (e == cudaSuccess) {
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(1);
    config.blockDim = dim3(kReduceThreads);
    config.stream = stream;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    const double* partials_const = partials;
    e = cudaLaunchKernelEx(&config, reduce_team_finalize_kernel, partials_const, blocks,
                           team->peers, team->rank, team->world, output, watchdog_word());
  }
  const cudaError_t f = cudaFreeAsync(workspace, stream);
  return e != cudaSuccess ? e : f;
}

int opl_team_destroy(void* team_ptr) {
  using namespace opl;
  Team* team = static_cast<Team*>(team_ptr);
  if (team == nullptr) return cudaErrorInvalidValue;
  cudaError_t first = cudaSuccess;
  for (int r = 0; r < team->world; ++r)
    if (team->opened[r]) {
      const cudaError_t e = cudaIpcCloseMemHandle(team->peers.peer[r]);
      if (first == cudaSuccess) first = e;
    }
  const cudaError_t e = cudaFree(team->local);
  if (first == cudaSuccess) first = e;
  delete team;
  return first;
}

}  // extern "C"
