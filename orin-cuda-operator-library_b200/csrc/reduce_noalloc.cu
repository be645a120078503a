// Reduce-sum variant that allocates nothing, for callers that cannot call
// cudaMalloc / cudaMallocAsync: code running where the allocator is off
// limits (inside an allocator hook or a memory-pool callback, under a
// framework that owns all device memory and forbids allocation on its
// streams, or with a fixed memory budget that a per-call workspace would
// break).
//
// Same kernels and the same deterministic result as opl_reduce_sum_f32; only
// the FP64 partial sums live in the file-scope array below instead of a
// stream-ordered workspace.  The array is a fixed 4096 FP64 slots (32 KiB)
// that every GPU loading this library keeps until the process exits.
//
// The array's name is a host-side stand-in in host code, not a device
// address: the device address is fetched with cudaGetSymbolAddress, once per
// device with that device current, on the first call made on that device
// (make that first call before any stream capture), and cached.  The cached
// address does not survive cudaDeviceReset: after a reset of a device, a
// process must not call this entry point on that device again.
//
// Every call shares the array and it keeps the previous call's contents.
// Nothing needs clearing: each call writes every slot it later reads.  Calls
// whose kernels overlap on the GPU (different streams, or different host
// threads on one device) race on the array and give wrong sums; serialise
// them on one stream.
#include <atomic>

#include "reduce_impl.cuh"

namespace opl {
namespace {

constexpr int kScratchSlots = 4096;
// reduce_grid never returns more than kReduceMaxCtas CTAs, one slot each.
static_assert(kScratchSlots >= kReduceMaxCtas,
              "the scratch array must hold one partial per reduce CTA");
constexpr int kMaxDevices = 64;

__device__ __align__(256) double g_reduce_scratch[kScratchSlots];

std::atomic<double*> g_scratch_ptr[kMaxDevices];

// Device address of g_reduce_scratch on the current device (set-up on first
// use per device).  Returns the CUDA error of the lookup on failure.
cudaError_t scratch_address(double** out) {
  const int device = current_device();
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  double* cached = g_scratch_ptr[device].load(std::memory_order_acquire);
  if (cached == nullptr) {
    void* address = nullptr;
    const cudaError_t error = cudaGetSymbolAddress(&address, g_reduce_scratch);
    if (error != cudaSuccess) return error;
    cached = static_cast<double*>(address);
    g_scratch_ptr[device].store(cached, std::memory_order_release);
  }
  *out = cached;
  return cudaSuccess;
}

}  // namespace
}  // namespace opl

extern "C" int opl_reduce_sum_f32_noalloc(const float* input, float* output,
                                          size_t n, opl_stream_t stream) {
  if (input == nullptr || output == nullptr || n == 0) return cudaErrorInvalidValue;
  const int blocks = opl::reduce_grid(input, n);
  double* scratch = nullptr;
  const cudaError_t error = opl::scratch_address(&scratch);
  if (error != cudaSuccess) return error;
  return opl::reduce_enqueue(input, n, scratch, blocks, output, nullptr, stream);
}
