// Library runtime: per-device caches, the watchdog word, utility entry points
// of the C-ABI and the C++ API (operators.h) forwarding onto the C-ABI.
#include <atomic>

#include "operatorlib/operators.h"
#include "opl_common.cuh"

namespace {

constexpr int kMaxDevices = 64;

__device__ int g_watchdog_word;

std::atomic<int> g_sm_count[kMaxDevices];
std::atomic<int*> g_watchdog_ptr[kMaxDevices];

}  // namespace

namespace opl {

int current_device() {
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) return -1;
  return device;
}

int sm_count() {
  const int device = current_device();
  if (device < 0 || device >= kMaxDevices) return 148;
  int cached = g_sm_count[device].load(std::memory_order_relaxed);
  if (cached > 0) return cached;
  int value = 0;
  if (cudaDeviceGetAttribute(&value, cudaDevAttrMultiProcessorCount, device) !=
          cudaSuccess ||
      value <= 0)
    return 148;
  g_sm_count[device].store(value, std::memory_order_relaxed);
  return value;
}

int* watchdog_word() {
  const int device = current_device();
  if (device < 0 || device >= kMaxDevices) return nullptr;
  int* cached = g_watchdog_ptr[device].load(std::memory_order_acquire);
  if (cached != nullptr) return cached;
  void* address = nullptr;
  if (cudaGetSymbolAddress(&address, g_watchdog_word) != cudaSuccess)
    return nullptr;
  g_watchdog_ptr[device].store(static_cast<int*>(address),
                               std::memory_order_release);
  return static_cast<int*>(address);
}

}  // namespace opl

extern "C" {

const char* opl_error_string(int error) {
  return cudaGetErrorString(static_cast<cudaError_t>(error));
}

int opl_read_and_clear_watchdog(int* code) {
  if (code == nullptr) return cudaErrorInvalidValue;
  int* word = opl::watchdog_word();
  if (word == nullptr) return cudaErrorInvalidDevice;
  cudaError_t error = cudaDeviceSynchronize();
  if (error != cudaSuccess) return error;
  error = cudaMemcpy(code, word, sizeof(int), cudaMemcpyDeviceToHost);
  if (error != cudaSuccess) return error;
  return cudaMemset(word, 0, sizeof(int));
}

const char* opl_version(void) { return "opl-b200 0.1.0 sm_100a"; }

}  // extern "C"

// C++ API of operators.h: one-to-one forwarders onto the C-ABI.
namespace operatorlib {

cudaError_t reduce_sum_f32(const float* input, float* output, std::size_t n,
                           cudaStream_t stream) {
  return static_cast<cudaError_t>(opl_reduce_sum_f32(input, output, n, stream));
}

cudaError_t softmax_f32(const float* input, float* output, int rows, int cols,
                        cudaStream_t stream) {
  return static_cast<cudaError_t>(
      opl_softmax_f32(input, output, rows, cols, stream));
}

cudaError_t transpose_f32(const float* input, float* output, int rows, int cols,
                          cudaStream_t stream) {
  return static_cast<cudaError_t>(
      opl_transpose_f32(input, output, rows, cols, stream));
}

cudaError_t rmsnorm_f32(const float* input, const float* weight, float* output,
                        int tokens, int hidden, float epsilon,
                        cudaStream_t stream) {
  return static_cast<cudaError_t>(
      opl_rmsnorm_f32(input, weight, output, tokens, hidden, epsilon, stream));
}

cudaError_t gemm_f32(const float* a, const float* b, float* c, int m, int n,
                     int k, cudaStream_t stream) {
  return static_cast<cudaError_t>(opl_gemm_f32(a, b, c, m, n, k, stream));
}

cudaError_t gemm_f16(const __half* a, const __half* b, float* c, int m, int n,
                     int k, cudaStream_t stream) {
  return static_cast<cudaError_t>(
      opl_gemm_f16(reinterpret_cast<const opl_half_t*>(a),
                   reinterpret_cast<const opl_half_t*>(b), c, m, n, k, stream));
}

cudaError_t attention_f32(const float* q, const float* k, const float* v,
                          float* output, int batch, int heads, int sequence,
                          int head_dim, bool causal, cudaStream_t stream) {
  return static_cast<cudaError_t>(opl_attention_f32(
      q, k, v, output, batch, heads, sequence, head_dim, causal ? 1 : 0,
      stream));
}

cudaError_t attention_f16(const __half* q, const __half* k, const __half* v,
                          float* output, int batch, int heads, int sequence,
                          int head_dim, bool causal, cudaStream_t stream) {
  return static_cast<cudaError_t>(opl_attention_f16(
      reinterpret_cast<const opl_half_t*>(q),
      reinterpret_cast<const opl_half_t*>(k),
      reinterpret_cast<const opl_half_t*>(v), output, batch, heads, sequence,
      head_dim, causal ? 1 : 0, stream));
}

}  // namespace operatorlib

// ---------------------------------------------------------------- TMA maps

#include <cudaTypedefs.h>

#include <mutex>

#include "tmap.cuh"

namespace opl {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

cudaError_t encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank,
                        const void* base, const uint64_t* dims,
                        const uint64_t* strides_bytes, const uint32_t* box,
                        CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault,
                                &status) == cudaSuccess &&
        status == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr) return cudaErrorNotSupported;
  cuuint64_t gdim[3];
  cuuint64_t gstride[2];
  cuuint32_t boxdim[3];
  cuuint32_t estride[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    boxdim[i] = box[i];
    if (i + 1 < rank) gstride[i] = strides_bytes[i];
  }
  const CUresult r = g_encode(map, dtype, static_cast<cuuint32_t>(rank),
                              const_cast<void*>(base), gdim, gstride, boxdim, estride,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace opl
