// Shared device/host helpers for the sm_100a operator kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstddef>
#include <cstdint>

#include "operatorlib/opl_capi.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "operatorlib-b200 kernels are written for sm_100a only"
#endif

namespace opl {

constexpr unsigned kFullMask = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFullMask, v, o));
  return v;
}

// Streaming 128-bit load that does not allocate in L1 (inputs are read once).
__device__ __forceinline__ float4 ld_stream(const float4* p) {
  float4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float ld_stream(const float* p) {
  float r;
  asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(r) : "l"(p));
  return r;
}

// Read-only loads as volatile asm.  In kernels launched with programmatic
// dependent launch, loads must stay after griddepcontrol.wait: an __ldg, or a
// plain load through a const __restrict__ pointer, lets the compiler assume
// the data never changes during the kernel and move the load ahead of the
// wait, where it can read what the previous kernel has not written yet.
__device__ __forceinline__ float ld_ro(const float* p) {
  float r;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ float4 ld_ro(const float4* p) {
  float4 r;
  asm volatile("ld.global.nc.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint4 ld_ro(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
// Coherent load of a value another grid wrote (FP64 partial sums).
__device__ __forceinline__ double ld_coherent(const double* p) {
  double r;
  asm volatile("ld.global.cg.f64 %0, [%1];" : "=d"(r) : "l"(p));  // L2, never a stale L1 line
  return r;
}

// Streaming stores: outputs are written once and not re-read by the kernel.
__device__ __forceinline__ void st_stream(float4* p, float4 v) { __stcs(p, v); }
__device__ __forceinline__ void st_stream(float* p, float v) { __stcs(p, v); }

// Kernels with bounded spin-waits write a non-zero code into the per-device
// watchdog word when a wait gives up (see opl_read_and_clear_watchdog); the
// word's device address comes from watchdog_word() and is a kernel argument.
__device__ __forceinline__ void watchdog_trip(int* word, int code) {
  atomicCAS(word, 0, code);
}

// Global nanosecond timer (%globaltimer), for wall-time bounds on spin-waits.
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Device address of the current device's watchdog word (nullptr on error).
int* watchdog_word();

// Number of SMs of the current device, cached per device (thread-safe).
int sm_count();
// Current device ordinal (cudaGetDevice), -1 on failure.
int current_device();

// Programmatic dependent launch for short row kernels: a kernel launched
// with launch_pdl may be scheduled while the previous kernel on the stream
// drains; pdl_begin() waits for that kernel's completion (and memory) before
// any global access, then lets the next such launch be scheduled.  Without
// the launch attribute both instructions return at once.
__device__ __forceinline__ void pdl_begin() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t stream,
                       Args... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = 0;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  return cudaLaunchKernelEx(&config, kernel, static_cast<KArgs>(args)...);
}

__host__ __device__ inline bool aligned16(const void* p) {
  return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0;
}

}  // namespace opl
