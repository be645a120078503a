#ifndef OPERATORLIB_OPL_CAPI_H_
#define OPERATORLIB_OPL_CAPI_H_

/* C-ABI of the B200 operator library (libopl_b200.so).
 *
 * Plain pointers, sizes and an opaque stream handle; no C++ or torch types,
 * so any FFI (ctypes, cffi, cgo, JNI) can bind it directly.  Each function
 * returns an int that is a cudaError_t value (0 == cudaSuccess,
 * 1 == cudaErrorInvalidValue for rejected arguments).  All pointers are
 * caller-owned device memory on the current device; outputs are
 * pre-allocated; work is only enqueued on `stream` (NULL = legacy default
 * stream) and nothing synchronises.  The C++ functions declared in
 * operatorlib/operators.h forward one-to-one to these entry points.
 *
 * Each entry point names the reference interface it replaces
 * (file:line in the reference project).
 */

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t (struct CUstream_st*), spelled without
 * including CUDA headers. */
typedef struct CUstream_st* opl_stream_t;

/* FP16 storage (IEEE binary16 bits), layout-compatible with __half. */
typedef uint16_t opl_half_t;

/* BF16 storage (bfloat16 bits), layout-compatible with __nv_bfloat16. */
typedef uint16_t opl_bf16_t;

/* Replaces operatorlib::reduce_sum_f32, include/operatorlib/operators.h:13-14
 * (implementation src/reduce.cu:54-69).  Sum of n floats, accumulated in
 * FP64 per block and combined in a fixed order: deterministic.  Uses a
 * stream-ordered workspace (cudaMallocAsync/cudaFreeAsync on `stream`). */
int opl_reduce_sum_f32(const float* input, float* output, size_t n,
                       opl_stream_t stream);

/* Multi-GPU building block with no single-call counterpart in the reference:
 * the same deterministic sum as opl_reduce_sum_f32 but written as one FP64
 * value, so per-GPU chunk partials can be all-reduced in FP64 before the
 * final cast (the reference combines block partials with a float atomicAdd,
 * src/reduce.cu:46). */
int opl_reduce_sum_partial_f64(const float* input, double* output, size_t n,
                               opl_stream_t stream);

/* No counterpart in the reference.  opl_reduce_sum_f32 without any
 * allocation, for callers that may not call cudaMalloc/cudaMallocAsync (code
 * inside allocator hooks or pool callbacks, frameworks that own all device
 * memory, fixed memory budgets).  Partial sums go to a fixed file-scope
 * device array of 4096 FP64 slots (32 KiB, held by every GPU that loads the
 * library until exit); the partial-sum grid never exceeds 4096 CTAs, so any
 * n fits.  The first call on each device looks the array up
 * (cudaGetSymbolAddress), caches the address and must come before any stream
 * capture; the cached address does not survive cudaDeviceReset.  All calls
 * share the array: calls that overlap on the GPU race; serialise them on one
 * stream.  Bit-identical result to opl_reduce_sum_f32. */
int opl_reduce_sum_f32_noalloc(const float* input, float* output, size_t n,
                               opl_stream_t stream);

/* Multi-GPU reduce fused with its all-reduce (no reference counterpart: the
 * reference is single-GPU; it replaces "per-GPU reduce + NCCL all-reduce").
 * A team is one rank per GPU of a node.  opl_team_create allocates this
 * GPU's team buffer and returns its CUDA IPC handle (64 bytes) to share with
 * the other ranks; opl_team_connect opens the peers' buffers from the
 * world * 64-byte array of all handles (rank order).  Every rank then calls
 * opl_team_reduce_sum_f32 on its own chunk, in the same order on all ranks:
 * each GPU sums its chunk, exchanges the FP64 partial with the peers over
 * NVLink and writes the identical total to *output.  A peer that does not
 * arrive within a bounded wait (about 2 s) yields NaN and the watchdog code.
 * A timeout is final for the team: every later call on that rank returns NaN
 * at once, the other ranks time out on their next call and do the same, and
 * the team has to be destroyed (opl_team_destroy) and created again. */
int opl_team_create(int rank, int world, void** team, void* ipc_handle_out);
int opl_team_connect(void* team, const void* all_ipc_handles);
int opl_team_reduce_sum_f32(void* team, const float* input, float* output, size_t n,
                            opl_stream_t stream);
int opl_team_destroy(void* team);

/* Replaces operatorlib::softmax_f32, operators.h:16-17 (src/softmax.cu:182-202). */
int opl_softmax_f32(const float* input, float* output, int rows, int cols,
                    opl_stream_t stream);

/* 16-bit I/O variants of softmax_f32 and rmsnorm_f32 (no counterpart in the
 * reference, whose launchers are FP32-only; it defers 16-bit I/O to a later
 * interface stage, docs/standalone_benchmark.md:14-16).  Inputs, weight and
 * outputs in FP16 or BF16; max / sums / normalisation in FP32; each result
 * rounded once to the storage type.  Same argument checks as the FP32
 * versions. */
int opl_softmax_f16(const opl_half_t* input, opl_half_t* output, int rows, int cols,
                    opl_stream_t stream);
int opl_softmax_bf16(const opl_bf16_t* input, opl_bf16_t* output, int rows, int cols,
                     opl_stream_t stream);
int opl_rmsnorm_f16(const opl_half_t* input, const opl_half_t* weight, opl_half_t* output,
                    int tokens, int hidden, float epsilon, opl_stream_t stream);
int opl_rmsnorm_bf16(const opl_bf16_t* input, const opl_bf16_t* weight, opl_bf16_t* output,
                     int tokens, int hidden, float epsilon, opl_stream_t stream);

/* Replaces operatorlib::transpose_f32, operators.h:19-20
 * (src/transpose.cu:38-47).  Bit-exact data movement. */
int opl_transpose_f32(const float* input, float* output, int rows, int cols,
                      opl_stream_t stream);

/* Replaces operatorlib::rmsnorm_f32, operators.h:22-24 (src/rmsnorm.cu:77-95).
 * epsilon <= 0 (or NaN) is rejected like the reference (src/rmsnorm.cu:80-82). */
int opl_rmsnorm_f32(const float* input, const float* weight, float* output,
                    int tokens, int hidden, float epsilon, opl_stream_t stream);

/* Replaces operatorlib::gemm_f32, operators.h:27-28 (src/gemm.cu:440-453).
 * Row-major C[M,N] = A[M,K] * B[K,N] on FP32 FFMA (no TF32 rounding). */
int opl_gemm_f32(const float* a, const float* b, float* c, int m, int n, int k,
                 opl_stream_t stream);

/* Replaces operatorlib::gemm_f16, operators.h:31-32 (src/gemm.cu:455-479).
 * FP16 A and B, tcgen05 tensor cores, FP32 accumulate and FP32 C.
 * Shapes whose row strides are not 16-byte multiples are staged through a
 * zero-padded stream-ordered workspace. */
int opl_gemm_f16(const opl_half_t* a, const opl_half_t* b, float* c, int m,
                 int n, int k, opl_stream_t stream);

/* Replaces operatorlib::attention_f32, operators.h:35-38
 * (src/attention.cu:445-484).  [B,H,S,D] contiguous, D <= 128, FP32 FFMA. */
int opl_attention_f32(const float* q, const float* k, const float* v,
                      float* output, int batch, int heads, int sequence,
                      int head_dim, int causal, opl_stream_t stream);

/* Replaces operatorlib::attention_f16, operators.h:41-44
 * (src/attention.cu:486-507).  FP16 Q/K/V, FP32 softmax state and output. */
int opl_attention_f16(const opl_half_t* q, const opl_half_t* k,
                      const opl_half_t* v, float* output, int batch, int heads,
                      int sequence, int head_dim, int causal,
                      opl_stream_t stream);

/* Library utilities (no reference counterpart). */

/* cudaGetErrorString of an error code returned above. */
const char* opl_error_string(int error);

/* Reads and clears the per-device watchdog word of the current device.
 * Kernels whose pipelines wait on mbarriers give up after a bounded number
 * of polls, record a non-zero code here and exit instead of hanging the
 * GPU.  Synchronises the current device (diagnostics only). */
int opl_read_and_clear_watchdog(int* code);

/* Library version, e.g. "opl-b200 0.1.0 sm_100a". */
const char* opl_version(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* OPERATORLIB_OPL_CAPI_H_ */
