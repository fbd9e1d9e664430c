// Shared helpers for the beam-decode kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>
#include <cstdlib>
#include <utility>

#include "beam_b200.h"

namespace be {

// Device-side status word: kernels that meet an out-of-range page id or slot
// record BE_EDEVICE_RANGE here and skip the access instead of faulting.
// (All device code is one translation unit, lib.cu, so it is defined here.)
__device__ int g_device_status = 0;

__device__ __forceinline__ void flag_range_error() { atomicCAS(&g_device_status, 0, BE_EDEVICE_RANGE); }

template <typename T> struct DT;
template <> struct DT<float> { static constexpr int id = BE_F32; };
template <> struct DT<__half> { static constexpr int id = BE_F16; };
template <> struct DT<__nv_bfloat16> { static constexpr int id = BE_BF16; };

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

inline int dtype_size(int dt) { return dt == BE_F32 ? 4 : 2; }

// Programmatic dependent launch: a kernel launched with launch_pdl may be
// scheduled while the previous kernel on its stream is still finishing (the
// launch latency overlaps that tail); it must call pdl_wait() before it reads
// anything the previous kernel writes.  BE_PDL=0 turns the attribute off.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Let the next PDL kernel on the stream start its preamble now (it still waits
// in pdl_wait() for this grid's completion before reading what it wrote).
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

inline bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("BE_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Host-side thread-local last-error text (read through be_last_error()).
void set_error(const char* fmt, ...);

#define BE_CUDA_CHECK(expr)                                                      \
  do {                                                                           \
    cudaError_t _e = (expr);                                                     \
    if (_e != cudaSuccess) {                                                     \
      ::be::set_error("%s: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, \
                      __LINE__);                                                 \
      return BE_ECUDA;                                                           \
    }                                                                            \
  } while (0)

#define BE_LAUNCH_CHECK()                                                             \
  do {                                                                                \
    cudaError_t _e = cudaGetLastError();                                              \
    if (_e != cudaSuccess) {                                                          \
      ::be::set_error("kernel launch: %s (%s:%d)", cudaGetErrorString(_e), __FILE__, \
                      __LINE__);                                                      \
      return BE_ECUDA;                                                                \
    }                                                                                 \
  } while (0)

}  // namespace be
