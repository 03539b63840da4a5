// Shared helpers for the qsp (qwen3_5 speculative step) CUDA library, sm_100a.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include <utility>

#include "../../include/qsp.h"

namespace qsp {

// ---------------------------------------------------------------- errors
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);

#define QSP_REQUIRE(cond, ...)                                   \
  do {                                                           \
    if (!(cond)) return ::qsp::set_error(QSP_ERR_INVALID, __VA_ARGS__); \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

// ---------------------------------------------------------------- programmatic dependent launch
// Kernels launched with launch_pdl may begin while the previous kernel on the stream is still
// finishing (its CTAs take whatever SM room is left). Such a kernel calls pdl_wait() in every
// CTA before it touches memory that earlier kernels write or read — only immutable data
// (weights) may be read before it — so "the previous kernel completed" stays transitive along
// the stream. pdl_trigger() lets the next kernel start launching; it is issued at the top of
// every kernel here, so a chain of kernels overlaps each one's launch, prologue and weight
// prefetch with its predecessor's tail.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline int launch_pdl(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return set_error(QSP_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  }
  return check_launch(what);
}

// ---------------------------------------------------------------- dtype plumbing
template <typename T> struct dt;
template <> struct dt<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
  // value after a round trip through the storage type (identity for fp32)
  static __device__ __forceinline__ float round(float x) { return x; }
};
template <> struct dt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
};

template <typename T> __device__ __forceinline__ float ld_f(const T* p) { return dt<T>::to_f(*p); }
template <typename T> __device__ __forceinline__ void st_f(T* p, float v) { *p = dt<T>::from_f(v); }

// ---------------------------------------------------------------- math
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float siluf_(float x) { return x / (1.0f + expf(-x)); }
// torch.nn.functional.softplus(x) with its default threshold of 20
__device__ __forceinline__ float softplusf_(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// Block-wide sum for blockDim.x <= 1024 (multiple of 32); `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = (lane < nw) ? red[lane] : 0.0f;
  t = warp_sum(t);
  return t;
}

}  // namespace qsp

#define QSP_DISPATCH_DTYPE(dtype, T, ...)                                  \
  do {                                                                     \
    if ((dtype) == QSP_F32) {                                              \
      using T = float;                                                     \
      __VA_ARGS__                                                          \
    } else if ((dtype) == QSP_BF16) {                                      \
      using T = __nv_bfloat16;                                             \
      __VA_ARGS__                                                          \
    } else {                                                               \
      return ::qsp::set_error(QSP_ERR_UNSUPPORTED, "unsupported dtype %d", (int)(dtype)); \
    }                                                                      \
  } while (0)
