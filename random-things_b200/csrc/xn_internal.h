// xn_internal.h - host-side helpers shared by the C-ABI entry points:
// error reporting (thread-local message + status code), argument checks and
// launch-error collection. No function here allocates device memory.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "xn_fused.h"

namespace xn {

// Records a formatted message for xn_last_error() and returns `code`.
int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));

// Clears the thread's message; returns XN_OK.
int ok();

// Collects the launch status of the kernel(s) just enqueued.
int check_launch(const char *op);

// Bytes per element, or 0 for an unknown dtype.
int dtype_bytes(int dtype);

// True for the floating-point dtypes the compute kernels handle.
inline bool is_float_dtype(int dtype) {
  return dtype == XN_F32 || dtype == XN_BF16 || dtype == XN_F16;
}

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool is_aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Smallest power of two >= v (v >= 1).
inline int64_t pow2_ceil(int64_t v) {
  int64_t p = 1;
  while (p < v) p <<= 1;
  return p;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Number of SMs of the current device (cached per device).
int sm_count();

// True unless the environment sets XN_PDL=0 (read once per process).
bool pdl_enabled();

// Grid of a persistent kernel: as many blocks of `block` threads (and `smem`
// bytes of dynamic shared memory) as are resident on the GPU at once, never
// more than `needed`.
template <typename K>
int64_t persistent_grid(K kernel, int block, int64_t needed, size_t smem = 0) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, block, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int64_t g = static_cast<int64_t>(per_sm) * sm_count();
  return g < needed ? g : needed;
}

// Launches `kernel` on `stream` with programmatic dependent launch allowed
// (cudaLaunchAttributeProgrammaticStreamSerialization): the kernel's blocks
// may be scheduled while the previous kernel of the stream drains. Every
// kernel of this library starts with griddep_wait() (xn_common.cuh), which
// holds it until that previous kernel has completed and its writes are
// visible, so results do not depend on the attribute. Errors are left for
// check_launch().
template <typename... KArgs, typename... Args>
void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
}

}  // namespace xn

// Dispatches a float dtype to a template parameter named T.
#define XN_DISPATCH_FLOAT(DTYPE, ...)          \
  switch (DTYPE) {                             \
    case XN_F32: {                             \
      using T = float;                         \
      __VA_ARGS__;                             \
      break;                                   \
    }                                          \
    case XN_BF16: {                            \
      using T = __nv_bfloat16;                 \
      __VA_ARGS__;                             \
      break;                                   \
    }                                          \
    case XN_F16: {                             \
      using T = __half;                        \
      __VA_ARGS__;                             \
      break;                                   \
    }                                          \
    default:                                   \
      break;                                   \
  }
