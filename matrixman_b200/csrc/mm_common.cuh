// Internal helpers shared by the runtime and the kernels of libmatrixman_b200.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <cstdlib>
#include <utility>
#include <string>

#include "../../include/matrixman_b200.h"

namespace mm {

// Thread-local last-error message (read through mm_last_error).
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t err, const char* action);

#define MM_CUDA(call, action)                         \
  do {                                                \
    cudaError_t _e = (call);                          \
    if (_e != cudaSuccess) return ::mm::cuda_fail(_e, action); \
  } while (0)

// Check the launch status of the kernel just queued.
#define MM_LAUNCH_CHECK(action)                       \
  do {                                                \
    cudaError_t _e = cudaGetLastError();              \
    if (_e != cudaSuccess) return ::mm::cuda_fail(_e, action); \
  } while (0)

cudaStream_t resolve_stream(void* stream);

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL).  A kernel launched with launch_pdl may
// be scheduled while the previous kernel in the stream drains; it must call
// pdl_wait() before its first global-memory access, which returns once every
// earlier kernel has completed and its writes are visible (a no-op in a launch
// without the attribute).  MATRIXMAN_PDL=0 launches everything plainly.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* env = std::getenv("MATRIXMAN_PDL");
    return !(env != nullptr && env[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Number of SMs of the current device (cached per device).
int sm_count();

// ---------------------------------------------------------------------------
// Tensor geometry helpers (host side).
// ---------------------------------------------------------------------------

struct Geom {
  int nd = 0;
  int64_t size[MM_MAX_DIMS];
  int64_t stride[MM_MAX_DIMS];
};

inline int64_t numel(const mm_tensor_t* t) {
  int64_t n = 1;
  for (int i = 0; i < t->ndim; ++i) n *= t->size[i];
  return n;
}

int validate(const mm_tensor_t* t, const char* name, int want_dtype = MM_F32);

// Collapse the common iteration space of up to 4 operands with the same
// logical shape: drop size-1 dims and merge adjacent dims that are contiguous
// in every operand.  Outputs are stored in g[k] (one Geom per operand, sharing
// nd and size).
int collapse(int nops, const mm_tensor_t* const* ops, Geom* g);

// Device-side strided offset computation for up to 6 collapsed dims.
struct DevGeom {
  int nd;
  int64_t size[MM_MAX_DIMS];
  int64_t stride[MM_MAX_DIMS];
};

inline DevGeom to_dev(const Geom& g) {
  DevGeom d;
  d.nd = g.nd;
  for (int i = 0; i < MM_MAX_DIMS; ++i) {
    d.size[i] = i < g.nd ? g.size[i] : 1;
    d.stride[i] = i < g.nd ? g.stride[i] : 0;
  }
  return d;
}

__device__ __forceinline__ int64_t dev_offset(int64_t linear, const DevGeom& g) {
  int64_t off = 0;
#pragma unroll
  for (int i = MM_MAX_DIMS - 1; i >= 0; --i) {
    if (i < g.nd) {
      int64_t s = g.size[i];
      int64_t q = linear / s;
      off += (linear - q * s) * g.stride[i];
      linear = q;
    }
  }
  return off;
}

inline unsigned grid_for(int64_t n, int block, int64_t max_blocks = 148LL * 32) {
  int64_t b = (n + block - 1) / block;
  if (b > max_blocks) b = max_blocks;
  if (b < 1) b = 1;
  return (unsigned)b;
}

}  // namespace mm
