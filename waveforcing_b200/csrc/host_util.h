// Host-side helpers shared by the C-ABI entry points: error strings,
// argument checks, TMA tensor-map encoding through the driver entry point.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/wfk.h"

namespace wfk {

// Last error message of the calling thread (returned by wf_last_error()).
void set_error(const std::string& msg);
int fail(int code, const char* fmt, ...);

#define WFK_CUDA_TRY(expr)                                                                \
  do {                                                                                    \
    cudaError_t _e = (expr);                                                              \
    if (_e != cudaSuccess)                                                                \
      return ::wfk::fail(WF_ERR_CUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, __LINE__); \
  } while (0)

// cuTensorMapEncodeTiled resolved once through cudaGetDriverEntryPoint, so
// the library does not link libcuda directly.
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* gaddr, const uint64_t* gdim,
                 const uint64_t* gstride_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

// Driver entry point lookup (nullptr when absent).
void* driver_fn(const char* name);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace wfk
