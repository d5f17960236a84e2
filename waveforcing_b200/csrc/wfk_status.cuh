// Device-side error status.  Every bounded wait that gives up ORs a code
// into a per-translation-unit status word; wf_status_take() collects and
// clears the words of all units on the current device.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace wfk {

enum StatusCode : uint32_t {
  ST_ATTN_PRODUCER = 1u << 0,
  ST_ATTN_MMA = 1u << 1,
  ST_ATTN_SOFTMAX = 1u << 2,
  ST_GEMM_PRODUCER = 1u << 3,
  ST_GEMM_MMA = 1u << 4,
  ST_GEMM_EPILOGUE = 1u << 5,
  ST_FLAG_TIMEOUT = 1u << 6,
  ST_DRAIN_TIMEOUT = 1u << 7,
  ST_ATTN_CONVERT = 1u << 8,
};

static __device__ unsigned int g_status;  // one word per translation unit

__device__ __forceinline__ void status_raise(uint32_t code) { atomicOr(&g_status, code); }

// Reads and clears this unit's word on the current device (synchronous).
static inline unsigned int status_take_local() {
  unsigned int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_status, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  cudaMemcpyToSymbol(g_status, &z, sizeof(z));
  return v;
}

}  // namespace wfk
