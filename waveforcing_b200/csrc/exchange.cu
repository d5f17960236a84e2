// Exchange primitives for the paged K/V publish (C++ replacement of
// wave_rt/distributed/ipc.py): CUDA IPC export/open/close, stream-ordered
// 32-bit release writes and acquire waits, peer copies, and a BOUNDED
// device-side flag wait that the reference lacks (its cuStreamWaitValue32
// hangs the consumer forever if a producer dies).
#include <cuda_runtime.h>

#include <cstring>

#include "host_util.h"
#include "sm100.cuh"

namespace wfk {
namespace xchg {

typedef CUresult (*StreamWriteValue32Fn)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
typedef CUresult (*StreamWaitValue32Fn)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
typedef CUresult (*MemGetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

// Spins (with backoff) until *flag >= value in the cyclic sense of
// CU_STREAM_WAIT_VALUE_GEQ, or until timeout_ns elapses.
__global__ void wait_flag_kernel(const unsigned int* __restrict__ flag, unsigned int value,
                                 unsigned long long timeout_ns, unsigned int* __restrict__ timeout_out) {
  const uint64_t t0 = globaltimer_ns();
  unsigned int ns = 32;
  while (true) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (static_cast<int>(v - value) >= 0) return;
    if (globaltimer_ns() - t0 > timeout_ns) {
      if (timeout_out) *timeout_out = 1u;
      status_raise(ST_FLAG_TIMEOUT);
      return;
    }
    __nanosleep(ns);
    if (ns < 1024) ns <<= 1;
  }
}

// Up to 32 flags in one launch: lane i spins on flags.p[i] like
// wait_flag_kernel; the kernel ends when every lane has seen its flag or
// given up.
constexpr int MAX_WAIT_FLAGS = 32;
struct FlagList {
  const unsigned int* p[MAX_WAIT_FLAGS];
};
__global__ void wait_flags_kernel(FlagList flags, int n, unsigned int value, unsigned long long timeout_ns,
                                  unsigned int* __restrict__ timeout_out) {
  const int i = threadIdx.x;
  if (i >= n) return;
  const uint64_t t0 = globaltimer_ns();
  unsigned int ns = 32;
  while (true) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags.p[i]) : "memory");
    if (static_cast<int>(v - value) >= 0) return;
    if (globaltimer_ns() - t0 > timeout_ns) {
      if (timeout_out) *timeout_out = 1u;
      status_raise(ST_FLAG_TIMEOUT);
      return;
    }
    __nanosleep(ns);
    if (ns < 1024) ns <<= 1;
  }
}

// Writes the device's %globaltimer (ns) to *dst when the stream reaches it.
__global__ void stamp_kernel(unsigned long long* __restrict__ dst) { *dst = globaltimer_ns(); }

}  // namespace xchg
}  // namespace wfk

using namespace wfk;
using namespace wfk::xchg;

extern "C" int wf_ipc_export(const void* p, uint8_t* handle64, uint64_t* offset) {
  if (!p || !handle64 || !offset) return fail(WF_ERR_INVALID_ARG, "wf_ipc_export: null argument");
  cudaIpcMemHandle_t h;
  WFK_CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void*>(p)));
  static_assert(sizeof(h) == 64, "IPC handle is 64 bytes");
  std::memcpy(handle64, &h, 64);
  auto range = reinterpret_cast<MemGetAddressRangeFn>(driver_fn("cuMemGetAddressRange"));
  if (!range) return fail(WF_ERR_CUDA, "cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(p));
  if (r != CUDA_SUCCESS) return fail(WF_ERR_CUDA, "cuMemGetAddressRange failed (%d)", (int)r);
  *offset = reinterpret_cast<uint64_t>(p) - static_cast<uint64_t>(base);
  return WF_OK;
}

extern "C" int wf_ipc_open(const uint8_t* handle64, void** base) {
  if (!handle64 || !base) return fail(WF_ERR_INVALID_ARG, "wf_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, 64);
  WFK_CUDA_TRY(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
  return WF_OK;
}

extern "C" int wf_ipc_close(void* base) {
  if (!base) return fail(WF_ERR_INVALID_ARG, "wf_ipc_close: null base");
  WFK_CUDA_TRY(cudaIpcCloseMemHandle(base));
  return WF_OK;
}

extern "C" int wf_enable_peer(int peer) {
  int dev = 0;
  WFK_CUDA_TRY(cudaGetDevice(&dev));
  if (peer == dev) return WF_OK;
  int can = 0;
  WFK_CUDA_TRY(cudaDeviceCanAccessPeer(&can, dev, peer));
  if (!can) return fail(WF_ERR_UNSUPPORTED, "device %d cannot access peer %d", dev, peer);
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return WF_OK;
  }
  WFK_CUDA_TRY(e);
  return WF_OK;
}

extern "C" int wf_stream_write_u32(void* stream, void* addr, uint32_t value) {
  if (!addr || (reinterpret_cast<uintptr_t>(addr) & 3)) return fail(WF_ERR_INVALID_ARG, "wf_stream_write_u32: bad addr");
  auto fn = reinterpret_cast<StreamWriteValue32Fn>(driver_fn("cuStreamWriteValue32"));
  if (!fn) return fail(WF_ERR_CUDA, "cuStreamWriteValue32 unavailable");
  const CUresult r = fn(static_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(addr), value, 0);
  if (r != CUDA_SUCCESS) return fail(WF_ERR_CUDA, "cuStreamWriteValue32 failed (%d)", (int)r);
  return WF_OK;
}

extern "C" int wf_stream_wait_u32(void* stream, const void* addr, uint32_t value) {
  if (!addr || (reinterpret_cast<uintptr_t>(addr) & 3)) return fail(WF_ERR_INVALID_ARG, "wf_stream_wait_u32: bad addr");
  auto fn = reinterpret_cast<StreamWaitValue32Fn>(driver_fn("cuStreamWaitValue32"));
  if (!fn) return fail(WF_ERR_CUDA, "cuStreamWaitValue32 unavailable");
  const CUresult r = fn(static_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(addr), value,
                        CU_STREAM_WAIT_VALUE_GEQ);
  if (r != CUDA_SUCCESS) return fail(WF_ERR_CUDA, "cuStreamWaitValue32 failed (%d)", (int)r);
  return WF_OK;
}

extern "C" int wf_wait_flag(const void* flag, uint32_t value, uint64_t timeout_ns, uint32_t* timeout_out,
                            void* stream) {
  if (!flag || (reinterpret_cast<uintptr_t>(flag) & 3)) return fail(WF_ERR_INVALID_ARG, "wf_wait_flag: bad flag");
  if (timeout_ns == 0 || timeout_ns > 600ull * 1000000000ull)
    return fail(WF_ERR_INVALID_ARG, "wf_wait_flag: timeout must be in (0, 600 s]");
  wait_flag_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const unsigned int*>(flag), value,
                                                                   timeout_ns, timeout_out);
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_wait_flags(const void* const* flags, int n, uint32_t value, uint64_t timeout_ns,
                             uint32_t* timeout_out, void* stream) {
  if (!flags || n < 0 || n > MAX_WAIT_FLAGS)
    return fail(WF_ERR_INVALID_ARG, "wf_wait_flags: need a host array of 0..32 flag addresses");
  if (timeout_ns == 0 || timeout_ns > 600ull * 1000000000ull)
    return fail(WF_ERR_INVALID_ARG, "wf_wait_flags: timeout must be in (0, 600 s]");
  FlagList fl{};
  for (int i = 0; i < n; ++i) {
    if (!flags[i] || (reinterpret_cast<uintptr_t>(flags[i]) & 3))
      return fail(WF_ERR_INVALID_ARG, "wf_wait_flags: flag %d is null or misaligned", i);
    fl.p[i] = static_cast<const unsigned int*>(flags[i]);
  }
  if (n == 0) return WF_OK;
  wait_flags_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(fl, n, value, timeout_ns, timeout_out);
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_stamp(uint64_t* dst, void* stream) {
  if (!dst || (reinterpret_cast<uintptr_t>(dst) & 7)) return fail(WF_ERR_INVALID_ARG, "wf_stamp: bad dst");
  stamp_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(reinterpret_cast<unsigned long long*>(dst));
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_memcpy_async(void* dst, const void* src, uint64_t bytes, void* stream) {
  if (bytes == 0) return WF_OK;
  if (!dst || !src) return fail(WF_ERR_INVALID_ARG, "wf_memcpy_async: null pointer");
  WFK_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)));
  return WF_OK;
}

extern "C" int wf_publish(void* const* dsts, const void* src, uint64_t bytes, void* const* flags, int n,
                          uint32_t value, void* stream) {
  if (n < 0 || (n > 0 && (!dsts || !flags || !src))) return fail(WF_ERR_INVALID_ARG, "wf_publish: bad arguments");
  for (int i = 0; i < n; ++i) {
    int rc = wf_memcpy_async(dsts[i], src, bytes, stream);
    if (rc != WF_OK) return rc;
    // The release write is ordered after the payload copy on the same stream.
    rc = wf_stream_write_u32(stream, flags[i], value);
    if (rc != WF_OK) return rc;
  }
  return WF_OK;
}

extern "C" unsigned int wfk_status_take_exchange(void) { return wfk::status_take_local(); }
