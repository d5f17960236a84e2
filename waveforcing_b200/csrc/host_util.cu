// Host helpers: per-thread error message, TMA descriptor encoding via the
// driver entry point, library-wide status collection.
#include <cstdarg>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "host_util.h"

namespace wfk {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

void* driver_fn(const char* name) {
  static std::mutex mu;
  static std::unordered_map<std::string, void*> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(name);
  if (it != cache.end()) return it->second;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    fn = nullptr;
  cache[name] = fn;
  return fn;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* gaddr, const uint64_t* gdim,
                 const uint64_t* gstride_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  auto fn = reinterpret_cast<EncodeTiledFn>(driver_fn("cuTensorMapEncodeTiled"));
  if (!fn) return fail(WF_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = gdim[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = gstride_bytes[i];
  }
  for (int i = 0; i + 1 < rank; ++i)
    if (s[i] % 16 != 0 || s[i] >= (1ull << 40))
      return fail(WF_ERR_INVALID_ARG, "TMA stride %d = %llu bytes is not a multiple of 16", i,
                  (unsigned long long)s[i]);
  CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(gaddr), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(WF_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return WF_OK;
}

}  // namespace wfk

extern "C" unsigned int wfk_status_take_attn(void);
extern "C" unsigned int wfk_status_take_codec(void);
extern "C" unsigned int wfk_status_take_gemm(void);
extern "C" unsigned int wfk_status_take_exchange(void);

extern "C" const char* wf_last_error(void) { return wfk::g_last_error.c_str(); }

extern "C" int wf_version(void) { return 2; }

extern "C" unsigned int wf_status_take(void) {
  cudaDeviceSynchronize();
  return wfk_status_take_attn() | wfk_status_take_codec() | wfk_status_take_gemm() | wfk_status_take_exchange();
}
