// Interleaved (non-neox) rotary embedding on bf16 [L, H, D] with per-token
// f32 cos/sin tables [L, D/2]: pairs (x[2i], x[2i+1]) rotate by angle i,
// f32 math, RNE back to bf16.  Used for the anchor re-RoPE of the paged
// exchange (wave_rt/denoiser/exchange/common.py:84-87) and the q/k RoPE of the
// patched attention (wave_rt/runtime/backend.py:119-121).
#include <cuda_runtime.h>

#include "host_util.h"
#include "sm100.cuh"

namespace wfk {
namespace rope {

// One thread per 8 elements (4 complex pairs); the head dimension is the
// fastest index so cos/sin loads are shared across heads through L1.
__global__ void rope_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                            const float* __restrict__ cos_t, const float* __restrict__ sin_t, int64_t L, int H,
                            int D, int64_t xs, int64_t ys) {
  const int per_tok = H * D / 8;
  const int64_t total = L * per_tok;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / per_tok;
    const int rem = static_cast<int>(i - t * per_tok) * 8;  // element offset within the token
    const int d = rem % D;                                  // offset within the head
    const uint4 v = *reinterpret_cast<const uint4*>(x + t * xs + rem);
    const float4 c = *reinterpret_cast<const float4*>(cos_t + t * (D / 2) + d / 2);
    const float4 s = *reinterpret_cast<const float4*>(sin_t + t * (D / 2) + d / 2);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    const float cc[4] = {c.x, c.y, c.z, c.w};
    const float ss[4] = {s.x, s.y, s.z, s.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float re = __uint_as_float(w[k] << 16);
      const float im = __uint_as_float(w[k] & 0xFFFF0000u);
      const float a = fmaf(re, cc[k], -im * ss[k]);
      const float b = fmaf(re, ss[k], im * cc[k]);
      o[k] = pack_bf16x2(a, b);
    }
    *reinterpret_cast<uint4*>(y + t * ys + rem) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace rope
}  // namespace wfk

extern "C" int wf_rope_apply(const void* x, void* y, const float* cos_t, const float* sin_t, int64_t L, int H, int D,
                             int64_t x_tok_stride, int64_t y_tok_stride, void* stream) {
  using namespace wfk;
  if (!x || !y || !cos_t || !sin_t || L < 0 || H < 1 || D < 8 || D % 8 != 0)
    return fail(WF_ERR_INVALID_ARG, "wf_rope_apply: bad arguments");
  if (!aligned16(x) || !aligned16(y) || !aligned16(cos_t) || !aligned16(sin_t) || x_tok_stride % 8 ||
      y_tok_stride % 8 || x_tok_stride < (int64_t)H * D || y_tok_stride < (int64_t)H * D)
    return fail(WF_ERR_INVALID_ARG, "wf_rope_apply: pointers must be 16-byte aligned, token strides >= H*D, %% 8");
  if (L == 0) return WF_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t work = L * H * D / 8;
  int64_t blocks = (work + 255) / 256;
  if (blocks > sms * 16) blocks = sms * 16;
  rope::rope_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), cos_t, sin_t, L, H, D, x_tok_stride,
      y_tok_stride);
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}
