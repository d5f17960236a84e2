// Row ops of the streaming VAE decoder (waveforcing_b200/pipelines/vae.py)
// on channels-last activations: every position's C channels are one
// contiguous bf16 row.
//   wf_channel_rmsnorm  out = x / max(||x||_2, eps) * sqrt(C) * gamma, then
//                       optionally SiLU -- the Wan VAE's RMS_norm over the
//                       channel dimension (naive_rt/rolling_forcing/wan/
//                       modules/vae.py:39-54) fused with the SiLU that
//                       follows it in every residual block and the head
//                       (:178-192, :466-470).
// f32 arithmetic, one bf16 rounding at the end.  16 threads per row: thread
// j handles the 16-byte chunks j, j + 16, ... of the row, and the row's
// sum of squares is reduced among the 16 lanes by shuffles.
#include <cuda_runtime.h>

#include <type_traits>

#include "host_util.h"
#include "sm100.cuh"

namespace wfk {
namespace vae {

constexpr int TPR = 16;  // threads per row

template <int CPT, bool SILU>
__global__ void __launch_bounds__(256)
    channel_rmsnorm_kernel(const __nv_bfloat16* x, __nv_bfloat16* out,  // may alias: a row is read before it is written
                           const __nv_bfloat16* __restrict__ gamma, int64_t rows, int C, float scale, float eps) {
  const int sub = threadIdx.x & (TPR - 1);
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / TPR;
  const bool live = row < rows;
  const int nch = C / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (live ? row : 0) * C);
  uint4 v[CPT];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int c = sub + i * TPR;
    v[i] = (live && c < nch) ? __ldcs(xr + c) : make_uint4(0, 0, 0, 0);
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float a = __uint_as_float(w[k] << 16), b = __uint_as_float(w[k] & 0xFFFF0000u);
      ss = fmaf(a, a, fmaf(b, b, ss));
    }
  }
#pragma unroll
  for (int o = TPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (!live) return;
  const float inv = scale / fmaxf(sqrtf(ss), eps);
  uint4* orow = reinterpret_cast<uint4*>(out + row * C);
  const uint4* g4 = reinterpret_cast<const uint4*>(gamma);
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int c = sub + i * TPR;
    if (c >= nch) continue;
    const uint4 g = __ldg(g4 + c);
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float a = __uint_as_float(w[k] << 16) * inv * __uint_as_float(gw[k] << 16);
      float b = __uint_as_float(w[k] & 0xFFFF0000u) * inv * __uint_as_float(gw[k] & 0xFFFF0000u);
      if constexpr (SILU) {
        a = a / (1.f + __expf(-a));
        b = b / (1.f + __expf(-b));
      }
      o[k] = pack_bf16x2(a, b);
    }
    orow[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Temporal x2 of the upsampling blocks on channels-last rows: src holds, per
// (frame i, position p), 2C channels [half 0 | half 1]; dst holds frames 2i
// (half 0) and 2i + 1 (half 1), each position's C channels contiguous.  One
// thread per 16-byte chunk of the output.
__global__ void __launch_bounds__(256) interleave_time2_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                               int64_t frames, int64_t hw, int64_t c16) {
  const int64_t n = frames * 2 * hw * c16;
  for (int64_t o = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; o < n;
       o += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t k = o % c16;
    const int64_t p = (o / c16) % hw;
    const int64_t j = (o / (c16 * hw)) & 1;
    const int64_t i = o / (c16 * hw * 2);
    dst[o] = __ldcs(src + ((i * hw + p) * 2 + j) * c16 + k);
  }
}

// out = x + bias[c] (+ res): the convolutions' bias (cuDNN returns 3-D
// convolutions without it) and the residual blocks' skip add in one
// vectorised pass over channels-last rows.  out may alias x.
__global__ void __launch_bounds__(256) bias_add_kernel(const uint4* x, const uint4* __restrict__ res,
                                                       const uint4* __restrict__ bias, uint4* out, int64_t n16,
                                                       int64_t c16) {
  for (int64_t o = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; o < n16;
       o += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4 a = x[o], b = __ldg(bias + o % c16);
    const uint4 r = res ? __ldcs(res + o) : make_uint4(0, 0, 0, 0);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w}, rw[4] = {r.x, r.y, r.z, r.w};
    uint32_t ow[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      // (x + bias) + res, each sum rounded as torch's separate bias and skip adds would
      float lo = __uint_as_float(aw[k] << 16) + __uint_as_float(bw[k] << 16);
      float hi = __uint_as_float(aw[k] & 0xFFFF0000u) + __uint_as_float(bw[k] & 0xFFFF0000u);
      if (res) {
        lo = __bfloat162float(__float2bfloat16_rn(lo)) + __uint_as_float(rw[k] << 16);
        hi = __bfloat162float(__float2bfloat16_rn(hi)) + __uint_as_float(rw[k] & 0xFFFF0000u);
      }
      ow[k] = pack_bf16x2(lo, hi);
    }
    out[o] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }
}

// Nearest x2 in H and W on channels-last rows: dst[n, y, x] = src[n, y / 2,
// x / 2] for every channel; each thread copies one 16-byte chunk of a source
// pixel to its four destination pixels.
__global__ void __launch_bounds__(256) upsample2x_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                         int64_t nimg, int64_t h, int64_t w, int64_t c16) {
  const int64_t n = nimg * h * w * c16;
  for (int64_t o = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; o < n;
       o += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t k = o % c16;
    const int64_t px = (o / c16) % w;
    const int64_t py = (o / (c16 * w)) % h;
    const int64_t im = o / (c16 * w * h);
    const uint4 v = __ldcs(src + o);
    const int64_t row0 = (im * 2 * h + 2 * py) * 2 * w + 2 * px;  // destination pixel (2py, 2px)
    dst[row0 * c16 + k] = v;
    dst[(row0 + 1) * c16 + k] = v;
    dst[(row0 + 2 * w) * c16 + k] = v;
    dst[(row0 + 2 * w + 1) * c16 + k] = v;
  }
}

// Rejects element counts whose product would overflow int64 or exceed 2^46
// 16-byte chunks (1 PiB): no device buffer is that large, so such sizes are
// caller errors, reported before any launch.
static bool too_big(int64_t a, int64_t b, int64_t c = 1, int64_t d = 1) {
  constexpr int64_t LIM = int64_t{1} << 46;
  int64_t p = 1;
  for (int64_t f : {a, b, c, d}) {
    if (f < 0 || (f > 0 && p > LIM / f)) return true;
    p *= f;
  }
  return false;
}

static unsigned grid_for(int64_t n) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n + 255) / 256, cap = static_cast<int64_t>(sms) * 16;
  return static_cast<unsigned>(want < cap ? want : cap);
}

}  // namespace vae
}  // namespace wfk

using namespace wfk;
using namespace wfk::vae;

extern "C" int wf_channel_rmsnorm(const void* x, void* out, int64_t rows, int64_t C, const void* gamma, float eps,
                                  int silu, void* stream) {
  if (!x || !out || !gamma || rows < 0 || C < 8 || C % 8 || C > 8 * TPR * 8 || !aligned16(x) || !aligned16(out) ||
      !aligned16(gamma))
    return fail(WF_ERR_INVALID_ARG, "wf_channel_rmsnorm: need C a multiple of 8 up to 1024 and 16-byte aligned rows");
  if (rows > (int64_t{0x7fffffff} * 256) / TPR)
    return fail(WF_ERR_INVALID_ARG, "wf_channel_rmsnorm: rows beyond one launch's grid");
  if (rows == 0) return WF_OK;
  const int64_t threads = rows * TPR;
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int cpt = static_cast<int>((C / 8 + TPR - 1) / TPR);
  const float scale = sqrtf(static_cast<float>(C));
  auto xb = static_cast<const __nv_bfloat16*>(x);
  auto ob = static_cast<__nv_bfloat16*>(out);
  auto gb = static_cast<const __nv_bfloat16*>(gamma);
  const int c = static_cast<int>(C);
  auto go = [&](auto cp) {
    constexpr int CP = decltype(cp)::value;
    if (silu)
      channel_rmsnorm_kernel<CP, true><<<blocks, 256, 0, s>>>(xb, ob, gb, rows, c, scale, eps);
    else
      channel_rmsnorm_kernel<CP, false><<<blocks, 256, 0, s>>>(xb, ob, gb, rows, c, scale, eps);
  };
  switch (cpt) {
    case 1: go(std::integral_constant<int, 1>()); break;
    case 2: go(std::integral_constant<int, 2>()); break;
    case 3: go(std::integral_constant<int, 3>()); break;
    case 4: go(std::integral_constant<int, 4>()); break;
    default: go(std::integral_constant<int, 8>()); break;
  }
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_interleave_time2(const void* src, void* dst, int64_t frames, int64_t hw, int64_t C, void* stream) {
  if (!src || !dst || frames < 0 || hw < 1 || C < 8 || C % 8 || !aligned16(src) || !aligned16(dst) || src == dst)
    return fail(WF_ERR_INVALID_ARG, "wf_interleave_time2: need C a multiple of 8, 16-byte aligned distinct buffers");
  if (too_big(frames, 2 * hw, C / 8)) return fail(WF_ERR_INVALID_ARG, "wf_interleave_time2: size overflows");
  if (frames == 0) return WF_OK;
  const int64_t n = frames * 2 * hw * (C / 8);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n + 255) / 256, cap = static_cast<int64_t>(sms) * 16;
  interleave_time2_kernel<<<static_cast<unsigned>(want < cap ? want : cap), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), frames, hw, C / 8);
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_channel_bias_add(const void* x, const void* bias, const void* res, void* out, int64_t rows,
                                   int64_t C, void* stream) {
  if (!x || !bias || !out || rows < 0 || C < 8 || C % 8 || !aligned16(x) || !aligned16(bias) || !aligned16(out) ||
      (res && !aligned16(res)))
    return fail(WF_ERR_INVALID_ARG, "wf_channel_bias_add: need C a multiple of 8 and 16-byte aligned rows");
  if (too_big(rows, C / 8)) return fail(WF_ERR_INVALID_ARG, "wf_channel_bias_add: size overflows");
  if (rows == 0) return WF_OK;
  const int64_t n16 = rows * (C / 8);
  bias_add_kernel<<<grid_for(n16), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(x), static_cast<const uint4*>(res), static_cast<const uint4*>(bias),
      static_cast<uint4*>(out), n16, C / 8);
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_upsample2x_nearest(const void* src, void* dst, int64_t images, int64_t h, int64_t w, int64_t C,
                                     void* stream) {
  if (!src || !dst || images < 0 || h < 1 || w < 1 || C < 8 || C % 8 || !aligned16(src) || !aligned16(dst) ||
      src == dst)
    return fail(WF_ERR_INVALID_ARG, "wf_upsample2x_nearest: need C a multiple of 8, 16-byte aligned distinct buffers");
  if (too_big(images, 4 * h, w, C / 8)) return fail(WF_ERR_INVALID_ARG, "wf_upsample2x_nearest: size overflows");
  if (images == 0) return WF_OK;
  const int64_t n = images * h * w * (C / 8);
  upsample2x_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), images, h, w, C / 8);
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}
