// Context assembly of the paged exchange in one launch: every row of the
// stage's K/V context buffer comes from one segment of a list, either
//   WF_SEG_COPY     bf16 rows copied (working pages, the stage's own chunk),
//   WF_SEG_ROPE     bf16 rows rotated by per-row f32 cos/sin tables (the
//                   anchor's re-RoPE, wave_rt/denoiser/exchange/common.py:84-87),
//   WF_SEG_DEQUANT  e4m3 codes with per-row f32 scales (FP8 pages received
//                   from other stages), bf16(e4m3(code) * scale).
// It replaces the per-layer copies of paged.py:226-237 plus the separate
// anchor RoPE pass and receive-side dequantisation: the anchor is rotated
// straight into the context buffer, and all segments of K and V of one layer
// share a launch.  A warp per row; lane l handles 16-byte output chunks l,
// l + 32, ... so loads and stores of a row are contiguous across the warp.
// Each lane issues UNR loads before their stores: without that the compiler,
// which cannot rule out that dst aliases src, keeps one load per lane in
// flight.
#include <cuda_runtime.h>

#include "host_util.h"
#include "quant_rows.cuh"
#include "sm100.cuh"

namespace wfk {
namespace assemble {

constexpr int MAX_SEGS = 24;
constexpr int WARPS = 8;
constexpr int UNR = 6;  // chunks per lane in flight (a 1536-column row is 6 per lane)

struct Params {
  wf_kv_segment seg[MAX_SEGS];
  int64_t row_start[MAX_SEGS + 1];  // prefix of segment rows
  int n;
  int64_t cols;
  int head_dim;
};

__device__ __forceinline__ uint4 rope8(const uint4& v, const float4& c, const float4& s) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  const float cc[4] = {c.x, c.y, c.z, c.w};
  const float ss[4] = {s.x, s.y, s.z, s.w};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float re = __uint_as_float(w[k] << 16);
    const float im = __uint_as_float(w[k] & 0xFFFF0000u);
    o[k] = pack_bf16x2(fmaf(re, cc[k], -im * ss[k]), fmaf(re, ss[k], im * cc[k]));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void __launch_bounds__(WARPS * 32) assemble_kernel(const __grid_constant__ Params p) {
  const int lane = threadIdx.x & 31;
  const int64_t total = p.row_start[p.n];
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * WARPS;
  const int64_t nch = p.cols / 8;
  const int half_d = p.head_dim / 2;
  int si = 0;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * WARPS + (threadIdx.x >> 5); r < total; r += nwarps) {
    while (r >= p.row_start[si + 1]) ++si;  // rows grow monotonically per warp
    const wf_kv_segment& sg = p.seg[si];
    const int64_t row = r - p.row_start[si];
    uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(sg.dst) + row * sg.dst_row_stride);
    if (sg.kind == WF_SEG_DEQUANT) {
      const uint2* src = reinterpret_cast<const uint2*>(static_cast<const uint8_t*>(sg.src) + row * sg.src_row_stride);
      const float s = __ldg(sg.aux0 + row);
      for (int64_t c0 = lane; c0 < nch; c0 += 32 * UNR) {
        uint2 v[UNR];
#pragma unroll
        for (int u = 0; u < UNR; ++u)
          if (c0 + u * 32 < nch) v[u] = __ldcs(src + c0 + u * 32);
#pragma unroll
        for (int u = 0; u < UNR; ++u)
          if (c0 + u * 32 < nch) dst[c0 + u * 32] = quant::dequant8(v[u], s);
      }
    } else {
      const uint4* src =
          reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(sg.src) + row * sg.src_row_stride);
      if (sg.kind == WF_SEG_ROPE) {
        const float* ct = sg.aux0 + row * half_d;
        const float* st = sg.aux1 + row * half_d;
        for (int64_t c0 = lane; c0 < nch; c0 += 32 * UNR) {
          uint4 v[UNR];
#pragma unroll
          for (int u = 0; u < UNR; ++u)
            if (c0 + u * 32 < nch) v[u] = __ldg(src + c0 + u * 32);
#pragma unroll
          for (int u = 0; u < UNR; ++u) {
            const int64_t c = c0 + u * 32;
            if (c < nch) {
              const int d2 = static_cast<int>((c * 8) % p.head_dim) / 2;
              dst[c] = rope8(v[u], *reinterpret_cast<const float4*>(ct + d2), *reinterpret_cast<const float4*>(st + d2));
            }
          }
        }
      } else {
        for (int64_t c0 = lane; c0 < nch; c0 += 32 * UNR) {
          uint4 v[UNR];
#pragma unroll
          for (int u = 0; u < UNR; ++u)
            if (c0 + u * 32 < nch) v[u] = __ldg(src + c0 + u * 32);
#pragma unroll
          for (int u = 0; u < UNR; ++u)
            if (c0 + u * 32 < nch) dst[c0 + u * 32] = v[u];
        }
      }
    }
  }
}

}  // namespace assemble
}  // namespace wfk

extern "C" int wf_kv_assemble(const wf_kv_segment* segs, int n_segs, int64_t cols, int head_dim, void* stream) {
  using namespace wfk;
  using namespace wfk::assemble;
  if (!segs || n_segs < 0 || n_segs > MAX_SEGS)
    return fail(WF_ERR_INVALID_ARG, "wf_kv_assemble: 0..%d segments required", MAX_SEGS);
  if (cols < 8 || cols % 8 || head_dim < 8 || head_dim % 8 || cols % head_dim)
    return fail(WF_ERR_INVALID_ARG, "wf_kv_assemble: cols must be a multiple of head_dim, both multiples of 8");
  Params p{};
  p.n = n_segs;
  p.cols = cols;
  p.head_dim = head_dim;
  int64_t acc = 0;
  for (int i = 0; i < n_segs; ++i) {
    const wf_kv_segment& s = segs[i];
    if (s.kind != WF_SEG_COPY && s.kind != WF_SEG_ROPE && s.kind != WF_SEG_DEQUANT)
      return fail(WF_ERR_INVALID_ARG, "wf_kv_assemble: segment %d has an unknown kind", i);
    if (s.rows < 0) return fail(WF_ERR_INVALID_ARG, "wf_kv_assemble: segment %d has negative rows", i);
    if (s.rows > 0) {
      const bool codes = s.kind == WF_SEG_DEQUANT;
      if (!s.src || !s.dst || !aligned16(s.dst) || s.dst_row_stride < cols || s.dst_row_stride % 8)
        return fail(WF_ERR_INVALID_ARG, "wf_kv_assemble: segment %d destination null, misaligned or short", i);
      if (codes ? ((reinterpret_cast<uintptr_t>(s.src) & 7) || s.src_row_stride < cols || s.src_row_stride % 8 ||
                   !s.aux0)
                : (!aligned16(s.src) || s.src_row_stride < cols || s.src_row_stride % 8))
        return fail(WF_ERR_INVALID_ARG, "wf_kv_assemble: segment %d source null, misaligned or short", i);
      if (s.kind == WF_SEG_ROPE && (!s.aux0 || !s.aux1 || !aligned16(s.aux0) || !aligned16(s.aux1)))
        return fail(WF_ERR_INVALID_ARG, "wf_kv_assemble: segment %d needs 16-byte aligned cos/sin tables", i);
    }
    p.seg[i] = s;
    p.row_start[i] = acc;
    acc += s.rows;
  }
  p.row_start[n_segs] = acc;
  for (int i = n_segs + 1; i <= MAX_SEGS; ++i) p.row_start[i] = acc;
  if (acc == 0) return WF_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (acc + WARPS - 1) / WARPS;
  const int64_t cap = static_cast<int64_t>(sms) * 8;
  const unsigned blocks = static_cast<unsigned>(want < cap ? want : cap);
  assemble_kernel<<<blocks, WARPS * 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}
