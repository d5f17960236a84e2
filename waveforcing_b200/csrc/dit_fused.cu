// Fused elementwise stages of the Wan block around the hot path (one warp
// per token row, f32 math, bf16 in/out), replacing chains of 4-8 torch ops:
//   wf_ln_modulate   out = LN(x) * (1 + scale[s]) + shift[s]
//                    naive_rt/rolling_forcing/wan/modules/causal_model.py:375-377, 405-408
//   wf_ln_modulate_quant  the same, quantised per token for the W8A8 linear
//                    that reads it (codes + scale; the bf16 row is not written)
//   wf_gate_residual x += y * gate[s]                       causal_model.py:383, 411-413
//   wf_qk_norm_rope  q, k from the fused QKV GEMM output:  RMSNorm over dim
//                    (model.py:70-88, rounding to bf16 before the weight as
//                    .type_as(x) * weight does), then interleaved RoPE per head
//                    (wave_rt/runtime/backend.py:119-121) with per-stage tables.
//   wf_qk_norm_rope_publish  the same, plus the per-token FP8 quantise-and-
//                    publish of each stage's roped K and its V (from the same
//                    QKV output) into that stage's destination slots.
// s = row / rows_per_stage selects the stage's modulation vector / RoPE table.
#include <cuda_runtime.h>

#include "host_util.h"
#include "quant_rows.cuh"
#include "sm100.cuh"

namespace wfk {
namespace fused {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// ---- row helpers: one warp holds a row of NCH * 256 elements, lane l the
// 8-element chunks l, l + 32, ...; every kernel below is built from these,
// so fused and unfused paths compute identical values.

// out = LN(v) * (1 + scale[st]) + shift[st], rounded to bf16 (packed)
template <int NCH>
__device__ __forceinline__ void row_ln_modulate(const float (&v)[NCH][8], const float* __restrict__ shift,
                                                const float* __restrict__ scale, int64_t st, int64_t mod_stride,
                                                float eps, int lane, uint4 (&packed)[NCH]) {
  constexpr int DIM = NCH * 256;
  float sum = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) sum += v[c][i];
  const float mean = warp_sum(sum) * (1.f / DIM);
  float q2 = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float d = v[c][i] - mean;
      q2 = fmaf(d, d, q2);
    }
  const float rstd = rsqrtf(warp_sum(q2) * (1.f / DIM) + eps);
  const float4* sh4 = reinterpret_cast<const float4*>(shift + st * mod_stride);
  const float4* sc4 = reinterpret_cast<const float4*>(scale + st * mod_stride);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int e = (lane + 32 * c) * 2;  // float4 index of this chunk's first element
    const float4 a0 = __ldg(sc4 + e), a1 = __ldg(sc4 + e + 1);
    const float4 b0 = __ldg(sh4 + e), b1 = __ldg(sh4 + e + 1);
    const float sc[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const float sf[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = fmaf((v[c][i] - mean) * rstd, 1.f + sc[i], sf[i]);
    packed[c] = pack8(o);
  }
}

// Per-token W8A8 quantisation of a bf16 row (act_quant_kernel's arithmetic,
// gemm_w8a8.cu, from the same quant_rows.cuh helpers): codes to xq_row, the
// scale to *x_scale (lane 0).
template <int NCH, bool I8>
__device__ __forceinline__ void row_quant_store(const uint4 (&packed)[NCH], uint8_t* __restrict__ xq_row,
                                                float* __restrict__ x_scale, int lane) {
  using namespace wfk::quant;
  uint32_t m2 = 0;
#pragma unroll
  for (int c = 0; c < NCH; ++c) m2 = amax8_bits(packed[c], m2);
  const RowQuant q = make_rowq(warp_amax_bits(m2), I8 ? 127.f : 448.f);
  uint2* out = reinterpret_cast<uint2*>(xq_row);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const uint4& pv = packed[c];
    uint2 code;
    if (q.finite) {
      if constexpr (I8)
        code = make_uint2(i8x2_fast(pv.x, q.r) | (i8x2_fast(pv.y, q.r) << 16),
                          i8x2_fast(pv.z, q.r) | (i8x2_fast(pv.w, q.r) << 16));
      else
        code = make_uint2(quant4_fast(pv.x, pv.y, q.r), quant4_fast(pv.z, pv.w, q.r));
    } else {
      const uint32_t w[4] = {pv.x, pv.y, pv.z, pv.w};
      uint32_t o2[2] = {0, 0};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float b0 = bf16_round_f(__fdiv_rn(__uint_as_float(w[i] << 16), q.s));
        const float b1 = bf16_round_f(__fdiv_rn(__uint_as_float(w[i] & 0xFFFF0000u), q.s));
        const uint32_t cc =
            I8 ? (i8_slow(b0) | (i8_slow(b1) << 8)) : (e4m3_encode_sw(b0) | (e4m3_encode_sw(b1) << 8));
        o2[i >> 1] |= cc << ((i & 1) * 16);
      }
      code = make_uint2(o2[0], o2[1]);
    }
    out[lane + 32 * c] = code;
  }
  if (lane == 0) *x_scale = q.s;
}

// NCH = dim / 256 chunks of 8 elements per lane
template <int NCH>
__global__ void __launch_bounds__(256) ln_modulate_kernel(const __nv_bfloat16* __restrict__ x, int64_t xs,
                                                          const float* __restrict__ shift,
                                                          const float* __restrict__ scale, int64_t mod_stride,
                                                          __nv_bfloat16* __restrict__ out, int64_t os, int64_t rows,
                                                          int64_t rows_per_stage, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  float v[NCH][8];
  const uint4* xr = reinterpret_cast<const uint4*>(x + r * xs);
#pragma unroll
  for (int c = 0; c < NCH; ++c) unpack8(__ldg(xr + lane + 32 * c), v[c]);
  uint4 packed[NCH];
  row_ln_modulate<NCH>(v, shift, scale, r / rows_per_stage, mod_stride, eps, lane, packed);
  uint4* orow = reinterpret_cast<uint4*>(out + r * os);
#pragma unroll
  for (int c = 0; c < NCH; ++c) orow[lane + 32 * c] = packed[c];
}

// ln_modulate_kernel fused with the per-token W8A8 activation quantiser of
// the linear that reads its output (the QKV projection, FFN fc_in): the row
// of bf16-rounded outputs stays in registers, its amax gives the row scale,
// and only codes (e4m3, or int8 when I8) and the scale are written, equal to
// wf_act_quant(wf_ln_modulate(x)) bit for bit.
template <int NCH, bool I8>
__global__ void __launch_bounds__(256) ln_modulate_quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t xs,
                                                                const float* __restrict__ shift,
                                                                const float* __restrict__ scale, int64_t mod_stride,
                                                                uint8_t* __restrict__ xq, float* __restrict__ x_scale,
                                                                int64_t rows, int64_t rows_per_stage, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  float v[NCH][8];
  const uint4* xr = reinterpret_cast<const uint4*>(x + r * xs);
#pragma unroll
  for (int c = 0; c < NCH; ++c) unpack8(__ldg(xr + lane + 32 * c), v[c]);
  uint4 packed[NCH];
  row_ln_modulate<NCH>(v, shift, scale, r / rows_per_stage, mod_stride, eps, lane, packed);
  row_quant_store<NCH, I8>(packed, xq + r * (NCH * 256), x_scale + r, lane);
}

// The gated residual x = bf16(x + y * gate[st]) (written back), then from the
// new row in registers, without reading it again:
//   MODE 0  its per-token quantisation (the cross-attention q projection's
//           W8A8 input), codes to xq and scales to x_scale;
//   MODE 1  LN-modulate with (shift, scale) to bf16 `out` (the FFN input, the
//           next layer's QKV input);
//   MODE 2  LN-modulate quantised per token (the same for W8A8 linears).
// Each output equals its two-launch form (wf_gate_residual, then
// wf_act_quant / wf_ln_modulate / wf_ln_modulate_quant) bit for bit.
template <int NCH, int MODE, bool I8>
__global__ void __launch_bounds__(256)
    gate_residual_then_kernel(__nv_bfloat16* __restrict__ x, int64_t xs, const __nv_bfloat16* __restrict__ y,
                              int64_t ys, const float* __restrict__ gate, int64_t gate_stride,
                              const float* __restrict__ shift, const float* __restrict__ scale, int64_t mod_stride,
                              __nv_bfloat16* __restrict__ out, int64_t os, uint8_t* __restrict__ xq,
                              float* __restrict__ x_scale, int64_t rows, int64_t gate_rows_per_stage,
                              int64_t mod_rows_per_stage, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  uint4* xr = reinterpret_cast<uint4*>(x + r * xs);
  const uint4* yr = reinterpret_cast<const uint4*>(y + r * ys);
  const float4* g4 = reinterpret_cast<const float4*>(gate + (r / gate_rows_per_stage) * gate_stride);
  float v[NCH][8];
  uint4 xn[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    float a[8], b[8];
    unpack8(xr[lane + 32 * c], a);
    unpack8(__ldg(yr + lane + 32 * c), b);
    const int e = (lane + 32 * c) * 2;
    const float4 g0 = __ldg(g4 + e), g1 = __ldg(g4 + e + 1);
    const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = fmaf(b[i], g[i], a[i]);
    xn[c] = pack8(a);
    xr[lane + 32 * c] = xn[c];
    unpack8(xn[c], v[c]);  // the bf16-rounded row, as a second kernel would read it
  }
  if constexpr (MODE == 0) {
    row_quant_store<NCH, I8>(xn, xq + r * (NCH * 256), x_scale + r, lane);
  } else {
    uint4 packed[NCH];
    row_ln_modulate<NCH>(v, shift, scale, r / mod_rows_per_stage, mod_stride, eps, lane, packed);
    if constexpr (MODE == 1) {
      uint4* orow = reinterpret_cast<uint4*>(out + r * os);
#pragma unroll
      for (int c = 0; c < NCH; ++c) orow[lane + 32 * c] = packed[c];
    } else {
      row_quant_store<NCH, I8>(packed, xq + r * (NCH * 256), x_scale + r, lane);
    }
  }
}

// x[r] = bf16(x[r] + y[r] * gate[stage])   (f32 math)
template <int NCH>
__global__ void __launch_bounds__(256) gate_residual_kernel(__nv_bfloat16* __restrict__ x, int64_t xs,
                                                            const __nv_bfloat16* __restrict__ y, int64_t ys,
                                                            const float* __restrict__ gate, int64_t gate_stride,
                                                            int64_t rows, int64_t rows_per_stage) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int64_t st = r / rows_per_stage;
  uint4* xr = reinterpret_cast<uint4*>(x + r * xs);
  const uint4* yr = reinterpret_cast<const uint4*>(y + r * ys);
  const float4* g4 = reinterpret_cast<const float4*>(gate + st * gate_stride);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    float a[8], b[8];
    unpack8(xr[lane + 32 * c], a);
    unpack8(__ldg(yr + lane + 32 * c), b);
    const int e = (lane + 32 * c) * 2;
    const float4 g0 = __ldg(g4 + e), g1 = __ldg(g4 + e + 1);
    const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = fmaf(b[i], g[i], a[i]);
    xr[lane + 32 * c] = pack8(a);
  }
}

// One warp per (token, q|k) row of the fused QKV output [rows, 3*dim].
// Writes roped q, roped k, and the normalised un-roped k.
template <int NCH>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ld,
                                                           const __nv_bfloat16* __restrict__ wq,
                                                           const __nv_bfloat16* __restrict__ wk,
                                                           const float* __restrict__ cos_t,
                                                           const float* __restrict__ sin_t, int head_dim,
                                                           __nv_bfloat16* __restrict__ q_out,
                                                           __nv_bfloat16* __restrict__ k_out,
                                                           __nv_bfloat16* __restrict__ k_unroped, int64_t rows,
                                                           int64_t rows_per_stage, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (wid >= 2 * rows) return;
  const int64_t r = wid >> 1;
  const bool is_k = wid & 1;
  constexpr int DIM = NCH * 256;
  const uint4* src = reinterpret_cast<const uint4*>(qkv + r * ld + (is_k ? DIM : 0));
  const uint4* w4 = reinterpret_cast<const uint4*>(is_k ? wk : wq);
  float v[NCH][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    unpack8(__ldg(src + lane + 32 * c), v[c]);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(v[c][i], v[c][i], ss);
  }
  const float rn = rsqrtf(warp_sum(ss) * (1.f / DIM) + eps);
  const int64_t tok = r % rows_per_stage;
  const int64_t st = r / rows_per_stage;
  const int half = head_dim / 2;
  const float* ct = cos_t + (st * rows_per_stage + tok) * half;
  const float* stab = sin_t + (st * rows_per_stage + tok) * half;
  __nv_bfloat16* dst = (is_k ? k_out : q_out) + r * DIM;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int e0 = (lane + 32 * c) * 8;  // element index within the row
    float w[8];
    unpack8(__ldg(w4 + lane + 32 * c), w);
    float n[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) n[i] = bf(bf(v[c][i] * rn) * w[i]);
    if (is_k && k_unroped) reinterpret_cast<uint4*>(k_unroped + r * DIM)[lane + 32 * c] = pack8(n);
    const int pd = (e0 % head_dim) / 2;  // first complex pair of this chunk within the head
    const float4 cv = *reinterpret_cast<const float4*>(ct + pd);
    const float4 sv = *reinterpret_cast<const float4*>(stab + pd);
    const float cc[4] = {cv.x, cv.y, cv.z, cv.w}, sn[4] = {sv.x, sv.y, sv.z, sv.w};
    float o[8];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float re = n[2 * p], im = n[2 * p + 1];
      o[2 * p] = fmaf(re, cc[p], -im * sn[p]);
      o[2 * p + 1] = fmaf(re, sn[p], im * cc[p]);
    }
    reinterpret_cast<uint4*>(dst)[lane + 32 * c] = pack8(o);
  }
}

template <int NCH>
__global__ void __launch_bounds__(256) rms_norm_kernel(const __nv_bfloat16* __restrict__ x, int64_t xs,
                                                       const __nv_bfloat16* __restrict__ w,
                                                       __nv_bfloat16* __restrict__ out, int64_t os, int64_t rows,
                                                       float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  constexpr int DIM = NCH * 256;
  const uint4* src = reinterpret_cast<const uint4*>(x + r * xs);
  float v[NCH][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    unpack8(__ldg(src + lane + 32 * c), v[c]);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(v[c][i], v[c][i], ss);
  }
  const float rn = rsqrtf(warp_sum(ss) * (1.f / DIM) + eps);
  const uint4* w4 = reinterpret_cast<const uint4*>(w);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    float wv[8], o[8];
    unpack8(__ldg(w4 + lane + 32 * c), wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = bf(v[c][i] * rn) * wv[i];
    reinterpret_cast<uint4*>(out + r * os)[lane + 32 * c] = pack8(o);
  }
}

template <typename F>
static int by_dim(int64_t dim, F&& f) {
  switch (dim) {
    case 256: f(std::integral_constant<int, 1>()); return WF_OK;
    case 1536: f(std::integral_constant<int, 6>()); return WF_OK;
    case 3072: f(std::integral_constant<int, 12>()); return WF_OK;
    case 5120: f(std::integral_constant<int, 20>()); return WF_OK;
    default: return fail(WF_ERR_UNSUPPORTED, "fused row kernels support dim 256/1536/3072/5120, got %lld",
                         (long long)dim);
  }
}

}  // namespace fused
}  // namespace wfk

using namespace wfk;
using namespace wfk::fused;

extern "C" int wf_ln_modulate(const void* x, int64_t x_stride, const float* shift, const float* scale,
                              int64_t mod_stride, void* out, int64_t out_stride, int64_t rows, int64_t dim,
                              int64_t rows_per_stage, float eps, void* stream) {
  if (!x || !shift || !scale || !out || rows < 0 || rows_per_stage < 1 || !aligned16(x) || !aligned16(out) ||
      !aligned16(shift) || !aligned16(scale) || x_stride % 8 || out_stride % 8 || mod_stride % 4)
    return fail(WF_ERR_INVALID_ARG, "wf_ln_modulate: bad arguments");
  if (rows == 0) return WF_OK;
  const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = by_dim(dim, [&](auto n) {
    ln_modulate_kernel<decltype(n)::value><<<blocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), x_stride, shift, scale, mod_stride, static_cast<__nv_bfloat16*>(out),
        out_stride, rows, rows_per_stage, eps);
  });
  if (rc != WF_OK) return rc;
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_ln_modulate_quant(const void* x, int64_t x_stride, const float* shift, const float* scale,
                                    int64_t mod_stride, void* xq, float* x_scale, int64_t rows, int64_t dim,
                                    int64_t rows_per_stage, float eps, int qtype, void* stream) {
  if (!x || !shift || !scale || !xq || !x_scale || rows < 0 || rows_per_stage < 1 || !aligned16(x) ||
      !aligned16(xq) || !aligned16(shift) || !aligned16(scale) || x_stride % 8 || mod_stride % 4)
    return fail(WF_ERR_INVALID_ARG, "wf_ln_modulate_quant: bad arguments");
  if (qtype != WF_DTYPE_E4M3 && qtype != WF_DTYPE_S8)
    return fail(WF_ERR_UNSUPPORTED, "wf_ln_modulate_quant: qtype must be WF_DTYPE_E4M3 or WF_DTYPE_S8");
  if (rows == 0) return WF_OK;
  const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = by_dim(dim, [&](auto n) {
    constexpr int N = decltype(n)::value;
    if (qtype == WF_DTYPE_S8)
      ln_modulate_quant_kernel<N, true><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), x_stride, shift,
                                                               scale, mod_stride, static_cast<uint8_t*>(xq), x_scale,
                                                               rows, rows_per_stage, eps);
    else
      ln_modulate_quant_kernel<N, false><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), x_stride,
                                                                shift, scale, mod_stride, static_cast<uint8_t*>(xq),
                                                                x_scale, rows, rows_per_stage, eps);
  });
  if (rc != WF_OK) return rc;
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_gate_residual(void* x, int64_t x_stride, const void* y, int64_t y_stride, const float* gate,
                                int64_t gate_stride, int64_t rows, int64_t dim, int64_t rows_per_stage,
                                void* stream) {
  if (!x || !y || !gate || rows < 0 || rows_per_stage < 1 || !aligned16(x) || !aligned16(y) || !aligned16(gate) ||
      x_stride % 8 || y_stride % 8 || gate_stride % 4)
    return fail(WF_ERR_INVALID_ARG, "wf_gate_residual: bad arguments");
  if (rows == 0) return WF_OK;
  const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = by_dim(dim, [&](auto n) {
    gate_residual_kernel<decltype(n)::value><<<blocks, 256, 0, s>>>(
        static_cast<__nv_bfloat16*>(x), x_stride, static_cast<const __nv_bfloat16*>(y), y_stride, gate,
        gate_stride, rows, rows_per_stage);
  });
  if (rc != WF_OK) return rc;
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_gate_residual_then(void* x, int64_t x_stride, const void* y, int64_t y_stride,
                                     const float* gate, int64_t gate_stride, int64_t gate_rows_per_stage,
                                     const float* shift, const float* scale, int64_t mod_stride,
                                     int64_t mod_rows_per_stage, float eps, void* out, int64_t out_stride, void* xq,
                                     float* x_scale, int qtype, int64_t rows, int64_t dim, void* stream) {
  const bool mod = shift != nullptr || scale != nullptr;
  if (!x || !y || !gate || rows < 0 || gate_rows_per_stage < 1 || !aligned16(x) || !aligned16(y) ||
      !aligned16(gate) || x_stride % 8 || y_stride % 8 || gate_stride % 4 || x_stride < dim || y_stride < dim ||
      gate_stride < 0 || rows > (int64_t{1} << 34))
    return fail(WF_ERR_INVALID_ARG, "wf_gate_residual_then: bad residual arguments");
  if (mod && (!shift || !scale || !aligned16(shift) || !aligned16(scale) || mod_stride % 4 || mod_rows_per_stage < 1))
    return fail(WF_ERR_INVALID_ARG, "wf_gate_residual_then: shift and scale go together (16-byte aligned)");
  if ((out != nullptr) == (xq != nullptr))
    return fail(WF_ERR_INVALID_ARG, "wf_gate_residual_then: exactly one of out / xq");
  if (!mod && !xq) return fail(WF_ERR_INVALID_ARG, "wf_gate_residual_then: without modulation only xq output");
  if (out && (!aligned16(out) || out_stride % 8 || out_stride < dim))
    return fail(WF_ERR_INVALID_ARG, "wf_gate_residual_then: out must be 16-byte aligned rows");
  if (xq && (!x_scale || !aligned16(xq)))
    return fail(WF_ERR_INVALID_ARG, "wf_gate_residual_then: xq (16-byte aligned) needs x_scale");
  if (xq && qtype != WF_DTYPE_E4M3 && qtype != WF_DTYPE_S8)
    return fail(WF_ERR_UNSUPPORTED, "wf_gate_residual_then: qtype must be WF_DTYPE_E4M3 or WF_DTYPE_S8");
  if (rows == 0) return WF_OK;
  const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int mode = !mod ? 0 : (out ? 1 : 2);
  const bool i8 = qtype == WF_DTYPE_S8;
  auto bx = static_cast<__nv_bfloat16*>(x);
  auto by = static_cast<const __nv_bfloat16*>(y);
  auto bo = static_cast<__nv_bfloat16*>(out);
  auto bq = static_cast<uint8_t*>(xq);
  int rc = by_dim(dim, [&](auto n) {
    constexpr int N = decltype(n)::value;
#define WFK_GRT(M, I)                                                                                           \
  gate_residual_then_kernel<N, M, I><<<blocks, 256, 0, s>>>(bx, x_stride, by, y_stride, gate, gate_stride, shift, \
                                                            scale, mod_stride, bo, out_stride, bq, x_scale, rows, \
                                                            gate_rows_per_stage, mod_rows_per_stage, eps)
    if (mode == 0) {
      if (i8) WFK_GRT(0, true); else WFK_GRT(0, false);
    } else if (mode == 1) {
      WFK_GRT(1, false);
    } else {
      if (i8) WFK_GRT(2, true); else WFK_GRT(2, false);
    }
#undef WFK_GRT
  });
  if (rc != WF_OK) return rc;
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

// ------------------------------------------------ fused FP8 K/V publish
// Destination slots per stage, kept in parameter space (__grid_constant__:
// indexed in place, not copied to local memory).
constexpr int PUB_STAGES = 8, PUB_DST = 8;
struct PublishTable {
  int n[PUB_STAGES];
  uint8_t* ck[PUB_STAGES][PUB_DST];
  uint8_t* cv[PUB_STAGES][PUB_DST];
  float* sk[PUB_STAGES][PUB_DST];
  float* sv[PUB_STAGES][PUB_DST];
};

// Three warps per token row r of the fused QKV output [rows, >= 3 dim]:
// role 0 writes roped q; role 1 writes roped k and the normalised un-roped k,
// exactly as qk_norm_rope_kernel, and, when the row's stage s has
// destinations, quantises the bf16 roped-k row per token (the codec's row
// helpers, bit-identical to wf_kv_quant_publish on k_out) into every
// destination; role 2 does the same for the row's V (columns [2 dim, 3 dim)
// of the QKV output), which needs no other pass.  Destination rows are
// indexed by the row's position within its stage, r % rows_per_stage.
template <int NCH>
__global__ void __launch_bounds__(256, NCH <= 6 ? 3 : 1) qk_norm_rope_publish_kernel(
    const __nv_bfloat16* __restrict__ qkv, int64_t ld, const __nv_bfloat16* __restrict__ wq,
    const __nv_bfloat16* __restrict__ wk, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
    int head_dim, __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_out,
    __nv_bfloat16* __restrict__ k_unroped, int64_t rows, int64_t rows_per_stage, float eps,
    const __grid_constant__ PublishTable pub) {
  using namespace wfk::quant;
  const int lane = threadIdx.x & 31;
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (wid >= 3 * rows) return;
  const int64_t r = wid / 3;
  const int role = static_cast<int>(wid - 3 * r);
  constexpr int DIM = NCH * 256;
  const int64_t tok = r % rows_per_stage;
  const int64_t st = r / rows_per_stage;
  const int nd = (role == 0 || st >= PUB_STAGES) ? 0 : pub.n[st];
  if (role == 2) {
    if (nd == 0) return;
    const uint4* src = reinterpret_cast<const uint4*>(qkv + r * ld + 2 * DIM);
    uint4 buf[NCH];
    uint32_t m2 = 0;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      buf[c] = __ldg(src + lane + 32 * c);
      m2 = amax8_bits(buf[c], m2);
    }
    const RowQuant q = make_rowq(warp_amax_bits(m2));
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const uint2 code = quant8(buf[c], q);
      for (int d = 0; d < nd; ++d) reinterpret_cast<uint2*>(pub.cv[st][d] + tok * DIM)[lane + 32 * c] = code;
    }
    if (lane == 0)
      for (int d = 0; d < nd; ++d) pub.sv[st][d][tok] = q.s;
    return;
  }
  const bool is_k = role == 1;
  const uint4* src = reinterpret_cast<const uint4*>(qkv + r * ld + (is_k ? DIM : 0));
  const uint4* w4 = reinterpret_cast<const uint4*>(is_k ? wk : wq);
  float v[NCH][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    unpack8(__ldg(src + lane + 32 * c), v[c]);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(v[c][i], v[c][i], ss);
  }
  const float rn = rsqrtf(warp_sum(ss) * (1.f / DIM) + eps);
  const int half = head_dim / 2;
  const float* ct = cos_t + (st * rows_per_stage + tok) * half;
  const float* stab = sin_t + (st * rows_per_stage + tok) * half;
  __nv_bfloat16* dst = (is_k ? k_out : q_out) + r * DIM;
  constexpr bool KEEP = NCH <= 12;  // roped k rows of up to 3072 stay in registers for the quantiser
  uint4 kept[KEEP ? NCH : 1];
  uint32_t m2 = 0;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int e0 = (lane + 32 * c) * 8;
    float w[8];
    unpack8(__ldg(w4 + lane + 32 * c), w);
    float n[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) n[i] = bf(bf(v[c][i] * rn) * w[i]);
    if (is_k && k_unroped) reinterpret_cast<uint4*>(k_unroped + r * DIM)[lane + 32 * c] = pack8(n);
    const int pd = (e0 % head_dim) / 2;
    const float4 cv = *reinterpret_cast<const float4*>(ct + pd);
    const float4 sv = *reinterpret_cast<const float4*>(stab + pd);
    const float cc[4] = {cv.x, cv.y, cv.z, cv.w}, sn[4] = {sv.x, sv.y, sv.z, sv.w};
    float o[8];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float re = n[2 * p], im = n[2 * p + 1];
      o[2 * p] = fmaf(re, cc[p], -im * sn[p]);
      o[2 * p + 1] = fmaf(re, sn[p], im * cc[p]);
    }
    const uint4 packed = pack8(o);
    reinterpret_cast<uint4*>(dst)[lane + 32 * c] = packed;
    if (nd > 0) {
      m2 = amax8_bits(packed, m2);
      if constexpr (KEEP) kept[c] = packed;
    }
  }
  if (nd == 0) return;
  const RowQuant q = make_rowq(warp_amax_bits(m2));
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    // wider rows read back this lane's own stores of k_out
    const uint4 packed = KEEP ? kept[c] : reinterpret_cast<const uint4*>(dst)[lane + 32 * c];
    const uint2 code = quant8(packed, q);
    for (int d = 0; d < nd; ++d) reinterpret_cast<uint2*>(pub.ck[st][d] + tok * DIM)[lane + 32 * c] = code;
  }
  if (lane == 0)
    for (int d = 0; d < nd; ++d) pub.sk[st][d][tok] = q.s;
}

extern "C" int wf_qk_norm_rope(const void* qkv, int64_t ld, const void* wq, const void* wk, const float* cos_t,
                               const float* sin_t, int head_dim, void* q_out, void* k_out, void* k_unroped,
                               int64_t rows, int64_t dim, int64_t rows_per_stage, float eps, void* stream) {
  if (!qkv || !wq || !wk || !cos_t || !sin_t || !q_out || !k_out || rows < 0 || rows_per_stage < 1 ||
      head_dim < 8 || head_dim % 8 || dim % head_dim || ld % 8 || !aligned16(qkv) || !aligned16(q_out) ||
      !aligned16(k_out) || !aligned16(cos_t) || !aligned16(sin_t) || (k_unroped && !aligned16(k_unroped)))
    return fail(WF_ERR_INVALID_ARG, "wf_qk_norm_rope: bad arguments");
  if (rows == 0) return WF_OK;
  const unsigned blocks = static_cast<unsigned>((2 * rows + 7) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = by_dim(dim, [&](auto n) {
    qk_norm_rope_kernel<decltype(n)::value><<<blocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(qkv), ld, static_cast<const __nv_bfloat16*>(wq),
        static_cast<const __nv_bfloat16*>(wk), cos_t, sin_t, head_dim, static_cast<__nv_bfloat16*>(q_out),
        static_cast<__nv_bfloat16*>(k_out), static_cast<__nv_bfloat16*>(k_unroped), rows, rows_per_stage, eps);
  });
  if (rc != WF_OK) return rc;
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_qk_norm_rope_publish(const void* qkv, int64_t ld, const void* wq, const void* wk,
                                       const float* cos_t, const float* sin_t, int head_dim, void* q_out,
                                       void* k_out, void* k_unroped, int64_t rows, int64_t dim,
                                       int64_t rows_per_stage, float eps, const wf_kv_publish_dst* dsts,
                                       const int32_t* n_dst, int n_stages, void* stream) {
  if (!qkv || !wq || !wk || !cos_t || !sin_t || !q_out || !k_out || rows < 0 || rows_per_stage < 1 ||
      head_dim < 8 || head_dim % 8 || dim % head_dim || ld % 8 || !aligned16(qkv) || !aligned16(q_out) ||
      !aligned16(k_out) || !aligned16(cos_t) || !aligned16(sin_t) || (k_unroped && !aligned16(k_unroped)))
    return fail(WF_ERR_INVALID_ARG, "wf_qk_norm_rope_publish: bad arguments");
  if (n_stages < 0 || n_stages > PUB_STAGES || (n_stages > 0 && (!dsts || !n_dst)))
    return fail(WF_ERR_INVALID_ARG, "wf_qk_norm_rope_publish: n_stages %d (at most %d, with dsts and n_dst)",
                n_stages, PUB_STAGES);
  if (rows > static_cast<int64_t>(PUB_STAGES) * rows_per_stage && n_stages > 0)
    return fail(WF_ERR_INVALID_ARG, "wf_qk_norm_rope_publish: rows of more than %d stages", PUB_STAGES);
  PublishTable tab{};
  for (int s = 0; s < n_stages; ++s) {
    if (n_dst[s] < 0 || n_dst[s] > PUB_DST)
      return fail(WF_ERR_INVALID_ARG, "wf_qk_norm_rope_publish: stage %d has %d destinations (0..%d)", s,
                  n_dst[s], PUB_DST);
    tab.n[s] = n_dst[s];
    for (int d = 0; d < n_dst[s]; ++d) {
      const wf_kv_publish_dst& e = dsts[s * PUB_DST + d];
      if (!e.codes_k || !e.codes_v || !e.scales_k || !e.scales_v ||
          (reinterpret_cast<uintptr_t>(e.codes_k) | reinterpret_cast<uintptr_t>(e.codes_v)) & 7 ||
          (reinterpret_cast<uintptr_t>(e.scales_k) | reinterpret_cast<uintptr_t>(e.scales_v)) & 3)
        return fail(WF_ERR_INVALID_ARG,
                    "wf_qk_norm_rope_publish: stage %d destination %d: null or misaligned (codes 8 B, scales 4 B)",
                    s, d);
      tab.ck[s][d] = e.codes_k;
      tab.cv[s][d] = e.codes_v;
      tab.sk[s][d] = e.scales_k;
      tab.sv[s][d] = e.scales_v;
    }
  }
  if (rows == 0) return WF_OK;
  const unsigned blocks = static_cast<unsigned>((3 * rows + 7) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = by_dim(dim, [&](auto n) {
    qk_norm_rope_publish_kernel<decltype(n)::value><<<blocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(qkv), ld, static_cast<const __nv_bfloat16*>(wq),
        static_cast<const __nv_bfloat16*>(wk), cos_t, sin_t, head_dim, static_cast<__nv_bfloat16*>(q_out),
        static_cast<__nv_bfloat16*>(k_out), static_cast<__nv_bfloat16*>(k_unroped), rows, rows_per_stage, eps, tab);
  });
  if (rc != WF_OK) return rc;
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_rms_norm(const void* x, int64_t x_stride, const void* w, void* out, int64_t out_stride,
                           int64_t rows, int64_t dim, float eps, void* stream) {
  if (!x || !w || !out || rows < 0 || !aligned16(x) || !aligned16(w) || !aligned16(out) || x_stride % 8 ||
      out_stride % 8)
    return fail(WF_ERR_INVALID_ARG, "wf_rms_norm: bad arguments");
  if (rows == 0) return WF_OK;
  const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = by_dim(dim, [&](auto n) {
    rms_norm_kernel<decltype(n)::value><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), x_stride,
                                                               static_cast<const __nv_bfloat16*>(w),
                                                               static_cast<__nv_bfloat16*>(out), out_stride, rows,
                                                               eps);
  });
  if (rc != WF_OK) return rc;
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}
