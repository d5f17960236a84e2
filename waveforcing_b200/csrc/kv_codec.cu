// FP8 e4m3 K/V codec (HBM-bound), bit-exact to the reference's dtype sequence
// (wave_rt/denoiser/exchange/common.py:143-164):
//     s    = f32(clamp(bf16(amax|x| / 448), 1e-8))
//     code = e4m3fn(bf16(x / s))          RNE, |v| > 464 -> NaN
//     deq  = e4m3(code) * s
// Layout: x is [rows, cols] bf16 with a row stride; codes are dense [rows, cols]
// u8; per-token scales [rows] f32 (or one f32 for the per-tensor mode).
//
// Exactness notes.
//  * The reference rounds x / s to f32 and then to bf16.  x and s are both
//    bf16 (8-bit significands A, B), so x / s = (A / B) 2^k is never a bf16
//    rounding midpoint (that would need B / gcd(A, B) to be a power of two of
//    at least 2^8) and lies at least 2^-17 (relative) away from every
//    midpoint.  RN(x * RN(1/s)) is within 2^-23 of x / s, so its bf16 rounding
//    equals the bf16 rounding of the correctly rounded quotient: the fast path
//    is one multiply by the row's reciprocal.  Rows whose scale is not finite
//    take the IEEE division and the software encoder.
//  * bf16 and e4m3 round-to-nearest are symmetric, so the fast path rounds
//    |x| / s and ORs x's sign into each code afterwards (torch keeps -0 as
//    0x80; the hardware conversion of a value that rounds to zero does not).
//  * The hardware e4m3 conversion saturates, torch's does not.  For a finite
//    row amax the bf16 quotient is at most 450 in magnitude (s is amax/448
//    rounded to bf16, so |x|/s <= 448.9 before rounding), where saturating and
//    non-saturating RNE agree; non-finite rows use the exact software encoder.
#include <cuda_runtime.h>

#include <mutex>

#include "host_util.h"
#include "quant_rows.cuh"
#include "sm100.cuh"

namespace wfk {
namespace codec {

constexpr int WARPS = 8;

using namespace wfk::quant;

// One warp per row; NCH 16-byte chunks per lane kept in registers (cols ==
// NCH * 256), or NCH == 0 for any cols % 8 == 0 (two passes over the row).
template <int NCH>
__device__ __forceinline__ void quant_row(const __nv_bfloat16* __restrict__ xrow, int64_t cols, int lane,
                                          uint8_t* const* dst_codes, float* const* dst_scales, int n_dst,
                                          int64_t row) {
  const uint4* x4 = reinterpret_cast<const uint4*>(xrow);
  const int64_t nch = cols / 8;
  uint32_t m2 = 0;
  uint4 buf[NCH > 0 ? NCH : 1];
  if constexpr (NCH > 0) {
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      buf[i] = __ldcs(x4 + lane + 32 * i);
      m2 = amax8_bits(buf[i], m2);
    }
  } else {
    for (int64_t c = lane; c < nch; c += 32) m2 = amax8_bits(__ldg(x4 + c), m2);
  }
  const RowQuant q = make_rowq(warp_amax_bits(m2));
  if constexpr (NCH > 0) {
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const uint2 c = quant8(buf[i], q);
      for (int d = 0; d < n_dst; ++d) reinterpret_cast<uint2*>(dst_codes[d] + row * cols)[lane + 32 * i] = c;
    }
  } else {
    for (int64_t c = lane; c < nch; c += 32) {
      const uint2 cc = quant8(__ldg(x4 + c), q);
      for (int d = 0; d < n_dst; ++d) reinterpret_cast<uint2*>(dst_codes[d] + row * cols)[c] = cc;
    }
  }
  if (lane == 0)
    for (int d = 0; d < n_dst; ++d) dst_scales[d][row] = q.s;
}

constexpr int MAX_DST = 8;
struct DstList {
  uint8_t* codes[MAX_DST];
  float* scales[MAX_DST];
};

template <int NCH>
__global__ void __launch_bounds__(WARPS * 32)
    quant_token_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int64_t cols, int64_t row_stride,
                       DstList dst, int n_dst) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  quant_row<NCH>(x + row * row_stride, cols, lane, dst.codes, dst.scales, n_dst, row);
}

// K and V of one layer in one launch: rows [0, rows) from k, [rows, 2 rows) from v.
template <int NCH>
__global__ void __launch_bounds__(WARPS * 32)
    quant_publish_kernel(const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v, int64_t rows,
                         int64_t cols, int64_t k_stride, int64_t v_stride, DstList dk, DstList dv, int n_dst) {
  const int lane = threadIdx.x & 31;
  int64_t row = static_cast<int64_t>(blockIdx.x) * WARPS + (threadIdx.x >> 5);
  if (row >= 2 * rows) return;
  if (row < rows) {
    quant_row<NCH>(k + row * k_stride, cols, lane, dk.codes, dk.scales, n_dst, row);
  } else {
    row -= rows;
    quant_row<NCH>(v + row * v_stride, cols, lane, dv.codes, dv.scales, n_dst, row);
  }
}

// Fused publish: NDST destinations known at compile time (pointer table stays in
// parameter space), each lane owns 16 consecutive elements per chunk so every
// destination receives 16-byte code stores, and warps loop over rows.
// NCH16 = cols / 512.
template <int NCH16, int NDST>
__global__ void __launch_bounds__(WARPS * 32)
    quant_publish16_kernel(const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v, int64_t rows,
                           int64_t k_stride, int64_t v_stride, DstList dk, DstList dv) {
  constexpr int64_t COLS = NCH16 * 512;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * WARPS;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * WARPS + (threadIdx.x >> 5); w < 2 * rows; w += nwarps) {
    const bool is_v = w >= rows;
    const int64_t row = is_v ? w - rows : w;
    const uint4* x4 = reinterpret_cast<const uint4*>((is_v ? v : k) + row * (is_v ? v_stride : k_stride));
    uint4 buf[2 * NCH16];
    uint32_t m2 = 0;
#pragma unroll
    for (int i = 0; i < NCH16; ++i) {
      buf[2 * i] = __ldcs(x4 + 2 * (lane + 32 * i));
      buf[2 * i + 1] = __ldcs(x4 + 2 * (lane + 32 * i) + 1);
      m2 = amax8_bits(buf[2 * i], m2);
      m2 = amax8_bits(buf[2 * i + 1], m2);
    }
    const RowQuant q = make_rowq(warp_amax_bits(m2));
    const DstList& d = is_v ? dv : dk;
#pragma unroll
    for (int i = 0; i < NCH16; ++i) {
      const uint4 c = quant16(buf[2 * i], buf[2 * i + 1], q);
#pragma unroll
      for (int j = 0; j < NDST; ++j) reinterpret_cast<uint4*>(d.codes[j] + row * COLS)[lane + 32 * i] = c;
    }
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < NDST; ++j) d.scales[j][row] = q.s;
    }
  }
}

// Scale-free cast of the onesided exchange (wave_rt/denoiser/exchange/onesided.py:152):
// code = e4m3fn(x) for bf16 x with torch's non-saturating RNE (|x| > 464 -> NaN),
// through the exact software encoder since no scale bounds the inputs.
__global__ void cast_e4m3_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int64_t cols,
                                 int64_t row_stride, uint8_t* __restrict__ codes) {
  const int64_t nch = cols / 8;
  const int64_t total = rows * nch;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nch, c = i - r * nch;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(x + r * row_stride) + c);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t out[2] = {0, 0};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t c2 = e4m3_encode_sw(__uint_as_float(w[k] << 16)) |
                          (e4m3_encode_sw(__uint_as_float(w[k] & 0xFFFF0000u)) << 8);
      out[k >> 1] |= c2 << ((k & 1) * 16);
    }
    reinterpret_cast<uint2*>(codes + r * cols)[c] = make_uint2(out[0], out[1]);
  }
}

// ------------------------------------------------------------ per-tensor
__global__ void amax_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int64_t cols, int64_t row_stride,
                            unsigned int* __restrict__ amax_bits) {
  const int64_t nch = cols / 8;
  const int64_t total = rows * nch;
  float m = 0.f;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nch, c = i - r * nch;
    m = amax8(__ldg(reinterpret_cast<const uint4*>(x + r * row_stride) + c), m);
  }
  m = warp_max_nan(m);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    m = warp_max_nan(m);
    // non-negative floats (and +NaN, which sorts above +inf) order like their bits
    if (threadIdx.x == 0) atomicMax(amax_bits, __float_as_uint(m) & 0x7FFFFFFFu);
  }
}

__global__ void quant_tensor_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int64_t cols,
                                    int64_t row_stride, const unsigned int* __restrict__ amax_bits,
                                    uint8_t* __restrict__ codes, float* __restrict__ scale_out) {
  const RowQuant q = make_rowq(__uint_as_float(*amax_bits));
  const int64_t nch = cols / 8;
  const int64_t total = rows * nch;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nch, c = i - r * nch;
    const uint2 cc = quant8(__ldg(reinterpret_cast<const uint4*>(x + r * row_stride) + c), q);
    reinterpret_cast<uint2*>(codes + r * cols)[c] = cc;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = q.s;
}

// ------------------------------------------------------------- dequant
__global__ void dequant_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ scales,
                               __nv_bfloat16* __restrict__ out, int64_t rows, int64_t cols, int64_t out_stride,
                               int mode) {
  const int64_t nch = cols / 8;
  const int64_t total = rows * nch;
  const float s_tensor = (mode == WF_SCALE_TENSOR) ? scales[0] : 1.f;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nch, c = i - r * nch;
    const float s = (mode == WF_SCALE_TOKEN) ? __ldg(scales + r) : s_tensor;
    const uint2 cc = __ldcs(reinterpret_cast<const uint2*>(codes + r * cols) + c);
    const uint32_t w[2] = {cc.x, cc.y};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint32_t lo2, hi2;
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(lo2) : "h"(static_cast<uint16_t>(w[j] & 0xFFFF)));
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(hi2) : "h"(static_cast<uint16_t>(w[j] >> 16)));
      const float f0 = __half2float(__ushort_as_half(static_cast<unsigned short>(lo2 & 0xFFFF))) * s;
      const float f1 = __half2float(__ushort_as_half(static_cast<unsigned short>(lo2 >> 16))) * s;
      const float f2 = __half2float(__ushort_as_half(static_cast<unsigned short>(hi2 & 0xFFFF))) * s;
      const float f3 = __half2float(__ushort_as_half(static_cast<unsigned short>(hi2 >> 16))) * s;
      o[2 * j] = pack_bf16x2(f0, f1);
      o[2 * j + 1] = pack_bf16x2(f2, f3);
    }
    reinterpret_cast<uint4*>(out + r * out_stride)[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Warp per row, NCH8 chunks of 8 codes per lane (cols = NCH8 * 256): lane l
// handles chunks l, l + 32, ... so each warp load covers 256 contiguous code
// bytes and each warp store 512 contiguous output bytes.
template <int NCH8>
__global__ void __launch_bounds__(WARPS * 32)
    dequant_row_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ scales,
                       __nv_bfloat16* __restrict__ out, int64_t rows, int64_t out_stride, int mode) {
  constexpr int64_t COLS = NCH8 * 256;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * WARPS;
  const float s_tensor = (mode == WF_SCALE_TENSOR) ? scales[0] : 1.f;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * WARPS + (threadIdx.x >> 5); r < rows; r += nwarps) {
    const float s = (mode == WF_SCALE_TOKEN) ? __ldg(scales + r) : s_tensor;
    const uint2* c2 = reinterpret_cast<const uint2*>(codes + r * COLS);
    uint4* o4 = reinterpret_cast<uint4*>(out + r * out_stride);
    uint2 c[NCH8];
#pragma unroll
    for (int i = 0; i < NCH8; ++i) c[i] = __ldcs(c2 + lane + 32 * i);
#pragma unroll
    for (int i = 0; i < NCH8; ++i) o4[lane + 32 * i] = dequant8(c[i], s);
  }
}

static int grid_for(int64_t work_items, int threads) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t blocks = (work_items + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sms) * 16;
  if (blocks > cap) blocks = cap;
  return static_cast<int>(blocks < 1 ? 1 : blocks);
}

static bool rows_ok(const void* x, int64_t rows, int64_t cols, int64_t stride) {
  return x && rows >= 0 && cols > 0 && cols % 8 == 0 && stride >= cols && stride % 8 == 0 && aligned16(x);
}

template <typename Launch>
static void dispatch_nch(int64_t cols, Launch&& launch) {
  if (cols == 1536)
    launch(std::integral_constant<int, 6>());
  else if (cols == 5120)
    launch(std::integral_constant<int, 20>());
  else if (cols == 3072)
    launch(std::integral_constant<int, 12>());
  else
    launch(std::integral_constant<int, 0>());
}

}  // namespace codec
}  // namespace wfk

using namespace wfk;
using namespace wfk::codec;

extern "C" int wf_kv_quant(const void* x, uint8_t* codes, float* scales, int64_t rows, int64_t cols,
                           int64_t x_row_stride, int mode, void* workspace, void* stream) {
  if (!rows_ok(x, rows, cols, x_row_stride) || !codes || (mode != WF_SCALE_NONE && !scales) ||
      (reinterpret_cast<uintptr_t>(codes) & 7))
    return fail(WF_ERR_INVALID_ARG, "wf_kv_quant: bad arguments (cols %% 8, 16-byte x, 8-byte codes)");
  if (rows == 0) return WF_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (mode == WF_SCALE_TOKEN) {
    DstList d{};
    d.codes[0] = codes;
    d.scales[0] = scales;
    const unsigned blocks = static_cast<unsigned>((rows + WARPS - 1) / WARPS);
    dispatch_nch(cols, [&](auto nch) {
      quant_token_kernel<decltype(nch)::value>
          <<<blocks, WARPS * 32, 0, s>>>(static_cast<const __nv_bfloat16*>(x), rows, cols, x_row_stride, d, 1);
    });
  } else if (mode == WF_SCALE_TENSOR) {
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 3))
      return fail(WF_ERR_INVALID_ARG, "wf_kv_quant: per-tensor mode needs a 4-byte aligned workspace");
    unsigned int* amax = static_cast<unsigned int*>(workspace);
    WFK_CUDA_TRY(cudaMemsetAsync(amax, 0, sizeof(unsigned int), s));
    const int g = grid_for(rows * (cols / 8), 256);
    amax_kernel<<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), rows, cols, x_row_stride, amax);
    quant_tensor_kernel<<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), rows, cols, x_row_stride, amax,
                                          codes, scales);
  } else if (mode == WF_SCALE_NONE) {
    const int g = grid_for(rows * (cols / 8), 256);
    cast_e4m3_kernel<<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), rows, cols, x_row_stride, codes);
  } else {
    return fail(WF_ERR_INVALID_ARG, "wf_kv_quant: mode must be WF_SCALE_NONE, WF_SCALE_TENSOR or WF_SCALE_TOKEN");
  }
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_kv_dequant(const uint8_t* codes, const float* scales, void* out, int64_t rows, int64_t cols,
                             int64_t out_row_stride, int mode, void* stream) {
  if (!rows_ok(out, rows, cols, out_row_stride) || !codes || (reinterpret_cast<uintptr_t>(codes) & 7))
    return fail(WF_ERR_INVALID_ARG, "wf_kv_dequant: bad arguments");
  if (mode != WF_SCALE_NONE && !scales) return fail(WF_ERR_INVALID_ARG, "wf_kv_dequant: scales required");
  if (mode != WF_SCALE_NONE && mode != WF_SCALE_TENSOR && mode != WF_SCALE_TOKEN)
    return fail(WF_ERR_INVALID_ARG, "wf_kv_dequant: bad mode");
  if (rows == 0) return WF_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool fast = (cols == 1536 || cols == 5120) && aligned16(out) && out_row_stride % 8 == 0;
  if (fast) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t want = (rows + WARPS - 1) / WARPS;
    const int64_t cap = static_cast<int64_t>(sms) * 8;
    const unsigned blocks = static_cast<unsigned>(want < cap ? want : cap);
    auto bf = static_cast<__nv_bfloat16*>(out);
    if (cols == 1536)
      dequant_row_kernel<6><<<blocks, WARPS * 32, 0, s>>>(codes, scales, bf, rows, out_row_stride, mode);
    else
      dequant_row_kernel<20><<<blocks, WARPS * 32, 0, s>>>(codes, scales, bf, rows, out_row_stride, mode);
  } else {
    const int g = grid_for(rows * (cols / 8), 256);
    dequant_kernel<<<g, 256, 0, s>>>(codes, scales, static_cast<__nv_bfloat16*>(out), rows, cols, out_row_stride,
                                     mode);
  }
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_kv_quant_publish(const void* k, const void* v, int64_t rows, int64_t cols, int64_t k_row_stride,
                                   int64_t v_row_stride, uint8_t* const* dst_codes_k, uint8_t* const* dst_codes_v,
                                   float* const* dst_scales_k, float* const* dst_scales_v, int n_dst,
                                   void* stream) {
  if (!rows_ok(k, rows, cols, k_row_stride) || !rows_ok(v, rows, cols, v_row_stride))
    return fail(WF_ERR_INVALID_ARG, "wf_kv_quant_publish: bad K/V arguments");
  if (n_dst < 1 || n_dst > MAX_DST || !dst_codes_k || !dst_codes_v || !dst_scales_k || !dst_scales_v)
    return fail(WF_ERR_INVALID_ARG, "wf_kv_quant_publish: 1..%d destinations required", MAX_DST);
  DstList dk{}, dv{};
  for (int i = 0; i < n_dst; ++i) {
    if (!dst_codes_k[i] || !dst_codes_v[i] || !dst_scales_k[i] || !dst_scales_v[i] ||
        (reinterpret_cast<uintptr_t>(dst_codes_k[i]) & 7) || (reinterpret_cast<uintptr_t>(dst_codes_v[i]) & 7))
      return fail(WF_ERR_INVALID_ARG, "wf_kv_quant_publish: destination %d null or misaligned", i);
    dk.codes[i] = dst_codes_k[i];
    dk.scales[i] = dst_scales_k[i];
    dv.codes[i] = dst_codes_v[i];
    dv.scales[i] = dst_scales_v[i];
  }
  if (rows == 0) return WF_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  bool aligned = true;
  for (int i = 0; i < n_dst; ++i)
    aligned = aligned && aligned16(dst_codes_k[i]) && aligned16(dst_codes_v[i]);
  const int nch16 = (cols % 512 == 0) ? static_cast<int>(cols / 512) : 0;
  if (aligned && (nch16 == 3 || nch16 == 6 || nch16 == 10)) {
    const int64_t want = (2 * rows + WARPS - 1) / WARPS;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t cap = static_cast<int64_t>(sms) * 6;
    const unsigned blocks = static_cast<unsigned>(want < cap ? want : cap);
    auto go = [&](auto nch, auto nd) {
      quant_publish16_kernel<decltype(nch)::value, decltype(nd)::value><<<blocks, WARPS * 32, 0, s>>>(
          static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v), rows, k_row_stride,
          v_row_stride, dk, dv);
    };
    auto by_n = [&](auto nch) {
      switch (n_dst) {
        case 1: go(nch, std::integral_constant<int, 1>()); break;
        case 2: go(nch, std::integral_constant<int, 2>()); break;
        case 3: go(nch, std::integral_constant<int, 3>()); break;
        case 4: go(nch, std::integral_constant<int, 4>()); break;
        case 5: go(nch, std::integral_constant<int, 5>()); break;
        case 6: go(nch, std::integral_constant<int, 6>()); break;
        case 7: go(nch, std::integral_constant<int, 7>()); break;
        default: go(nch, std::integral_constant<int, 8>()); break;
      }
    };
    if (nch16 == 3)
      by_n(std::integral_constant<int, 3>());
    else if (nch16 == 6)
      by_n(std::integral_constant<int, 6>());
    else
      by_n(std::integral_constant<int, 10>());
  } else {
    const unsigned blocks = static_cast<unsigned>((2 * rows + WARPS - 1) / WARPS);
    dispatch_nch(cols, [&](auto nch) {
      quant_publish_kernel<decltype(nch)::value><<<blocks, WARPS * 32, 0, s>>>(
          static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v), rows, cols, k_row_stride,
          v_row_stride, dk, dv, n_dst);
    });
  }
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

// ------------------------------------------------ allocation-free variant
// wf_kv_quant_tensor_static: the per-tensor quantiser with its grid-wide
// reduction scratch in this file-scope device array instead of caller memory.
// The amax pass writes one partial maximum per block of NOALLOC_SPAN
// elements; the quantise pass reduces those partials.  Every partial the
// second pass reads is written earlier by the same call, so nothing has to be
// cleared between calls, and slots beyond the current call's block count
// (left over from an earlier, larger call) are never read.  All calls on a
// device share the array: two calls whose kernels overlap on the GPU (for
// example on different streams) race and must be serialised by the caller.
namespace wfk {
namespace codec {

constexpr int NOALLOC_PARTIALS = 4096;                                 // 16 KB per GPU
constexpr int64_t NOALLOC_SPAN = 8192;                                 // elements per partial
constexpr int64_t NOALLOC_MAX_ELEMS = NOALLOC_PARTIALS * NOALLOC_SPAN;  // 33,554,432
static __device__ __align__(256) float g_noalloc_partials[NOALLOC_PARTIALS];

// block b reduces chunks [b * 1024, (b + 1) * 1024) of 8 elements
__global__ void __launch_bounds__(256) amax_partials_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows,
                                                            int64_t cols, int64_t row_stride,
                                                            float* __restrict__ partials) {
  const int64_t nch = cols / 8;
  const int64_t total = rows * nch;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * (NOALLOC_SPAN / 8);
  float m = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int64_t i = base + threadIdx.x + 256 * k;
    if (i < total) {
      const int64_t r = i / nch, c = i - r * nch;
      m = amax8(__ldg(reinterpret_cast<const uint4*>(x + r * row_stride) + c), m);
    }
  }
  m = warp_max_nan(m);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
    m = warp_max_nan(m);
    if (threadIdx.x == 0) partials[blockIdx.x] = m;
  }
}

__global__ void __launch_bounds__(256) quant_from_partials_kernel(const __nv_bfloat16* __restrict__ x,
                                                                  int64_t rows, int64_t cols, int64_t row_stride,
                                                                  const float* __restrict__ partials,
                                                                  int nparts, uint8_t* __restrict__ codes,
                                                                  float* __restrict__ scale_out) {
  __shared__ float red[8];
  float m = 0.f;
  for (int i = threadIdx.x; i < nparts; i += 256) {
    const float p = partials[i];
    m = (p > m || p != p) ? p : m;
  }
  m = warp_max_nan(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = red[0];
  for (int w = 1; w < 8; ++w) m = (red[w] > m || red[w] != red[w]) ? red[w] : m;
  const RowQuant q = make_rowq(m);
  const int64_t nch = cols / 8;
  const int64_t total = rows * nch;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nch, c = i - r * nch;
    const uint2 cc = quant8(__ldg(reinterpret_cast<const uint4*>(x + r * row_stride) + c), q);
    reinterpret_cast<uint2*>(codes + r * cols)[c] = cc;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = q.s;
}

// Device address of g_noalloc_partials per device ordinal, resolved on the
// first call made with that device current.  The cache also records the
// context the address was resolved in: after cudaDeviceReset (or any other
// teardown of the primary context) the module is loaded again and the array
// may move, so a call in a new context resolves the address again.
static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[256] = {};
static CUcontext g_noalloc_ctx[256] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

static int noalloc_scratch(float** out) {
  int dev = 0;
  WFK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 256) return fail(WF_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  auto get_ctx = reinterpret_cast<CtxGetCurrentFn>(driver_fn("cuCtxGetCurrent"));
  if (!get_ctx) return fail(WF_ERR_CUDA, "cuCtxGetCurrent unavailable from the driver");
  // Before the first runtime call that needs it, no context may be current
  // yet (ctx == nullptr); cudaGetSymbolAddress below makes the primary
  // context current, and the context is read again afterwards.
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) return fail(WF_ERR_CUDA, "cuCtxGetCurrent failed on device %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!ctx || !g_noalloc_ptr[dev] || g_noalloc_ctx[dev] != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_partials);
    if (e != cudaSuccess || !p)
      return fail(WF_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed on device %d: %s", dev, cudaGetErrorString(e));
    if (get_ctx(&ctx) != CUDA_SUCCESS || !ctx) return fail(WF_ERR_CUDA, "no current context on device %d", dev);
    g_noalloc_ptr[dev] = static_cast<float*>(p);
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_ptr[dev];
  return WF_OK;
}

}  // namespace codec
}  // namespace wfk

extern "C" int wf_kv_quant_tensor_static(const void* x, uint8_t* codes, float* scale, int64_t rows, int64_t cols,
                                         int64_t x_row_stride, void* stream) {
  if (!rows_ok(x, rows, cols, x_row_stride) || !codes || !scale || (reinterpret_cast<uintptr_t>(codes) & 7))
    return fail(WF_ERR_INVALID_ARG, "wf_kv_quant_tensor_static: bad arguments (cols %% 8, 16-byte x, 8-byte codes)");
  // Compared by division so that no product of two unchecked sizes can wrap.
  if (cols > NOALLOC_MAX_ELEMS || rows > NOALLOC_MAX_ELEMS / cols)
    return fail(WF_ERR_INVALID_ARG,
                "wf_kv_quant_tensor_static: %lld x %lld elements exceed the static scratch limit of %lld "
                "(4096 partial maxima of 8192 elements); use wf_kv_quant with a workspace",
                (long long)rows, (long long)cols, (long long)NOALLOC_MAX_ELEMS);
  if (rows == 0) return WF_OK;
  float* partials = nullptr;
  int rc = noalloc_scratch(&partials);
  if (rc != WF_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nparts = static_cast<int>((rows * cols + NOALLOC_SPAN - 1) / NOALLOC_SPAN);
  amax_partials_kernel<<<nparts, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), rows, cols, x_row_stride,
                                              partials);
  WFK_CUDA_TRY(cudaGetLastError());  // the quantise pass must not run on partials that were never written
  const int g = grid_for(rows * (cols / 8), 256);
  quant_from_partials_kernel<<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), rows, cols, x_row_stride,
                                               partials, nparts, codes, scale);
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" unsigned int wfk_status_take_codec(void) { return wfk::status_take_local(); }
