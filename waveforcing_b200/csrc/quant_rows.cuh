// Row quantisation helpers shared by the FP8 K/V codec (kv_codec.cu) and the
// W8A8 activation quantiser (gemm_w8a8.cu).  The exactness argument for the
// fast path is at the top of kv_codec.cu: for bf16 x and bf16 s,
// bf16(RN(x * RN(1/s))) equals bf16(RN(x / s)).
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

#include "sm100.cuh"

namespace wfk {
namespace quant {

__device__ __forceinline__ float bf16_round_f(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float scale_from_amax(float amax, float qmax = 448.f) {
  // bf16(amax / qmax) with IEEE division, clamped below by bf16(1e-8).
  const float s = bf16_round_f(__fdiv_rn(amax, qmax));
  const float smin = bf16_round_f(1e-8f);
  return (s >= smin || s != s) ? s : smin;  // NaN propagates like torch.clamp
}

// Exact software e4m3fn encoder for a bf16-valued float (torch semantics).
__device__ __forceinline__ uint32_t e4m3_encode_sw(float f) {
  const uint32_t bits = __float_as_uint(f);
  const uint32_t sign = (bits >> 24) & 0x80u;
  const float a = fabsf(f);
  if (!(a <= 464.f)) return 0x7Fu | sign;  // NaN, inf, or rounds past 448
  if (a < 0.015625f) {                     // below 2^-6: subnormal grid 2^-9
    return static_cast<uint32_t>(rintf(a * 512.f)) | sign;
  }
  const uint32_t ab = __float_as_uint(a);
  int e = static_cast<int>((ab >> 23) & 0xFF) - 127;
  uint32_t q = (ab >> 20) & 7u;
  const uint32_t rem = ab & 0xFFFFFu;
  if (rem > 0x80000u || (rem == 0x80000u && (q & 1u))) ++q;
  if (q == 8u) {
    q = 0;
    ++e;
  }
  return ((static_cast<uint32_t>(e + 7) << 3) | q) | sign;
}

// Two bf16-valued floats -> two e4m3 codes (lo in bits 0-7).
__device__ __forceinline__ uint32_t e4m3x2_hw(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

struct RowQuant {
  float s;      // scale (as stored)
  float r;      // RN(1/s)
  bool finite;  // fast path valid
};

__device__ __forceinline__ RowQuant make_rowq(float amax, float qmax = 448.f) {
  RowQuant q;
  q.s = scale_from_amax(amax, qmax);
  q.finite = isfinite(q.s);
  q.r = __frcp_rn(q.s);
  return q;
}

// Two bf16 magnitudes (one bf16x2 word, signs ignored) -> two e4m3 codes of
// bf16(|x| * r) in the low 16 bits.
__device__ __forceinline__ uint32_t e4m3x2_mag(uint32_t w, float r) {
  const uint32_t a = w & 0x7FFF7FFFu;
  const float2 p = fmul2(make_float2(__uint_as_float(a << 16), __uint_as_float(a & 0xFFFF0000u)), make_float2(r, r));
  const __nv_bfloat162 b = __floats2bfloat162_rn(p.x, p.y);
  const uint32_t bb = *reinterpret_cast<const uint32_t*>(&b);
  return e4m3x2_hw(__uint_as_float(bb << 16), __uint_as_float(bb & 0xFFFF0000u));
}

// Four bf16 (two bf16x2 words) -> four codes, fast path (finite scale).
__device__ __forceinline__ uint32_t quant4_fast(uint32_t w0, uint32_t w1, float r) {
  const uint32_t mag = __byte_perm(e4m3x2_mag(w0, r), e4m3x2_mag(w1, r), 0x5410);
  // the sign bits of the four bf16 (bit 15 / 31 of each word) into bit 7 of each code byte
  return mag | (__byte_perm(w0, w1, 0x7531) & 0x80808080u);
}

// 8 bf16 (uint4) -> 8 codes (uint2)
__device__ __forceinline__ uint2 quant8(const uint4& v, const RowQuant& q) {
  if (q.finite) return make_uint2(quant4_fast(v.x, v.y, q.r), quant4_fast(v.z, v.w, q.r));
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t out[2] = {0, 0};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float b0 = bf16_round_f(__fdiv_rn(__uint_as_float(w[i] << 16), q.s));
    const float b1 = bf16_round_f(__fdiv_rn(__uint_as_float(w[i] & 0xFFFF0000u), q.s));
    const uint32_t c = e4m3_encode_sw(b0) | (e4m3_encode_sw(b1) << 8);
    out[i >> 1] |= c << ((i & 1) * 16);
  }
  return make_uint2(out[0], out[1]);
}

// 16 bf16 (two uint4) -> 16 codes (uint4)
__device__ __forceinline__ uint4 quant16(const uint4& a, const uint4& b, const RowQuant& q) {
  const uint2 lo = quant8(a, q), hi = quant8(b, q);
  return make_uint4(lo.x, lo.y, hi.x, hi.y);
}

__device__ __forceinline__ float amax8(const uint4& v, float m) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float x0 = fabsf(__uint_as_float(w[i] << 16));
    const float x1 = fabsf(__uint_as_float(w[i] & 0xFFFF0000u));
    // NaN-propagating max (torch.amax propagates NaN)
    m = (x0 > m || x0 != x0) ? x0 : m;
    m = (x1 > m || x1 != x1) ? x1 : m;
  }
  return m;
}

// Running maximum of |x| over bf16x2 words, kept as two u16 lanes of bf16
// magnitude bits.  Non-negative floats, +inf and NaN order like their bit
// patterns, so the integer maximum is torch.amax's NaN-propagating maximum.
__device__ __forceinline__ uint32_t vmax_u16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t amax8_bits(const uint4& v, uint32_t m2) {
  m2 = vmax_u16x2(m2, v.x & 0x7FFF7FFFu);
  m2 = vmax_u16x2(m2, v.y & 0x7FFF7FFFu);
  m2 = vmax_u16x2(m2, v.z & 0x7FFF7FFFu);
  return vmax_u16x2(m2, v.w & 0x7FFF7FFFu);
}

// Warp-wide maximum of packed magnitudes -> f32 amax (bf16-valued).
__device__ __forceinline__ float warp_amax_bits(uint32_t m2) {
  const uint32_t m = __reduce_max_sync(0xffffffffu, max(m2 & 0xFFFFu, m2 >> 16));
  return __uint_as_float(m << 16);
}

__device__ __forceinline__ float warp_max_nan(float m) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float t = __shfl_xor_sync(0xffffffffu, m, o);
    m = (t > m || t != t) ? t : m;
  }
  return m;
}

// Two bf16 (one bf16x2 word) -> two int8 codes of clamp(rint(bf16(x * r)),
// -127, 127) in the low 16 bits (round half to even, like numpy/torch round).
__device__ __forceinline__ uint32_t i8x2_fast(uint32_t w, float r) {
  const float2 p = fmul2(make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u)), make_float2(r, r));
  const __nv_bfloat162 b = __floats2bfloat162_rn(p.x, p.y);
  const uint32_t bb = *reinterpret_cast<const uint32_t*>(&b);
  const int a = __float2int_rn(fminf(fmaxf(__uint_as_float(bb << 16), -127.f), 127.f));
  const int c = __float2int_rn(fminf(fmaxf(__uint_as_float(bb & 0xFFFF0000u), -127.f), 127.f));
  return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(c) & 0xFFu) << 8);
}

// Integer code of one bf16-valued ratio when the scale is not finite (IEEE
// division already applied): rint, then fmax/fmin against +-127 (NaN -> -127).
__device__ __forceinline__ uint32_t i8_slow(float ratio) {
  return static_cast<uint32_t>(static_cast<int>(fminf(fmaxf(rintf(ratio), -127.f), 127.f))) & 0xFFu;
}

// 8 codes (uint2) -> 8 bf16 (uint4) of e4m3(code) * s: the e4m3 value is
// exact in f16 and f32, the f32 product rounds once to bf16.
__device__ __forceinline__ uint4 dequant8(const uint2& c, float s) {
  const uint32_t w[2] = {c.x, c.y};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t f2;
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(f2) : "h"(static_cast<uint16_t>(h ? w[j] >> 16 : w[j] & 0xFFFF)));
      const float2 p = fmul2(make_float2(__half2float(__ushort_as_half(static_cast<unsigned short>(f2 & 0xFFFF))),
                                         __half2float(__ushort_as_half(static_cast<unsigned short>(f2 >> 16)))),
                             make_float2(s, s));
      o[2 * j + h] = pack_bf16x2(p.x, p.y);
    }
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace quant
}  // namespace wfk
