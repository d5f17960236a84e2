// W8A8 linear on tcgen05: y = (xq . wq^T) * x_scale[m] * w_scale[n] + bias[n]
// replacing torch._scaled_mm in WaveFp8Linear (wave_rt/runtime/fp8.py:49-56).
//
//   xq [M, K] and wq [N, K] are 8-bit, K-contiguous; e4m3 uses
//   tcgen05.mma kind::f8f6f4 (f32 accumulate), s8 uses kind::i8 (s32).
//   CTA tile 128 x 256, K step 128 bytes (one 128-byte swizzle row), 4-stage
//   TMA ring.  warp 0 = TMA producer, warp 1 = TMEM owner + MMA issuer,
//   warps 4-7 = epilogue (thread t owns accumulator row t = TMEM lane t):
//   scale and bias from per-tile shared-memory copies, bf16 convert into a
//   double-buffered 128 x 64 swizzled staging tile, TMA bulk store.
// Also here: load-time per-channel weight quantisation and per-token dynamic
// activation quantisation (the per-row forms of fp8.py:32-36 and :47-48).
#include <cuda_runtime.h>

#include <cstdlib>
#include <type_traits>

#include "host_util.h"
#include "quant_rows.cuh"
#include "sm100.cuh"

namespace wfk {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes (= elements for 8-bit types)
constexpr int NS = 4;
constexpr int A_TILE = BM * BK;  // 16 KB
constexpr int B_TILE = BN * BK;  // 32 KB
constexpr int OUT_COLS = 64;               // bf16 columns per staging tile (128 bytes)
constexpr int OUT_TILE = BM * OUT_COLS * 2;  // 16 KB
constexpr int NBARS = 2 * NS + 5;
constexpr int SMEM_BYTES = 1024 + NS * (A_TILE + B_TILE) + 2 * OUT_TILE + BN * 4 /*w_scale*/ + BN * 2 /*bias*/ +
                           16 /*flags*/ + NBARS * 8 + 16;
constexpr int THREADS = 256;
constexpr uint32_t EPI_BAR = 1;  // named barrier of the four epilogue warps

__device__ __forceinline__ bool wait_drain(uint64_t* bar, uint32_t parity, uint64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > timeout_ns) {
      status_raise(ST_DRAIN_TIMEOUT);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// GELU with the tanh approximation (torch GELU(approximate="tanh")):
// 0.5 x (1 + tanh(u)) with u = sqrt(2/pi) (x + 0.044715 x^3), evaluated as
// x * sigmoid(2u) = x / (1 + e^(-2u)).  That form has no cancellation for
// negative x (where 1 + tanh(u) is small): e^(-2u) from ex2.approx and the
// reciprocal from rcp.approx keep the relative error near 2^-22; e^(-2u)
// saturates to +inf / 0 for large |u|, giving 0 / x.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  const float e = ex2_approx(u * -2.8853900817779268f);  // e^(-2u)
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + e));
  return x * r;
}

// bf16 GELU(tanh) of two bf16 values in one word (f32 math, RNE back to bf16).
__device__ __forceinline__ uint32_t gelu_bf16x2(uint32_t w) {
  return pack_bf16x2(gelu_tanh(__uint_as_float(w << 16)), gelu_tanh(__uint_as_float(w & 0xFFFF0000u)));
}

// 1 / d for a pair, d in [1, 2^126], on the FMA pipe: Newton-Raphson
// r <- r (2 - d r) from the exponent-reflection first guess (the integer
// constant minus the bits of d, which maps 2^k to about 2^-k; 5.1 % max
// relative error on [1, 2^126], measured here), three steps: within 2 ulp of
// 1/d.  Frees the MUFU for the exponential in the activation quantiser,
// where one MUFU op per element otherwise bounds the kernel.
__device__ __forceinline__ float2 rcp2_newton(float2 d) {
  float2 r = make_float2(__uint_as_float(0x7EF311C3u - __float_as_uint(d.x)),
                         __uint_as_float(0x7EF311C3u - __float_as_uint(d.y)));
  const float2 nd = make_float2(-d.x, -d.y), two = make_float2(2.f, 2.f);
#pragma unroll
  for (int i = 0; i < 3; ++i) r = fmul2(r, ffma2(nd, r, two));
  return r;
}

// gelu_bf16x2 with one MUFU op per element: the same u and e^(-2u) as
// gelu_tanh, the reciprocal of 1 + e^(-2u) by rcp2_newton.  Where that
// denominator exceeds 2^126 the result is x * 0, as with rcp.approx.ftz.
__device__ __forceinline__ uint32_t gelu_bf16x2_fma(uint32_t w) {
  const float2 x = make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  const float2 x2 = fmul2(x, x);
  const float2 inner = ffma2(fmul2(make_float2(0.044715f, 0.044715f), x), x2, x);
  const float2 u = fmul2(make_float2(0.7978845608028654f, 0.7978845608028654f), inner);
  const float2 e = make_float2(ex2_approx(u.x * -2.8853900817779268f), ex2_approx(u.y * -2.8853900817779268f));
  const float2 d = fadd2(make_float2(1.f, 1.f), e);
  constexpr float kMax = 8.507059173023462e37f;  // 2^126
  float2 r = rcp2_newton(make_float2(fminf(d.x, kMax), fminf(d.y, kMax)));
  r.x = d.x > kMax ? 0.f : r.x;
  r.y = d.y > kMax ? 0.f : r.y;
  const float2 g = fmul2(x, r);
  return pack_bf16x2(g.x, g.y);
}

// Epilogue of one 64-column group of accumulator row et (already in
// registers): y = acc * x_scale * w_scale + bias (f32), optional GELU(tanh)
// of the bf16-rounded value, bf16 into the row's 128-byte line `so` of the
// swizzled staging tile.
template <bool IS_INT8>
__device__ __forceinline__ void epi_convert_group(const uint32_t (&r)[OUT_COLS], const float* sw_g,
                                                  const __nv_bfloat16* bias_g, float2 sx2, int act, int et,
                                                  uint8_t* so) {
#pragma unroll
  for (int c = 0; c < OUT_COLS / 8; ++c) {
    const float* sw = sw_g + c * 8;
    const uint4 bb = *reinterpret_cast<const uint4*>(bias_g + c * 8);
    const uint32_t bw[4] = {bb.x, bb.y, bb.z, bb.w};
    uint32_t pk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t r0 = r[c * 8 + 2 * i], r1 = r[c * 8 + 2 * i + 1];
      const float2 acc = IS_INT8 ? make_float2(static_cast<float>(static_cast<int>(r0)),
                                               static_cast<float>(static_cast<int>(r1)))
                                 : make_float2(__uint_as_float(r0), __uint_as_float(r1));
      const float2 b2 = make_float2(__uint_as_float(bw[i] << 16), __uint_as_float(bw[i] & 0xFFFF0000u));
      const float2 f = ffma2(fmul2(acc, sx2), make_float2(sw[2 * i], sw[2 * i + 1]), b2);
      pk[i] = act == WF_ACT_GELU_TANH ? pack_bf16x2(gelu_tanh(bf16_round(f.x)), gelu_tanh(bf16_round(f.y)))
                                      : pack_bf16x2(f.x, f.y);
    }
    // 128-byte swizzle: 16-byte chunk c of row et lives at chunk c ^ (et & 7)
    *reinterpret_cast<uint4*>(so + ((c ^ (et & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  }
}

// Persistent: CTA c processes output tiles c, c + gridDim.x, ... (tile t ->
// m-tile t % m_tiles, n-tile t / m_tiles, so CTAs running together share the
// same weight tile in L2).  The TMEM accumulator is double buffered: the MMA
// warp fills buffer (i & 1) while the epilogue drains the other one.
template <bool IS_INT8>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_w8a8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const float* __restrict__ x_scale, const float* __restrict__ w_scale,
                     const __nv_bfloat16* __restrict__ bias, const __grid_constant__ CUtensorMap tmY, int M, int N,
                     int K, int per_token, int act) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + NS * A_TILE;
  uint8_t* sOut = sB + NS * B_TILE;                                    // [2][OUT_TILE], 1024-aligned
  float* sSW = reinterpret_cast<float*>(sOut + 2 * OUT_TILE);          // [BN]
  __nv_bfloat16* sBias = reinterpret_cast<__nv_bfloat16*>(sSW + BN);  // [BN]
  int* sOk = reinterpret_cast<int*>(sBias + BN);                       // [4]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOk + 4);
  uint64_t* full = bars;
  uint64_t* empty = bars + NS;
  uint64_t* acc_full = empty + NS;  // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint64_t* fin = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fin + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM;
  const int n_tiles = (N + BN - 1) / BN;
  const int n_total = m_tiles * n_tiles;
  const int nk = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int it = 0;  // global k-block counter across tiles
      int issued = 0;
      for (int t = blockIdx.x; t < n_total && !*abort_flag; t += gridDim.x) {
        const int m0 = (t % m_tiles) * BM, n0 = (t / m_tiles) * BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % NS;
          if (it >= NS && !mbar_wait(&empty[s], ((it / NS) - 1) & 1, abort_flag, ST_GEMM_PRODUCER)) break;
          mbar_arrive_expect_tx(&full[s], A_TILE + B_TILE);
          tma_load_2d(sA + s * A_TILE, &tmA, &full[s], kb * BK, m0);
          tma_load_2d(sB + s * B_TILE, &tmB, &full[s], kb * BK, n0);
          issued = it + 1;
        }
      }
      if (*abort_flag)
        for (int i = (issued > NS ? issued - NS : 0); i < issued; ++i)
          wait_drain(&full[i % NS], (i / NS) & 1, 200000000ull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = IS_INT8 ? make_idesc(2, FMT_S8, FMT_S8, 0, BM, BN)
                                         : make_idesc(1, FMT_E4M3, FMT_E4M3, 0, BM, BN);
      int it = 0, local = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_total; t += gridDim.x, ++local) {
        const int buf = local & 1;
        // the epilogue must have drained this accumulator (tile local-2)
        if (local >= 2 && !mbar_wait(&acc_empty[buf], ((local >> 1) - 1) & 1, abort_flag, ST_GEMM_MMA)) break;
        tc_fence_after();
        const uint32_t d = tbase + buf * BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % NS;
          if (!mbar_wait(&full[s], (it / NS) & 1, abort_flag, ST_GEMM_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(sA + s * A_TILE), b = smem_u32(sB + s * B_TILE);
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const uint64_t da = desc_sw128(a + kk * 32, 16, 1024), db = desc_sw128(b + kk * 32, 16, 1024);
            if constexpr (IS_INT8)
              umma_i8_ss(d, da, db, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            else
              umma_f8_ss(d, da, db, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[buf]);
      }
      umma_commit(fin);
      wait_drain(fin, 0, 200000000ull);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    // Per tile: the four warps agree (through sOk and the named barrier) on
    // whether the accumulator arrived, so either all of them run the tile or
    // none does and no named barrier is left waiting.  Per 64-column group:
    // TMEM -> registers -> scale/bias -> bf16 into staging buffer (grp & 1),
    // then one thread stores the 128 x 64 box with TMA.  Before the barrier
    // that precedes store grp, that thread waits until store grp-1 has read
    // its buffer, so the next group can refill it.
    const int et = threadIdx.x - 128;  // epilogue thread = accumulator row = TMEM lane
    const int wq = warp - 4;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const float sw_t = per_token ? 0.f : __ldg(w_scale);
    const __nv_bfloat16 zero_b = __float2bfloat16_rn(0.f);
    int local = 0, grp = 0;
    for (int t = blockIdx.x; t < n_total; t += gridDim.x, ++local) {
      const int buf = local & 1;
      const bool okw =
          __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (local >> 1) & 1, abort_flag, ST_GEMM_EPILOGUE));
      const int m0 = (t % m_tiles) * BM, n0 = (t / m_tiles) * BN;
      for (int j = et; j < BN; j += 128) {
        const int n = n0 + j < N ? n0 + j : N - 1;
        sSW[j] = per_token ? __ldg(w_scale + n) : sw_t;
        sBias[j] = bias ? bias[n] : zero_b;
      }
      if (lane == 0) sOk[wq] = okw ? 1 : 0;
      named_bar_sync(EPI_BAR, 128);
      if (!(sOk[0] & sOk[1] & sOk[2] & sOk[3])) break;
      tc_fence_after();
      const int row = m0 + et;
      const float sx = (row < M) ? (per_token ? __ldg(x_scale + row) : __ldg(x_scale)) : 0.f;
      const float2 sx2 = make_float2(sx, sx);
#pragma unroll 1
      for (int g = 0; g < BN / OUT_COLS; ++g, ++grp) {
        uint32_t r[OUT_COLS];
        tmem_ld32x32b_x64(tbase + buf * BN + lane_off + g * OUT_COLS, r);
        if (g == BN / OUT_COLS - 1) {
          // every column of this accumulator is in registers: hand it back
          tc_fence_before();
          mbar_arrive(&acc_empty[buf]);
        }
        epi_convert_group<IS_INT8>(r, sSW + g * OUT_COLS, sBias + g * OUT_COLS, sx2, act, et,
                                   sOut + (grp & 1) * OUT_TILE + et * 128);
        fence_proxy_async_smem();
        if (et == 0) bulk_wait_read_all();
        named_bar_sync(EPI_BAR, 128);
        if (et == 0) {
          tma_store_2d(&tmY, sOut + (grp & 1) * OUT_TILE, n0 + g * OUT_COLS, m0);
          bulk_commit_group();
        }
      }
    }
    if (et == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 2 * BN);
  }
}

// ------------------------------------------------------------- CTA pairs
// The same GEMM on 256 x 256 output tiles per CTA pair (cluster of 2,
// tcgen05 cta_group::2).  Each CTA loads 128 rows of A and 128 rows of B (its
// half of the tile's N) per k block into its own shared memory; one thread
// of the even CTA issues M = 256, N = 256 MMAs that read both CTAs' halves
// and accumulate rows [0,128) of the tile in the even CTA's TMEM and rows
// [128,256) in the odd CTA's.  Per SM and k block that is 32 KB from L2
// instead of 48 KB, and six pipeline stages fit where four did.  No load
// multicasts.
//   full[s]      even CTA only: count 1 (its expect_tx of both CTAs' bytes);
//                both CTAs' TMA loads complete their bytes on it
//   empty[s]     each CTA: count 1, the MMA thread's commit after stage s
//   acc_full[b]  each CTA: count 1, commit after the tile's last k block
//   acc_empty[b] even CTA: count 8, one arrival per epilogue warp of each CTA
//   fin          even CTA: every MMA has completed
// Aborts (a timed-out wait) are raised in both CTAs, so the partner's waits
// end too; the CTAs leave together through a cluster barrier.
constexpr int PNS = 6;
constexpr int PA_TILE = BM * BK;  // 16 KB per CTA
constexpr int PB_TILE = 128 * BK;  // 16 KB per CTA (half of the pair's 256 columns)
constexpr int PNBARS = 2 * PNS + 5;
constexpr int PSMEM_BYTES = 1024 + PNS * (PA_TILE + PB_TILE) + 2 * OUT_TILE + BN * 4 + BN * 2 + 16 + PNBARS * 8 + 16;
static_assert(PSMEM_BYTES <= 232448, "pair GEMM shared memory");

template <bool IS_INT8>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_w8a8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const float* __restrict__ x_scale, const float* __restrict__ w_scale,
                          const __nv_bfloat16* __restrict__ bias, const __grid_constant__ CUtensorMap tmY, int M,
                          int N, int K, int per_token, int act, int n_fast) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + PNS * PA_TILE;
  uint8_t* sOut = sB + PNS * PB_TILE;
  float* sSW = reinterpret_cast<float*>(sOut + 2 * OUT_TILE);
  __nv_bfloat16* sBias = reinterpret_cast<__nv_bfloat16*>(sSW + BN);
  int* sOk = reinterpret_cast<int*>(sBias + BN);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOk + 4);
  uint64_t* full = bars;
  uint64_t* empty = bars + PNS;
  uint64_t* acc_full = empty + PNS;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* fin = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fin + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: the CTA whose thread issues the MMAs
  const uint32_t peer = rank ^ 1u;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int m_tiles = (M + 2 * BM - 1) / (2 * BM);
  const int n_tiles = (N + BN - 1) / BN;
  const int n_total = m_tiles * n_tiles;
  const int nk = (K + BK - 1) / BK;
  // the even CTA's full barriers and both CTAs' empty / acc_full barriers, as shared::cluster addresses
  const uint32_t lead_full = mapa_shared(smem_u32(full), 0);
  const uint32_t peer_empty = mapa_shared(smem_u32(empty), peer);
  const uint32_t peer_acc_full = mapa_shared(smem_u32(acc_full), peer);
  const uint32_t lead_acc_empty = mapa_shared(smem_u32(acc_empty), 0);
  const uint32_t peer_abort = mapa_shared(smem_u32(const_cast<int*>(abort_flag)), peer);
  auto raise_abort = [&]() {
    *abort_flag = 1;
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_abort), "r"(1) : "memory");
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < PNS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);
    }
    mbar_init(fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before either signals the other's
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int it = 0;
      for (int t = pair; t < n_total && !*abort_flag; t += npairs) {
        const int mt = n_fast ? t / n_tiles : t % m_tiles, nt = n_fast ? t % n_tiles : t / m_tiles;
        const int m0 = mt * 2 * BM + static_cast<int>(rank) * BM;
        const int n0 = nt * BN + static_cast<int>(rank) * 128;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % PNS;
          if (it >= PNS && !mbar_wait(&empty[s], ((it / PNS) - 1) & 1, abort_flag, ST_GEMM_PRODUCER)) {
            raise_abort();
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * (PA_TILE + PB_TILE));
          tma_load_2d_pair(sA + s * PA_TILE, &tmA, lead_full + 8u * s, kb * BK, m0);
          tma_load_2d_pair(sB + s * PB_TILE, &tmB, lead_full + 8u * s, kb * BK, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = IS_INT8 ? make_idesc(2, FMT_S8, FMT_S8, 0, 2 * BM, BN)
                                         : make_idesc(1, FMT_E4M3, FMT_E4M3, 0, 2 * BM, BN);
      int it = 0, local = 0;
      bool ok = true;
      for (int t = pair; ok && t < n_total; t += npairs, ++local) {
        const int buf = local & 1;
        if (local >= 2 && !mbar_wait(&acc_empty[buf], ((local >> 1) - 1) & 1, abort_flag, ST_GEMM_MMA)) {
          raise_abort();
          break;
        }
        tc_fence_after();
        const uint32_t d = tbase + buf * BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % PNS;
          if (!mbar_wait(&full[s], (it / PNS) & 1, abort_flag, ST_GEMM_MMA)) {
            raise_abort();
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(sA + s * PA_TILE), b = smem_u32(sB + s * PB_TILE);
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const uint64_t da = desc_sw128(a + kk * 32, 16, 1024), db = desc_sw128(b + kk * 32, 16, 1024);
            if constexpr (IS_INT8)
              umma_i8_pair(d, da, db, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            else
              umma_f8_pair(d, da, db, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit_pair(smem_u32(&empty[s]));
          umma_commit_pair(peer_empty + 8u * s);
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&acc_full[buf]));
        umma_commit_pair(peer_acc_full + 8u * buf);
      }
      umma_commit_pair(smem_u32(fin));
      wait_drain(fin, 0, 200000000ull);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // epilogue: rows [m0, m0 + 128) of the pair tile are this CTA's TMEM lanes
    const int et = threadIdx.x - 128;
    const int wq = warp - 4;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const float sw_t = per_token ? 0.f : __ldg(w_scale);
    const __nv_bfloat16 zero_b = __float2bfloat16_rn(0.f);
    int local = 0, grp = 0;
    for (int t = pair; t < n_total; t += npairs, ++local) {
      const int buf = local & 1;
      const bool okw =
          __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (local >> 1) & 1, abort_flag, ST_GEMM_EPILOGUE));
      const int mt = n_fast ? t / n_tiles : t % m_tiles, nt = n_fast ? t % n_tiles : t / m_tiles;
      const int m0 = mt * 2 * BM + static_cast<int>(rank) * BM, n0 = nt * BN;
      for (int j = et; j < BN; j += 128) {
        const int n = n0 + j < N ? n0 + j : N - 1;
        sSW[j] = per_token ? __ldg(w_scale + n) : sw_t;
        sBias[j] = bias ? bias[n] : zero_b;
      }
      if (lane == 0) sOk[wq] = okw ? 1 : 0;
      named_bar_sync(EPI_BAR, 128);
      if (!(sOk[0] & sOk[1] & sOk[2] & sOk[3])) {
        if (et == 0) raise_abort();
        break;
      }
      tc_fence_after();
      const int row = m0 + et;
      const float sx = (row < M) ? (per_token ? __ldg(x_scale + row) : __ldg(x_scale)) : 0.f;
      const float2 sx2 = make_float2(sx, sx);
#pragma unroll 1
      for (int g = 0; g < BN / OUT_COLS; ++g, ++grp) {
        uint32_t r[OUT_COLS];
        tmem_ld32x32b_x64(tbase + buf * BN + lane_off + g * OUT_COLS, r);
        if (g == BN / OUT_COLS - 1) {
          // the whole accumulator row is in registers: one arrival per warp on
          // the even CTA's acc_empty (remote from the odd CTA)
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (rank == 0)
              mbar_arrive(&acc_empty[buf]);
            else
              mbar_arrive_cluster(lead_acc_empty + 8u * buf);
          }
        }
        epi_convert_group<IS_INT8>(r, sSW + g * OUT_COLS, sBias + g * OUT_COLS, sx2, act, et,
                                   sOut + (grp & 1) * OUT_TILE + et * 128);
        fence_proxy_async_smem();
        if (et == 0) bulk_wait_read_all();
        named_bar_sync(EPI_BAR, 128);
        if (et == 0 && m0 < M) {  // the odd CTA's half of the last row tile may lie wholly past M
          tma_store_2d(&tmY, sOut + (grp & 1) * OUT_TILE, n0 + g * OUT_COLS, m0);
          bulk_commit_group();
        }
      }
    }
    if (et == 0) bulk_wait_all();
  }
  // After an abort a CTA's own loads may still be landing in its shared
  // memory (the odd CTA's are counted on the even CTA's barriers): give them
  // a bounded moment before either CTA leaves.
  if (*abort_flag && threadIdx.x == 0) {
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the even CTA's MMAs and the odd CTA's remote arrivals are done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, 2 * BN);
  }
}

// ----------------------------------------------------------- quantisers
__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float warp_max(float m) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  return m;
}

// Per-output-channel weight quantisation, f32 math (fp8.py:32-36 per row).
__global__ void weight_quant_kernel(const __nv_bfloat16* __restrict__ w, uint8_t* __restrict__ wq,
                                    float* __restrict__ w_scale, int64_t N, int64_t K, int is_int8) {
  const int lane = threadIdx.x & 31;
  const int64_t n = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (n >= N) return;
  const __nv_bfloat16* row = w + n * K;
  float m = 0.f;
  for (int64_t k = lane; k < K; k += 32) m = fmaxf(m, fabsf(__bfloat162float(row[k])));
  m = warp_max(m);
  const float qmax = is_int8 ? 127.f : 448.f;
  float s = __fdiv_rn(m, qmax);
  s = s < 1e-8f ? 1e-8f : s;
  for (int64_t k = lane; k < K; k += 32) {
    const float r = __fdiv_rn(__bfloat162float(row[k]), s);
    uint8_t c;
    if (is_int8) {
      const float t = fminf(fmaxf(rintf(r), -127.f), 127.f);
      c = static_cast<uint8_t>(static_cast<int8_t>(t));
    } else {
      uint16_t p;
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(p) : "f"(0.f), "f"(fabsf(r)));
      c = static_cast<uint8_t>((p & 0x7F) | ((__float_as_uint(r) >> 24) & 0x80u));
    }
    wq[n * K + k] = c;
  }
  if (lane == 0) w_scale[n] = s;
}

// Per-token activation quantisation with bf16 scale math (fp8.py:47-48 per
// row): s = max(bf16(amax|x| / qmax), bf16(1e-8)), code = e4m3(bf16(x / s)) or
// clamp(rint(bf16(x / s)), -127, 127).  A warp per row for K <= 3072 (wider
// rows: act_quant_cta_kernel); the row stays in registers for NCH8 > 0
// (K = NCH8 * 256), otherwise it is read twice.  The
// division is one multiply by RN(1/s) (exact for bf16 x and s; see
// quant_rows.cuh); rows with a non-finite scale take the IEEE division.
// GELU: the row is first mapped through bf16(GELU_tanh(x)) -- the FFN's
// activation, quantised for fc_out without its bf16 output ever being stored.
template <bool I8, bool GELU, int NCH8>
__global__ void __launch_bounds__(256)
    act_quant_kernel(const __nv_bfloat16* __restrict__ x, uint8_t* __restrict__ xq, float* __restrict__ x_scale,
                     int64_t M, int64_t K, int64_t xs) {
  using namespace wfk::quant;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t nch = K / 8;
  auto load = [&](const uint4* p) -> uint4 {
    uint4 v = __ldcs(p);
    if constexpr (GELU) v = make_uint4(gelu_bf16x2(v.x), gelu_bf16x2(v.y), gelu_bf16x2(v.z), gelu_bf16x2(v.w));
    return v;
  };
  for (int64_t m = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); m < M; m += nwarps) {
    const uint4* r4 = reinterpret_cast<const uint4*>(x + m * xs);
    uint2* out = reinterpret_cast<uint2*>(xq + m * K);
    uint32_t m2 = 0;
    uint4 buf[NCH8 > 0 ? NCH8 : 1];
    if constexpr (NCH8 > 0) {
#pragma unroll
      for (int i = 0; i < NCH8; ++i) {
        buf[i] = load(r4 + lane + 32 * i);
        m2 = amax8_bits(buf[i], m2);
      }
    } else {
      for (int64_t c = lane; c < nch; c += 32) m2 = amax8_bits(load(r4 + c), m2);
    }
    const RowQuant q = make_rowq(warp_amax_bits(m2), I8 ? 127.f : 448.f);
    auto quant8v = [&](const uint4& v) -> uint2 {
      if (q.finite) {
        if constexpr (I8)
          return make_uint2(i8x2_fast(v.x, q.r) | (i8x2_fast(v.y, q.r) << 16),
                            i8x2_fast(v.z, q.r) | (i8x2_fast(v.w, q.r) << 16));
        else
          return make_uint2(quant4_fast(v.x, v.y, q.r), quant4_fast(v.z, v.w, q.r));
      }
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[2] = {0, 0};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float b0 = bf16_round_f(__fdiv_rn(__uint_as_float(w[i] << 16), q.s));
        const float b1 = bf16_round_f(__fdiv_rn(__uint_as_float(w[i] & 0xFFFF0000u), q.s));
        const uint32_t c = I8 ? (i8_slow(b0) | (i8_slow(b1) << 8)) : (e4m3_encode_sw(b0) | (e4m3_encode_sw(b1) << 8));
        o[i >> 1] |= c << ((i & 1) * 16);
      }
      return make_uint2(o[0], o[1]);
    };
    if constexpr (NCH8 > 0) {
#pragma unroll
      for (int i = 0; i < NCH8; ++i) out[lane + 32 * i] = quant8v(buf[i]);
    } else {
      for (int64_t c = lane; c < nch; c += 32) out[c] = quant8v(load(r4 + c));
    }
    if (lane == 0) x_scale[m] = q.s;
  }
}

// The same quantisation for wide rows (K > 3072: the FFN's 8960 / 13824
// columns, the 14B model's 5120): a CTA per row, CPT 16-byte chunks per
// thread, so the row stays in registers at full occupancy instead of 140
// registers per lane in one warp; the row maximum is reduced through shared
// memory.  With GELU the activation takes one MUFU op per element
// (gelu_bf16x2_fma).  Codes, scales and the non-finite fallback are those of
// act_quant_kernel.
template <bool I8, bool GELU, int CPT>
__global__ void __launch_bounds__(512)
    act_quant_cta_kernel(const __nv_bfloat16* __restrict__ x, uint8_t* __restrict__ xq, float* __restrict__ x_scale,
                         int64_t M, int64_t K, int64_t xs) {
  using namespace wfk::quant;
  __shared__ uint32_t red[16];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
  const int64_t nch = K / 8;
  for (int64_t m = blockIdx.x; m < M; m += gridDim.x) {
    const uint4* r4 = reinterpret_cast<const uint4*>(x + m * xs);
    uint2* out = reinterpret_cast<uint2*>(xq + m * K);
    uint4 buf[CPT];
    uint32_t m2 = 0;
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
      const int64_t c = tid + static_cast<int64_t>(i) * blockDim.x;
      if (c < nch) {
        uint4 v = __ldcs(r4 + c);
        if constexpr (GELU)
          v = make_uint4(gelu_bf16x2_fma(v.x), gelu_bf16x2_fma(v.y), gelu_bf16x2_fma(v.z), gelu_bf16x2_fma(v.w));
        buf[i] = v;
        m2 = amax8_bits(v, m2);
      }
    }
    // f32 amax values are non-negative (NaN above inf), so their bits order as unsigned
    const uint32_t wm = __float_as_uint(warp_amax_bits(m2));
    if (lane == 0) red[wid] = wm;
    __syncthreads();
    uint32_t bm = red[0];
    for (int w = 1; w < nw; ++w) bm = max(bm, red[w]);
    __syncthreads();  // red is rewritten for the next row
    const RowQuant q = make_rowq(__uint_as_float(bm), I8 ? 127.f : 448.f);
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
      const int64_t c = tid + static_cast<int64_t>(i) * blockDim.x;
      if (c >= nch) continue;
      const uint4 v = buf[i];
      if (q.finite) {
        if constexpr (I8)
          out[c] = make_uint2(i8x2_fast(v.x, q.r) | (i8x2_fast(v.y, q.r) << 16),
                              i8x2_fast(v.z, q.r) | (i8x2_fast(v.w, q.r) << 16));
        else
          out[c] = make_uint2(quant4_fast(v.x, v.y, q.r), quant4_fast(v.z, v.w, q.r));
      } else {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[2] = {0, 0};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float b0 = bf16_round_f(__fdiv_rn(__uint_as_float(w[j] << 16), q.s));
          const float b1 = bf16_round_f(__fdiv_rn(__uint_as_float(w[j] & 0xFFFF0000u), q.s));
          const uint32_t cc =
              I8 ? (i8_slow(b0) | (i8_slow(b1) << 8)) : (e4m3_encode_sw(b0) | (e4m3_encode_sw(b1) << 8));
          o[j >> 1] |= cc << ((j & 1) * 16);
        }
        out[c] = make_uint2(o[0], o[1]);
      }
    }
    if (tid == 0) x_scale[m] = q.s;
  }
}

static int make_map_out(CUtensorMap* map, const void* p, int rows, int cols, int64_t row_stride) {
  const uint64_t gdim[2] = {(uint64_t)cols, (uint64_t)rows};
  const uint64_t gstr[1] = {(uint64_t)row_stride * 2};
  const uint32_t box[2] = {(uint32_t)OUT_COLS, (uint32_t)BM};
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p, gdim, gstr, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

static int make_map_2d(CUtensorMap* map, const void* p, int rows, int cols, int box_rows) {
  const uint64_t gdim[2] = {(uint64_t)cols, (uint64_t)rows};
  const uint64_t gstr[1] = {(uint64_t)cols};
  const uint32_t box[2] = {(uint32_t)BK, (uint32_t)box_rows};
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p, gdim, gstr, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace gemm
}  // namespace wfk

using namespace wfk;
using namespace wfk::gemm;

extern "C" int wf_gemm_w8a8_act(const void* xq, const float* x_scale, const void* wq, const float* w_scale,
                                const void* bias, void* y, int M, int N, int K, int64_t y_row_stride, int qtype,
                                int scale_mode, int activation, void* stream) {
  if (activation != WF_ACT_NONE && activation != WF_ACT_GELU_TANH)
    return fail(WF_ERR_INVALID_ARG, "wf_gemm_w8a8_act: activation must be WF_ACT_NONE or WF_ACT_GELU_TANH");
  if (qtype != WF_DTYPE_E4M3 && qtype != WF_DTYPE_S8)
    return fail(WF_ERR_UNSUPPORTED, "wf_gemm_w8a8: qtype must be WF_DTYPE_E4M3 or WF_DTYPE_S8");
  if (scale_mode != WF_SCALE_TENSOR && scale_mode != WF_SCALE_TOKEN)
    return fail(WF_ERR_INVALID_ARG, "wf_gemm_w8a8: scale_mode must be WF_SCALE_TENSOR or WF_SCALE_TOKEN");
  if (M < 1 || N < 16 || K < 16 || N % 16 || K % 16 || M > (1 << 30))
    return fail(WF_ERR_INVALID_ARG, "wf_gemm_w8a8: need M>=1, N and K multiples of 16 (M=%d N=%d K=%d)", M, N, K);
  if (!xq || !wq || !y || !x_scale || !w_scale || !aligned16(xq) || !aligned16(wq) || !aligned16(y) ||
      y_row_stride < N || y_row_stride % 8)
    return fail(WF_ERR_INVALID_ARG, "wf_gemm_w8a8: null/misaligned pointer or bad y stride");
  // CTA pairs (256 x 256 tiles) for M >= 1024 and K >= 4096 (measured at the
  // N=1 tick's M = 28080: 4.5 % faster on fc_out, K = 8960, but 3-4 % slower
  // than one CTA per tile at K = 1536, where a tile has only 12 k blocks);
  // WFK_GEMM_PAIR=0 disables and =1 forces them (M >= 1024) for A/B runs
  static const int pair_env = [] {
    const char* e = std::getenv("WFK_GEMM_PAIR");
    return e ? (e[0] == '0' ? 0 : 1) : -1;
  }();
  const bool use_pair = M >= 1024 && (pair_env == 1 || (pair_env == -1 && K >= 4096));
  CUtensorMap ta, tb, ty;
  int rc;
  if ((rc = make_map_2d(&ta, xq, M, K, BM)) != WF_OK) return rc;
  if ((rc = make_map_2d(&tb, wq, N, K, use_pair ? 128 : BN)) != WF_OK) return rc;
  if ((rc = make_map_out(&ty, y, M, N, y_row_stride)) != WF_OK) return rc;
  static thread_local int configured_dev = -1;
  int dev = 0;
  WFK_CUDA_TRY(cudaGetDevice(&dev));
  if (configured_dev != dev) {
    WFK_CUDA_TRY(cudaFuncSetAttribute(gemm_w8a8_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      SMEM_BYTES));
    WFK_CUDA_TRY(cudaFuncSetAttribute(gemm_w8a8_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      SMEM_BYTES));
    WFK_CUDA_TRY(cudaFuncSetAttribute(gemm_w8a8_pair_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      PSMEM_BYTES));
    WFK_CUDA_TRY(cudaFuncSetAttribute(gemm_w8a8_pair_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      PSMEM_BYTES));
    configured_dev = dev;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int per_token = scale_mode == WF_SCALE_TOKEN;
  if (use_pair) {
    // as many pairs as can be resident at once (a GPC with an odd number of
    // free SMs leaves one idle), queried once per device
    static thread_local int pair_dev = -1, max_pairs = 0;
    if (pair_dev != dev) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(sms);
      cfg.blockDim = dim3(THREADS);
      cfg.dynamicSmemBytes = PSMEM_BYTES;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, gemm_w8a8_pair_kernel<false>, &cfg) != cudaSuccess || n < 1) {
        cudaGetLastError();
        n = sms / 2;
      }
      max_pairs = n < sms / 2 ? n : sms / 2;
      pair_dev = dev;
    }
    const int pair_tiles = ((N + BN - 1) / BN) * ((M + 2 * BM - 1) / (2 * BM));
    const int pairs = pair_tiles < max_pairs ? pair_tiles : max_pairs;
    const dim3 pgrid(2 * pairs);
    // Tile order: m fastest keeps the pairs running together on one weight
    // tile; when the activations exceed half the 126 MB L2 (fc_out at
    // M = 28080: 251 MB), that order re-reads them from DRAM once per column of
    // tiles (1.53 GB at fc_out), so walk n fastest there: each activation tile
    // is then read once and the weights (13.8 MB) stay in L2
    const int n_fast = static_cast<int64_t>(M) * K > (int64_t{64} << 20) ? 1 : 0;
    if (qtype == WF_DTYPE_S8)
      gemm_w8a8_pair_kernel<true><<<pgrid, THREADS, PSMEM_BYTES, s>>>(
          ta, tb, x_scale, w_scale, static_cast<const __nv_bfloat16*>(bias), ty, M, N, K, per_token, activation,
          n_fast);
    else
      gemm_w8a8_pair_kernel<false><<<pgrid, THREADS, PSMEM_BYTES, s>>>(
          ta, tb, x_scale, w_scale, static_cast<const __nv_bfloat16*>(bias), ty, M, N, K, per_token, activation,
          n_fast);
    WFK_CUDA_TRY(cudaGetLastError());
    return WF_OK;
  }
  const int tiles = ((N + BN - 1) / BN) * ((M + BM - 1) / BM);
  const dim3 grid(tiles < sms ? tiles : sms);
  if (qtype == WF_DTYPE_S8)
    gemm_w8a8_kernel<true><<<grid, THREADS, SMEM_BYTES, s>>>(
        ta, tb, x_scale, w_scale, static_cast<const __nv_bfloat16*>(bias), ty, M, N, K, per_token, activation);
  else
    gemm_w8a8_kernel<false><<<grid, THREADS, SMEM_BYTES, s>>>(
        ta, tb, x_scale, w_scale, static_cast<const __nv_bfloat16*>(bias), ty, M, N, K, per_token, activation);
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_gemm_w8a8(const void* xq, const float* x_scale, const void* wq, const float* w_scale,
                            const void* bias, void* y, int M, int N, int K, int64_t y_row_stride, int qtype,
                            int scale_mode, void* stream) {
  return wf_gemm_w8a8_act(xq, x_scale, wq, w_scale, bias, y, M, N, K, y_row_stride, qtype, scale_mode, WF_ACT_NONE,
                          stream);
}

extern "C" int wf_weight_quant(const void* w, void* wq, float* w_scale, int64_t N, int64_t K, int qtype,
                               void* stream) {
  if (!w || !wq || !w_scale || N < 1 || K < 1) return fail(WF_ERR_INVALID_ARG, "wf_weight_quant: bad arguments");
  if (qtype != WF_DTYPE_E4M3 && qtype != WF_DTYPE_S8) return fail(WF_ERR_UNSUPPORTED, "wf_weight_quant: qtype");
  const unsigned blocks = static_cast<unsigned>((N + 7) / 8);
  weight_quant_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(w), static_cast<uint8_t*>(wq), w_scale, N, K, qtype == WF_DTYPE_S8);
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_act_quant_act(const void* x, void* xq, float* x_scale, int64_t M, int64_t K,
                                int64_t x_row_stride, int qtype, int activation, void* stream) {
  if (!x || !xq || !x_scale || M < 0 || K < 8 || K % 8 || x_row_stride < K || x_row_stride % 8 || !aligned16(x) ||
      (reinterpret_cast<uintptr_t>(xq) & 7))
    return fail(WF_ERR_INVALID_ARG, "wf_act_quant: bad arguments");
  if (qtype != WF_DTYPE_E4M3 && qtype != WF_DTYPE_S8) return fail(WF_ERR_UNSUPPORTED, "wf_act_quant: qtype");
  if (activation != WF_ACT_NONE && activation != WF_ACT_GELU_TANH)
    return fail(WF_ERR_INVALID_ARG, "wf_act_quant_act: activation must be WF_ACT_NONE or WF_ACT_GELU_TANH");
  if (M == 0) return WF_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (M + 7) / 8;
  const int64_t cap = static_cast<int64_t>(sms) * 8;
  const unsigned blocks = static_cast<unsigned>(want < cap ? want : cap);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto xb = static_cast<const __nv_bfloat16*>(x);
  auto qb = static_cast<uint8_t*>(xq);
  auto go = [&](auto i8, auto gelu, auto nch) {
    act_quant_kernel<decltype(i8)::value, decltype(gelu)::value, decltype(nch)::value>
        <<<blocks, 256, 0, s>>>(xb, qb, x_scale, M, K, x_row_stride);
  };
  constexpr int kCpt = 5;
  const int64_t nch = K / 8;
  const int64_t cta_threads = ((nch + kCpt - 1) / kCpt + 31) / 32 * 32;
  auto by_k = [&](auto i8, auto gelu) {
    if (K > 3072 && cta_threads <= 512) {
      const unsigned rows = static_cast<unsigned>(M < (int64_t{1} << 31) - 1 ? M : (int64_t{1} << 31) - 1);
      act_quant_cta_kernel<decltype(i8)::value, decltype(gelu)::value, kCpt>
          <<<rows, static_cast<unsigned>(cta_threads), 0, s>>>(xb, qb, x_scale, M, K, x_row_stride);
    } else if (K == 1536)
      go(i8, gelu, std::integral_constant<int, 6>());
    else if (K == 3072)
      go(i8, gelu, std::integral_constant<int, 12>());
    else
      go(i8, gelu, std::integral_constant<int, 0>());
  };
  const bool gelu = activation == WF_ACT_GELU_TANH;
  if (qtype == WF_DTYPE_S8)
    gelu ? by_k(std::true_type(), std::true_type()) : by_k(std::true_type(), std::false_type());
  else
    gelu ? by_k(std::false_type(), std::true_type()) : by_k(std::false_type(), std::false_type());
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" int wf_act_quant(const void* x, void* xq, float* x_scale, int64_t M, int64_t K, int64_t x_row_stride,
                            int qtype, void* stream) {
  return wf_act_quant_act(x, xq, x_scale, M, K, x_row_stride, qtype, WF_ACT_NONE, stream);
}

extern "C" unsigned int wfk_status_take_gemm(void) { return wfk::status_take_local(); }
