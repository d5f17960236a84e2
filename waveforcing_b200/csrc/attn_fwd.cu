// tcgen05/TMEM flash attention forward (bf16, head_dim 128) for the chunk
// self-attention of WaveRT's wavefront step (wave_rt/runtime/backend.py:141-148).
//
// Work item = 128 queries of one head (of one batch entry) against all Lk keys,
// in 256-key tiles.  The grid is persistent: CTA c processes items c,
// c + gridDim.x, ...; the next item's Q and K/V loads and its first QK^T run
// while the previous item's epilogue drains O.
//   warp 0       TMA producer: Q per item; K in 256-key tiles (2-stage ring,
//                one tile ahead of V); V in 128-key halves (one slot per
//                half); 128-byte swizzle, 64-column boxes
//   warp 1       allocates 512 TMEM columns; lane 0 issues the MMAs:
//                S_j  = Q K_j^T  as one M=128, N=256 MMA per 16-wide k step
//                O   += P_j V_j  as M=128, N=128 MMAs (A = P from TMEM,
//                                B = V MN-major), 16 k steps per tile
//   warps 4-7    softmax of keys [0,128) of each tile   (warpgroup 0)
//   warps 8-11   softmax of keys [128,256) of each tile (warpgroup 1)
//                thread t of a warpgroup owns query row t (= TMEM lane t);
//                the two halves of a row agree on the row max through a
//                shared-memory exchange; each warpgroup writes its half of
//                P_j (bf16) to TMEM, rescales its 64 columns of O lazily
//                (only when the running max grows by more than 2^8), and
//                finally normalises and stores its 64 output columns.
// TMEM columns: S [0,256)  P [256,384)  O [384,512).
// S is released as soon as both warpgroups have read it into registers, so
// QK^T of tile j+1 runs on the tensor pipe while P_j is being computed; P is
// written only after PV_{j-1} has completed.
// FP8 K/V (attn_fwd_e4m3_kernel): K and V arrive as e4m3 codes with a scale
// per token row (or one per tensor).  Each code tile lands by TMA in the upper
// half of its operand slot and warps 2-3 expand it in place to f16 products
// f16(e4m3(code) * scale) in the operand layout the bf16 path gets from TMA;
// Q is converted bf16 -> f16 in place once per item and P is written as f16,
// so both MMAs run kind::f16 on f16 operands with the same protocol.
// Barrier phases run on per-CTA counters that continue across items (tiles
// for the S/P/PV/K/V barriers, items for Q/last/o_free).  Every wait is
// bounded (sm100.cuh mbar_wait); a timed-out wait raises the status word and
// the CTA drains its in-flight work and exits.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdlib>
#include <cstring>

#include "host_util.h"
#include "sm100.cuh"

namespace wfk {
namespace attn {

constexpr int BM = 128;          // queries per item
constexpr int BN = 256;          // keys per tile
constexpr int KH = 128;          // keys per softmax warpgroup / per V slot
constexpr int HD = 128;
constexpr int NSK = 2;           // K ring depth (256-key tiles)
constexpr int QTILE = BM * HD * 2;   // 32 KB
constexpr int KTILE = BN * HD * 2;   // 64 KB: [d 0-63: 256 rows x 128 B][d 64-127]
constexpr int KHALF = KTILE / 2;     // 32 KB
constexpr int VSLOT = KH * HD * 2;   // 32 KB: [d 0-63: 128 rows x 128 B][d 64-127]
constexpr int VHALF = VSLOT / 2;     // 16 KB
constexpr int QHALF = QTILE / 2;     // 16 KB
constexpr int BIG = QTILE + NSK * KTILE + 2 * VSLOT;  // 224 KB
constexpr int NBARS = 1 + 2 * NSK + 4 + 9 + (1 + NSK + 2);  // + FP8 arrival barriers (q_raw, raw_k, raw_v)
constexpr int NCONV = 64;                                     // converter threads (warps 2-3), FP8 K/V only
constexpr int SMEM_BYTES = 1024 /*align slack*/ + BIG + NBARS * 8 + 2 * BM * 4 /*row exchange*/ + 16;
constexpr int THREADS = 384;

constexpr uint32_t COL_S = 0, COL_P = 256, COL_O = 384;

__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, uint64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > timeout_ns) {
      status_raise(ST_DRAIN_TIMEOUT);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tmem_st_x1(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t tmem_ld_x1(uint32_t taddr) {
  uint32_t v;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];\n\ttcgen05.wait::ld.sync.aligned;"
               : "=r"(v)
               : "r"(taddr)
               : "memory");
  return v;
}

struct Item {
  int q0, h, bz;
};
__device__ __forceinline__ Item item_of(int it, int n_qt, int H) {
  Item r;
  r.q0 = (it % n_qt) * BM;
  const int rest = it / n_qt;
  r.h = rest % H;
  r.bz = rest / H;
  return r;
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  const __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t cvt_f16x2_e4m3x2(uint32_t two_codes) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(static_cast<uint16_t>(two_codes)));
  return r;
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Row scales of one K tile or V half, fetched before the converters wait for
// the codes so the loads overlap that wait: warp cw converts rows
// [cw * rpw, (cw + 1) * rpw) of the tile, and lane l holds the scales of its
// rows l, l + 32, l + 64 and l + 96 (rows past rpw or past Lk read 0; with
// per-tensor or no scales every slot holds the one value).
template <int NS>
__device__ __forceinline__ void fetch_row_scales(float (&sv)[NS], const float* __restrict__ scale, int mode,
                                                 int bz, int Lk, int key0, int rpw, int cw, int lane) {
#pragma unroll
  for (int c = 0; c < NS; ++c) {
    const int r = c * 32 + lane;
    const int key = key0 + cw * rpw + r;
    float sc = 1.f;
    if (mode == WF_SCALE_TOKEN)
      sc = (r < rpw && key < Lk) ? __ldg(scale + (long long)bz * Lk + key) : 0.f;
    else if (mode == WF_SCALE_TENSOR)
      sc = __ldg(scale);
    sv[c] = sc;
  }
}

// Expands rpw e4m3 rows per converter warp (2 * rpw rows of 128 codes),
// TMA-landed (128-byte swizzle) in the upper half of an operand slot at
// base + half_bytes, into f16 products over both halves [d 0-63 | d 64-127]
// at base, in the layout a 16-bit TMA load of the same tile produces.  Row
// r's codes and the upper half's row r share one 128-byte line: the 8 lanes
// converting a row read all of it before any of them writes (__syncwarp),
// and rows are split between the two warps.  A warp converts 4 rows per
// step and STEPS steps per batch: the batch's loads are issued together and
// one __syncwarp separates all its reads from all its writes.  Scales come
// from the lanes that fetched them (a batch's rows lie in one group of 32,
// so the register index is static).
template <int NS>
__device__ __forceinline__ void convert_rows(uint8_t* base, int half_bytes, int cw, int lane, const float (&sv)[NS]) {
  constexpr int RPW = NS * 32;
  constexpr int STEPS = 2;  // 4 spills under warpgroup 0's 72-register budget
  static_assert(32 % (4 * STEPS) == 0, "a batch must not cross a group of 32 rows");
  const int c = lane & 7;
#pragma unroll
  for (int g = 0; g < NS; ++g) {
#pragma unroll 1
    for (int i0 = 0; i0 < 32; i0 += 4 * STEPS) {
      // 16-byte stores are serviced 8 lanes (one row) at a time.  Lanes
      // c < 4 write their even output chunk first and lanes c >= 4 (the
      // other half, 32 or 16 KB away, so at the same banks) their odd one:
      // each group of 8 stores then covers all 8 bank groups.  The order is
      // chosen on the input words (codes 0-7 make the even chunk, 8-15 the
      // odd one), and the odd chunk is the even one ^ 1 (2k + 1 = 2k ^ 1).
      const int hi = c >> 2;
      uint32_t h[STEPS][8];
#pragma unroll
      for (int t = 0; t < STEPS; ++t) {
        const int rl = g * 32 + i0 + 4 * t + (lane >> 3);  // row within this warp's share
        const int r = cw * RPW + rl;
        const float sc = __shfl_sync(0xffffffffu, sv[g], rl & 31);
        const uint32_t s2 = pack_f16x2(sc, sc);
        const uint4 raw = *reinterpret_cast<const uint4*>(base + half_bytes + r * 128 + ((c ^ (r & 7)) << 4));
        const uint32_t w4[4] = {hi ? raw.z : raw.x, hi ? raw.w : raw.y, hi ? raw.x : raw.z, hi ? raw.y : raw.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          h[t][2 * k] = hmul2(cvt_f16x2_e4m3x2(w4[k] & 0xFFFFu), s2);
          h[t][2 * k + 1] = hmul2(cvt_f16x2_e4m3x2(w4[k] >> 16), s2);
        }
      }
      __syncwarp();
#pragma unroll
      for (int t = 0; t < STEPS; ++t) {
        const int r = cw * RPW + g * 32 + i0 + 4 * t + (lane >> 3);
        uint8_t* row = base + hi * half_bytes + r * 128;
        const int first = ((2 * (c & 3)) ^ (r & 7)) ^ hi;
        *reinterpret_cast<uint4*>(row + (first << 4)) = make_uint4(h[t][0], h[t][1], h[t][2], h[t][3]);
        *reinterpret_cast<uint4*>(row + ((first ^ 1) << 4)) = make_uint4(h[t][4], h[t][5], h[t][6], h[t][7]);
      }
      // the next batch reads other rows' lines, which this batch does not write
    }
  }
}

// bf16 -> f16 in place over `bytes` of shared memory (element order is kept,
// so the swizzled layout is unchanged).
__device__ __forceinline__ void convert_q_f16(uint8_t* base, int bytes, int t) {
  for (int off = t * 16; off < bytes; off += NCONV * 16) {
    uint4 v = *reinterpret_cast<const uint4*>(base + off);
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = pack_f16x2(__uint_as_float(w[k] << 16), __uint_as_float(w[k] & 0xFFFF0000u));
    *reinterpret_cast<uint4*>(base + off) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <bool KV8, bool PX>
__device__ __forceinline__ void attn_body(const CUtensorMap& tmQ, const CUtensorMap& tmK, const CUtensorMap& tmV,
                                          __nv_bfloat16* __restrict__ out, long long o_tok, long long o_head,
                                          long long o_batch, int Lq, int Lk, int H, int n_items, float scale_log2,
                                          const float* __restrict__ k_scale, const float* __restrict__ v_scale,
                                          int scale_mode) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + QTILE;
  uint8_t* sV = sK + NSK * KTILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * VSLOT);
  uint64_t* bar_q = bars;             // Q of the current item landed
  uint64_t* full_k = bars + 1;
  uint64_t* empty_k = full_k + NSK;
  uint64_t* full_v = empty_k + NSK;   // [2], one per 128-key half
  uint64_t* empty_v = full_v + 2;     // [2]
  uint64_t* bar_s = empty_v + 2;      // S_j complete
  uint64_t* bar_sfree = bar_s + 1;    // both warpgroups have read S_j and exchanged the row max
  uint64_t* bar_p = bar_sfree + 1;    // P_j written
  uint64_t* bar_pv = bar_p + 1;       // PV_j complete
  uint64_t* bar_xch = bar_pv + 1;     // row exchange between the warpgroups
  uint64_t* bar_last = bar_xch + 1;   // every PV of the current item has completed
  uint64_t* q_empty = bar_last + 1;   // the current item's last QK^T has completed (Q may be reloaded)
  uint64_t* o_free = q_empty + 1;     // the epilogue has read O (the next item's first PV may overwrite it)
  uint64_t* bar_fin = o_free + 1;
  uint64_t* q_raw = bar_fin + 1;      // FP8 K/V: the bf16 Q tile landed (bar_q: converted to f16)
  uint64_t* raw_k = q_raw + 1;        // [NSK] FP8 K codes landed (full_k: converted)
  uint64_t* raw_v = raw_k + NSK;      // [2]   FP8 V codes landed (full_v: converted)
  float* xch = reinterpret_cast<float*>(raw_v + 2);  // [2][BM]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xch + 2 * BM);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nk = (Lk + BN - 1) / BN;
  const int n_qt = (Lq + BM - 1) / BM;

  if (threadIdx.x == 0) {
    // With FP8 K/V the operand barriers complete on the converters' arrivals
    // instead of TMA transaction bytes.
    const uint32_t operand_arrivals = KV8 ? NCONV : 1;
    mbar_init(bar_q, operand_arrivals);
    for (int s = 0; s < NSK; ++s) {
      mbar_init(&full_k[s], operand_arrivals);
      mbar_init(&empty_k[s], 1);
      mbar_init(&raw_k[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&full_v[s], operand_arrivals);
      mbar_init(&empty_v[s], 1);
      mbar_init(&raw_v[s], 1);
    }
    mbar_init(q_raw, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_sfree, 256);
    mbar_init(bar_p, 256);
    mbar_init(bar_pv, 1);
    mbar_init(bar_xch, 256);
    mbar_init(bar_last, 1);
    mbar_init(q_empty, 1);
    mbar_init(o_free, 256);
    mbar_init(bar_fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  // Register split: 384 threads launch with 168 registers each (64,512).
  // Warpgroup 0 (producer, MMA, two idle warps) drops to 72 and the two
  // softmax warpgroups rise to 216: 128 * 72 + 256 * 216 = 64,512.  The
  // setmaxnreg sits at the top of each warpgroup's branch and the branches
  // never rejoin (each ends with its own copy of the teardown), so no code
  // runs at an ambiguous register count.
  auto teardown = [&]() {
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tbase, 512);
    }
  };
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 72;\n" ::: "memory");
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------ producer
      // Per item: Q (once the previous item's last QK^T has completed), then
      // K_0, and per tile j: K_{j+1}, V_j (both halves).  K runs a tile ahead
      // because QK^T_{j+1} is queued on the tensor pipe before PV_j, and
      // V_j's slots only free up when PV_{j-1} completes.  The counters kt
      // (K tiles) and vt (V tiles) run across items.
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int kt = 0, vt = 0, n_it = 0;
      int q_loads = 0, v_loads[2] = {0, 0};  // loads issued per barrier, for the drain on abort
      bool run = true;
      auto load_k = [&](const Item& w, int j) -> bool {
        const int s = kt % NSK;
        if (kt >= NSK && !mbar_wait(&empty_k[s], ((kt / NSK) - 1) & 1, abort_flag, ST_ATTN_PRODUCER)) return false;
        uint8_t* dst = sK + s * KTILE;
        if constexpr (KV8) {
          // 256 rows of 128 codes into the upper half; the converters expand them
          mbar_arrive_expect_tx(&raw_k[s], BN * 128);
          tma_load_4d(dst + KHALF, &tmK, &raw_k[s], 0, w.h, j * BN, w.bz);
        } else {
          mbar_arrive_expect_tx(&full_k[s], KTILE);
          tma_load_4d(dst, &tmK, &full_k[s], 0, w.h, j * BN, w.bz);
          tma_load_4d(dst + KH * 128, &tmK, &full_k[s], 0, w.h, j * BN + KH, w.bz);
          tma_load_4d(dst + KHALF, &tmK, &full_k[s], 64, w.h, j * BN, w.bz);
          tma_load_4d(dst + KHALF + KH * 128, &tmK, &full_k[s], 64, w.h, j * BN + KH, w.bz);
        }
        ++kt;
        return true;
      };
      for (int it = blockIdx.x; run && it < n_items; it += gridDim.x, ++n_it) {
        const Item w = item_of(it, n_qt, H);
        if (n_it > 0 && !mbar_wait(q_empty, (n_it - 1) & 1, abort_flag, ST_ATTN_PRODUCER)) break;
        uint64_t* qb = KV8 ? q_raw : bar_q;
        mbar_arrive_expect_tx(qb, QTILE);
        tma_load_4d(sQ, &tmQ, qb, 0, w.h, w.q0, w.bz);
        tma_load_4d(sQ + QHALF, &tmQ, qb, 64, w.h, w.q0, w.bz);
        ++q_loads;
        if (!(run = load_k(w, 0))) break;
        for (int j = 0; run && j < nk; ++j) {
          if (j + 1 < nk && !(run = load_k(w, j + 1))) break;
          for (int half = 0; half < 2; ++half) {
            if (vt >= 1 && !mbar_wait(&empty_v[half], (vt - 1) & 1, abort_flag, ST_ATTN_PRODUCER)) {
              run = false;
              break;
            }
            uint8_t* dst = sV + half * VSLOT;
            if constexpr (KV8) {
              mbar_arrive_expect_tx(&raw_v[half], KH * 128);
              tma_load_4d(dst + VHALF, &tmV, &raw_v[half], 0, w.h, j * BN + half * KH, w.bz);
            } else {
              mbar_arrive_expect_tx(&full_v[half], VSLOT);
              tma_load_4d(dst, &tmV, &full_v[half], 0, w.h, j * BN + half * KH, w.bz);
              tma_load_4d(dst + VHALF, &tmV, &full_v[half], 64, w.h, j * BN + half * KH, w.bz);
            }
            ++v_loads[half];
          }
          if (run) ++vt;
        }
      }
      if (*abort_flag) {
        // Let the copies this thread issued land before the CTA exits: the
        // last Q, the last NSK K tiles and the last load of each V half
        // (the phase of load n on a barrier is n & 1).
        // (With FP8 K/V the copies complete on the raw barriers.)
        if (q_loads > 0) mbar_wait_drain(KV8 ? q_raw : bar_q, (q_loads - 1) & 1, 200000000ull);
        for (int t = (kt > NSK ? kt - NSK : 0); t < kt; ++t)
          mbar_wait_drain(KV8 ? &raw_k[t % NSK] : &full_k[t % NSK], (t / NSK) & 1, 200000000ull);
        for (int half = 0; half < 2; ++half)
          if (v_loads[half] > 0)
            mbar_wait_drain(KV8 ? &raw_v[half] : &full_v[half], (v_loads[half] - 1) & 1, 200000000ull);
      }
    } else if (warp == 1 && lane == 0) {
      // ----------------------------------------------------------------- MMA
      constexpr uint32_t OPF = KV8 ? FMT_F16 : FMT_BF16;  // operand type (A and B alike)
      constexpr uint32_t idesc_qk = make_idesc(1, OPF, OPF, 0, BM, BN);
      constexpr uint32_t idesc_pv = make_idesc(1, OPF, OPF, 1, BM, HD);
      const uint32_t aQ = smem_u32(sQ);
      int kt = 0, st = 0, n_it = 0;  // K tiles, S tiles (= PV tiles) issued, items
      bool ok = true;
      for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++n_it) {
        if (!mbar_wait(bar_q, n_it & 1, abort_flag, ST_ATTN_MMA)) break;
        for (int j = 0; ok && j <= nk; ++j) {
          if (j < nk) {
            const int s = kt % NSK;
            if (!mbar_wait(&full_k[s], (kt / NSK) & 1, abort_flag, ST_ATTN_MMA)) {
              ok = false;
              break;
            }
            // S is single-buffered: both warpgroups must have read the previous S tile.
            if (st + j >= 1 && !mbar_wait(bar_sfree, (st + j - 1) & 1, abort_flag, ST_ATTN_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t aK = smem_u32(sK + s * KTILE);
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
              const uint32_t qoff = (kk >> 2) * QHALF + (kk & 3) * 32;
              const uint32_t koff = (kk >> 2) * KHALF + (kk & 3) * 32;
              umma_f16_ss(tbase + COL_S, desc_sw128(aQ + qoff, 16, 1024), desc_sw128(aK + koff, 16, 1024),
                          idesc_qk, kk > 0);
            }
            umma_commit(&empty_k[s]);
            umma_commit(bar_s);
            if (j == nk - 1) umma_commit(q_empty);
            ++kt;
          }
          if (j >= 1) {
            const int g = st + j - 1;  // global index of the PV tile
            if (!mbar_wait(bar_p, g & 1, abort_flag, ST_ATTN_MMA)) {
              ok = false;
              break;
            }
            // The item's first PV overwrites O: the previous item's epilogue must have read it.
            if (j == 1 && n_it > 0 && !mbar_wait(o_free, (n_it - 1) & 1, abort_flag, ST_ATTN_MMA)) {
              ok = false;
              break;
            }
            for (int half = 0; half < 2; ++half) {
              if (!mbar_wait(&full_v[half], g & 1, abort_flag, ST_ATTN_MMA)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t aV = smem_u32(sV + half * VSLOT);
              const uint32_t tP = tbase + COL_P + half * (KH / 2);
#pragma unroll
              for (int kk = 0; kk < KH / 16; ++kk) {
                umma_f16_ts(tbase + COL_O, tP + kk * 8, desc_sw128(aV + kk * 2048, VHALF, 1024), idesc_pv,
                            (j > 1 || half > 0 || kk > 0) ? 1u : 0u);
              }
              umma_commit(&empty_v[half]);
            }
            if (!ok) break;
            umma_commit(bar_pv);
          }
        }
        if (!ok) break;
        st += nk;
        umma_commit(bar_last);
      }
      // Nothing of ours may still be running when TMEM is released.
      umma_commit(bar_fin);
      mbar_wait_drain(bar_fin, 0, 200000000ull);
    } else if (KV8 && (warp == 2 || warp == 3)) {
      // ----------------------------------------------------------- converter
      // The producer's order: per item Q, K_0, then per tile j K_{j+1} and the
      // two halves of V_j.  Each converted tile is made visible to the
      // tensor pipe (fence.proxy.async) before the arrival on its operand
      // barrier.  kt / vt / n_it count like the producer's.
      const int cw = warp - 2;
      const int t = cw * 32 + lane;
      int kt = 0, vt = 0, n_it = 0;
      bool ok = true;
      auto conv_k = [&](const Item& w, int j) -> bool {
        const int s = kt % NSK;
        float sv[BN / 64];  // this lane's 4 of the warp's 128 rows
        fetch_row_scales(sv, k_scale, scale_mode, w.bz, Lk, j * BN, BN / 2, cw, lane);
        if (!__all_sync(0xffffffffu, mbar_wait(&raw_k[s], (kt / NSK) & 1, abort_flag, ST_ATTN_CONVERT)))
          return false;
        convert_rows(sK + s * KTILE, KHALF, cw, lane, sv);
        fence_proxy_async_smem();
        mbar_arrive(&full_k[s]);
        ++kt;
        return true;
      };
      for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++n_it) {
        const Item w = item_of(it, n_qt, H);
        ok = __all_sync(0xffffffffu, mbar_wait(q_raw, n_it & 1, abort_flag, ST_ATTN_CONVERT));
        if (!ok) break;
        convert_q_f16(sQ, QTILE, t);
        fence_proxy_async_smem();
        mbar_arrive(bar_q);
        if (!(ok = conv_k(w, 0))) break;
        for (int j = 0; ok && j < nk; ++j) {
          if (j + 1 < nk && !(ok = conv_k(w, j + 1))) break;
          for (int half = 0; half < 2; ++half) {
            float sv[KH / 64];  // this lane's 2 of the warp's 64 rows
            fetch_row_scales(sv, v_scale, scale_mode, w.bz, Lk, j * BN + half * KH, KH / 2, cw, lane);
            if (!(ok = __all_sync(0xffffffffu,
                                  mbar_wait(&raw_v[half], vt & 1, abort_flag, ST_ATTN_CONVERT))))
              break;
            convert_rows(sV + half * VSLOT, VHALF, cw, lane, sv);
            fence_proxy_async_smem();
            mbar_arrive(&full_v[half]);
          }
          if (ok) ++vt;
        }
      }
    }
    __syncwarp();
    teardown();
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 216;\n" ::: "memory");
    // ------------------------------------------------------------ softmax
    const int wg = (warp - 4) >> 2;  // 0: keys [0,128) of a tile, 1: keys [128,256)
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    float* my_x = xch + wg * BM + row;
    const float* other_x = xch + (wg ^ 1) * BM + row;
    int st = 0, xc = 0, n_it = 0;  // S tiles consumed, row exchanges, items
    bool ok = true;
    for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++n_it) {
      const Item w = item_of(it, n_qt, H);
      float m_run = -INFINITY;
      float l_run = 0.f;
      for (int j = 0; j < nk; ++j, ++st, ++xc) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar_s, st & 1, abort_flag, ST_ATTN_SOFTMAX));
        if (!ok) break;
        tc_fence_after();
        float s[KH];
        {
          uint32_t r[64];
          tmem_ld32x32b_x64(tbase + lane_off + COL_S + wg * KH, r);
#pragma unroll
          for (int i = 0; i < 64; ++i) s[i] = __uint_as_float(r[i]);
          tmem_ld32x32b_x64(tbase + lane_off + COL_S + wg * KH + 64, r);
#pragma unroll
          for (int i = 0; i < 64; ++i) s[64 + i] = __uint_as_float(r[i]);
        }
        const int kvalid = Lk - j * BN - wg * KH;
        if (kvalid < KH) {
#pragma unroll
          for (int i = 0; i < KH; ++i)
            if (i >= kvalid) s[i] = -INFINITY;
        }
        // Row max of the 128 scores as four independent 3-input max chains
        // (chain c takes keys c, c + 4, c + 8, ...) joined at the end: 19
        // dependent steps instead of 127.  (Eight chains spill under the
        // softmax warpgroups' register budget.)
        static_assert(KH == 128, "max chains cover 128 keys");
        float mx;
        {
          constexpr int NC = 4;
          float mc[NC];
#pragma unroll
          for (int c = 0; c < NC; ++c) mc[c] = fmaxf(s[c], s[NC + c]);
#pragma unroll
          for (int i = 2 * NC; i < KH; i += 2 * NC) {
#pragma unroll
            for (int c = 0; c < NC; ++c) mc[c] = fmax3(mc[c], s[i + c], s[i + NC + c]);
          }
          mx = fmaxf(fmax3(mc[0], mc[1], mc[2]), mc[3]);
        }
        // Row max across the two halves.  The exchange slot is reused every
        // tile: the next S tile (and with it this thread's next write) waits on
        // bar_sfree, which every thread passes only after its read below.
        *my_x = mx;
        mbar_arrive(bar_xch);
        ok = __all_sync(0xffffffffu, mbar_wait(bar_xch, xc & 1, abort_flag, ST_ATTN_SOFTMAX));
        if (!ok) break;
        mx = fmaxf(mx, *other_x);
        tc_fence_before();
        mbar_arrive(bar_sfree);
        const float mx2 = mx * scale_log2;
        float m_new = m_run;
        bool grow = false;
        if (j == 0) {
          m_new = mx2;
        } else if (mx2 > m_run + 8.f) {
          m_new = mx2;
          grow = true;
        }
        const float2 sc2 = make_float2(scale_log2, scale_log2);
        const float2 nm2 = make_float2(-m_new, -m_new);
        // four partial row sums, so the additions do not form one 64-long chain
        constexpr int NSUM = 4;
        float2 sum_a = make_float2(0.f, 0.f), sum_b = sum_a, sum_c = sum_a, sum_d = sum_a;
        auto add_sum = [&](int i, float2 pr) {
          if (NSUM == 1 || (i & 3) == 0)
            sum_a = fadd2(sum_a, pr);
          else if ((i & 3) == 1)
            sum_b = fadd2(sum_b, pr);
          else if ((i & 3) == 2)
            sum_c = fadd2(sum_c, pr);
          else
            sum_d = fadd2(sum_d, pr);
        };
        uint32_t pk[KH / 2];
        if constexpr (PX) {
          // P = 2^(s * scale_log2 - m) on MUFU's packed 16-bit path: the
          // exponent pair is rounded to the MMA's P type (bf16, or f16 for
          // FP8 K/V) and one ex2 gives both P values in that type.  The row
          // sum adds exactly the P the MMA multiplies.
#pragma unroll
          for (int i = 0; i < KH / 2; ++i) {
            const float2 x = ffma2(make_float2(s[2 * i], s[2 * i + 1]), sc2, nm2);
            uint32_t p;
            float2 pr;
            if constexpr (KV8) {
              asm("ex2.approx.f16x2 %0, %1;" : "=r"(p) : "r"(pack_f16x2(x.x, x.y)));
              const __half2 h = *reinterpret_cast<const __half2*>(&p);
              pr = __half22float2(h);
            } else {
              asm("ex2.approx.ftz.bf16x2 %0, %1;" : "=r"(p) : "r"(pack_bf16x2(x.x, x.y)));
              pr = make_float2(__uint_as_float(p << 16), __uint_as_float(p & 0xFFFF0000u));
            }
            add_sum(i, pr);
            pk[i] = p;
          }
        } else {
          // P = 2^(s * scale_log2 - m): pairs through packed f32x2 FMAs; 3 of
          // every 8 pairs take the FMA-pipe polynomial, the rest MUFU ex2, so
          // the two pipes finish together.
#pragma unroll
          for (int i = 0; i < KH / 2; ++i) {
            const float2 x = ffma2(make_float2(s[2 * i], s[2 * i + 1]), sc2, nm2);
            float2 pr;
            if ((i & 7) < 3) {
              pr = exp2_poly2(x);
            } else {
              pr.x = ex2_approx(x.x);
              pr.y = ex2_approx(x.y);
            }
            add_sum(i, pr);
            pk[i] = KV8 ? pack_f16x2(pr.x, pr.y) : pack_bf16x2(pr.x, pr.y);
          }
        }
        float2 sumv = sum_a;
        if constexpr (NSUM == 4) sumv = fadd2(fadd2(sum_a, sum_b), fadd2(sum_c, sum_d));
        const float sum = sumv.x + sumv.y;
        const float alpha = grow ? ex2_approx(m_run - m_new) : 1.f;
        // P and O may only be written once PV_{j-1} has completed.  This
        // parity wait is unambiguous: S_j's commit (one issuing thread, in
        // order) already covered PV_{j-2}, and PV_j needs this thread's
        // arrival.  For j == 0 the previous item's epilogue already waited on
        // bar_last, which covers its last PV.
        if (j > 0) {
          ok = __all_sync(0xffffffffu, mbar_wait(bar_pv, (st - 1) & 1, abort_flag, ST_ATTN_SOFTMAX));
          if (!ok) break;
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
          for (int c = 0; c < HD / 2; c += 32) {
            uint32_t r[32];
            tmem_ld32x32b_x32(tbase + lane_off + COL_O + wg * (HD / 2) + c, r);
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32x32b_x32(tbase + lane_off + COL_O + wg * (HD / 2) + c, r);
          }
        }
        l_run = l_run * alpha + sum;
        m_run = m_new;
        tmem_st32x32b_x64(tbase + lane_off + COL_P + wg * (KH / 2), pk);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(bar_p);
      }
      if (!ok) break;
      ok = __all_sync(0xffffffffu, mbar_wait(bar_last, n_it & 1, abort_flag, ST_ATTN_SOFTMAX));
      if (!ok) break;
      tc_fence_after();
      // Row sum across the two halves, through TMEM: each warpgroup writes its
      // partial sum into the first column of its own P half (P is free: every
      // PV of this item has completed) and reads the other's after the
      // exchange barrier.  The next item's P writes come after the next row
      // max exchange, which the partner reaches only after this read.
      tmem_st_x1(tbase + lane_off + COL_P + wg * (KH / 2), __float_as_uint(l_run));
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar_xch);
      ok = __all_sync(0xffffffffu, mbar_wait(bar_xch, xc & 1, abort_flag, ST_ATTN_SOFTMAX));
      ++xc;
      if (!ok) break;
      tc_fence_after();
      const float l_other = __uint_as_float(tmem_ld_x1(tbase + lane_off + COL_P + (wg ^ 1) * (KH / 2)));
      const float inv_l = 1.f / (l_run + l_other);
      const int qrow = w.q0 + row;
      __nv_bfloat16* dst =
          out + (long long)w.bz * o_batch + (long long)qrow * o_tok + (long long)w.h * o_head + wg * (HD / 2);
#pragma unroll
      for (int c = 0; c < HD / 2; c += 32) {
        uint32_t r[32];
        tmem_ld32x32b_x32(tbase + lane_off + COL_O + wg * (HD / 2) + c, r);
        if (qrow < Lq) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 wv;
            wv.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]) * inv_l, __uint_as_float(r[8 * v + 1]) * inv_l);
            wv.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv_l, __uint_as_float(r[8 * v + 3]) * inv_l);
            wv.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv_l, __uint_as_float(r[8 * v + 5]) * inv_l);
            wv.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv_l, __uint_as_float(r[8 * v + 7]) * inv_l);
            d4[v] = wv;
          }
        }
      }
      // O is in registers (tcgen05.ld waits for completion): the next item's
      // first PV may overwrite it.
      tc_fence_before();
      mbar_arrive(o_free);
    }
    teardown();
  }
}

#define WFK_ATTN_KERNELS(NAME, KV8, PX)                                                                       \
  __global__ void __launch_bounds__(THREADS, 1)                                                               \
      NAME(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,                  \
           const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ out, long long o_tok,         \
           long long o_head, long long o_batch, int Lq, int Lk, int H, int n_items, float scale_log2,         \
           const float* __restrict__ k_scale, const float* __restrict__ v_scale, int scale_mode) {           \
    attn_body<KV8, PX>(tmQ, tmK, tmV, out, o_tok, o_head, o_batch, Lq, Lk, H, n_items, scale_log2, k_scale,  \
                       v_scale, scale_mode);                                                                 \
  }

// bf16 K/V (scales unused) and e4m3 K/V codes [batch, Lk, H, 128] with
// per-token (k_scale[bz * Lk + key]), per-tensor (k_scale[0]) or no scales;
// the _px forms take the exponentials on MUFU's packed 16-bit path.
WFK_ATTN_KERNELS(attn_fwd_bf16_kernel, false, false)
WFK_ATTN_KERNELS(attn_fwd_bf16_px_kernel, false, true)
WFK_ATTN_KERNELS(attn_fwd_e4m3_kernel, true, false)
WFK_ATTN_KERNELS(attn_fwd_e4m3_px_kernel, true, true)
#undef WFK_ATTN_KERNELS

// Tensor map over a [batch, L, H, 128] bf16 tensor with {batch, token, head}
// element strides; box = 64 head-dim columns x 1 head x 128 tokens.
static int make_qkv_map(CUtensorMap* m, const void* p, int batch, int L, int H, const int64_t* st) {
  const uint64_t gdim[4] = {(uint64_t)HD, (uint64_t)H, (uint64_t)L, (uint64_t)batch};
  const uint64_t gstr[3] = {(uint64_t)st[2] * 2, (uint64_t)st[1] * 2,
                            (uint64_t)(batch > 1 ? st[0] : st[1] * (int64_t)L) * 2};
  const uint32_t box[4] = {64, 1, 128, 1};
  return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, p, gdim, gstr, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Tensor map over [batch, L, H, 128] e4m3 codes (one byte per element) with
// {batch, token, head} strides in bytes; box = 128 codes x 1 head x `rows`
// tokens (one 128-byte swizzled line per token).
static int make_code_map(CUtensorMap* m, const void* p, int batch, int L, int H, const int64_t* st, int rows) {
  const uint64_t gdim[4] = {(uint64_t)HD, (uint64_t)H, (uint64_t)L, (uint64_t)batch};
  const uint64_t gstr[3] = {(uint64_t)st[2], (uint64_t)st[1], (uint64_t)(batch > 1 ? st[0] : st[1] * (int64_t)L)};
  const uint32_t box[4] = {128, 1, (uint32_t)rows, 1};
  return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, p, gdim, gstr, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

static bool strides_ok(const int64_t* st, int batch) {
  if (st == nullptr) return false;
  for (int i = 0; i < 3; ++i)
    if (st[i] < 0 || (st[i] % 8) != 0) return false;
  if (batch > 1 && st[0] == 0) return false;
  return st[1] > 0 && st[2] > 0;
}

}  // namespace attn
}  // namespace wfk

extern "C" int wf_attn_fwd(const void* q, const void* k, const void* v, void* o, int batch, int Lq, int Lk, int H,
                           int D, const int64_t* q_stride, const int64_t* k_stride, const int64_t* v_stride,
                           const int64_t* o_stride, int kv_dtype, const float* k_scale, const float* v_scale,
                           int scale_mode, float softmax_scale, void* stream) {
  using namespace wfk;
  using namespace wfk::attn;
  if (D != HD) return fail(WF_ERR_UNSUPPORTED, "wf_attn_fwd: head_dim %d unsupported (only 128)", D);
  const bool kv8 = kv_dtype == WF_DTYPE_E4M3;
  if (kv_dtype != WF_DTYPE_BF16 && !kv8)
    return fail(WF_ERR_UNSUPPORTED, "wf_attn_fwd: kv_dtype %d unsupported (bf16 or e4m3)", kv_dtype);
  if (!kv8 && (k_scale != nullptr || v_scale != nullptr || scale_mode != WF_SCALE_NONE))
    return fail(WF_ERR_INVALID_ARG, "wf_attn_fwd: bf16 K/V take no scales (k_scale/v_scale NULL, WF_SCALE_NONE)");
  if (kv8 && scale_mode != WF_SCALE_NONE && scale_mode != WF_SCALE_TENSOR && scale_mode != WF_SCALE_TOKEN)
    return fail(WF_ERR_INVALID_ARG, "wf_attn_fwd: unknown scale_mode %d", scale_mode);
  if (kv8 && scale_mode != WF_SCALE_NONE && (!k_scale || !v_scale))
    return fail(WF_ERR_INVALID_ARG, "wf_attn_fwd: e4m3 K/V with scales need k_scale and v_scale");
  if (batch < 1 || Lq < 1 || Lk < 1 || H < 1 || H > 65535 || batch > 65535)
    return fail(WF_ERR_INVALID_ARG, "wf_attn_fwd: bad sizes batch=%d Lq=%d Lk=%d H=%d", batch, Lq, Lk, H);
  if (!q || !k || !v || !o) return fail(WF_ERR_INVALID_ARG, "wf_attn_fwd: null tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return fail(WF_ERR_INVALID_ARG, "wf_attn_fwd: tensors must be 16-byte aligned");
  if (!strides_ok(q_stride, batch) || !strides_ok(k_stride, batch) || !strides_ok(v_stride, batch) ||
      !strides_ok(o_stride, batch))
    return fail(WF_ERR_INVALID_ARG, "wf_attn_fwd: strides must be positive multiples of 8 elements");
  if (kv8)
    for (int i = 0; i < 3; ++i)
      if (k_stride[i] % 16 || v_stride[i] % 16)
        return fail(WF_ERR_INVALID_ARG, "wf_attn_fwd: e4m3 K/V strides must be multiples of 16 bytes");
  if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale))
    return fail(WF_ERR_INVALID_ARG, "wf_attn_fwd: softmax_scale must be positive");

  CUtensorMap tq, tk, tv;
  int rc;
  if ((rc = make_qkv_map(&tq, q, batch, Lq, H, q_stride)) != WF_OK) return rc;
  if (kv8) {
    if ((rc = make_code_map(&tk, k, batch, Lk, H, k_stride, BN)) != WF_OK) return rc;
    if ((rc = make_code_map(&tv, v, batch, Lk, H, v_stride, KH)) != WF_OK) return rc;
  } else {
    if ((rc = make_qkv_map(&tk, k, batch, Lk, H, k_stride)) != WF_OK) return rc;
    if ((rc = make_qkv_map(&tv, v, batch, Lk, H, v_stride)) != WF_OK) return rc;
  }

  static thread_local int configured_dev = -1;
  int dev = 0;
  WFK_CUDA_TRY(cudaGetDevice(&dev));
  if (configured_dev != dev) {
    for (auto fn : {attn_fwd_bf16_kernel, attn_fwd_bf16_px_kernel, attn_fwd_e4m3_kernel, attn_fwd_e4m3_px_kernel})
      WFK_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    configured_dev = dev;
  }
  const long long items = (long long)((Lq + BM - 1) / BM) * H * batch;
  if (items > (1LL << 30)) return fail(WF_ERR_INVALID_ARG, "wf_attn_fwd: too many query tiles (%lld)", items);
  static thread_local int sms = 0, sms_dev = -1;
  if (sms_dev != dev) {
    WFK_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    sms_dev = dev;
  }
  // Persistent grid: at most one CTA per SM; with more items than SMs each
  // CTA walks items blockIdx.x, blockIdx.x + gridDim.x, ...  When items do
  // not fill whole waves, the grid is the smallest count that keeps every
  // CTA's item count within one of the others'.
  long long grid = items < sms ? items : sms;
  if (items > sms) {
    const long long per = (items + sms - 1) / sms;
    grid = (items + per - 1) / per;
  }
  const float scale_log2 = softmax_scale * 1.4426950408889634f;
  // Exponential path: WFK_ATTN_EXP=packed selects MUFU's packed 16-bit ex2,
  // =split the f32 MUFU / FMA-polynomial split (read once per process).
  static const bool packed_exp = [] {
    const char* e = std::getenv("WFK_ATTN_EXP");
    return e != nullptr && std::strcmp(e, "packed") == 0;
  }();
  auto kern = kv8 ? (packed_exp ? attn_fwd_e4m3_px_kernel : attn_fwd_e4m3_kernel)
                  : (packed_exp ? attn_fwd_bf16_px_kernel : attn_fwd_bf16_kernel);
  kern<<<(unsigned)grid, THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(
      tq, tk, tv, static_cast<__nv_bfloat16*>(o), (long long)o_stride[1], (long long)o_stride[2],
      (long long)o_stride[0], Lq, Lk, H, (int)items, scale_log2, kv8 ? k_scale : nullptr, kv8 ? v_scale : nullptr,
      kv8 ? scale_mode : WF_SCALE_NONE);
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

namespace wfk {
namespace attn {
__global__ void exp2_selftest_kernel(const float* __restrict__ x, float* __restrict__ y_poly,
                                     float* __restrict__ y_mufu, int n) {
  const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (i + 1 >= n + 1) return;
  const float2 in = make_float2(x[i], i + 1 < n ? x[i + 1] : 0.f);
  const float2 p = exp2_poly2(in);
  y_poly[i] = p.x;
  y_mufu[i] = ex2_approx(in.x);
  if (i + 1 < n) {
    y_poly[i + 1] = p.y;
    y_mufu[i + 1] = ex2_approx(in.y);
  }
}
}  // namespace attn
}  // namespace wfk

extern "C" int wf_selftest_exp2(const float* x, float* y_poly, float* y_mufu, int n, void* stream) {
  if (!x || !y_poly || !y_mufu || n < 0) return wfk::fail(WF_ERR_INVALID_ARG, "wf_selftest_exp2: bad arguments");
  if (n == 0) return WF_OK;
  const int pairs = (n + 1) / 2;
  wfk::attn::exp2_selftest_kernel<<<(pairs + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y_poly,
                                                                                                      y_mufu, n);
  WFK_CUDA_TRY(cudaGetLastError());
  return WF_OK;
}

extern "C" unsigned int wfk_status_take_attn(void) { return wfk::status_take_local(); }
