/*
 * wfk.h -- C ABI of libwfk.so, the B200 (sm_100a) implementation of WaveRT's
 * per-layer DiT hot path.
 *
 * Conventions (all entry points):
 *   - plain pointers and sizes only; device pointers are device addresses of
 *     the current CUDA device, `stream` is a cudaStream_t passed as void*;
 *   - every call is stream-ordered and returns 0 (WF_OK) or a WF_ERR_* code;
 *     wf_last_error() gives the calling thread's message for the last
 *     failure (the Python shim raises RuntimeError with it, the convention of
 *     wave_rt/distributed/ipc.py:28-37);
 *   - no entry point allocates device memory unless its comment says so; the
 *     caller owns every buffer;
 *   - strides are in elements, the innermost dimension is contiguous.
 *
 * Reference interfaces are cited as path:line inside SJTU-DENG-Lab/WaveForcing.
 */
#ifndef WFK_H_
#define WFK_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WF_OK 0
#define WF_ERR_INVALID_ARG 1
#define WF_ERR_UNSUPPORTED 2
#define WF_ERR_CUDA 3
#define WF_ERR_TIMEOUT 4

#define WF_DTYPE_BF16 0
#define WF_DTYPE_E4M3 1
#define WF_DTYPE_S8 2

#define WF_SCALE_NONE 0
#define WF_SCALE_TENSOR 1
#define WF_SCALE_TOKEN 2

#define WF_ACT_NONE 0
#define WF_ACT_GELU_TANH 1

/* ------------------------------------------------------------ library */

/* Message of the last failed call on this host thread ("" if none). */
const char* wf_last_error(void);

/* ABI version (incremented on any signature change). */
int wf_version(void);

/* Reads and clears the device status word of the current device (bitmask of
 * bounded waits that gave up; 0 = healthy).  Synchronises the device. */
unsigned int wf_status_take(void);

/* ---------------------------------------------------------- attention */

/* O = softmax(Q K^T * softmax_scale) V, non-causal, NHD layout, D = 128.
 * Replaces the attention call of the patched self-attention,
 * wave_rt/runtime/backend.py:141-148 (SGLang torch_sdpa / flash_attn_func /
 * sageattn on (roped_query, ctx_k, ctx_v)); block causality is given by which
 * chunks the caller places in K/V (wave_rt/denoiser/exchange/paged.py:247-248).
 * Shapes: q/o [batch, Lq, H, D], k/v [batch, Lk, H, D]; strides are
 * {batch, token, head} in elements.  Requires 16-byte aligned base pointers
 * and strides that are multiples of 8.
 *   kv_dtype WF_DTYPE_BF16: k/v bf16; k_scale/v_scale NULL, WF_SCALE_NONE.
 *   kv_dtype WF_DTYPE_E4M3: k/v are e4m3 codes (one byte per element, strides
 *   multiples of 16), as the FP8 transport carries them; scale_mode
 *   WF_SCALE_TOKEN reads one f32 scale per token row, k_scale[b * Lk + key]
 *   (the per-token codec, over all heads of the row), WF_SCALE_TENSOR reads
 *   k_scale[0] (common.py:143-164), WF_SCALE_NONE uses the codes as values
 *   (onesided.py:151-153).  The kernel expands each TMA-loaded code tile in
 *   shared memory to f16 products f16(e4m3(code) * scale) and runs both
 *   contractions on f16 operands (q converted from bf16, P written as f16),
 *   so |q| and |code * scale| must stay below 65504. */
int wf_attn_fwd(const void* q, const void* k, const void* v, void* o, int batch, int Lq, int Lk, int H, int D,
                const int64_t* q_stride, const int64_t* k_stride, const int64_t* v_stride,
                const int64_t* o_stride, int kv_dtype, const float* k_scale, const float* v_scale,
                int scale_mode, float softmax_scale, void* stream);

/* Diagnostic (no counterpart in the reference): evaluates the attention
 * softmax's two exponential paths on x[n] -- the FMA-pipe polynomial
 * (y_poly) and the MUFU ex2.approx (y_mufu) -- so their error bounds can be
 * tested against exp2. */
int wf_selftest_exp2(const float* x, float* y_poly, float* y_mufu, int n, void* stream);

/* ------------------------------------------------------- FP8 K/V codec */

/* Quantise a bf16 [rows, cols] matrix (row stride x_row_stride) to e4m3fn
 * codes [rows, cols] (dense) with the reference's dtype sequence
 *   s = f32(clamp(bf16(amax|x| / 448), 1e-8)); code = e4m3(bf16(x / s))
 * wave_rt/denoiser/exchange/common.py:143-150 (per-tensor, mode
 * WF_SCALE_TENSOR: one scale in scales[0]) or the same sequence per row
 * (mode WF_SCALE_TOKEN: scales[rows]).  Per-tensor mode needs a grid-wide
 * amax and uses `workspace` (>= 4 bytes of device memory, caller-owned,
 * overwritten); per-token mode ignores it.  Mode WF_SCALE_NONE is the
 * scale-free cast of the onesided exchange, code = e4m3fn(x)
 * (wave_rt/denoiser/exchange/onesided.py:151-153); scales may be NULL. */
int wf_kv_quant(const void* x, uint8_t* codes, float* scales, int64_t rows, int64_t cols, int64_t x_row_stride,
                int mode, void* workspace, void* stream);

/* Allocation-free form of wf_kv_quant(..., WF_SCALE_TENSOR, ...).  It has no
 * counterpart in the reference.  It exists for callers that cannot allocate
 * device memory where they quantise: hosts reaching this library through a C
 * FFI with no CUDA allocator of their own, processes whose device memory is
 * already reserved by a framework's caching allocator (a raw cudaMalloc can
 * fail there), and per-layer loops that must not pay cudaMalloc's implicit
 * synchronisation.  Its grid-wide amax scratch is a fixed 16 KB device array
 * inside libwfk (4096 partial maxima), which every GPU that loads the library
 * holds until the process exits; it calls no cudaMalloc, cudaFree or
 * allocating library routine.  Limit: rows * cols <= 33,554,432 elements
 * (4096 x 8192); larger inputs are rejected with WF_ERR_INVALID_ARG.  The first
 * call on a device resolves the array's device address (cudaGetSymbolAddress
 * with that device current); make that first call before any stream capture.
 * The address is cached per device and context: the first call in a new
 * context (after cudaDeviceReset, for example) resolves it again.
 * All calls on a device share the array: calls whose kernels overlap on the
 * GPU race.  Codes and scale are bit-identical to wf_kv_quant's. */
int wf_kv_quant_tensor_static(const void* x, uint8_t* codes, float* scale, int64_t rows, int64_t cols,
                              int64_t x_row_stride, void* stream);

/* Dequantise codes [rows, cols] to bf16 out (row stride out_row_stride):
 * out = bf16(e4m3(code) * scale), the receive side of
 * wave_rt/denoiser/exchange/common.py:162 and onesided.py:177-179
 * (mode WF_SCALE_NONE: scale-free cast back, scales ignored). */
int wf_kv_dequant(const uint8_t* codes, const float* scales, void* out, int64_t rows, int64_t cols,
                  int64_t out_row_stride, int mode, void* stream);

/* Per-token quantise K and V of one layer and write codes + scales straight
 * into n_dst destination slots (local or peer device memory), the FP8 form of
 * the layer-wise publish wave_rt/denoiser/exchange/paged.py:120-145.
 * k, v: bf16 [rows, cols] with row strides; dst_codes_k[i]/dst_codes_v[i]:
 * [rows, cols] u8; dst_scales_k[i]/dst_scales_v[i]: [rows] f32. */
int wf_kv_quant_publish(const void* k, const void* v, int64_t rows, int64_t cols, int64_t k_row_stride,
                        int64_t v_row_stride, uint8_t* const* dst_codes_k, uint8_t* const* dst_codes_v,
                        float* const* dst_scales_k, float* const* dst_scales_v, int n_dst, void* stream);

/* ------------------------------------------------------------- W8A8 */

/* Per-output-channel weight quantisation (load time), the per-channel form of
 * wave_rt/runtime/fp8.py:32-36: s[n] = clamp(amax|w[n,:]| / Q, 1e-8) in f32,
 * q = e4m3(w / s) (qtype WF_DTYPE_E4M3, Q = 448) or rne-int8 clamp(+-127)
 * (WF_DTYPE_S8, Q = 127).  w: bf16 [N, K]. */
int wf_weight_quant(const void* w, void* wq, float* w_scale, int64_t N, int64_t K, int qtype, void* stream);

/* Per-token dynamic activation quantisation, the per-row form of
 * wave_rt/runtime/fp8.py:47-48 (bf16 scale math).  x: bf16 [M, K] with row
 * stride x_row_stride -> xq [M, K] dense, x_scale [M]. */
int wf_act_quant(const void* x, void* xq, float* x_scale, int64_t M, int64_t K, int64_t x_row_stride, int qtype,
                 void* stream);

/* wf_act_quant of bf16(activation(x)): WF_ACT_GELU_TANH maps each element
 * through the FFN's GELU(approximate="tanh") first, so fc_out's input
 * quantisation reads fc_in's bf16 output once and the activation's bf16
 * tensor is never written (the Wan FFN, causal_model.py:309-420).
 * WF_ACT_NONE is wf_act_quant. */
int wf_act_quant_act(const void* x, void* xq, float* x_scale, int64_t M, int64_t K, int64_t x_row_stride, int qtype,
                     int activation, void* stream);

/* y[M, N] (bf16, row stride y_row_stride) = (xq[M, K] . wq[N, K]^T) * x_scale[m] * w_scale[n] + bias[n]
 * on tcgen05 (kind::f8f6f4 for e4m3, kind::i8 for s8), replacing the
 * torch._scaled_mm call of wave_rt/runtime/fp8.py:49-56.  scale_mode
 * WF_SCALE_TENSOR reads x_scale[0] and w_scale[0] (the reference's
 * per-tensor form), WF_SCALE_TOKEN reads x_scale[M] and w_scale[N].
 * bias may be NULL.  K must be a multiple of 128 and N of 16. */
int wf_gemm_w8a8(const void* xq, const float* x_scale, const void* wq, const float* w_scale, const void* bias,
                 void* y, int M, int N, int K, int64_t y_row_stride, int qtype, int scale_mode, void* stream);

/* wf_gemm_w8a8 with an activation applied to the bf16-rounded output in the
 * epilogue.  WF_ACT_GELU_TANH is the FFN's GELU(approximate="tanh") after
 * fc_in (the Wan block FFN, causal_model.py:309-420): fc_in and the GELU of the
 * reference become one call.  WF_ACT_NONE is wf_gemm_w8a8. */
int wf_gemm_w8a8_act(const void* xq, const float* x_scale, const void* wq, const float* w_scale, const void* bias,
                     void* y, int M, int N, int K, int64_t y_row_stride, int qtype, int scale_mode, int activation,
                     void* stream);

/* ------------------------------------------------------ context assembly */

#define WF_SEG_COPY 0    /* bf16 rows copied */
#define WF_SEG_ROPE 1    /* bf16 rows rotated by per-row f32 cos/sin [rows, head_dim/2] (interleaved pairs) */
#define WF_SEG_DEQUANT 2 /* e4m3 codes with per-row f32 scales -> bf16(e4m3(code) * scale) */

/* One source of rows of a K or V context buffer. */
typedef struct wf_kv_segment {
  int32_t kind;           /* WF_SEG_* */
  int32_t reserved;       /* 0 */
  const void* src;        /* bf16 rows (COPY, ROPE) or u8 codes (DEQUANT); 16-byte aligned (8 for codes) */
  const float* aux0;      /* ROPE: cos table [rows, head_dim/2]; DEQUANT: scales [rows]; COPY: NULL */
  const float* aux1;      /* ROPE: sin table [rows, head_dim/2]; else NULL */
  void* dst;              /* bf16 rows, 16-byte aligned */
  int64_t rows;
  int64_t src_row_stride; /* elements of the source type (bf16 or bytes), >= cols, multiple of 8 */
  int64_t dst_row_stride; /* bf16 elements, >= cols, multiple of 8 */
} wf_kv_segment;

/* Assembles the paged exchange's K/V context of one layer in one launch:
 * up to 24 segments, each row copied, re-RoPEd or dequantised into place.
 * Replaces the per-layer anchor/working/self copies of
 * wave_rt/denoiser/exchange/paged.py:226-237, the anchor re-RoPE of
 * exchange/common.py:84-87 (rotated straight into the buffer) and the
 * receive-side dequantisation of FP8 pages.  cols = H * head_dim. */
int wf_kv_assemble(const wf_kv_segment* segs, int n_segs, int64_t cols, int head_dim, void* stream);

/* ---------------------------------------------------------------- RoPE */

/* Interleaved (non-neox) rotary embedding, y = x * (cos + i sin) on complex
 * pairs, f32 math, bf16 out: the anchor re-RoPE of
 * wave_rt/denoiser/exchange/common.py:84-87 (SGLang _apply_rotary_emb with
 * is_neox_style=False) and the q/k RoPE of wave_rt/runtime/backend.py:119-121.
 * x, y: bf16 [L, H, D] with token strides (head stride D); cos/sin: f32
 * [L, D/2].  y may alias x. */
int wf_rope_apply(const void* x, void* y, const float* cos_t, const float* sin_t, int64_t L, int H, int D,
                  int64_t x_tok_stride, int64_t y_tok_stride, void* stream);

/* ------------------------------------- fused Wan-block row kernels */
/* Caller-side epilogues around the hot path, one warp per token row, f32 math,
 * bf16 in/out.  dim must be 256, 1536, 3072 or 5120.  Row r belongs to stage
 * r / rows_per_stage, which selects that stage's modulation / RoPE table. */

/* out = LayerNorm(x) * (1 + scale[s]) + shift[s]  (no affine, eps), the
 * modulated norms of naive_rt/rolling_forcing/wan/modules/causal_model.py:375-377
 * and :405-408.  shift/scale: f32 [stages, dim] with row stride mod_stride. */
int wf_ln_modulate(const void* x, int64_t x_stride, const float* shift, const float* scale, int64_t mod_stride,
                   void* out, int64_t out_stride, int64_t rows, int64_t dim, int64_t rows_per_stage, float eps,
                   void* stream);

/* wf_ln_modulate whose bf16 output goes straight into the per-token W8A8
 * activation quantiser of the linear that reads it (the QKV projection and
 * FFN fc_in of causal_model.py:375-377, 405-408 with W8A8 linears,
 * wave_rt/runtime/fp8.py:47-48 per row): xq [rows, dim] e4m3 or int8 codes
 * (qtype) and x_scale [rows], equal bit for bit to wf_act_quant applied to
 * wf_ln_modulate's output, without writing or re-reading that output. */
int wf_ln_modulate_quant(const void* x, int64_t x_stride, const float* shift, const float* scale,
                         int64_t mod_stride, void* xq, float* x_scale, int64_t rows, int64_t dim,
                         int64_t rows_per_stage, float eps, int qtype, void* stream);

/* x = bf16(x + y * gate[s]) in place, the gated residuals of
 * causal_model.py:383 and :411-413 (gate of ones for the cross-attention add). */
int wf_gate_residual(void* x, int64_t x_stride, const void* y, int64_t y_stride, const float* gate,
                     int64_t gate_stride, int64_t rows, int64_t dim, int64_t rows_per_stage, void* stream);

/* wf_gate_residual fused with the row op that reads its result, so the new
 * row is used from registers instead of being read back:
 *   shift == scale == NULL, xq/x_scale set: per-token W8A8 quantisation of
 *     the new x (as wf_act_quant), for the cross-attention q projection;
 *   shift, scale and out set: LN-modulate of the new x to bf16 out [rows,
 *     out_stride] (as wf_ln_modulate), for the FFN input and the next
 *     layer's QKV input;
 *   shift, scale, xq and x_scale set: the same quantised per token (as
 *     wf_ln_modulate_quant).
 * Exactly one of out / xq is given.  gate rows select their stage by
 * gate_rows_per_stage, modulation rows by mod_rows_per_stage.  Every output,
 * and x itself, equals the two-launch form bit for bit. */
int wf_gate_residual_then(void* x, int64_t x_stride, const void* y, int64_t y_stride, const float* gate,
                          int64_t gate_stride, int64_t gate_rows_per_stage, const float* shift, const float* scale,
                          int64_t mod_stride, int64_t mod_rows_per_stage, float eps, void* out, int64_t out_stride,
                          void* xq, float* x_scale, int qtype, int64_t rows, int64_t dim, void* stream);

/* Streaming VAE decode: the channel RMSNorm of channels-last bf16
 * activations, rows [rows, C] contiguous (C a multiple of 8, at most 1024):
 * out = x / max(||x||_2, eps) * sqrt(C) * gamma (bf16 [C]), then SiLU when
 * silu != 0 (naive_rt/rolling_forcing/wan/modules/vae.py:39-54 with the
 * SiLU of :178-192); f32 math, out may alias x. */
int wf_channel_rmsnorm(const void* x, void* out, int64_t rows, int64_t C, const void* gamma, float eps, int silu,
                       void* stream);

/* Streaming VAE decode, temporal x2 on channels-last rows: src [frames, hw,
 * 2C] (bf16) becomes dst [2 * frames, hw, C], frame 2i from channels [0, C)
 * of src frame i and frame 2i + 1 from [C, 2C)
 * (naive_rt/rolling_forcing/wan/modules/vae.py:127-131). */
int wf_interleave_time2(const void* src, void* dst, int64_t frames, int64_t hw, int64_t C, void* stream);

/* Streaming VAE decode, on channels-last bf16 rows [rows, C] (C a multiple
 * of 8): out = x + bias[c], then + res when res is not NULL, each sum rounded
 * to bf16 (the convolution bias that cuDNN leaves to a separate pass, and the
 * residual blocks' skip add, vae.py:194-214); out may alias x. */
int wf_channel_bias_add(const void* x, const void* bias, const void* res, void* out, int64_t rows, int64_t C,
                        void* stream);

/* Streaming VAE decode: nearest x2 in H and W of channels-last bf16 images
 * src [images, h, w, C] into dst [images, 2h, 2w, C] (vae.py:62-66, 77-80). */
int wf_upsample2x_nearest(const void* src, void* dst, int64_t images, int64_t h, int64_t w, int64_t C,
                          void* stream);

/* From the fused QKV GEMM output qkv [rows, ld] (q at column 0, k at dim):
 * RMSNorm over dim (rounded to bf16, then times the bf16 weight, as
 * naive_rt/rolling_forcing/wan/modules/model.py:70-88) followed by interleaved
 * RoPE with per-stage f32 tables cos/sin [stages * rows_per_stage, head_dim/2]
 * (wave_rt/runtime/backend.py:119-121).  Writes roped q, roped k, and the
 * normalised un-roped k (k_unroped may be NULL), each [rows, dim] dense. */
int wf_qk_norm_rope(const void* qkv, int64_t ld, const void* wq, const void* wk, const float* cos_t,
                    const float* sin_t, int head_dim, void* q_out, void* k_out, void* k_unroped, int64_t rows,
                    int64_t dim, int64_t rows_per_stage, float eps, void* stream);

/* One destination slot of a fused FP8 K/V publish: codes [T, dim] u8 (8-byte
 * aligned) and per-row scales [T] f32 for K and for V. */
typedef struct wf_kv_publish_dst {
  uint8_t* codes_k;
  uint8_t* codes_v;
  float* scales_k;
  float* scales_v;
} wf_kv_publish_dst;

/* wf_qk_norm_rope fused with the per-token FP8 publish of the same layer:
 * for every stage s < n_stages with n_dst[s] > 0, the stage's roped K rows
 * (as written to k_out) and its V rows (columns [2 dim, 3 dim) of qkv) are
 * quantised per token, with the codec of wf_kv_quant_publish, bit for bit,
 * and written to dsts[s * 8 + d], d < n_dst[s] (local or peer memory; row
 * r of the stage goes to row r of each slot).  This is the layer-wise K/V
 * publish of wave_rt/denoiser/exchange/paged.py:120-145 moved into the
 * kernel that produces K, so the bf16 K and V are not read a second time.
 * dsts: host array of n_stages * 8 entries; n_stages <= 8, n_dst[s] <= 8.
 * The caller orders the consumers' release flags after this call. */
int wf_qk_norm_rope_publish(const void* qkv, int64_t ld, const void* wq, const void* wk, const float* cos_t,
                            const float* sin_t, int head_dim, void* q_out, void* k_out, void* k_unroped,
                            int64_t rows, int64_t dim, int64_t rows_per_stage, float eps,
                            const wf_kv_publish_dst* dsts, const int32_t* n_dst, int n_stages, void* stream);

/* out = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w), model.py:70-88. */
int wf_rms_norm(const void* x, int64_t x_stride, const void* w, void* out, int64_t out_stride, int64_t rows,
                int64_t dim, float eps, void* stream);

/* ------------------------------------------------ exchange primitives */

/* IPC export of the allocation holding `p`; replaces ipc_export,
 * wave_rt/distributed/ipc.py:147-152 (handle bytes + offset of p in it). */
int wf_ipc_export(const void* p, uint8_t* handle64, uint64_t* offset);

/* Opens a peer handle in the current context with lazy peer access;
 * replaces ipc_open_handle, wave_rt/distributed/ipc.py:112-118. */
int wf_ipc_open(const uint8_t* handle64, void** base);

/* Closes a mapping opened by wf_ipc_open; replaces ipc_close_handle,
 * wave_rt/distributed/ipc.py:135-136. */
int wf_ipc_close(void* base);

/* Enables peer access from the current device to `peer` (idempotent). */
int wf_enable_peer(int peer);

/* Stream-ordered 32-bit release write; replaces stream_write_u32,
 * wave_rt/distributed/ipc.py:43-47. */
int wf_stream_write_u32(void* stream, void* addr, uint32_t value);

/* Stream-ordered unbounded acquire wait (*addr >= value); replaces
 * stream_wait_u32, wave_rt/distributed/ipc.py:50-54.  Prefer wf_wait_flag. */
int wf_stream_wait_u32(void* stream, const void* addr, uint32_t value);

/* Bounded device-side acquire: a one-thread kernel on `stream` spins with
 * ld.acquire.sys until *flag >= value or timeout_ns elapses.  On timeout it
 * writes 1 to *timeout_out (device or host-mapped memory, may be NULL), raises
 * the device status word and returns, leaving the stream usable.  Replaces the
 * wait of wave_rt/denoiser/exchange/paged.py:147-154, which has no timeout. */
int wf_wait_flag(const void* flag, uint32_t value, uint64_t timeout_ns, uint32_t* timeout_out, void* stream);

/* wf_wait_flag over n (0..32) flags in one launch: `flags` is a HOST array of
 * n device addresses (4-byte aligned); the stream continues once every flag
 * is >= value or its wait timed out (same timeout report as wf_wait_flag).
 * A consumer's waits for all its producers of one layer, which the reference
 * issues one per producer (wave_rt/denoiser/exchange/paged.py:147-154). */
int wf_wait_flags(const void* const* flags, int n, uint32_t value, uint64_t timeout_ns, uint32_t* timeout_out,
                  void* stream);

/* Diagnostic (no counterpart in the reference): a one-thread kernel on
 * `stream` writes the device's %globaltimer (ns) to *dst (8-byte aligned
 * device memory) when the stream reaches it.  Stamps of one tick on every
 * rank, aligned at a common collective, give the cross-rank timeline of the
 * wavefront. */
int wf_stamp(uint64_t* dst, void* stream);

/* Asynchronous device-to-device (or peer) copy of `bytes`; replaces
 * memcpy_dtod_async, wave_rt/distributed/ipc.py:60-67. */
int wf_memcpy_async(void* dst, const void* src, uint64_t bytes, void* stream);

/* One layer's publish to n destinations: for each i, copy bytes from src to
 * dsts[i] and then write `value` to flags[i] on the same stream (payload
 * before flag), as wave_rt/denoiser/exchange/paged.py:134-141. */
int wf_publish(void* const* dsts, const void* src, uint64_t bytes, void* const* flags, int n, uint32_t value,
               void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WFK_H_ */
