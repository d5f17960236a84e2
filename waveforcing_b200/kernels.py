"""torch-facing wrappers over the libwfk C ABI.

Each wrapper validates dtype/device/layout, launches on the caller's current
CUDA stream and raises on any error.  There is no CPU or library fallback:
CPU tensors or a missing libwfk.so raise.
"""

from __future__ import annotations

import ctypes as C
import math

import torch

from waveforcing_b200 import _lib as L

# Number of libwfk kernel launches issued through these wrappers (reported by
# bench.py as gpu_launches for its timed region).
LAUNCHES = [0]


def _stream() -> int:
    LAUNCHES[0] += 1
    return torch.cuda.current_stream().cuda_stream


def _check(cond: bool, msg: str) -> None:
    """Shape/dtype validation the C ABI cannot do: it sees pointers, not sizes,
    so a mis-shaped output or side tensor would be read or written out of
    bounds.  Runs before the device check."""
    if not cond:
        raise ValueError(msg)


def _need_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("waveforcing_b200 kernels need CUDA tensors (no CPU path exists)")


def _strides_bthd(t: torch.Tensor):
    """[B, L, H, D] or [L, H, D] -> (batch, L, H, D, {batch, token, head} strides)."""
    if t.dim() == 3:
        Lt, H, D = t.shape
        return 1, Lt, H, D, (t.stride(0) * Lt, t.stride(0), t.stride(1))
    if t.dim() == 4:
        B, Lt, H, D = t.shape
        return B, Lt, H, D, (t.stride(0), t.stride(1), t.stride(2))
    raise ValueError(f"expected [B,L,H,D] or [L,H,D], got {tuple(t.shape)}")


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, softmax_scale: float | None = None,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(q k^T * scale) v on the tcgen05 kernel; NHD bf16, head_dim 128."""
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise TypeError("attention: q, k, v must be bfloat16")
    for t in (q, k, v):
        if t.stride(-1) != 1:
            raise ValueError("attention: last dim must be contiguous")
    B, Lq, H, D, qs = _strides_bthd(q)
    Bk, Lk, Hk, Dk, ks = _strides_bthd(k)
    Bv, Lv, Hv, Dv, vs = _strides_bthd(v)
    if (Bk, Hk, Dk) != (B, H, D) or (Bv, Lv, Hv, Dv) != (B, Lk, H, D):
        raise ValueError(f"attention: shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    _check(out.shape == q.shape and out.dtype == torch.bfloat16 and out.device == q.device and out.stride(-1) == 1,
           "attention: out must be bf16 with q's shape and device and a contiguous last dim")
    _need_cuda(q, k, v, out)
    _, _, _, _, os_ = _strides_bthd(out)
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    L.check(
        L.lib().wf_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, Lq, Lk, H, D,
                            L.i64_array(qs), L.i64_array(ks), L.i64_array(vs), L.i64_array(os_),
                            L.WF_DTYPE_BF16, None, None, L.WF_SCALE_NONE, scale, _stream()),
        "wf_attn_fwd",
    )
    return out


def attention_fp8(q: torch.Tensor, k_codes: torch.Tensor, v_codes: torch.Tensor, k_scale: torch.Tensor | None,
                  v_scale: torch.Tensor | None, scale_mode: int = L.WF_SCALE_TOKEN, softmax_scale: float | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Attention over FP8 K/V pages: q bf16 [B, Lq, H, 128]; k_codes/v_codes
    uint8 e4m3 codes [B, Lk, H, 128]; scales f32 per token row [B, Lk]
    (WF_SCALE_TOKEN), one per tensor [1] (WF_SCALE_TENSOR) or none.  The
    kernel expands the codes to f16 products code * scale in shared memory and
    runs both contractions on f16 operands (|q| and |k|, |v| below 65504)."""
    if q.dtype != torch.bfloat16 or k_codes.dtype != torch.uint8 or v_codes.dtype != torch.uint8:
        raise TypeError("attention_fp8: q must be bfloat16, k/v uint8 e4m3 codes")
    for t in (q, k_codes, v_codes):
        if t.stride(-1) != 1:
            raise ValueError("attention_fp8: last dim must be contiguous")
    B, Lq, H, D, qs = _strides_bthd(q)
    Bk, Lk, Hk, Dk, ks = _strides_bthd(k_codes)
    Bv, Lv, Hv, Dv, vs = _strides_bthd(v_codes)
    if (Bk, Hk, Dk) != (B, H, D) or (Bv, Lv, Hv, Dv) != (B, Lk, H, D):
        raise ValueError(f"attention_fp8: shape mismatch q{tuple(q.shape)} k{tuple(k_codes.shape)} "
                         f"v{tuple(v_codes.shape)}")
    need = {L.WF_SCALE_TOKEN: B * Lk, L.WF_SCALE_TENSOR: 1, L.WF_SCALE_NONE: 0}.get(scale_mode)
    _check(need is not None, "attention_fp8: unknown scale_mode")
    if need:
        _check(all(t is not None and t.dtype == torch.float32 and t.is_contiguous() and t.numel() >= need
                   for t in (k_scale, v_scale)),
               "attention_fp8: k_scale/v_scale must be contiguous f32 with B*Lk (token) or 1 (tensor) elements")
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    _check(out.shape == q.shape and out.dtype == torch.bfloat16 and out.stride(-1) == 1,
           "attention_fp8: out must be bf16 with q's shape and a contiguous last dim")
    _need_cuda(q, k_codes, v_codes, out)
    _, _, _, _, os_ = _strides_bthd(out)
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    L.check(
        L.lib().wf_attn_fwd(q.data_ptr(), k_codes.data_ptr(), v_codes.data_ptr(), out.data_ptr(), B, Lq, Lk, H, D,
                            L.i64_array(qs), L.i64_array(ks), L.i64_array(vs), L.i64_array(os_),
                            L.WF_DTYPE_E4M3, k_scale.data_ptr() if need else None,
                            v_scale.data_ptr() if need else None, scale_mode, scale, _stream()),
        "wf_attn_fwd(e4m3)",
    )
    return out


def _as_rows(x: torch.Tensor):
    """View x as [rows, cols] with a row stride (last dim contiguous)."""
    if x.dim() == 1:
        return 1, x.shape[0], x.shape[0]
    cols = x.shape[-1]
    x2 = x.reshape(-1, cols) if not x.is_contiguous() else x.view(-1, cols)
    return x2.shape[0], cols, x2.stride(0)


def kv_quant(x: torch.Tensor, mode: int = L.WF_SCALE_TOKEN, codes: torch.Tensor | None = None,
             scales: torch.Tensor | None = None, workspace: torch.Tensor | None = None):
    """bf16 [rows, cols] -> (u8 codes [rows, cols], f32 scales [rows] or [1])."""
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(-1) != 1:
        raise ValueError("kv_quant: x must be a 2-D bf16 matrix with contiguous rows")
    rows, cols = x.shape
    n_scales = rows if mode == L.WF_SCALE_TOKEN else 1
    if codes is not None:
        _check(codes.dtype == torch.uint8 and codes.is_contiguous() and codes.numel() == rows * cols,
               "kv_quant: codes must be a contiguous uint8 tensor of rows * cols elements")
    if scales is not None and mode != L.WF_SCALE_NONE:
        _check(scales.dtype == torch.float32 and scales.is_contiguous() and scales.numel() >= n_scales,
               "kv_quant: scales must be contiguous f32 with one element per row (token) or one (tensor)")
    if workspace is not None:
        _check(workspace.dtype == torch.int32 and workspace.numel() >= 1,
               "kv_quant: workspace must be an int32 tensor of at least one element")
    _need_cuda(x)
    if codes is None:
        codes = torch.empty((rows, cols), dtype=torch.uint8, device=x.device)
    if scales is None and mode != L.WF_SCALE_NONE:
        scales = torch.empty((n_scales,), dtype=torch.float32, device=x.device)
    ws = 0
    if mode == L.WF_SCALE_TENSOR:
        if workspace is None:
            workspace = torch.empty((1,), dtype=torch.int32, device=x.device)
        ws = workspace.data_ptr()
    L.check(L.lib().wf_kv_quant(x.data_ptr(), codes.data_ptr(), scales.data_ptr() if scales is not None else None,
                                rows, cols, x.stride(0), mode, ws, _stream()), "wf_kv_quant")
    return codes, scales


def kv_dequant(codes: torch.Tensor, scales: torch.Tensor | None, mode: int = L.WF_SCALE_TOKEN,
               out: torch.Tensor | None = None) -> torch.Tensor:
    if codes.dtype != torch.uint8 or codes.dim() != 2 or not codes.is_contiguous():
        raise ValueError("kv_dequant: codes must be a contiguous 2-D uint8 matrix")
    rows, cols = codes.shape
    if mode != L.WF_SCALE_NONE:
        _check(scales is not None and scales.dtype == torch.float32
               and scales.numel() >= (rows if mode == L.WF_SCALE_TOKEN else 1),
               "kv_dequant: f32 scales needed, one per row (token) or one (tensor)")
    if out is not None:
        _check(out.dim() == 2 and tuple(out.shape) == (rows, cols) and out.dtype == torch.bfloat16
               and out.stride(-1) == 1, "kv_dequant: out must be bf16 [rows, cols] with contiguous rows")
    _need_cuda(codes)
    if out is None:
        out = torch.empty((rows, cols), dtype=torch.bfloat16, device=codes.device)
    sp = scales.data_ptr() if scales is not None else 0
    L.check(L.lib().wf_kv_dequant(codes.data_ptr(), sp, out.data_ptr(), rows, cols, out.stride(0), mode, _stream()),
            "wf_kv_dequant")
    return out


def kv_quant_publish(k: torch.Tensor, v: torch.Tensor, dst_codes_k, dst_codes_v, dst_scales_k, dst_scales_v) -> None:
    """Per-token quantise K and V [rows, cols] and write codes/scales to every
    destination (device pointers as ints, local or peer)."""
    _check(k.dim() == 2 and v.shape == k.shape and k.dtype == v.dtype == torch.bfloat16,
           "kv_quant_publish: k and v must be bf16 matrices of one shape")
    n = len(dst_codes_k)
    _check(n >= 1 and len(dst_codes_v) == len(dst_scales_k) == len(dst_scales_v) == n,
           "kv_quant_publish: one code and one scale destination per K and V, same count")
    _need_cuda(k, v)
    rows, cols = k.shape
    L.check(L.lib().wf_kv_quant_publish(k.data_ptr(), v.data_ptr(), rows, cols, k.stride(0), v.stride(0),
                                        L.ptr_array(dst_codes_k), L.ptr_array(dst_codes_v),
                                        L.ptr_array(dst_scales_k), L.ptr_array(dst_scales_v), n, _stream()),
            "wf_kv_quant_publish")


def weight_quant(w: torch.Tensor, qtype: int = L.WF_DTYPE_E4M3):
    """bf16 [N, K] -> (codes [N, K] uint8/int8 storage, f32 scales [N])."""
    _check(w.dim() == 2 and w.dtype == torch.bfloat16, "weight_quant: w must be a bf16 [N, K] matrix")
    _need_cuda(w)
    w = w.contiguous()
    N, K = w.shape
    wq = torch.empty((N, K), dtype=torch.uint8, device=w.device)
    ws = torch.empty((N,), dtype=torch.float32, device=w.device)
    L.check(L.lib().wf_weight_quant(w.data_ptr(), wq.data_ptr(), ws.data_ptr(), N, K, qtype, _stream()),
            "wf_weight_quant")
    return wq, ws


def act_quant(x: torch.Tensor, qtype: int = L.WF_DTYPE_E4M3, xq: torch.Tensor | None = None,
              xs: torch.Tensor | None = None, activation: int = L.WF_ACT_NONE):
    """Per-token activation quantisation of x [M, K] bf16; activation
    WF_ACT_GELU_TANH quantises bf16(GELU_tanh(x)) instead."""
    _check(x.dim() == 2 and x.dtype == torch.bfloat16 and x.stride(-1) == 1,
           "act_quant: x must be a bf16 [M, K] matrix with contiguous rows")
    M, K = x.shape
    _check(xq is None or tuple(xq.shape) == (M, K), "act_quant: xq must be [M, K]")
    _check(xs is None or (xs.dtype == torch.float32 and xs.numel() >= M), "act_quant: xs must hold M f32 scales")
    _need_cuda(x)
    if xq is None:
        xq = torch.empty((M, K), dtype=torch.uint8, device=x.device)
    if xs is None:
        xs = torch.empty((M,), dtype=torch.float32, device=x.device)
    L.check(L.lib().wf_act_quant_act(x.data_ptr(), xq.data_ptr(), xs.data_ptr(), M, K, x.stride(0), qtype,
                                     activation, _stream()), "wf_act_quant_act")
    return xq, xs


def gemm_w8a8(xq, xs, wq, ws, bias=None, qtype: int = L.WF_DTYPE_E4M3, scale_mode: int = L.WF_SCALE_TOKEN,
              out: torch.Tensor | None = None, activation: int = L.WF_ACT_NONE) -> torch.Tensor:
    """y = (xq wq^T) * xs * ws + bias in bf16; activation WF_ACT_GELU_TANH applies
    GELU(tanh) to the bf16-rounded result in the same kernel."""
    _check(xq.dim() == 2 and wq.dim() == 2 and xq.shape[1] == wq.shape[1],
           "gemm_w8a8: xq [M, K] and wq [N, K] must share K")
    M, K = xq.shape
    N = wq.shape[0]
    per_token = scale_mode == L.WF_SCALE_TOKEN
    _check(xs.dtype == ws.dtype == torch.float32 and xs.numel() >= (M if per_token else 1)
           and ws.numel() >= (N if per_token else 1),
           "gemm_w8a8: f32 scales needed, x_scale per row and w_scale per channel (one each per tensor)")
    _check(bias is None or bias.numel() == N, "gemm_w8a8: bias must have N elements")
    _check(out is None or (tuple(out.shape) == (M, N) and out.dtype == torch.bfloat16 and out.stride(-1) == 1),
           "gemm_w8a8: out must be bf16 [M, N] with contiguous rows")
    _need_cuda(xq, wq)
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=xq.device)
    bp = bias.data_ptr() if bias is not None else 0
    L.check(L.lib().wf_gemm_w8a8_act(xq.data_ptr(), xs.data_ptr(), wq.data_ptr(), ws.data_ptr(), bp, out.data_ptr(),
                                     M, N, K, out.stride(0), qtype, scale_mode, activation, _stream()),
            "wf_gemm_w8a8_act")
    return out


def kv_assemble(segments, cols: int, head_dim: int) -> None:
    """One launch that fills K/V context rows from a list of segments
    (kind, src, aux0, aux1, dst, rows, src_row_stride, dst_row_stride), with
    kind WF_SEG_COPY / WF_SEG_ROPE / WF_SEG_DEQUANT, pointers as ints (aux as 0
    when unused) and strides in elements of the source / bf16 destination."""
    n = len(segments)
    arr = (L.KvSegment * max(1, n))()
    for i, (kind, src, a0, a1, dst, rows, ss, ds) in enumerate(segments):
        arr[i] = L.KvSegment(kind, 0, src, a0 or None, a1 or None, dst, rows, ss, ds)
    L.check(L.lib().wf_kv_assemble(arr, n, cols, head_dim, _stream()), "wf_kv_assemble")


def rope_apply(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, out: torch.Tensor | None = None):
    """Interleaved RoPE on bf16 [L, H, D] with f32 cos/sin [L, D/2]."""
    if x.dim() == 4:
        x = x[0]
    Lt, H, D = x.shape
    _check(x.dtype == torch.bfloat16 and x.stride(2) == 1 and x.stride(1) == D,
           "rope_apply: x must be bf16 [L, H, D] with contiguous heads (token stride is free)")
    for tab in (cos, sin):
        _check(tab.dtype == torch.float32 and tab.dim() == 2 and tab.shape[0] >= Lt and tab.shape[1] == D // 2
               and tab.is_contiguous(), "rope_apply: cos/sin must be contiguous f32 [>= L, D/2]")
    _check(out is None or (out.shape == x.shape and out.dtype == x.dtype and out.stride(2) == 1
                           and out.stride(1) == D), "rope_apply: out must match x, with contiguous heads")
    _need_cuda(x, cos, sin)
    if out is None:
        out = torch.empty_like(x)
    L.check(L.lib().wf_rope_apply(x.data_ptr(), out.data_ptr(), cos.data_ptr(), sin.data_ptr(), Lt, H, D,
                                  x.stride(0), out.stride(0), _stream()), "wf_rope_apply")
    return out


# ------------------------------------------------------ fused Wan-block rows
def ln_modulate(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, rows_per_stage: int, eps: float,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """out = LN(x) * (1 + scale[s]) + shift[s]; x bf16 [rows, dim], shift/scale f32 [S, dim] row-strided."""
    _check(x.dim() == 2 and x.dtype == torch.bfloat16, "ln_modulate: x must be a bf16 [rows, dim] matrix")
    rows, dim = x.shape
    for t in (shift, scale):
        _check(t.dtype == torch.float32 and t.dim() == 2 and t.shape[1] == dim and t.stride(1) == 1
               and t.shape[0] * rows_per_stage >= rows, "ln_modulate: shift/scale must be f32 [stages, dim]")
    _check(shift.stride(0) == scale.stride(0), "ln_modulate: shift and scale must share their row stride")
    _check(out is None or (out.shape == x.shape and out.dtype == torch.bfloat16), "ln_modulate: out must match x")
    _need_cuda(x)
    if out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
    L.check(L.lib().wf_ln_modulate(x.data_ptr(), x.stride(0), shift.data_ptr(), scale.data_ptr(), shift.stride(0),
                                   out.data_ptr(), out.stride(0), rows, dim, rows_per_stage, eps, _stream()),
            "wf_ln_modulate")
    return out


def ln_modulate_quant(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, rows_per_stage: int, eps: float,
                      qtype: int = L.WF_DTYPE_E4M3):
    """ln_modulate followed by the per-token W8A8 activation quantiser, in one
    kernel: returns (codes uint8 [rows, dim], scales f32 [rows]), equal to
    act_quant(ln_modulate(x)) without the bf16 output being written."""
    _check(x.dim() == 2 and x.dtype == torch.bfloat16, "ln_modulate_quant: x must be a bf16 [rows, dim] matrix")
    rows, dim = x.shape
    for t in (shift, scale):
        _check(t.dtype == torch.float32 and t.dim() == 2 and t.shape[1] == dim and t.stride(1) == 1
               and t.shape[0] * rows_per_stage >= rows, "ln_modulate_quant: shift/scale must be f32 [stages, dim]")
    _check(shift.stride(0) == scale.stride(0), "ln_modulate_quant: shift and scale must share their row stride")
    _need_cuda(x)
    xq = torch.empty((rows, dim), device=x.device, dtype=torch.uint8)
    xs = torch.empty((rows,), device=x.device, dtype=torch.float32)
    L.check(L.lib().wf_ln_modulate_quant(x.data_ptr(), x.stride(0), shift.data_ptr(), scale.data_ptr(),
                                         shift.stride(0), xq.data_ptr(), xs.data_ptr(), rows, dim, rows_per_stage,
                                         eps, qtype, _stream()), "wf_ln_modulate_quant")
    return xq, xs


def gate_residual(x: torch.Tensor, y: torch.Tensor, gate: torch.Tensor, rows_per_stage: int) -> torch.Tensor:
    """x += y * gate[s] in place (f32 math, bf16 storage)."""
    _check(x.dim() == 2 and y.shape == x.shape and x.dtype == y.dtype == torch.bfloat16,
           "gate_residual: x and y must be bf16 matrices of one shape")
    rows, dim = x.shape
    _check(gate.dtype == torch.float32 and gate.shape[-1] == dim and gate.stride(-1) == 1
           and (gate.dim() == 1 or (gate.dim() == 2 and gate.shape[0] * rows_per_stage >= rows)),
           "gate_residual: gate must be f32 [dim] or [stages, dim]")
    _need_cuda(x, y)
    gs = gate.stride(0) if gate.dim() == 2 else 0
    L.check(L.lib().wf_gate_residual(x.data_ptr(), x.stride(0), y.data_ptr(), y.stride(0), gate.data_ptr(), gs,
                                     rows, dim, rows_per_stage, _stream()), "wf_gate_residual")
    return x


def gate_residual_then(x: torch.Tensor, y: torch.Tensor, gate: torch.Tensor, gate_rows_per_stage: int,
                       shift: torch.Tensor | None = None, scale: torch.Tensor | None = None,
                       mod_rows_per_stage: int = 1, eps: float = 1e-6, quant: bool = False,
                       qtype: int = L.WF_DTYPE_E4M3):
    """x += y * gate[s] in place, then from the new rows without reading them
    back: with shift/scale, LN-modulate to a new bf16 [rows, dim] (or, with
    ``quant``, its per-token W8A8 codes and scales); without, the per-token
    quantisation of x itself (``quant`` implied).  Returns the bf16 output or
    (codes uint8 [rows, dim], scales f32 [rows])."""
    _check(x.dim() == 2 and y.shape == x.shape and x.dtype == y.dtype == torch.bfloat16,
           "gate_residual_then: x and y must be bf16 matrices of one shape")
    rows, dim = x.shape
    _check(gate.dtype == torch.float32 and gate.shape[-1] == dim and gate.stride(-1) == 1
           and (gate.dim() == 1 or (gate.dim() == 2 and gate.shape[0] * gate_rows_per_stage >= rows)),
           "gate_residual_then: gate must be f32 [dim] or [stages, dim]")
    mod = shift is not None or scale is not None
    if mod:
        for t in (shift, scale):
            _check(t is not None and t.dtype == torch.float32 and t.dim() == 2 and t.shape[1] == dim
                   and t.stride(1) == 1 and t.shape[0] * mod_rows_per_stage >= rows,
                   "gate_residual_then: shift/scale must be f32 [stages, dim]")
        _check(shift.stride(0) == scale.stride(0), "gate_residual_then: shift and scale must share their row stride")
    _need_cuda(x, y)
    gs = gate.stride(0) if gate.dim() == 2 else 0
    quant = quant or not mod
    out = xq = xs = None
    if quant:
        xq = torch.empty((rows, dim), device=x.device, dtype=torch.uint8)
        xs = torch.empty((rows,), device=x.device, dtype=torch.float32)
    else:
        out = torch.empty((rows, dim), device=x.device, dtype=torch.bfloat16)
    L.check(L.lib().wf_gate_residual_then(
        x.data_ptr(), x.stride(0), y.data_ptr(), y.stride(0), gate.data_ptr(), gs, gate_rows_per_stage,
        shift.data_ptr() if mod else None, scale.data_ptr() if mod else None, shift.stride(0) if mod else 0,
        mod_rows_per_stage, eps, out.data_ptr() if out is not None else None, dim,
        xq.data_ptr() if quant else None, xs.data_ptr() if quant else None, qtype, rows, dim, _stream()),
        "wf_gate_residual_then")
    return (xq, xs) if quant else out


def channel_rmsnorm(x: torch.Tensor, gamma: torch.Tensor, silu: bool, eps: float = 1e-12,
                    out: torch.Tensor | None = None) -> torch.Tensor:  # out: any contiguous bf16 of x's shape
    """x / max(||x||, eps) * sqrt(C) * gamma over the LAST dimension of a
    contiguous bf16 tensor (the channel rows of channels-last activations),
    then SiLU when ``silu``; ``out`` may be x itself."""
    _check(x.dtype == torch.bfloat16 and x.is_contiguous(), "channel_rmsnorm: x must be contiguous bf16")
    C = x.shape[-1]
    _check(gamma.dtype == torch.bfloat16 and gamma.numel() == C and gamma.is_contiguous(),
           "channel_rmsnorm: gamma must be contiguous bf16 [C]")
    _check(out is None or (out.shape == x.shape and out.dtype == x.dtype and out.is_contiguous()),
           "channel_rmsnorm: out must match x")
    _need_cuda(x)
    if out is None:
        out = torch.empty_like(x)
    L.check(L.lib().wf_channel_rmsnorm(x.data_ptr(), out.data_ptr(), x.numel() // C, C, gamma.data_ptr(), eps,
                                       1 if silu else 0, _stream()), "wf_channel_rmsnorm")
    return out


def channel_bias_add(x: torch.Tensor, bias: torch.Tensor, res: torch.Tensor | None = None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """x + bias (over the channel dim 1) [+ res] for channels-last bf16 x of 4 or
    5 dims; out may be x.  Returns a tensor in x's layout."""
    cl = torch.channels_last_3d if x.dim() == 5 else torch.channels_last
    _check(x.dtype == torch.bfloat16 and x.dim() in (4, 5) and x.is_contiguous(memory_format=cl),
           "channel_bias_add: x must be channels-last bf16 of 4 or 5 dims")
    C = x.shape[1]
    _check(bias.dtype == torch.bfloat16 and bias.numel() == C and bias.is_contiguous(),
           "channel_bias_add: bias must be contiguous bf16 [C]")
    _check(res is None or (res.shape == x.shape and res.dtype == x.dtype and res.is_contiguous(memory_format=cl)),
           "channel_bias_add: res must match x (channels-last)")
    _need_cuda(x)
    if out is None:
        out = torch.empty_like(x, memory_format=cl)
    L.check(L.lib().wf_channel_bias_add(x.data_ptr(), bias.data_ptr(), res.data_ptr() if res is not None else None,
                                        out.data_ptr(), x.numel() // C, C, _stream()), "wf_channel_bias_add")
    return out


def upsample2x_nearest(f: torch.Tensor) -> torch.Tensor:
    """Nearest x2 in H and W of channels-last bf16 images [N, C, H, W]."""
    _check(f.dtype == torch.bfloat16 and f.dim() == 4 and f.is_contiguous(memory_format=torch.channels_last),
           "upsample2x_nearest: f must be channels-last bf16 [N, C, H, W]")
    n, c, h, w = f.shape
    _need_cuda(f)
    out = torch.empty((n, c, 2 * h, 2 * w), device=f.device, dtype=f.dtype, memory_format=torch.channels_last)
    L.check(L.lib().wf_upsample2x_nearest(f.data_ptr(), out.data_ptr(), n, h, w, c, _stream()),
            "wf_upsample2x_nearest")
    return out


def interleave_time2(y: torch.Tensor) -> torch.Tensor:
    """[b, 2C, T, H, W] channels-last bf16 -> [b, C, 2T, H, W] channels-last:
    frame 2i from channels [0, C) of frame i, frame 2i + 1 from [C, 2C)."""
    _check(y.dim() == 5 and y.dtype == torch.bfloat16 and y.is_contiguous(memory_format=torch.channels_last_3d)
           and y.shape[1] % 2 == 0, "interleave_time2: y must be channels-last bf16 [b, 2C, T, H, W]")
    b, c2, t, h, w = y.shape
    _need_cuda(y)
    out = torch.empty((b, c2 // 2, 2 * t, h, w), device=y.device, dtype=y.dtype,
                      memory_format=torch.channels_last_3d)
    L.check(L.lib().wf_interleave_time2(y.data_ptr(), out.data_ptr(), b * t, h * w, c2 // 2, _stream()),
            "wf_interleave_time2")
    return out


def qk_norm_rope(qkv: torch.Tensor, dim: int, wq: torch.Tensor, wk: torch.Tensor, cos: torch.Tensor,
                 sin: torch.Tensor, head_dim: int, rows_per_stage: int, eps: float, want_unroped: bool = True):
    """Fused RMSNorm(q), RMSNorm(k) + RoPE from the fused QKV GEMM output.
    Returns (roped q, roped k, normalised un-roped k or None), each [rows, dim]."""
    _check(qkv.dim() == 2 and qkv.dtype == torch.bfloat16 and qkv.shape[1] >= 3 * dim,
           "qk_norm_rope: qkv must be a bf16 [rows, >= 3*dim] matrix")
    rows = qkv.shape[0]
    _check(all(w.numel() == dim and w.dtype == torch.bfloat16 and w.is_contiguous() for w in (wq, wk)),
           "qk_norm_rope: norm weights must be contiguous bf16 with dim elements")
    for tab in (cos, sin):
        _check(tab.dtype == torch.float32 and tab.dim() == 2 and tab.shape[0] >= rows
               and tab.shape[1] == head_dim // 2 and tab.is_contiguous(),
               "qk_norm_rope: cos/sin must be contiguous f32 [>= rows, head_dim/2]")
    _need_cuda(qkv)
    q = torch.empty((rows, dim), device=qkv.device, dtype=torch.bfloat16)
    k = torch.empty_like(q)
    ku = torch.empty_like(q) if want_unroped else None
    L.check(L.lib().wf_qk_norm_rope(qkv.data_ptr(), qkv.stride(0), wq.data_ptr(), wk.data_ptr(), cos.data_ptr(),
                                    sin.data_ptr(), head_dim, q.data_ptr(), k.data_ptr(),
                                    ku.data_ptr() if ku is not None else None, rows, dim, rows_per_stage, eps,
                                    _stream()), "wf_qk_norm_rope")
    return q, k, ku


def qk_norm_rope_publish(qkv: torch.Tensor, dim: int, wq: torch.Tensor, wk: torch.Tensor, cos: torch.Tensor,
                         sin: torch.Tensor, head_dim: int, rows_per_stage: int, eps: float, publish,
                         want_unroped: bool = True):
    """qk_norm_rope plus the per-token FP8 publish of every stage's roped K and
    V (wf_qk_norm_rope_publish).  ``publish[s]`` lists stage s's destination
    slots as (codes_k, codes_v, scales_k, scales_v) device pointers (ints),
    each slot [rows_per_stage, dim] codes and [rows_per_stage] f32 scales."""
    _check(qkv.dim() == 2 and qkv.dtype == torch.bfloat16 and qkv.shape[1] >= 3 * dim,
           "qk_norm_rope_publish: qkv must be a bf16 [rows, >= 3*dim] matrix")
    rows = qkv.shape[0]
    _check(all(w.numel() == dim and w.dtype == torch.bfloat16 and w.is_contiguous() for w in (wq, wk)),
           "qk_norm_rope_publish: norm weights must be contiguous bf16 with dim elements")
    for tab in (cos, sin):
        _check(tab.dtype == torch.float32 and tab.dim() == 2 and tab.shape[0] >= rows
               and tab.shape[1] == head_dim // 2 and tab.is_contiguous(),
               "qk_norm_rope_publish: cos/sin must be contiguous f32 [>= rows, head_dim/2]")
    n_stages = len(publish)
    _check(n_stages <= L.PUBLISH_MAX_STAGES and n_stages * rows_per_stage >= rows
           and all(len(p) <= L.PUBLISH_MAX_DST for p in publish),
           "qk_norm_rope_publish: one destination list per stage, at most 8 stages of 8 destinations")
    _need_cuda(qkv)
    dsts = (L.KvPublishDst * max(1, n_stages * L.PUBLISH_MAX_DST))()
    counts = (C.c_int32 * max(1, n_stages))()
    for s, lst in enumerate(publish):
        counts[s] = len(lst)
        for d, (ck, cv, sk, sv) in enumerate(lst):
            dsts[s * L.PUBLISH_MAX_DST + d] = L.KvPublishDst(int(ck), int(cv), int(sk), int(sv))
    q = torch.empty((rows, dim), device=qkv.device, dtype=torch.bfloat16)
    k = torch.empty_like(q)
    ku = torch.empty_like(q) if want_unroped else None
    L.check(L.lib().wf_qk_norm_rope_publish(qkv.data_ptr(), qkv.stride(0), wq.data_ptr(), wk.data_ptr(),
                                            cos.data_ptr(), sin.data_ptr(), head_dim, q.data_ptr(), k.data_ptr(),
                                            ku.data_ptr() if ku is not None else None, rows, dim, rows_per_stage,
                                            eps, dsts, counts, n_stages, _stream()), "wf_qk_norm_rope_publish")
    return q, k, ku


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    _check(x.dim() == 2 and x.dtype == torch.bfloat16 and w.numel() == x.shape[1] and w.dtype == torch.bfloat16
           and w.is_contiguous(), "rms_norm: x must be bf16 [rows, dim] and w contiguous bf16 with dim elements")
    _need_cuda(x)
    rows, dim = x.shape
    out = torch.empty((rows, dim), device=x.device, dtype=torch.bfloat16)
    L.check(L.lib().wf_rms_norm(x.data_ptr(), x.stride(0), w.data_ptr(), out.data_ptr(), out.stride(0), rows, dim,
                                eps, _stream()), "wf_rms_norm")
    return out
