"""The torch-facing wrappers check shapes and dtypes before anything reaches the
C ABI (which sees pointers, not sizes).  On CPU tensors a well-formed call
passes those checks and stops at the device check (RuntimeError); a
mis-shaped call stops earlier (ValueError).  The well-formed calls use the
shapes of the package's own call sites."""

import pytest
import torch

from waveforcing_b200 import _lib as L
from waveforcing_b200 import kernels as K

bf = torch.bfloat16
f32 = torch.float32


def _passes(fn, *a, **kw):
    with pytest.raises(RuntimeError, match="CUDA"):
        fn(*a, **kw)


def _rejects(fn, *a, **kw):
    with pytest.raises(ValueError):
        fn(*a, **kw)


def test_attention_out():
    q = torch.zeros(1, 130, 2, 128, dtype=bf)
    kv = torch.zeros(1, 300, 2, 128, dtype=bf)
    _passes(K.attention, q, kv, kv)
    _passes(K.attention, q, kv, kv, out=torch.empty_like(q))
    _rejects(K.attention, q, kv, kv, out=torch.empty(1, 129, 2, 128, dtype=bf))
    _rejects(K.attention, q, kv, kv, out=torch.empty(1, 130, 2, 128, dtype=f32))


def test_codec_wrappers():
    rows, cols = 96, 1536
    codes = torch.zeros(rows, cols, dtype=torch.uint8)
    _passes(K.kv_dequant, codes, torch.ones(rows), L.WF_SCALE_TOKEN)
    _passes(K.kv_dequant, codes, torch.ones(1), L.WF_SCALE_TENSOR)
    _passes(K.kv_dequant, codes, None, L.WF_SCALE_NONE)
    _passes(K.kv_dequant, codes, torch.ones(rows), L.WF_SCALE_TOKEN, out=torch.empty(rows, cols, dtype=bf))
    _rejects(K.kv_dequant, codes, torch.ones(rows - 1), L.WF_SCALE_TOKEN)
    _rejects(K.kv_dequant, codes, None, L.WF_SCALE_TOKEN)
    _rejects(K.kv_dequant, codes, torch.ones(rows), L.WF_SCALE_TOKEN, out=torch.empty(rows, cols - 8, dtype=bf))
    k = torch.zeros(rows, cols, dtype=bf)
    _passes(K.kv_quant_publish, k, k.clone(), [1, 2], [3, 4], [5, 6], [7, 8])
    _rejects(K.kv_quant_publish, k, torch.zeros(rows, cols + 8, dtype=bf), [1], [2], [3], [4])
    _rejects(K.kv_quant_publish, k, k.clone(), [1, 2], [3], [5, 6], [7, 8])


def test_w8a8_wrappers():
    M, N, Kd = 130, 256, 512
    _passes(K.weight_quant, torch.zeros(N, Kd, dtype=bf))
    _rejects(K.weight_quant, torch.zeros(N, Kd, dtype=f32))
    _passes(K.act_quant, torch.zeros(M, Kd, dtype=bf))
    _rejects(K.act_quant, torch.zeros(M, Kd, dtype=bf), xs=torch.empty(M - 1))
    xq, wq = torch.zeros(M, Kd, dtype=torch.uint8), torch.zeros(N, Kd, dtype=torch.uint8)
    # per-channel weights with per-token activations, and the per-tensor form
    _passes(K.gemm_w8a8, xq, torch.ones(M), wq, torch.ones(N), torch.zeros(N, dtype=bf))
    _passes(K.gemm_w8a8, xq, torch.ones(1), wq, torch.ones(1), None, L.WF_DTYPE_E4M3, L.WF_SCALE_TENSOR)
    _rejects(K.gemm_w8a8, xq, torch.ones(M), torch.zeros(N, Kd + 16, dtype=torch.uint8), torch.ones(N))
    _rejects(K.gemm_w8a8, xq, torch.ones(M), wq, torch.ones(N - 1))
    _rejects(K.gemm_w8a8, xq, torch.ones(M), wq, torch.ones(N), torch.zeros(N + 1, dtype=bf))
    _rejects(K.gemm_w8a8, xq, torch.ones(M), wq, torch.ones(N), out=torch.empty(M, N + 8, dtype=bf))


def test_row_kernel_wrappers():
    S, T, dim, hd = 3, 40, 256, 128
    x = torch.zeros(S * T, dim, dtype=bf)
    e = torch.zeros(S, 6, dim)  # the DiT's per-stage modulation, f32
    _passes(K.ln_modulate, x, e[:, 0], e[:, 1], T, 1e-6)
    _rejects(K.ln_modulate, x, e[:2, 0], e[:2, 1], T, 1e-6)  # too few stages for the rows
    _rejects(K.ln_modulate, x, e[:, 0], e[:, 1].contiguous(), T, 1e-6)  # row strides differ
    _passes(K.gate_residual, x, x.clone(), e[:, 2], T)
    _passes(K.gate_residual, x, x.clone(), torch.ones(dim), S * T)
    _rejects(K.gate_residual, x, torch.zeros(S * T, dim + 8, dtype=bf), e[:, 2], T)
    _rejects(K.gate_residual, x, x.clone(), e[:, 2].to(bf), T)
    qkv = torch.zeros(S * T, 3 * dim, dtype=bf)
    w = torch.ones(dim, dtype=bf)
    tab = torch.zeros(S * T, hd // 2)
    _passes(K.qk_norm_rope, qkv, dim, w, w, tab, tab, hd, T, 1e-6)
    _rejects(K.qk_norm_rope, qkv, dim, w, w, tab[:T], tab[:T], hd, T, 1e-6)
    _passes(K.rms_norm, x, w, 1e-6)
    _rejects(K.rms_norm, x, torch.ones(dim - 1, dtype=bf), 1e-6)
    page = torch.zeros(T, dim // hd, hd, dtype=bf)
    _passes(K.rope_apply, page, tab[:T], tab[:T])
    _passes(K.rope_apply, page[None], tab[:T], tab[:T])
    _rejects(K.rope_apply, page, tab[:T].double(), tab[:T].double())
    _rejects(K.rope_apply, page, tab[:T - 1], tab[:T - 1])


def test_codec_quant_side_buffers():
    rows, cols = 96, 1536
    x = torch.zeros(rows, cols, dtype=bf)
    _passes(K.kv_quant, x, L.WF_SCALE_TOKEN)
    _passes(K.kv_quant, x, L.WF_SCALE_TOKEN, codes=torch.empty(rows, cols, dtype=torch.uint8),
            scales=torch.empty(rows))
    _rejects(K.kv_quant, x, L.WF_SCALE_TOKEN, codes=torch.empty(rows, cols - 8, dtype=torch.uint8))
    _rejects(K.kv_quant, x, L.WF_SCALE_TOKEN, codes=torch.empty(rows, cols, dtype=bf))
    _rejects(K.kv_quant, x, L.WF_SCALE_TOKEN, scales=torch.empty(rows - 1))
    _rejects(K.kv_quant, x, L.WF_SCALE_TOKEN, scales=torch.empty(rows, dtype=bf))
    _rejects(K.kv_quant, x, L.WF_SCALE_TENSOR, workspace=torch.empty(1, dtype=f32))


def test_rope_and_norm_weight_dtypes():
    x = torch.zeros(10, 2, 128, dtype=bf)
    tab = torch.zeros(10, 64)
    _passes(K.rope_apply, x, tab, tab)
    _rejects(K.rope_apply, x.float(), tab, tab)
    _rejects(K.rope_apply, x.transpose(1, 2).contiguous().transpose(1, 2), tab, tab)  # heads not contiguous
    dim = 256
    _passes(K.rms_norm, torch.zeros(4, dim, dtype=bf), torch.ones(dim, dtype=bf), 1e-6)
    _rejects(K.rms_norm, torch.zeros(4, dim, dtype=bf), torch.ones(dim), 1e-6)  # f32 weight
    qkv = torch.zeros(4, 3 * dim, dtype=bf)
    t = torch.zeros(4, 64)
    _passes(K.qk_norm_rope, qkv, dim, torch.ones(dim, dtype=bf), torch.ones(dim, dtype=bf), t, t, 128, 4, 1e-6)
    _rejects(K.qk_norm_rope, qkv, dim, torch.ones(dim), torch.ones(dim, dtype=bf), t, t, 128, 4, 1e-6)
