"""Chunk self-attention over an assembled K/V context (test infrastructure only).

The reference calls ``self.attn(q, K, V)`` (SGLang torch_sdpa) at
wave_rt/runtime/backend.py:141-148: softmax(Q K^T / sqrt(D)) V, non-causal,
NHD layout.  Block causality comes from which chunks are in K/V, not from a
mask.  The vendored statement of the same call is the torch SDPA fallback
at naive_rt/rolling_forcing/wan/modules/attention.py:75-89 (transpose to
[B, N, L, D], ``F.scaled_dot_product_attention``, transpose back).

``sdpa_numpy`` restates the math in float64/float32 numpy for small cases;
``sdpa_reference_torch`` is the reference's own CPU call, used as the timed
CPU baseline and to pin the numpy restatement.
"""

from __future__ import annotations

import math

import numpy as np


def sdpa_numpy(q, k, v, scale=None, k_scale=None, v_scale=None, block=512, dtype=np.float64):
    """q [Lq,H,D], k/v [Lk,H,D] (float arrays) -> out [Lq,H,D] in ``dtype``.

    ``k_scale``/``v_scale`` (optional, [Lk] or scalar) multiply K/V rows, the
    dequantisation of common.py:162 applied per token.
    """
    Lq, H, D = q.shape
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    k = k.astype(dtype)
    v = v.astype(dtype)
    if k_scale is not None:
        ks = np.asarray(k_scale, dtype)
        k = k * (ks[:, None, None] if ks.ndim else ks)
    if v_scale is not None:
        vs = np.asarray(v_scale, dtype)
        v = v * (vs[:, None, None] if vs.ndim else vs)
    out = np.empty((Lq, H, D), dtype)
    kh = np.transpose(k, (1, 2, 0))  # [H, D, Lk]
    vh = np.transpose(v, (1, 0, 2))  # [H, Lk, D]
    for s in range(0, Lq, block):
        qb = np.transpose(q[s : s + block].astype(dtype), (1, 0, 2))  # [H, b, D]
        sc = np.matmul(qb, kh) * scale
        sc -= sc.max(axis=-1, keepdims=True)
        p = np.exp(sc)
        p /= p.sum(axis=-1, keepdims=True)
        out[s : s + block] = np.transpose(np.matmul(p, vh), (1, 0, 2))
    return out


def sdpa_reference_torch(q, k, v, scale=None):
    """attention.py:76-89 on CPU tensors [B, L, H, D] -> [B, Lq, H, D]."""
    import torch
    import torch.nn.functional as F

    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    out = F.scaled_dot_product_attention(qh, kh, vh, scale=scale)
    return out.transpose(1, 2).contiguous()


def attn_flops(Lq: int, Lk: int, H: int, D: int) -> float:
    """Algorithmic FLOPs of one call: QK^T and PV, 2 flops per MAC."""
    return 4.0 * Lq * Lk * H * D
