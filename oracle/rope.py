"""Wan 3-axis RoPE restated in numpy (test infrastructure only).

Follows the vendored naive model, which states the same arithmetic SGLang
applies on the production path:
  * rope_params          -- naive_rt/rolling_forcing/wan/modules/model.py:29-37
  * frequency table      -- naive_rt/rolling_forcing/wan/modules/causal_model.py:549-554
    (head_dim 128 -> complex widths [22, 21, 21] for (frame, height, width))
  * causal_rope_apply    -- naive_rt/rolling_forcing/wan/modules/causal_model.py:27-54
    (interleaved complex pairs, float64 math, result cast back to x's dtype)
The anchor re-RoPE of the paged exchange calls the same rotation at a
different ``start_frame`` (wave_rt/denoiser/exchange/common.py:45-91).
"""

from __future__ import annotations

import numpy as np


def rope_params(max_seq_len: int, dim: int, theta: float = 10000.0) -> np.ndarray:
    """model.py:29-37 -> complex128 [max_seq_len, dim/2]."""
    assert dim % 2 == 0
    inv = 1.0 / np.power(theta, np.arange(0, dim, 2, dtype=np.float64) / dim)
    ang = np.outer(np.arange(max_seq_len, dtype=np.float64), inv)
    return np.exp(1j * ang)


def freq_table(head_dim: int = 128, max_seq_len: int = 1024) -> np.ndarray:
    """causal_model.py:549-554 -> complex128 [1024, head_dim/2]."""
    d = head_dim
    return np.concatenate(
        [
            rope_params(max_seq_len, d - 4 * (d // 6)),
            rope_params(max_seq_len, 2 * (d // 6)),
            rope_params(max_seq_len, 2 * (d // 6)),
        ],
        axis=1,
    )


def token_freqs(f: int, h: int, w: int, start_frame: int, head_dim: int = 128) -> np.ndarray:
    """Per-token complex multipliers [f*h*w, head_dim/2] (causal_model.py:31-47)."""
    freqs = freq_table(head_dim)
    c = head_dim // 2
    c0 = c - 2 * (c // 3)
    c1 = c // 3
    f0, f1, f2 = freqs[:, :c0], freqs[:, c0 : c0 + c1], freqs[:, c0 + c1 :]
    ff = np.broadcast_to(f0[start_frame : start_frame + f][:, None, None, :], (f, h, w, c0))
    fh = np.broadcast_to(f1[:h][None, :, None, :], (f, h, w, c1))
    fw = np.broadcast_to(f2[:w][None, None, :, :], (f, h, w, c1))
    return np.concatenate([ff, fh, fw], axis=-1).reshape(f * h * w, c)


def causal_rope_apply(x: np.ndarray, f: int, h: int, w: int, start_frame: int) -> np.ndarray:
    """causal_model.py:27-54 for batch 1: x [L, n, d] float -> rotated float64 [L, n, d].

    Tokens beyond f*h*w pass through unchanged.  The caller rounds to the
    tensor dtype (``.type_as(v)``).
    """
    L, n, d = x.shape
    seq = f * h * w
    fr = token_freqs(f, h, w, start_frame, d)  # [seq, d/2]
    xc = x[:seq].astype(np.float64).reshape(seq, n, d // 2, 2)
    xc = xc[..., 0] + 1j * xc[..., 1]
    y = xc * fr[:, None, :]
    out = np.stack([y.real, y.imag], axis=-1).reshape(seq, n, d)
    if seq < L:
        out = np.concatenate([out, x[seq:].astype(np.float64)], axis=0)
    return out


def cos_sin_tables(f: int, h: int, w: int, start_frame: int, head_dim: int = 128):
    """float32 cos/sin [f*h*w, head_dim/2] built in float64 (common.py:45-68)."""
    fr = token_freqs(f, h, w, start_frame, head_dim)
    return fr.real.astype(np.float32), fr.imag.astype(np.float32)
