"""W8A8 linear restated in numpy (test infrastructure only).

Per-tensor FP8 (the reference): wave_rt/runtime/fp8.py:21-61
  weight (fp32 math, fp8.py:32-36):
      w_scale = clamp(amax(|w|) / 448, 1e-8)        (float32)
      w_fp8   = e4m3(w / w_scale)                   (float32 -> e4m3, RNE)
  activation (bf16 math, fp8.py:46-48):
      a_scale = clamp(bf16(amax(|x|) / 448), 1e-8)  (bf16)
      x_fp8   = e4m3(bf16(x / a_scale))
  output (fp8.py:49-56, torch._scaled_mm):
      y = bf16(sum_k x_fp8*w_fp8 * a_scale * w_scale + bias)

Per-channel / per-token (the granularity this build adds): the same dtype
sequences with the weight amax taken per output channel (row of w) and the
activation amax per token (row of x).  The INT8 variant replaces 448 by 127
and the e4m3 rounding by round-half-even to an integer clamped to [-127, 127].
"""

from __future__ import annotations

import numpy as np

from oracle.codec import E4M3_MAX, SCALE_MIN, bf16_round, e4m3_decode, e4m3_encode

I8_MAX = 127.0


def _clamp_min(s):
    return np.maximum(s, np.float32(SCALE_MIN)).astype(np.float32)


def quant_weight(w, qtype="e4m3", per_channel=True):
    """w [N,K] float -> (codes [N,K] uint8|int8, scales [N] or scalar float32)."""
    w = np.asarray(w, np.float32)
    qmax = E4M3_MAX if qtype == "e4m3" else I8_MAX
    amax = np.max(np.abs(w), axis=1) if per_channel else np.max(np.abs(w))
    s = _clamp_min(np.float32(amax) / np.float32(qmax) if np.ndim(amax) == 0 else amax / np.float32(qmax))
    ratio = w / (s[:, None] if per_channel else s)
    if qtype == "e4m3":
        return e4m3_encode(ratio.astype(np.float32)), s
    return np.clip(np.round(ratio), -I8_MAX, I8_MAX).astype(np.int8), s


def quant_act(x, qtype="e4m3", per_token=True):
    """x [M,K] bf16 values -> (codes, scales [M] or scalar), bf16 scale math (fp8.py:47-48)."""
    x = bf16_round(np.asarray(x, np.float32))
    qmax = E4M3_MAX if qtype == "e4m3" else I8_MAX
    amax = np.max(np.abs(x), axis=1) if per_token else np.max(np.abs(x))
    s = bf16_round(np.asarray(amax, np.float32) / np.float32(qmax))
    s = np.maximum(s, bf16_round(np.float32(SCALE_MIN))).astype(np.float32)
    ratio = bf16_round(x / (s[:, None] if per_token else s))
    if qtype == "e4m3":
        return e4m3_encode(ratio), s
    return np.clip(np.round(ratio), -I8_MAX, I8_MAX).astype(np.int8), s


def decode(codes, qtype):
    if qtype == "e4m3":
        return e4m3_decode(codes).astype(np.float64)
    return np.asarray(codes, np.float64)


def gemm(xq, sx, wq, sw, bias=None, qtype="e4m3"):
    """y[m,n] = bf16(sum_k dec(xq)[m,k] dec(wq)[n,k] * sx[m] * sw[n] + bias[n]) (float64 accumulate)."""
    acc = decode(xq, qtype) @ decode(wq, qtype).T
    sx = np.asarray(sx, np.float64)
    sw = np.asarray(sw, np.float64)
    y = acc * (sx[:, None] if sx.ndim else sx) * (sw[None, :] if sw.ndim else sw)
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[None, :]
    return bf16_round(y.astype(np.float32))


def linear(x, w, bias=None, qtype="e4m3", per_channel=True):
    """Full W8A8 linear: quantise both sides then ``gemm``."""
    wq, sw = quant_weight(w, qtype, per_channel)
    xq, sx = quant_act(x, qtype, per_channel)
    return gemm(xq, sx, wq, sw, bias, qtype)
