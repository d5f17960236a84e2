"""FP8 e4m3 K/V codec restated in numpy (test infrastructure only).

Reference arithmetic (per-tensor, ``sync`` mode):
  wave_rt/denoiser/exchange/common.py:143-164 (``_all_gather_fp8``)
      scale = f32(clamp(bf16(amax(|x|) / 448.0), 1e-8))
      codes = e4m3fn(bf16(x / scale))              # bf16 math, RNE, non-saturating
      deq   = f32(bf16(e4m3(codes)) * scale)       # shape-(1,) scale promotes to f32
  wave_rt/denoiser/settings.py:20-23 (FP8_E4M3_MAX = 448, e4m3fn dtype)
Scale-free cast (``onesided``): wave_rt/denoiser/exchange/onesided.py:151-153,177-179.

The per-token codec is the same dtype sequence applied to each token row
(amax over that row's H*D values), which is the per-token granularity the
build adds for the paged exchange.

All bf16 values are carried as float32 arrays holding bf16-representable
numbers; ``bf16_round`` performs round-to-nearest-even exactly as torch's
float->bfloat16 conversion does.
"""

from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0
SCALE_MIN = 1e-8


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest-even bf16, returned as float32 (NaN stays NaN)."""
    x = np.asarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    bias = 0x7FFF + ((bits >> 16) & 1)
    out = ((bits + bias) & 0xFFFF0000).astype(np.uint32)
    nan = np.isnan(x)
    out = np.where(nan, (bits.astype(np.uint32) | 0x00400000) & 0xFFFF0000, out)
    return out.astype(np.uint32).view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """bf16-representable float32 -> uint16 bit pattern."""
    return (np.asarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint32) << 16).astype(np.uint32).view(np.float32)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """float32 -> e4m3fn code (uint8), RNE, non-saturating: |x| > 464 -> NaN (0x7F).

    Restates torch's ``Tensor.to(torch.float8_e4m3fn)`` as used at
    wave_rt/denoiser/exchange/common.py:150 and wave_rt/runtime/fp8.py:35,48.
    """
    x = np.asarray(x, dtype=np.float32)
    sign = ((x.view(np.uint32) >> 31) & 1).astype(np.uint8)
    with np.errstate(invalid="ignore"):
        a = np.abs(x).astype(np.float64)
    code = np.zeros(a.shape, dtype=np.uint8)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        # subnormal range: quantum 2^-9, values below 2^-6
        sub = a < 2.0**-6
        qs = np.round(a / 2.0**-9)  # round-half-even
        # normal range: 3 mantissa bits
        e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
        e = np.clip(e, -6, 30)
        qn = np.round(a / 2.0 ** (e - 3)) * 2.0 ** (e - 3)
    q = np.where(sub, qs * 2.0**-9, qn)
    # encode q (exactly representable in e4m3 unless > 448)
    with np.errstate(divide="ignore", invalid="ignore"):
        sub_q = q < 2.0**-6
        m_sub = np.round(q / 2.0**-9).astype(np.int64)
        eq = np.floor(np.log2(np.where(q > 0, q, 1.0))).astype(np.int64)
        m_n = np.round(q / 2.0 ** eq.astype(np.float64) * 8 - 8).astype(np.int64)
    enc_n = ((eq + 7) << 3) | m_n
    enc = np.where(sub_q, m_sub, enc_n)
    bad = np.isnan(a) | (q > E4M3_MAX)
    enc = np.where(bad, 0x7F, enc)
    code = (enc.astype(np.uint8) & 0x7F) | (sign << 7)
    return code.astype(np.uint8)


def e4m3_decode(code: np.ndarray) -> np.ndarray:
    """e4m3fn code -> float32 value (exact; 0x7F/0xFF -> NaN)."""
    c = np.asarray(code, dtype=np.uint8).astype(np.int64)
    s = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 7
    val = np.where(e == 0, m * 2.0**-9, (1 + m / 8.0) * 2.0 ** (e - 7))
    val = np.where((c & 0x7F) == 0x7F, np.nan, val)
    return (s * val).astype(np.float32)


def _scale_from_amax(amax: np.ndarray) -> np.ndarray:
    """scale = f32(clamp(bf16(amax / 448), 1e-8)) -- common.py:145-149."""
    s = bf16_round(np.asarray(amax, np.float32) / np.float32(E4M3_MAX))
    return np.maximum(s, bf16_round(np.float32(SCALE_MIN))).astype(np.float32)


def quant_per_tensor(x: np.ndarray):
    """common.py:145-150 -> (codes uint8 same shape, scale float32 scalar)."""
    x = bf16_round(x)
    amax = np.max(np.abs(x)) if x.size else np.float32(0)
    scale = _scale_from_amax(amax)
    q = bf16_round(x / scale)  # bf16 tensor / 0-dim f32 tensor -> bf16 result
    return e4m3_encode(q), np.float32(scale)


def quant_per_token(x2: np.ndarray):
    """Row-wise restatement of common.py:145-150 over a [rows, cols] bf16 matrix.

    Returns (codes uint8 [rows, cols], scales float32 [rows]).
    """
    x2 = bf16_round(np.asarray(x2, np.float32))
    amax = np.max(np.abs(x2), axis=1) if x2.shape[1] else np.zeros(x2.shape[0], np.float32)
    scales = _scale_from_amax(amax)
    q = bf16_round(x2 / scales[:, None])
    return e4m3_encode(q), scales.astype(np.float32)


def dequant(codes: np.ndarray, scales: np.ndarray, per_token: bool) -> np.ndarray:
    """common.py:162 -- f32(bf16(e4m3 value) * scale); the product is exact in f32."""
    v = e4m3_decode(codes)
    if per_token:
        return (v * np.asarray(scales, np.float32)[:, None]).astype(np.float32)
    return (v * np.float32(scales)).astype(np.float32)


def cast_scale_free(x: np.ndarray) -> np.ndarray:
    """onesided.py:152 -- kv.to(e4m3fn) with no scale (bf16 input)."""
    return e4m3_encode(bf16_round(x))


# ------------------------------------------------------------------ torch CPU
# The same dtype sequences written with torch CPU ops, i.e. the reference's
# own lines (common.py:145-150, :162) run on the host.  numpy's integer and
# log2 ufuncs are slow on some hosts; these forms quantise the full-size K/V
# of BASELINE config 1 (43 M elements) in well under a second.  They are
# pinned to the numpy restatement above by tests/test_oracle_golden.py.
def quant_per_tensor_torch(x):
    """x: CPU bf16 tensor -> (uint8 codes, f32 0-dim scale) as common.py:145-150."""
    import torch

    x = x.to(torch.bfloat16)
    scale = (x.abs().amax() / E4M3_MAX).clamp(min=SCALE_MIN).to(torch.float32)
    return (x / scale).to(torch.float8_e4m3fn).view(torch.uint8), scale


def quant_per_token_torch(x2):
    """x2: CPU bf16 [rows, cols] -> (uint8 codes, f32 scales [rows]); the row-wise
    form of common.py:145-150 (bf16 scale math, bf16 quotient)."""
    import torch

    x2 = x2.to(torch.bfloat16)
    scales = (x2.abs().amax(dim=1) / E4M3_MAX).clamp(min=SCALE_MIN).to(torch.float32)
    q = (x2.float() / scales[:, None]).to(torch.bfloat16)
    return q.to(torch.float8_e4m3fn).view(torch.uint8), scales


def dequant_torch(codes, scales, per_token: bool):
    """common.py:162 on CPU tensors: f32(bf16(e4m3 value) * scale)."""
    import torch

    v = codes.view(torch.float8_e4m3fn).to(torch.bfloat16)
    s = scales.reshape(-1, 1) if per_token else scales.reshape(1)
    return v * s
