"""The FP8 codec's fast path replaces the reference's f32 division x / s by a
multiply with RN(1/s) before the bf16 rounding (waveforcing_b200/csrc/kv_codec.cu).
That is exact because x and s are bf16: x / s is never a bf16 rounding
midpoint and stays far from all of them.  This checks the claim over every
pair of bf16 significands at a spread of exponents, in numpy on the CPU."""

import numpy as np


def _bf16_rn(x):
    b = x.view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def test_reciprocal_multiply_rounds_like_division():
    a = np.arange(1, 256, dtype=np.float32)[:, None]   # x significands (incl. subnormal-like)
    b = np.arange(128, 256, dtype=np.float32)[None, :]  # s significands
    for ea in range(-12, 14, 2):
        for eb in range(-14, 12, 2):
            x = np.broadcast_to(a * np.float32(2.0 ** ea), (255, 128)).astype(np.float32)
            s = np.broadcast_to(b * np.float32(2.0 ** eb), (255, 128)).astype(np.float32)
            q_div = (x.astype(np.float64) / s.astype(np.float64)).astype(np.float32)
            q_mul = x * (np.float32(1) / s)
            assert np.array_equal(_bf16_rn(q_div), _bf16_rn(q_mul)), (ea, eb)
