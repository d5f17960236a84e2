"""BASELINE config 1 exactly, on the B200 path against the reference's CPU path.

Config 1 is one Wan2.1-1.3B self-attention layer: q = one 3-frame chunk
(4680 tokens), K/V = two prior chunks plus the current one (14040 tokens),
12 heads x 128, q/k/v fp32 N(0,1)/sqrt(128) from seed 0, and k/v passed
through the FP8 e4m3 K/V quantise -> dequantise round trip before the
attention.

Two codecs are covered:
  * per-tensor, the reference's own: one scale over stack(K, V), as
    wave_rt/denoiser/exchange/common.py:143-164 quantises the stacked pair;
  * per-token: one scale per token row of K and of V (over H*D).

GPU side: libwfk's codec (wf_kv_quant, wf_kv_dequant) and attention
(wf_attn_fwd) on the bf16 runtime copies of q/k/v, and the same codes fed
straight to the FP8-input attention (wf_attn_fwd with kv_dtype e4m3).  CPU side: the oracle's
codec (its torch-CPU form, pinned bit for bit to the numpy restatement by
the oracle tests; bit-exact bar for codes and scales) and the
reference's attention call, F.scaled_dot_product_attention on CPU in fp32
(naive_rt/rolling_forcing/wan/modules/attention.py:76-89), on the fp32
dequantised K/V that common.py:162 returns.  Attention bar: max|out - ref| /
max|ref| <= 1e-2.
"""

import math

import pytest
import torch

from oracle import attention as o_attn
from oracle import codec as o_codec

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

T, CTX, H, D = 4680, 3 * 4680, 12, 128


@pytest.fixture(scope="module")
def config1():
    g = torch.Generator(device="cpu").manual_seed(0)
    q = torch.randn(1, T, H, D, generator=g) / math.sqrt(D)
    k = torch.randn(1, CTX, H, D, generator=g) / math.sqrt(D)
    v = torch.randn(1, CTX, H, D, generator=g) / math.sqrt(D)
    # the runtime dtype of the published K/V (the DiT computes in bf16)
    return q, k.bfloat16(), v.bfloat16()


def _cpu_attention(q, k_f32, v_f32):
    """The reference's CPU attention call on the dequantised fp32 K/V."""
    return o_attn.sdpa_reference_torch(q, k_f32.reshape(1, CTX, H, D), v_f32.reshape(1, CTX, H, D))


def _rel(a, b):
    return (a.float() - b.float()).abs().max().item() / b.float().abs().max().item()


def test_config1_per_tensor_round_trip(config1):
    from waveforcing_b200 import _lib as L
    from waveforcing_b200 import kernels as K

    q, k, v = config1
    kv = torch.stack([k[0], v[0]]).reshape(2 * CTX, H * D)  # the stacked pair of common.py:143-150
    codes_ref, scale_ref = o_codec.quant_per_tensor_torch(kv)
    codes, scale = K.kv_quant(kv.cuda(), L.WF_SCALE_TENSOR)
    assert torch.equal(codes.cpu(), codes_ref)
    assert scale.item() == scale_ref.item()
    kv_deq = o_codec.dequant_torch(codes_ref, scale_ref, per_token=False)  # fp32, common.py:162
    ref = _cpu_attention(q, kv_deq[:CTX], kv_deq[CTX:])

    deq = K.kv_dequant(codes, scale, L.WF_SCALE_TENSOR).view(2, 1, CTX, H, D)
    out = K.attention(q.cuda().bfloat16(), deq[0], deq[1])
    rel = _rel(out.cpu(), ref)
    assert rel <= 1e-2, rel
    # the same codes straight into the FP8-input attention (per-tensor scale)
    c2 = codes.view(2, 1, CTX, H, D)
    out8 = K.attention_fp8(q.cuda().bfloat16(), c2[0], c2[1], scale, scale, L.WF_SCALE_TENSOR)
    rel8 = _rel(out8.cpu(), ref)
    assert rel8 <= 1e-2, rel8
    assert L.status_take() == 0


def test_config1_per_token_round_trip(config1):
    from waveforcing_b200 import _lib as L
    from waveforcing_b200 import kernels as K

    q, k, v = config1
    deq_ref = []
    deq_gpu = []
    pages = []
    for x in (k, v):
        x2 = x.reshape(CTX, H * D)
        codes_ref, scales_ref = o_codec.quant_per_token_torch(x2)
        codes, scales = K.kv_quant(x2.cuda(), L.WF_SCALE_TOKEN)
        assert torch.equal(codes.cpu(), codes_ref)
        assert torch.equal(scales.cpu(), scales_ref)
        deq_ref.append(o_codec.dequant_torch(codes_ref, scales_ref, per_token=True))
        deq_gpu.append(K.kv_dequant(codes, scales, L.WF_SCALE_TOKEN).view(1, CTX, H, D))
        pages.append((codes.view(1, CTX, H, D), scales))
    ref = _cpu_attention(q, deq_ref[0], deq_ref[1])
    out = K.attention(q.cuda().bfloat16(), deq_gpu[0], deq_gpu[1])
    rel = _rel(out.cpu(), ref)
    assert rel <= 1e-2, rel
    # the same codes straight into the FP8-input attention (per-token scales)
    (kc, ks), (vc, vs) = pages
    out8 = K.attention_fp8(q.cuda().bfloat16(), kc, vc, ks, vs, L.WF_SCALE_TOKEN)
    rel8 = _rel(out8.cpu(), ref)
    assert rel8 <= 1e-2, rel8
    assert L.status_take() == 0
