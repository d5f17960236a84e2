"""Parity of the libwfk CUDA kernels with the CPU oracle (B200 only).

Tolerances (stated per BASELINE north_star):
  * codec codes and scales, W8A8 quantised operands: bit-exact;
  * attention and GEMM outputs: max|out - ref| / max|ref| <= 1e-2 (bf16 out);
  * RoPE: within 2 bf16 ulps of the float64 oracle (f32 vs f64 rotation).
"""

import math
import os

import numpy as np
import pytest
import torch

from oracle import attention as o_attn
from oracle import codec as o_codec
from oracle import rope as o_rope
from oracle import w8a8 as o_w8a8
from tests.conftest import bits_to_f32

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

DEV = "cuda"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _kernels():
    from waveforcing_b200 import kernels

    return kernels


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


def _bf16_gpu(x_np):
    return torch.from_numpy(np.ascontiguousarray(x_np, np.float32)).to(DEV).to(torch.bfloat16)


def _f32(t):
    return t.float().cpu().numpy()


# ------------------------------------------------------------------ attention
ATTN_CASES = [
    (128, 128, 1), (130, 300, 2), (5, 517, 3), (257, 1000, 2), (64, 64, 2), (1, 1, 1),
    (300, 129, 4), (4680, 4680, 1), (200, 700, 40), (256, 256, 1), (100, 384, 2),
    (1024, 600, 40), (28080, 512, 2), (2048, 100, 20),  # more items than SMs: several per CTA
]


@pytest.mark.parametrize("Lq,Lk,H", ATTN_CASES)
def test_attention_matches_oracle(Lq, Lk, H):
    K = _kernels()
    rng = np.random.default_rng(Lq * 7 + Lk * 3 + H)
    q = o_codec.bf16_round(rng.standard_normal((Lq, H, 128)).astype(np.float32))
    k = o_codec.bf16_round(rng.standard_normal((Lk, H, 128)).astype(np.float32))
    v = o_codec.bf16_round(rng.standard_normal((Lk, H, 128)).astype(np.float32))
    out = K.attention(_bf16_gpu(q), _bf16_gpu(k), _bf16_gpu(v))
    torch.cuda.synchronize()
    ref = o_attn.sdpa_numpy(q, k, v)
    assert _rel(_f32(out), ref) <= 1e-2


FP8_CASES = [(130, 300, 2), (4680, 4680, 1), (256, 1000, 12), (5, 517, 3), (200, 700, 40), (2048, 100, 20)]


def _fp8_pages(x2, mode):
    """Codes and scales of a [rows, cols] bf16 page for an attention scale mode."""
    from waveforcing_b200 import _lib as L

    K = _kernels()
    if mode == L.WF_SCALE_NONE:
        return K.kv_quant(x2, L.WF_SCALE_NONE)[0], None
    return K.kv_quant(x2, mode)


@pytest.mark.parametrize("Lq,Lk,H", FP8_CASES)
@pytest.mark.parametrize("mode", ["token", "tensor", "none"])
def test_attention_fp8_kv_matches_oracle(Lq, Lk, H, mode):
    """wf_attn_fwd on e4m3 K/V codes (kv_dtype WF_DTYPE_E4M3) against the fp64
    oracle on the dequantised K/V (common.py:162): <= 1e-2 max relative."""
    from waveforcing_b200 import _lib as L

    K = _kernels()
    m = {"token": L.WF_SCALE_TOKEN, "tensor": L.WF_SCALE_TENSOR, "none": L.WF_SCALE_NONE}[mode]
    rng = np.random.default_rng(Lq * 3 + Lk + H)
    q = o_codec.bf16_round(rng.standard_normal((Lq, H, 128)).astype(np.float32))
    kscale = 1.0 if mode == "none" else 3.0
    k = o_codec.bf16_round((rng.standard_normal((Lk, H, 128)) * kscale).astype(np.float32))
    v = o_codec.bf16_round((rng.standard_normal((Lk, H, 128)) * kscale).astype(np.float32))
    kc, ks = _fp8_pages(_bf16_gpu(k).view(Lk, H * 128), m)
    vc, vs = _fp8_pages(_bf16_gpu(v).view(Lk, H * 128), m)
    out = K.attention_fp8(_bf16_gpu(q)[None], kc.view(1, Lk, H, 128), vc.view(1, Lk, H, 128), ks, vs, m)
    torch.cuda.synchronize()
    per_token = mode == "token"
    if mode == "none":
        kd = o_codec.e4m3_decode(kc.cpu().numpy())
        vd = o_codec.e4m3_decode(vc.cpu().numpy())
    else:
        kd = o_codec.dequant(kc.cpu().numpy(), ks.cpu().numpy() if per_token else ks.item(), per_token)
        vd = o_codec.dequant(vc.cpu().numpy(), vs.cpu().numpy() if per_token else vs.item(), per_token)
    ref = o_attn.sdpa_numpy(q, kd.reshape(Lk, H, 128), vd.reshape(Lk, H, 128))
    assert _rel(_f32(out[0]), ref) <= 1e-2
    from waveforcing_b200 import _lib as L2

    assert L2.status_take() == 0


def test_attention_fp8_strided_batch_and_large_logits():
    """FP8 K/V views into a wider slab, batch 2, and late keys that dominate
    (the lazy O rescale), against fp32 SDPA on the exactly dequantised pages
    (e4m3(code) * scale in f32, common.py:162).  The logits here spread over
    tens of units, so a bf16 rounding of K (as wf_kv_dequant writes it) would
    move them more than the kernel's f16 products do: the reference keeps f32."""
    from waveforcing_b200 import _lib as L

    K = _kernels()
    torch.manual_seed(3)
    B, Lq, Lk, H = 2, 200, 700, 3
    k = torch.randn(B, 900, H, 128, device=DEV)
    k[:, 600:700] *= 6.0
    v = torch.randn(B, 900, H, 128, device=DEV)
    q = (torch.randn(B, Lq, H, 128, device=DEV) * 3).bfloat16()
    kc, ks = K.kv_quant(k.bfloat16().view(-1, H * 128), L.WF_SCALE_TOKEN)
    vc, vs = K.kv_quant(v.bfloat16().view(-1, H * 128), L.WF_SCALE_TOKEN)
    kc, vc = kc.view(B, 900, H, 128), vc.view(B, 900, H, 128)
    ks, vs = ks.view(B, 900), vs.view(B, 900)
    # the first Lk tokens of each batch entry; scales follow the view as [B, Lk]
    out = K.attention_fp8(q, kc[:, :Lk], vc[:, :Lk], ks[:, :Lk].contiguous(), vs[:, :Lk].contiguous(),
                          L.WF_SCALE_TOKEN)
    kd = kc.view(torch.float8_e4m3fn).float() * ks[:, :, None, None]
    vd = vc.view(torch.float8_e4m3fn).float() * vs[:, :, None, None]
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.float().transpose(1, 2), kd[:, :Lk].float().transpose(1, 2), vd[:, :Lk].float().transpose(1, 2))
    ref = ref.transpose(1, 2)
    assert (out.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()
    assert L.status_take() == 0


def test_attention_golden(golden):
    K = _kernels()
    g = golden("sdpa.npz")
    for i in range(int(g["n"])):
        q, k, v = (bits_to_f32(g[f"c{i}_{t}"]) for t in "qkv")
        out = K.attention(_bf16_gpu(q), _bf16_gpu(k), _bf16_gpu(v))
        assert _rel(_f32(out), g[f"c{i}_o"]) <= 1e-2, i


def test_attention_large_logits_rescale():
    """Rows whose max grows late exercise the lazy O rescale path."""
    K = _kernels()
    rng = np.random.default_rng(5)
    Lq, Lk, H = 200, 700, 2
    q = o_codec.bf16_round((rng.standard_normal((Lq, H, 128)) * 3).astype(np.float32))
    k = rng.standard_normal((Lk, H, 128)).astype(np.float32)
    k[600:] *= 6.0  # late keys dominate
    k = o_codec.bf16_round(k)
    v = o_codec.bf16_round(rng.standard_normal((Lk, H, 128)).astype(np.float32))
    out = K.attention(_bf16_gpu(q), _bf16_gpu(k), _bf16_gpu(v))
    assert _rel(_f32(out), o_attn.sdpa_numpy(q, k, v)) <= 1e-2


def test_attention_strided_views_and_batch():
    """Non-contiguous slab prefixes (paged Kb[:active_len]) and batch > 1."""
    K = _kernels()
    torch.manual_seed(0)
    slab_k = torch.randn(2, 900, 3, 128, device=DEV).to(torch.bfloat16)
    slab_v = torch.randn(2, 900, 3, 128, device=DEV).to(torch.bfloat16)
    q = torch.randn(2, 150, 3, 128, device=DEV).to(torch.bfloat16)
    k, v = slab_k[:, :700], slab_v[:, :700]
    out = K.attention(q, k, v)
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.float().transpose(1, 2), k.float().transpose(1, 2), v.float().transpose(1, 2)).transpose(1, 2)
    assert (out.float() - ref).abs().max().item() / ref.abs().max().item() <= 1e-2


def test_attention_rejects_bad_args():
    K = _kernels()
    q = torch.zeros(4, 1, 64, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        K.attention(q, q, q)  # head_dim 64 unsupported
    with pytest.raises(RuntimeError):
        K.attention(q.cpu(), q.cpu(), q.cpu())


# ---------------------------------------------------------------------- codec
def _codec_inputs():
    rng = np.random.default_rng(11)
    yield "normal", rng.standard_normal((300, 1536)).astype(np.float32)
    wide = rng.standard_normal((97, 1536)) * np.exp(rng.standard_normal((97, 1536)) * 4)
    yield "wide", wide.astype(np.float32)
    yield "tiny", (rng.standard_normal((33, 1536)) * 1e-9).astype(np.float32)
    z = rng.standard_normal((17, 5120)).astype(np.float32)
    z[3] = 0
    yield "zero-row", z
    yield "odd-cols", rng.standard_normal((21, 264)).astype(np.float32)


@pytest.mark.parametrize("mode", ["token", "tensor"])
def test_kv_quant_bit_exact(mode):
    K = _kernels()
    from waveforcing_b200._lib import WF_SCALE_TENSOR, WF_SCALE_TOKEN

    for name, x in _codec_inputs():
        xb = o_codec.bf16_round(x)
        if mode == "token":
            ref_c, ref_s = o_codec.quant_per_token(xb)
            codes, scales = K.kv_quant(_bf16_gpu(xb), WF_SCALE_TOKEN)
        else:
            ref_c, ref_s = o_codec.quant_per_tensor(xb)
            codes, scales = K.kv_quant(_bf16_gpu(xb), WF_SCALE_TENSOR)
        assert np.array_equal(codes.cpu().numpy(), ref_c), name
        assert np.array_equal(scales.cpu().numpy().reshape(-1), np.asarray(ref_s, np.float32).reshape(-1)), name


def test_kv_quant_golden_reference_vectors(golden):
    K = _kernels()
    from waveforcing_b200._lib import WF_SCALE_TENSOR

    g = golden("codec_per_tensor.npz")
    for i in range(int(g["n"])):
        x = bits_to_f32(g[f"c{i}_x"])
        x2 = x.reshape(-1, x.shape[-1])
        codes, scales = K.kv_quant(_bf16_gpu(x2), WF_SCALE_TENSOR)
        assert np.array_equal(codes.cpu().numpy().reshape(g[f"c{i}_codes"].shape), g[f"c{i}_codes"]), i
        assert scales.item() == float(g[f"c{i}_scale"]), i


def test_kv_quant_all_bf16_values():
    """Every finite bf16 pattern quantised under a fixed row amax."""
    K = _kernels()
    from waveforcing_b200._lib import WF_SCALE_TOKEN

    b = np.arange(65536, dtype=np.uint32)
    f = o_codec.bf16_from_bits(b)
    f = f[np.isfinite(f)]
    for amax in (1.0, 3.0e4, 7.5e-3, 1e-12):
        vals = np.clip(f, -amax, amax)
        n = (vals.size // 1536) * 1536
        x = vals[:n].reshape(-1, 1536).copy()
        x[:, 0] = amax
        ref_c, ref_s = o_codec.quant_per_token(x)
        codes, scales = K.kv_quant(_bf16_gpu(x), WF_SCALE_TOKEN)
        got = codes.cpu().numpy()
        bad = np.argwhere(got != ref_c)
        assert np.array_equal(scales.cpu().numpy(), ref_s), amax
        assert bad.size == 0, (amax, bad[:4].tolist(), x[tuple(bad[0])], got[tuple(bad[0])], ref_c[tuple(bad[0])])


@pytest.mark.parametrize("mode", ["token", "tensor", "none"])
def test_kv_dequant_bit_exact(mode):
    K = _kernels()
    from waveforcing_b200._lib import WF_SCALE_NONE, WF_SCALE_TENSOR, WF_SCALE_TOKEN

    rng = np.random.default_rng(3)
    x = o_codec.bf16_round(rng.standard_normal((129, 1536)).astype(np.float32) * 5)
    if mode == "token":
        c, s = o_codec.quant_per_token(x)
        ref = o_codec.bf16_round(o_codec.dequant(c, s, True))
        m = WF_SCALE_TOKEN
    elif mode == "tensor":
        c, s = o_codec.quant_per_tensor(x)
        ref = o_codec.bf16_round(o_codec.dequant(c, s, False))
        s = np.array([s], np.float32)
        m = WF_SCALE_TENSOR
    else:
        c = o_codec.cast_scale_free(x)
        s = None
        ref = o_codec.e4m3_decode(c)
        m = WF_SCALE_NONE
    sc = torch.from_numpy(np.asarray(s, np.float32)).to(DEV) if s is not None else None
    out = K.kv_dequant(torch.from_numpy(c).to(DEV), sc, m)
    assert np.array_equal(_f32(out), ref)


def test_kv_quant_publish_fans_out():
    K = _kernels()
    from waveforcing_b200._lib import WF_SCALE_TOKEN

    torch.manual_seed(1)
    k = torch.randn(300, 1536, device=DEV).to(torch.bfloat16)
    v = torch.randn(300, 1536, device=DEV).to(torch.bfloat16) * 3
    ck, sk = K.kv_quant(k, WF_SCALE_TOKEN)
    cv, sv = K.kv_quant(v, WF_SCALE_TOKEN)
    dst = [(torch.empty_like(ck), torch.empty_like(cv), torch.empty_like(sk), torch.empty_like(sv)) for _ in range(3)]
    K.kv_quant_publish(k, v, [d[0].data_ptr() for d in dst], [d[1].data_ptr() for d in dst],
                       [d[2].data_ptr() for d in dst], [d[3].data_ptr() for d in dst])
    for d in dst:
        assert torch.equal(d[0], ck) and torch.equal(d[1], cv)
        assert torch.equal(d[2], sk) and torch.equal(d[3], sv)


@pytest.mark.parametrize("n_dst", [1, 4, 5])
def test_kv_quant_publish_matches_oracle(n_dst):
    """The fused publish against the row-wise restatement, including a row
    with a NaN (non-finite scale path), zero rows, -0 and huge values.  (A
    row holding inf is left out: inf / inf gives a NaN whose sign bit differs
    between x86 and CUDA, so the code byte is platform-defined.)"""
    K = _kernels()
    rng = np.random.default_rng(7 + n_dst)
    k = rng.standard_normal((261, 1536)).astype(np.float32)
    v = (rng.standard_normal((261, 1536)) * np.exp(rng.standard_normal((261, 1536)) * 3)).astype(np.float32)
    k[9, 3] = np.nan
    v[11] = 0.0
    v[12] = -0.0
    v[13, ::7] = -0.0
    k[20] *= 3e37
    k, v = o_codec.bf16_round(k), o_codec.bf16_round(v)
    ref_ck, ref_sk = o_codec.quant_per_token(k)
    ref_cv, ref_sv = o_codec.quant_per_token(v)
    kg, vg = _bf16_gpu(k), _bf16_gpu(v)
    dst = [(torch.empty(261, 1536, dtype=torch.uint8, device=DEV), torch.empty(261, 1536, dtype=torch.uint8, device=DEV),
            torch.empty(261, device=DEV), torch.empty(261, device=DEV)) for _ in range(n_dst)]
    K.kv_quant_publish(kg, vg, [d[0].data_ptr() for d in dst], [d[1].data_ptr() for d in dst],
                       [d[2].data_ptr() for d in dst], [d[3].data_ptr() for d in dst])
    torch.cuda.synchronize()
    for d in dst:
        assert np.array_equal(d[0].cpu().numpy(), ref_ck) and np.array_equal(d[1].cpu().numpy(), ref_cv)
        # scales: equal values (a NaN scale's payload bits are platform-defined)
        assert np.array_equal(d[2].cpu().numpy(), np.asarray(ref_sk, np.float32), equal_nan=True)
        assert np.array_equal(d[3].cpu().numpy(), np.asarray(ref_sv, np.float32), equal_nan=True)


# ----------------------------------------------------------------------- W8A8
@pytest.mark.parametrize("qtype", ["e4m3", "s8"])
@pytest.mark.parametrize("Kd", [256, 1536, 4104, 5120, 8960, 13824])
def test_quantisers_bit_exact(qtype, Kd):
    """Weight and activation quantisers against the oracle; K covers the
    warp-per-row kernel with the row in registers (1536) or read twice (256)
    and the CTA-per-row kernel for wide rows (4104: a ragged last thread;
    5120, 8960, 13824); activations include wide magnitudes, zero rows and -0."""
    K = _kernels()
    from waveforcing_b200._lib import WF_DTYPE_E4M3, WF_DTYPE_S8

    qt = WF_DTYPE_E4M3 if qtype == "e4m3" else WF_DTYPE_S8
    rng = np.random.default_rng(2 + Kd)
    w = o_codec.bf16_round((rng.standard_normal((96, Kd)) * 0.02).astype(np.float32))
    x = rng.standard_normal((70, Kd)) * 2 * np.exp(rng.standard_normal((70, Kd)) * 2)
    x[3] = 0.0
    x[4] = -0.0
    x[5, ::3] = -0.0
    x = o_codec.bf16_round(x.astype(np.float32))
    wq, ws = K.weight_quant(_bf16_gpu(w), qt)
    xq, xs = K.act_quant(_bf16_gpu(x), qt)
    rwq, rws = o_w8a8.quant_weight(w, qtype, per_channel=True)
    rxq, rxs = o_w8a8.quant_act(x, qtype, per_token=True)
    assert np.array_equal(ws.cpu().numpy(), rws)
    assert np.array_equal(xs.cpu().numpy(), rxs)
    assert np.array_equal(wq.cpu().numpy().view(rwq.dtype), rwq)
    assert np.array_equal(xq.cpu().numpy().view(rxq.dtype), rxq)


@pytest.mark.parametrize("qtype", ["e4m3", "s8"])
@pytest.mark.parametrize("M,N,K_", [(128, 256, 128), (300, 512, 384), (4680, 1536, 1536), (77, 96, 256),
                                    (500, 13824, 5120), (300, 5120, 13824),
                                    # M >= 1024 and K >= 4096: CTA-pair tiles (256 x 256); ragged M and N,
                                    # one pair tile, the fc_out shape
                                    (1100, 400, 4096), (1024, 256, 4608), (2049, 1536, 8960)])
def test_gemm_w8a8_matches_oracle(qtype, M, N, K_):
    K = _kernels()
    from waveforcing_b200._lib import WF_DTYPE_E4M3, WF_DTYPE_S8

    qt = WF_DTYPE_E4M3 if qtype == "e4m3" else WF_DTYPE_S8
    rng = np.random.default_rng(M + N + K_)
    w = o_codec.bf16_round((rng.standard_normal((N, K_)) * 0.02).astype(np.float32))
    x = o_codec.bf16_round((rng.standard_normal((M, K_)) * 2).astype(np.float32))
    b = o_codec.bf16_round((rng.standard_normal(N) * 0.1).astype(np.float32))
    wq, ws = K.weight_quant(_bf16_gpu(w), qt)
    xq, xs = K.act_quant(_bf16_gpu(x), qt)
    y = K.gemm_w8a8(xq, xs, wq, ws, _bf16_gpu(b), qt)
    rwq, rws = o_w8a8.quant_weight(w, qtype)
    rxq, rxs = o_w8a8.quant_act(x, qtype)
    ref = o_w8a8.gemm(rxq, rxs, rwq, rws, b, qtype)
    assert _rel(_f32(y), ref) <= 1e-2


_PAIR_SCRIPT = r"""
import sys, numpy as np, torch
from waveforcing_b200 import kernels as K
from waveforcing_b200._lib import WF_DTYPE_E4M3, WF_DTYPE_S8
qt = WF_DTYPE_E4M3 if sys.argv[1] == "e4m3" else WF_DTYPE_S8
M, N, K_ = (int(v) for v in sys.argv[3].split(","))
g = torch.Generator(device="cuda").manual_seed(7)
x = torch.randn(M, K_, device="cuda", generator=g).bfloat16()
w = (torch.randn(N, K_, device="cuda", generator=g) * 0.02).bfloat16()
b = (torch.randn(N, device="cuda", generator=g) * 0.1).bfloat16()
wq, ws = K.weight_quant(w, qt)
xq, xs = K.act_quant(x, qt)
y = K.gemm_w8a8(xq, xs, wq, ws, b, qt)
np.save(sys.argv[2], y.float().cpu().numpy())
"""


@pytest.mark.parametrize("qtype", ["e4m3", "s8"])
@pytest.mark.parametrize("shape", ["3000,4608,1536", "8192,512,8960"])  # m-fastest, n-fastest tile order
def test_gemm_pair_matches_single_cta(qtype, shape, tmp_path):
    """The CTA-pair kernel (WFK_GEMM_PAIR=1) against the one-CTA kernel
    (WFK_GEMM_PAIR=0) on the same inputs, each in its own process: both accumulate every
    output in f32 (s32) over the same k order; outputs agree to one bf16 ulp."""
    import subprocess
    import sys

    outs = []
    for env_pair in ("1", "0"):  # forced on (the shape's K would pick one CTA per tile), then off
        f = tmp_path / f"y{env_pair}.npy"
        env = dict(os.environ, WFK_GEMM_PAIR=env_pair)
        r = subprocess.run([sys.executable, "-c", _PAIR_SCRIPT, qtype, str(f), shape], env=env, capture_output=True,
                           text=True, timeout=300, cwd=ROOT)
        assert r.returncode == 0, r.stderr[-2000:]
        outs.append(np.load(f))
    a, b = outs
    assert np.all(np.isfinite(a)) and np.abs(a).max() > 0
    assert np.all(np.abs(a - b) <= np.abs(b) * 2.0**-7 + 1e-6)


@pytest.mark.parametrize("qtype", ["e4m3", "s8"])
@pytest.mark.parametrize("M_", [600, 1300])
def test_gemm_w8a8_gelu_epilogue(qtype, M_):
    """fc_in + GELU(tanh) in one kernel against the oracle linear followed by
    torch's tanh GELU on the bf16-rounded output (600 and 1300 rows; the
    pair kernel's GELU epilogue is the same code, covered through the
    WFK_GEMM_PAIR test)."""
    K = _kernels()
    from waveforcing_b200._lib import WF_ACT_GELU_TANH, WF_DTYPE_E4M3, WF_DTYPE_S8

    qt = WF_DTYPE_E4M3 if qtype == "e4m3" else WF_DTYPE_S8
    rng = np.random.default_rng(31)
    M, N, K_ = M_, 8960, 1536
    w = o_codec.bf16_round((rng.standard_normal((N, K_)) * 0.02).astype(np.float32))
    x = o_codec.bf16_round((rng.standard_normal((M, K_)) * 2).astype(np.float32))
    b = o_codec.bf16_round((rng.standard_normal(N) * 0.1).astype(np.float32))
    wq, ws = K.weight_quant(_bf16_gpu(w), qt)
    xq, xs = K.act_quant(_bf16_gpu(x), qt)
    y = K.gemm_w8a8(xq, xs, wq, ws, _bf16_gpu(b), qt, activation=WF_ACT_GELU_TANH)
    rwq, rws = o_w8a8.quant_weight(w, qtype)
    rxq, rxs = o_w8a8.quant_act(x, qtype)
    lin = o_codec.bf16_round(o_w8a8.gemm(rxq, rxs, rwq, rws, b, qtype).astype(np.float32))
    ref = torch.nn.functional.gelu(torch.from_numpy(lin).double(), approximate="tanh").numpy()
    assert _rel(_f32(y), ref) <= 1e-2


@pytest.mark.parametrize("qtype", ["e4m3", "s8"])
@pytest.mark.parametrize("Kd", [1536, 8960, 13824])
def test_act_quant_with_gelu_input(qtype, Kd):
    """Per-token quantisation of bf16(GELU_tanh(x)) against the oracle applied
    to the exactly computed GELU.  The kernel evaluates x / (1 + e^(-2u)) with
    ex2.approx and an approximate reciprocal (rcp.approx, or Newton steps on
    the FMA pipe for the wide rows), so a code may differ where the bf16
    rounding of the activation flips: at most 1 in 1000 codes, each by one
    step."""
    K = _kernels()
    from waveforcing_b200._lib import WF_ACT_GELU_TANH, WF_DTYPE_E4M3, WF_DTYPE_S8

    qt = WF_DTYPE_E4M3 if qtype == "e4m3" else WF_DTYPE_S8
    rng = np.random.default_rng(Kd)
    x = o_codec.bf16_round((rng.standard_normal((64, Kd)) * 3).astype(np.float32))
    g = o_codec.bf16_round(torch.nn.functional.gelu(torch.from_numpy(x).double(), approximate="tanh").float().numpy())
    rq, rs = o_w8a8.quant_act(g, qtype)
    xq, xs = K.act_quant(_bf16_gpu(x), qt, activation=WF_ACT_GELU_TANH)
    xs = xs.cpu().numpy()
    assert np.all(np.abs(xs - rs) <= rs * 2.0**-7)
    got = xq.cpu().numpy().view(rq.dtype)
    mism = got != rq
    assert mism.mean() <= 1e-3
    if qtype == "e4m3":
        dg, dr = o_codec.e4m3_decode(got[mism]), o_codec.e4m3_decode(rq[mism])
        assert np.all(np.abs(dg - dr) <= np.maximum(np.abs(dr) * 0.126, 2.0**-9 * 1.001))  # one e4m3 step
    else:
        assert np.all(np.abs(got[mism].astype(np.int32) - rq[mism].astype(np.int32)) <= 1)


def test_gemm_per_tensor_matches_reference_golden(golden):
    """The reference's per-tensor WaveFp8Linear outputs, through our GEMM."""
    K = _kernels()
    from waveforcing_b200._lib import WF_DTYPE_E4M3, WF_SCALE_TENSOR

    g = golden("w8a8_per_tensor.npz")
    for i in range(int(g["n"])):
        x = bits_to_f32(g[f"c{i}_x"])
        M, Kd = x.shape
        if Kd % 16:
            continue
        wq = torch.from_numpy(g[f"c{i}_wq"]).to(DEV)
        ws = torch.tensor([float(g[f"c{i}_ws"])], device=DEV, dtype=torch.float32)
        xq, xs = o_w8a8.quant_act(x, "e4m3", per_token=False)
        b = _bf16_gpu(bits_to_f32(g[f"c{i}_b"])) if f"c{i}_b" in g else None
        y = K.gemm_w8a8(torch.from_numpy(xq).to(DEV), torch.tensor([float(xs)], device=DEV), wq, ws, b,
                        WF_DTYPE_E4M3, WF_SCALE_TENSOR)
        assert _rel(_f32(y), bits_to_f32(g[f"c{i}_y"])) <= 1e-2, i


# ----------------------------------------------------------- context assembly
def test_kv_assemble_segments_match_separate_kernels():
    """Copy, RoPE and dequant segments of one launch against torch copies,
    wf_rope_apply and wf_kv_dequant, into a strided destination."""
    K = _kernels()
    from waveforcing_b200 import _lib as L

    torch.manual_seed(3)
    T, H, D = 300, 3, 128
    HD = H * D
    ku = torch.randn(T, H, D, device=DEV).to(torch.bfloat16)
    kr = torch.randn(2 * T, H, D, device=DEV).to(torch.bfloat16)[::2]  # strided rows
    cos = torch.rand(T, D // 2, device=DEV) * 2 - 1
    sin = torch.rand(T, D // 2, device=DEV) * 2 - 1
    x = torch.randn(T + 17, HD, device=DEV).to(torch.bfloat16)
    codes, scales = K.kv_quant(x, L.WF_SCALE_TOKEN)
    dst = torch.zeros(4 * T, HD + 64, device=DEV, dtype=torch.bfloat16)
    dst_ptr, dst_st = dst.data_ptr(), dst.stride(0)
    segs = [(L.WF_SEG_ROPE, ku.data_ptr(), cos.data_ptr(), sin.data_ptr(), dst_ptr, T, HD, dst_st),
            (L.WF_SEG_COPY, kr.data_ptr(), 0, 0, dst_ptr + T * dst_st * 2, T, kr.stride(0), dst_st),
            (L.WF_SEG_COPY, kr.data_ptr(), 0, 0, dst_ptr + 2 * T * dst_st * 2, 0, kr.stride(0), dst_st),
            (L.WF_SEG_DEQUANT, codes.data_ptr(), scales.data_ptr(), 0, dst_ptr + 2 * T * dst_st * 2, T + 17, HD,
             dst_st)]
    K.kv_assemble(segs, HD, D)
    torch.cuda.synchronize()
    assert torch.equal(dst[:T, :HD], K.rope_apply(ku, cos, sin).reshape(T, HD))
    assert torch.equal(dst[T:2 * T, :HD], kr.reshape(T, HD))
    assert torch.equal(dst[2 * T:3 * T + 17, :HD], K.kv_dequant(codes, scales, L.WF_SCALE_TOKEN))
    assert torch.count_nonzero(dst[:, HD:]) == 0 and torch.count_nonzero(dst[3 * T + 17:]) == 0
    with pytest.raises(RuntimeError):
        K.kv_assemble([(7, ku.data_ptr(), 0, 0, dst_ptr, T, HD, dst_st)], HD, D)
    with pytest.raises(RuntimeError):
        K.kv_assemble([(L.WF_SEG_ROPE, ku.data_ptr(), 0, 0, dst_ptr, T, HD, dst_st)], HD, D)


# ----------------------------------------------------------------------- RoPE
def test_rope_matches_oracle(golden):
    K = _kernels()
    g = golden("rope.npz")
    for i in range(int(g["n"])):
        f, h, w, sf, n = [int(v) for v in g[f"c{i}_meta"]]
        x = bits_to_f32(g[f"c{i}_x"])
        cos, sin = o_rope.cos_sin_tables(f, h, w, sf)
        y = K.rope_apply(_bf16_gpu(x), torch.from_numpy(cos).to(DEV), torch.from_numpy(sin).to(DEV))
        ref = bits_to_f32(g[f"c{i}_y"])
        ulp = np.abs(ref) * 2.0**-7 + 1e-30
        assert np.all(np.abs(_f32(y) - ref) <= 2 * ulp + 1e-6), i


# ------------------------------------------------------------- bounded waits
def test_wait_flag_returns_when_set_and_times_out_when_not():
    from waveforcing_b200 import _lib as L

    lib = L.lib()
    s = torch.cuda.current_stream().cuda_stream
    flag = torch.zeros(4, dtype=torch.int32, device=DEV)
    tout = torch.zeros(2, dtype=torch.int32, device=DEV)
    L.status_take()
    # already satisfied (GEQ): returns immediately
    flag[0] = 7
    L.check(lib.wf_wait_flag(flag.data_ptr(), 7, 200_000_000, tout.data_ptr(), s), "wf_wait_flag")
    torch.cuda.synchronize()
    assert tout[0].item() == 0 and L.status_take() == 0
    # never written: gives up after ~0.2 s, reports it, stream stays usable
    L.check(lib.wf_wait_flag(flag[1:].data_ptr(), 1, 200_000_000, tout[1:].data_ptr(), s), "wf_wait_flag")
    torch.cuda.synchronize()
    assert tout[1].item() == 1
    assert L.status_take() & (1 << 6)
    assert (flag + 1).sum().item() == 7 + 4


def test_stream_write_then_wait_value():
    from waveforcing_b200 import _lib as L

    lib = L.lib()
    s = torch.cuda.current_stream().cuda_stream
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    L.check(lib.wf_stream_write_u32(s, flag.data_ptr(), 5), "write")
    L.check(lib.wf_stream_wait_u32(s, flag.data_ptr(), 5), "wait")
    torch.cuda.synchronize()
    assert flag.item() == 5


def test_publish_payload_then_flag():
    from waveforcing_b200 import _lib as L

    lib = L.lib()
    s = torch.cuda.current_stream().cuda_stream
    src = torch.arange(4096, dtype=torch.int32, device=DEV)
    dsts = [torch.zeros_like(src) for _ in range(2)]
    flags = torch.zeros(2, dtype=torch.int32, device=DEV)
    L.check(lib.wf_publish(L.ptr_array([d.data_ptr() for d in dsts]), src.data_ptr(), src.numel() * 4,
                           L.ptr_array([flags[i:].data_ptr() for i in range(2)]), 2, 9, s), "publish")
    torch.cuda.synchronize()
    assert all(torch.equal(d, src) for d in dsts) and flags.tolist() == [9, 9]


def test_ipc_export_offset():
    from waveforcing_b200 import _lib as L
    import ctypes as C

    base = torch.empty(1 << 20, dtype=torch.uint8, device=DEV)
    view = base[4096:]
    h = (C.c_uint8 * 64)()
    off = C.c_uint64()
    L.check(L.lib().wf_ipc_export(view.data_ptr(), h, C.byref(off)), "export")
    h0 = (C.c_uint8 * 64)()
    off0 = C.c_uint64()
    L.check(L.lib().wf_ipc_export(base.data_ptr(), h0, C.byref(off0)), "export")
    assert off.value - off0.value == 4096


# ------------------------------------------------------- fused block rows
@pytest.mark.parametrize("dim", [256, 1536, 5120])
def test_fused_rows_match_torch(dim):
    import torch.nn.functional as F

    K = _kernels()
    torch.manual_seed(dim)
    S, T, hd = 3, 40, 128
    x = torch.randn(S * T, dim, device=DEV).bfloat16()
    e = torch.randn(S, 6, dim, device=DEV) * 0.3
    # LayerNorm + modulation
    out = K.ln_modulate(x, e[:, 0], e[:, 1], T, 1e-6)
    ref = (F.layer_norm(x.float().view(S, T, dim), (dim,), eps=1e-6) * (1 + e[:, 1][:, None]) + e[:, 0][:, None])
    assert (out.float().view(S, T, dim) - ref).abs().max().item() <= 0.02 * ref.abs().max().item()
    # gated residual
    y = torch.randn(S * T, dim, device=DEV).bfloat16()
    ref = (x.float().view(S, T, dim) + y.float().view(S, T, dim) * e[:, 2][:, None]).bfloat16().float()
    got = K.gate_residual(x.clone(), y, e[:, 2], T).float().view(S, T, dim)
    assert (got - ref).abs().max().item() <= 0.01 * ref.abs().max().item()
    # RMSNorm (q, k) + RoPE from a fused QKV matrix
    qkv = torch.randn(S * T, 3 * dim, device=DEV).bfloat16()
    wq = (torch.randn(dim, device=DEV) * 0.5 + 1).bfloat16()
    wk = (torch.randn(dim, device=DEV) * 0.5 + 1).bfloat16()
    cos = torch.rand(S * T, hd // 2, device=DEV) * 2 - 1
    sin = torch.sqrt(1 - cos * cos)
    q, k, ku = K.qk_norm_rope(qkv, dim, wq, wk, cos, sin, hd, T, 1e-6)

    def rms(t, w):
        tf = t.float()
        return (tf * torch.rsqrt(tf.pow(2).mean(-1, keepdim=True) + 1e-6)).bfloat16() * w

    def rope(t):
        t = t.float().view(S * T, dim // hd, hd // 2, 2)
        re, im = t[..., 0], t[..., 1]
        c, s = cos[:, None, :], sin[:, None, :]
        return torch.stack([re * c - im * s, re * s + im * c], -1).view(S * T, dim)

    kn = rms(qkv[:, dim:2 * dim], wk)
    assert torch.equal(ku, kn)
    for got, want in ((q, rope(rms(qkv[:, :dim], wq))), (k, rope(kn))):
        assert (got.float() - want).abs().max().item() <= 0.01 * want.abs().max().item()
    # plain RMSNorm
    r = K.rms_norm(x, wq, 1e-6)
    assert (r.float() - rms(x, wq).float()).abs().max().item() <= 0.01 * r.float().abs().max().item()


@pytest.mark.parametrize("dim", [256, 1536, 3072, 5120])
@pytest.mark.parametrize("qtype", ["e4m3", "s8"])
def test_ln_modulate_quant_matches_separate_passes(dim, qtype):
    """wf_ln_modulate_quant: codes and scales bit-identical to wf_act_quant on
    wf_ln_modulate's bf16 output (e4m3 and int8; rows of three stages, one
    of them all zeros)."""
    from waveforcing_b200 import _lib as L

    K = _kernels()
    qt = L.WF_DTYPE_E4M3 if qtype == "e4m3" else L.WF_DTYPE_S8
    torch.manual_seed(dim + 7)
    S, T = 3, 40
    x = (torch.randn(S * T, dim, device=DEV) * torch.rand(S * T, 1, device=DEV) * 5).bfloat16()
    x[17] = 0
    e = torch.randn(S, 6, dim, device=DEV) * 0.3
    xq, xs = K.ln_modulate_quant(x, e[:, 0], e[:, 1], T, 1e-6, qt)
    h = K.ln_modulate(x, e[:, 0], e[:, 1], T, 1e-6)
    rq, rs = K.act_quant(h, qt)
    assert torch.equal(xq, rq) and torch.equal(xs, rs)
    assert L.status_take() == 0


@pytest.mark.parametrize("dim", [256, 1536, 5120])
@pytest.mark.parametrize("mode", ["quant", "ln", "ln_quant_e4m3", "ln_quant_s8"])
def test_gate_residual_then_matches_two_launches(dim, mode):
    """wf_gate_residual_then: the updated x and its output (per-token codes and
    scales, LN-modulate, or LN-modulate quantised) bit-identical to
    wf_gate_residual followed by wf_act_quant / wf_ln_modulate /
    wf_ln_modulate_quant; per-stage gates and modulation over three stages."""
    from waveforcing_b200 import _lib as L

    K = _kernels()
    torch.manual_seed(dim + 11)
    S, T = 3, 40
    x0 = (torch.randn(S * T, dim, device=DEV) * 3).bfloat16()
    y = (torch.randn(S * T, dim, device=DEV) * torch.rand(S * T, 1, device=DEV) * 2).bfloat16()
    x0[9] = 0
    y[9] = 0  # an all-zero row after the residual
    g = torch.randn(S, dim, device=DEV) * 0.5
    e = torch.randn(S, 6, dim, device=DEV) * 0.3
    qt = L.WF_DTYPE_S8 if mode.endswith("s8") else L.WF_DTYPE_E4M3
    xa = x0.clone()
    K.gate_residual(xa, y, g, T)
    xb = x0.clone()
    if mode == "quant":
        got = K.gate_residual_then(xb, y, g, T, quant=True, qtype=qt)
        want = K.act_quant(xa, qt)
    elif mode == "ln":
        got = (K.gate_residual_then(xb, y, g, T, e[:, 3], e[:, 4], T, 1e-6),)
        want = (K.ln_modulate(xa, e[:, 3], e[:, 4], T, 1e-6),)
    else:
        got = K.gate_residual_then(xb, y, g, T, e[:, 0], e[:, 1], T, 1e-6, quant=True, qtype=qt)
        want = K.ln_modulate_quant(xa, e[:, 0], e[:, 1], T, 1e-6, qt)
    assert torch.equal(xa, xb)
    for a, b in zip(got, want):
        assert torch.equal(a, b)
    assert L.status_take() == 0


@pytest.mark.parametrize("dim", [256, 1536, 5120])
def test_qk_norm_rope_publish_matches_separate_passes(dim):
    """wf_qk_norm_rope_publish: q, k and the un-roped k bit-identical to
    wf_qk_norm_rope; every destination's codes and scales bit-identical to
    wf_kv_quant_publish on the same K and V rows and to the oracle's per-token
    codec (the torch-CPU form); stages without destinations publish nothing."""
    K = _kernels()
    torch.manual_seed(dim + 1)
    S, T, hd = 3, 40, 128
    qkv = (torch.randn(S * T, 3 * dim, device=DEV) * torch.rand(S * T, 1, device=DEV) * 4).bfloat16()
    qkv[5, 2 * dim:] = 0  # an all-zero V row (the scale clamps to bf16(1e-8))
    wq = (torch.randn(dim, device=DEV) * 0.5 + 1).bfloat16()
    wk = (torch.randn(dim, device=DEV) * 0.5 + 1).bfloat16()
    cos = torch.rand(S * T, hd // 2, device=DEV) * 2 - 1
    sin = torch.sqrt(1 - cos * cos)
    ndst = [2, 0, 5]
    slots = [[(torch.full((T, dim), 0xAB, device=DEV, dtype=torch.uint8),
               torch.full((T, dim), 0xAB, device=DEV, dtype=torch.uint8),
               torch.full((T,), -7.0, device=DEV), torch.full((T,), -7.0, device=DEV)) for _ in range(n)]
             for n in ndst]
    pub = [[tuple(t.data_ptr() for t in d) for d in st] for st in slots]
    q, k, ku = K.qk_norm_rope_publish(qkv, dim, wq, wk, cos, sin, hd, T, 1e-6, pub)
    q0, k0, ku0 = K.qk_norm_rope(qkv, dim, wq, wk, cos, sin, hd, T, 1e-6)
    assert torch.equal(q, q0) and torch.equal(k, k0) and torch.equal(ku, ku0)
    for s, st in enumerate(slots):
        rows = slice(s * T, (s + 1) * T)
        if not st:
            continue
        ref = [(torch.empty(T, dim, device=DEV, dtype=torch.uint8), torch.empty(T, dim, device=DEV, dtype=torch.uint8),
                torch.empty(T, device=DEV), torch.empty(T, device=DEV))]
        K.kv_quant_publish(k0[rows], qkv[rows, 2 * dim:], *[[t.data_ptr()] for t in ref[0]])
        ok_c, ok_s = o_codec.quant_per_token_torch(k0[rows].cpu())
        ov_c, ov_s = o_codec.quant_per_token_torch(qkv[rows, 2 * dim:].cpu())
        for ck, cv, sk, sv in st:
            assert torch.equal(ck, ref[0][0]) and torch.equal(cv, ref[0][1]), s
            assert torch.equal(sk, ref[0][2]) and torch.equal(sv, ref[0][3]), s
            assert torch.equal(ck.cpu(), ok_c) and torch.equal(sk.cpu(), ok_s), s
            assert torch.equal(cv.cpu(), ov_c) and torch.equal(sv.cpu(), ov_s), s
    assert K.LAUNCHES[0] > 0


def test_softmax_exp2_paths_error_bounds():
    """The FMA-pipe polynomial 2^x used for part of the softmax stays within
    1e-4 relative error of exp2 on the range the kernel feeds it ([-125, 8]),
    the same order as the MUFU ex2.approx path it replaces."""
    from waveforcing_b200 import _lib as L

    x = torch.cat([torch.linspace(-125.0, 8.0, 400001, device=DEV), torch.tensor([-0.5, 0.5, 0.0, 7.99], device=DEV)])
    yp = torch.empty_like(x)
    ym = torch.empty_like(x)
    L.check(L.lib().wf_selftest_exp2(x.data_ptr(), yp.data_ptr(), ym.data_ptr(), x.numel(),
                                     torch.cuda.current_stream().cuda_stream), "wf_selftest_exp2")
    ref = torch.exp2(x.double())
    rel_p = ((yp.double() - ref).abs() / ref).max().item()
    rel_m = ((ym.double() - ref).abs() / ref).max().item()
    assert rel_p < 1e-4, rel_p
    assert rel_m < 1e-4, rel_m
    # masked scores (-inf) map to a tiny positive normal value, not NaN
    z = torch.tensor([float("-inf"), -1000.0], device=DEV)
    L.check(L.lib().wf_selftest_exp2(z.data_ptr(), yp.data_ptr(), ym.data_ptr(), 2,
                                     torch.cuda.current_stream().cuda_stream), "wf_selftest_exp2")
    assert torch.all(yp[:2] >= 0) and torch.all(yp[:2] < 1e-37)


def test_kv_scale_free_cast_bit_exact():
    """onesided.py:152 cast (no scale) over every finite bf16 pattern, NaN-producing range included."""
    K = _kernels()
    from waveforcing_b200._lib import WF_SCALE_NONE

    b = np.arange(65536, dtype=np.uint32)
    f = o_codec.bf16_from_bits(b)
    f = f[np.isfinite(f)]
    n = (f.size // 1536) * 1536
    x = f[:n].reshape(-1, 1536)
    codes, _ = K.kv_quant(_bf16_gpu(x), WF_SCALE_NONE)
    ref = o_codec.cast_scale_free(x)
    got = codes.cpu().numpy()
    nan = (ref & 0x7F) == 0x7F
    assert np.array_equal(got[~nan], ref[~nan])
    assert np.all((got[nan] & 0x7F) == 0x7F)
