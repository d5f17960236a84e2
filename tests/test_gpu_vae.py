"""Streaming VAE decode on a B200: the bf16 channels-last GPU decoder against
the f32 CPU decoder with the same weights, and chunked GPU pushes against the
frame-by-frame GPU decode.  The decoder is a library path (cuDNN convolutions,
torch SDPA); parity of its arithmetic with the reference's Wan2.1 decoder is
pinned on CPU in tests/test_vae.py."""

import pytest
import torch

from waveforcing_b200.pipelines import vae as V

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

CFG = V.VAEConfig(dim=32, z_dim=16)


def _cos(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float(torch.nn.functional.cosine_similarity(a, b, dim=0))


def test_gpu_bf16_decode_matches_cpu_f32():
    z = torch.randn(CFG.z_dim, 4, 12, 20, generator=torch.Generator().manual_seed(1))
    cpu = V.VAEDecoder.random(CFG, seed=7)
    want = V.decode_framewise(cpu, z)
    gpu = V.VAEDecoder.random(CFG, seed=7).for_gpu("cuda")
    s = V.DecodeStream(gpu)
    got = torch.cat([s.push(z[:, :3].cuda()), s.push(z[:, 3:].cuda())], 1).float().cpu()
    assert tuple(got.shape) == tuple(want.shape) == (3, 13, 96, 160)
    assert _cos(got, want) >= 0.999
    assert float((got - want).abs().max()) <= 0.1


def test_gpu_chunked_equals_framewise():
    z = torch.randn(CFG.z_dim, 7, 12, 20, generator=torch.Generator().manual_seed(2)).cuda()
    dec = V.VAEDecoder.random(CFG, seed=3).for_gpu("cuda")
    want = V.decode_framewise(dec, z).float()
    s = V.DecodeStream(dec)
    got = torch.cat([s.push(z[:, a:b]) for a, b in ((0, 3), (3, 6), (6, 7))], 1).float()
    assert tuple(got.shape) == (3, 25, 96, 160)
    assert _cos(got, want) >= 0.9999


@pytest.mark.parametrize("C", [16, 96, 192, 384])
@pytest.mark.parametrize("silu", [False, True])
def test_channel_rmsnorm_matches_f32(C, silu):
    """wf_channel_rmsnorm against normalize * sqrt(C) * gamma (+ SiLU) in f32 on
    the bf16 inputs: within one bf16 rounding; a zero row stays zero."""
    from waveforcing_b200 import kernels

    g = torch.Generator(device="cuda").manual_seed(C)
    x = (torch.randn(3, 5, 7, 9, C, device="cuda", generator=g) * 4).bfloat16()
    x[0, 0, 0, 0] = 0
    gamma = (1 + 0.2 * torch.randn(C, device="cuda", generator=g)).bfloat16()
    got = kernels.channel_rmsnorm(x, gamma, silu).float()
    xf = x.float()
    ref = torch.nn.functional.normalize(xf, dim=-1) * C ** 0.5 * gamma.float()
    if silu:
        ref = torch.nn.functional.silu(ref)
    assert torch.all((got - ref).abs() <= ref.abs() * 2.0**-7 + 1e-3)
    assert torch.all(got[0, 0, 0, 0] == 0)


def test_interleave_time2_matches_reference_reshape():
    """wf_interleave_time2 against the reference's view/stack of the temporal
    conv output (vae.py:127-131): frame 2i from channels [0, C), 2i + 1 from
    [C, 2C)."""
    from waveforcing_b200 import kernels

    b, c, t, h, w = 1, 24, 3, 5, 7
    y = torch.randn(b, 2 * c, t, h, w, device="cuda").bfloat16().contiguous(memory_format=torch.channels_last_3d)
    got = kernels.interleave_time2(y)
    v = y.view(b, 2, c, t, h, w)
    want = torch.stack((v[:, 0], v[:, 1]), 3).reshape(b, c, 2 * t, h, w)
    assert got.is_contiguous(memory_format=torch.channels_last_3d)
    assert torch.equal(got, want)


@pytest.mark.parametrize("with_res", [False, True])
def test_channel_bias_add_matches_torch(with_res):
    """wf_channel_bias_add against torch's bias add and skip add in bf16
    (each sum rounded), bit for bit, in place."""
    from waveforcing_b200 import kernels

    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(1, 96, 3, 10, 12, device="cuda", generator=g).bfloat16()
    x = x.contiguous(memory_format=torch.channels_last_3d)
    b = torch.randn(96, device="cuda", generator=g).bfloat16()
    r = torch.randn(1, 96, 3, 10, 12, device="cuda", generator=g).bfloat16().contiguous(
        memory_format=torch.channels_last_3d)
    want = x + b.view(1, -1, 1, 1, 1)
    if with_res:
        want = want + r
    got = kernels.channel_bias_add(x.clone(memory_format=torch.channels_last_3d), b, r if with_res else None)
    assert torch.equal(got, want)


def test_upsample2x_nearest_matches_interpolate():
    from waveforcing_b200 import kernels

    f = torch.randn(5, 48, 7, 9, device="cuda").bfloat16().contiguous(memory_format=torch.channels_last)
    got = kernels.upsample2x_nearest(f)
    want = torch.nn.functional.interpolate(f, scale_factor=2.0, mode="nearest")
    assert torch.equal(got, want)
