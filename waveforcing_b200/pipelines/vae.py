"""Streaming decode of finished latent chunks by a Wan2.1-shaped VAE decoder.

The reference turns the store rank's finished chunks into pixels in one of two
ways (wave_rt/pipelines/vae.py):
  * serially at the end of the run (``finalize_on_store`` :210-258, through
    the backend's decode);
  * frame by frame in a pipeline of VAE processes on the spare GPUs
    (``vae_stage`` :42-207): the decoder's layers are cut into contiguous
    groups, one group per process, and each latent frame's activations pass
    from group to group with NCCL send/recv.

Both drive the Wan2.1 VAE decoder (naive_rt/rolling_forcing/wan/modules/
vae.py, ``WanVAE_.decode`` :612-637 over ``Decoder3d`` :418-531), which is
causal in time.  Every 3-D convolution sees its input padded by two zero
frames on the left, and a stream carries those two frames from call to call
(the reference's ``feat_cache``).  The first latent frame skips the temporal
upsampling convolutions ('Rep', :96-131), so F latent frames become 1 + 4 (F - 1)
pixel frames.

This module restates that decoder for the wavefront's chunks:
  * ``VAEDecoder`` holds the weights (random-init; there are no checkpoints)
    as a flat list of units, the granularity at which a pipeline cuts it.
  * ``DecodeStream`` keeps the per-unit causal state of one video.  It decodes
    a chunk's frames as they arrive: frame 0 alone, any later frames
    together, since every operation is causal or per frame.
  * ``VAEPipelineStage`` runs a contiguous group of units on one rank and
    hands activations to the next rank (the reference's ``vae_stage``).
    ``partition_units`` balances the groups by FLOPs.

Layout: NCDHW tensors in bf16 on the GPU, stored channels-last (NDHWC) all
the way through, for cuDNN's implicit-GEMM convolutions.  The convolutions
run on cuDNN and the attention on torch SDPA (library calls); the channel
RMSNorm + SiLU is a libwfk kernel.  The decoder sits outside the DiT hot path
and counts only for FPS with VAE.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from waveforcing_b200 import kernels


@dataclass(frozen=True)
class VAEConfig:
    """Decoder shape (naive_rt/rolling_forcing/wan/modules/vae.py:418-470 and
    the Wan2.1 VAE's construction: base width 96, z 16)."""

    dim: int = 96
    z_dim: int = 16
    dim_mult: tuple = (1, 2, 4, 4)
    num_res_blocks: int = 2
    temporal_upsample: tuple = (False, True, True)  # reversed encoder downsampling (:565)

    @property
    def widths(self) -> list[int]:
        return [self.dim * m for m in (self.dim_mult[-1],) + tuple(reversed(self.dim_mult))]


# ------------------------------------------------------------------ layers
class _CausalConv(nn.Module):
    """Convolution causal in time with kernel (kt, kh, kw) and spatial
    padding (kh // 2, kw // 2).  A stream carries the last kt - 1 input frames,
    starting from zeros, so calls over consecutive frame groups equal one call
    over the whole sequence with kt - 1 zero frames in front."""

    def __init__(self, cin: int, cout: int, k) -> None:
        super().__init__()
        self.k = (k, k, k) if isinstance(k, int) else tuple(k)
        self.weight = nn.Parameter(torch.empty(cout, cin, *self.k))
        self.bias = nn.Parameter(torch.empty(cout))

    def forward(self, x: torch.Tensor, state: dict, key: str) -> torch.Tensor:
        kt = self.k[0]
        if kt > 1:
            prev = state.get(key)
            if prev is None:
                prev = _like_layout(x, torch.zeros((x.shape[0], x.shape[1], kt - 1) + tuple(x.shape[3:]),
                                                   dtype=x.dtype, device=x.device))
            x = _like_layout(prev, torch.cat([prev, x], 2))
            state[key] = x[:, :, -(kt - 1):].clone()
        return self._conv(x)

    def run_buffer(self, buf: torch.Tensor, state: dict, key: str, res: torch.Tensor | None = None) -> torch.Tensor:
        """The same convolution on an input that already carries the stream's
        kt - 1 frames in front (``_RMSNorm.into_causal``): no concatenation.
        ``res`` is added to the result (the residual block's skip)."""
        p = self.k[0] - 1
        state[key] = buf[:, :, -p:].clone()
        return self._conv(buf, res)

    def _conv(self, x: torch.Tensor, res: torch.Tensor | None = None) -> torch.Tensor:
        pad = (0, self.k[1] // 2, self.k[2] // 2)
        if x.is_cuda and self.weight.shape[0] % 8 == 0:
            # cuDNN leaves a 3-D convolution's bias to a strided broadcast add;
            # one libwfk pass adds it, and the skip, on channels-last rows
            y = _like_layout(x, F.conv3d(x, self.weight, None, padding=pad))
            return kernels.channel_bias_add(y, self.bias, _like_layout(y, res) if res is not None else None, out=y)
        y = F.conv3d(x, self.weight, self.bias, padding=pad)
        return y + res if res is not None else y


def _like_layout(ref: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
    """On the GPU every activation stays channels-last (NDHWC): a tensor in
    another layout reaching a convolution is converted by a strided copy of
    the whole activation, which cost three quarters of the decode time."""
    if t.is_cuda and t.dim() == 5 and not t.is_contiguous(memory_format=torch.channels_last_3d):
        return t.contiguous(memory_format=torch.channels_last_3d)
    return t


class _RMSNorm(nn.Module):
    """L2-normalise over channels, times sqrt(C) and a per-channel gain
    (RMS_norm, vae.py:39-54), optionally followed by SiLU.  On the GPU
    (channels-last bf16) one libwfk kernel does both (wf_channel_rmsnorm):
    torch's normalize on channels-last activations runs as strided
    elementwise passes, three quarters of the decoder's time."""

    def __init__(self, dim: int) -> None:
        super().__init__()
        self.gain = nn.Parameter(torch.ones(dim))
        self.scale = dim ** 0.5

    def forward(self, x: torch.Tensor, silu: bool = False) -> torch.Tensor:
        if x.is_cuda:
            return _channel_rows(x, lambda r: kernels.channel_rmsnorm(r, self.gain, silu))
        g = self.gain.view((1, -1) + (1,) * (x.dim() - 2))
        y = F.normalize(x, dim=1) * self.scale * g
        return F.silu(y) if silu else y


    def into_causal(self, x: torch.Tensor, silu: bool, conv: "_CausalConv", state: dict, key: str) -> torch.Tensor:
        """GPU, batch 1: norm (+ SiLU) of x written straight into the input
        buffer of the causal ``conv`` that follows, behind the kt - 1 frames the
        stream carries for it (``conv.run_buffer``), so the convolution input is
        never concatenated."""
        p = conv.k[0] - 1
        b, c, t, h, w = x.shape
        buf = torch.empty((b, t + p, h, w, c), device=x.device, dtype=x.dtype)
        prev = state.get(key)
        if prev is None:
            buf[:, :p].zero_()
        else:
            buf[:, :p].copy_(prev.permute(0, 2, 3, 4, 1))
        rows = x.permute(0, 2, 3, 4, 1)
        if not rows.is_contiguous():
            rows = rows.contiguous()
        kernels.channel_rmsnorm(rows, self.gain, silu, out=buf[:, p:])
        return buf.permute(0, 4, 1, 2, 3)


def _channel_rows(x: torch.Tensor, fn) -> torch.Tensor:
    """Apply a row op over the channels of an NC... tensor stored channels-last
    (the channel rows contiguous) and return the result in the same layout."""
    nd = x.dim()
    perm = (0,) + tuple(range(2, nd)) + (1,)
    rows = x.permute(*perm)
    if not rows.is_contiguous():
        rows = rows.contiguous()
    out = fn(rows)
    inv = (0, nd - 1) + tuple(range(1, nd - 1))
    return out.permute(*inv)


class _ResBlock(nn.Module):
    """norm, SiLU, 3x3x3 causal conv, norm, SiLU, 3x3x3 causal conv, plus a
    1x1x1 projection of the input when the width changes (vae.py:178-214)."""

    def __init__(self, cin: int, cout: int) -> None:
        super().__init__()
        self.n1, self.c1 = _RMSNorm(cin), _CausalConv(cin, cout, 3)
        self.n2, self.c2 = _RMSNorm(cout), _CausalConv(cout, cout, 3)
        self.short = _CausalConv(cin, cout, 1) if cin != cout else None

    def forward(self, x, state, key):
        h = self.short(x, state, key + ".s") if self.short is not None else x
        if x.is_cuda and x.shape[0] == 1:
            y = self.c1.run_buffer(self.n1.into_causal(x, True, self.c1, state, key + ".c1"), state, key + ".c1")
            return self.c2.run_buffer(self.n2.into_causal(y, True, self.c2, state, key + ".c2"), state, key + ".c2",
                                      res=h)
        else:
            y = self.c1(self.n1(x, silu=True), state, key + ".c1")
            y = self.c2(self.n2(y, silu=True), state, key + ".c2")
        return y + h


class _FrameAttention(nn.Module):
    """Single-head self-attention over the H x W positions of each frame,
    residual (vae.py:217-258)."""

    def __init__(self, dim: int) -> None:
        super().__init__()
        self.norm = _RMSNorm(dim)
        self.qkv = nn.Parameter(torch.empty(3 * dim, dim))
        self.qkv_b = nn.Parameter(torch.empty(3 * dim))
        self.proj = nn.Parameter(torch.empty(dim, dim))
        self.proj_b = nn.Parameter(torch.empty(dim))

    def forward(self, x, state, key):
        b, c, t, h, w = x.shape
        f = x.permute(0, 2, 3, 4, 1).reshape(b * t, h * w, c)  # tokens of each frame
        if f.is_cuda:
            n = kernels.channel_rmsnorm(f.contiguous(), self.norm.gain, False)
        else:
            n = F.normalize(f, dim=-1) * self.norm.scale * self.norm.gain
        q, k, v = F.linear(n, self.qkv, self.qkv_b).chunk(3, dim=-1)
        o = F.scaled_dot_product_attention(q[:, None], k[:, None], v[:, None])[:, 0]
        o = F.linear(o, self.proj, self.proj_b)
        return x + o.reshape(b, t, h, w, c).permute(0, 4, 1, 2, 3)


class _Upsample(nn.Module):
    """x2 in H and W (nearest, then a 3x3 conv halving the width); with
    ``temporal``, first x2 in time: a (3, 1, 1) causal conv to twice the width
    whose two halves become frames 2i and 2i + 1 (vae.py:62-139).  The
    stream's first call bypasses the temporal conv; its causal state then
    starts from zeros at the second call."""

    def __init__(self, dim: int, temporal: bool) -> None:
        super().__init__()
        self.temporal = temporal
        self.tconv = _CausalConv(dim, 2 * dim, (3, 1, 1)) if temporal else None
        self.conv_w = nn.Parameter(torch.empty(dim // 2, dim, 3, 3))
        self.conv_b = nn.Parameter(torch.empty(dim // 2))

    def forward(self, x, state, key):
        if self.temporal:
            if state.get(key + ".seen"):
                b, c, t, h, w = x.shape
                y = self.tconv(x, state, key + ".t")  # [b, 2c, t, h, w]
                if y.is_cuda:
                    # channels-last: frame i's two channel halves become frames
                    # 2i, 2i+1 in one vectorised pass (wf_interleave_time2)
                    x = kernels.interleave_time2(_like_layout(y, y))
                else:
                    x = y.view(b, 2, c, t, h, w).permute(0, 2, 3, 1, 4, 5).reshape(b, c, 2 * t, h, w)
            else:
                state[key + ".seen"] = True
        b, c, t, h, w = x.shape
        f = x.transpose(1, 2).reshape(b * t, c, h, w)
        if f.is_cuda and c % 8 == 0 and (c // 2) % 8 == 0:
            f = kernels.upsample2x_nearest(f.contiguous(memory_format=torch.channels_last))
            f = F.conv2d(f, self.conv_w, None, padding=1).contiguous(memory_format=torch.channels_last)
            f = kernels.channel_bias_add(f, self.conv_b, out=f)
        else:
            f = F.interpolate(f, scale_factor=2.0, mode="nearest")
            f = F.conv2d(f, self.conv_w, self.conv_b, padding=1)
        return f.reshape(b, t, c // 2, 2 * h, 2 * w).transpose(1, 2)


class _Input(nn.Module):
    """Latent de-normalisation z / std + mean, the VAE's 1x1x1 conv2 and the
    decoder's first 3x3x3 causal conv (vae.py:612-620, :476-489)."""

    def __init__(self, z_dim: int, width: int) -> None:
        super().__init__()
        self.mean = nn.Parameter(torch.zeros(z_dim))
        self.inv_std = nn.Parameter(torch.ones(z_dim))
        self.pre = _CausalConv(z_dim, z_dim, 1)
        self.conv = _CausalConv(z_dim, width, 3)

    def forward(self, z, state, key):
        v = (1, -1, 1, 1, 1)
        x = z / self.inv_std.view(v) + self.mean.view(v)
        return self.conv(self.pre(x, state, key + ".pre"), state, key + ".conv")


class _Head(nn.Module):
    """norm, SiLU, 3x3x3 causal conv to RGB, clamped to [-1, 1]
    (vae.py:466-470, wave_rt/pipelines/vae.py:167)."""

    def __init__(self, dim: int) -> None:
        super().__init__()
        self.norm = _RMSNorm(dim)
        self.conv = _CausalConv(dim, 3, 3)

    def forward(self, x, state, key):
        if x.is_cuda and x.shape[0] == 1:
            y = self.conv.run_buffer(self.norm.into_causal(x, True, self.conv, state, key + ".conv"), state,
                                     key + ".conv")
        else:
            y = self.conv(self.norm(x, silu=True), state, key + ".conv")
        return y.clamp(-1, 1)


# ----------------------------------------------------------------- decoder
class VAEDecoder(nn.Module):
    """The decoder as an ordered list of units (input, middle, upsampling
    stages, head); ``units[i](x, state, name)`` maps activations to
    activations, with causal state kept in the caller's ``state`` dict."""

    def __init__(self, cfg: VAEConfig = VAEConfig()) -> None:
        super().__init__()
        self.cfg = cfg
        w = cfg.widths
        names, units = ["in"], [_Input(cfg.z_dim, w[0])]
        names += ["mid.res0", "mid.attn", "mid.res1"]
        units += [_ResBlock(w[0], w[0]), _FrameAttention(w[0]), _ResBlock(w[0], w[0])]
        self.upsample_at = []
        for i in range(len(cfg.dim_mult)):
            cin, cout = (w[i] // 2 if i > 0 else w[i]), w[i + 1]
            for j in range(cfg.num_res_blocks + 1):
                names.append(f"up{i}.res{j}")
                units.append(_ResBlock(cin, cout))
                cin = cout
            if i != len(cfg.dim_mult) - 1:
                names.append(f"up{i}.resample")
                units.append(_Upsample(cout, cfg.temporal_upsample[i]))
        names.append("head")
        units.append(_Head(w[-1]))
        self.names = names
        self.units = nn.ModuleList(units)

    @classmethod
    def random(cls, cfg: VAEConfig = VAEConfig(), device="cpu", dtype=torch.float32, seed: int = 0) -> "VAEDecoder":
        """Random-init weights: N(0, 1/fan_in) kernels, small biases and gains
        near one, so activations keep their scale through the depth."""
        m = cls(cfg)
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for name, p in m.named_parameters():
                if name.endswith(("gain", "inv_std")):
                    p.copy_(1 + 0.1 * torch.randn(p.shape, generator=g))
                elif p.dim() == 1:
                    p.copy_(0.02 * torch.randn(p.shape, generator=g))
                else:
                    fan_in = p[0].numel()
                    p.copy_(torch.randn(p.shape, generator=g) / math.sqrt(fan_in))
        return m.to(device=device, dtype=dtype).eval()

    def reference_names(self) -> dict:
        """Our parameter -> the reference WanVAE_'s parameter name and shape
        (naive_rt/rolling_forcing/wan/modules/vae.py: ``conv2``, ``decoder.*``)."""
        out = {}
        u = self.units

        def put(t, name, shape=None):
            out[id(t)] = (t, name, shape)

        put(u[0].pre.weight, "conv2.weight")
        put(u[0].pre.bias, "conv2.bias")
        put(u[0].conv.weight, "decoder.conv1.weight")
        put(u[0].conv.bias, "decoder.conv1.bias")

        def res(prefix, r):
            put(r.n1.gain, prefix + "residual.0.gamma", (-1, 1, 1, 1))
            put(r.c1.weight, prefix + "residual.2.weight")
            put(r.c1.bias, prefix + "residual.2.bias")
            put(r.n2.gain, prefix + "residual.3.gamma", (-1, 1, 1, 1))
            put(r.c2.weight, prefix + "residual.6.weight")
            put(r.c2.bias, prefix + "residual.6.bias")
            if r.short is not None:
                put(r.short.weight, prefix + "shortcut.weight")
                put(r.short.bias, prefix + "shortcut.bias")

        res("decoder.middle.0.", u[1])
        a = u[2]
        c = a.proj.shape[0]
        put(a.norm.gain, "decoder.middle.1.norm.gamma", (-1, 1, 1))
        put(a.qkv, "decoder.middle.1.to_qkv.weight", (3 * c, c, 1, 1))
        put(a.qkv_b, "decoder.middle.1.to_qkv.bias")
        put(a.proj, "decoder.middle.1.proj.weight", (c, c, 1, 1))
        put(a.proj_b, "decoder.middle.1.proj.bias")
        res("decoder.middle.2.", u[3])
        for j, m in enumerate(list(u)[4:-1]):
            p = f"decoder.upsamples.{j}."
            if isinstance(m, _ResBlock):
                res(p, m)
            else:
                put(m.conv_w, p + "resample.1.weight")
                put(m.conv_b, p + "resample.1.bias")
                if m.temporal:
                    put(m.tconv.weight, p + "time_conv.weight")
                    put(m.tconv.bias, p + "time_conv.bias")
        put(u[-1].norm.gain, "decoder.head.0.gamma", (-1, 1, 1, 1))
        put(u[-1].conv.weight, "decoder.head.2.weight")
        put(u[-1].conv.bias, "decoder.head.2.bias")
        return out

    @classmethod
    def from_reference(cls, ref_vae, mean, std, cfg: VAEConfig = VAEConfig()) -> "VAEDecoder":
        """This decoder with the weights of the reference's loaded ``WanVAE_``
        (its ``conv2`` and ``decoder``) and its latent statistics (``mean``,
        ``std``: the scale the reference's decode divides by is 1 / std), so a
        checkpointed VAE drops in unchanged."""
        m = cls(cfg)
        src = dict(ref_vae.named_parameters())
        with torch.no_grad():
            for t, name, _shape in m.reference_names().values():
                if name not in src:
                    raise KeyError(f"reference VAE has no parameter {name}")
                t.copy_(src[name].detach().reshape(t.shape).to(t.dtype))
            m.units[0].mean.copy_(torch.as_tensor(mean, dtype=torch.float32).reshape(-1))
            m.units[0].inv_std.copy_(1.0 / torch.as_tensor(std, dtype=torch.float32).reshape(-1))
        return m.eval()

    def for_gpu(self, device, dtype=torch.bfloat16) -> "VAEDecoder":
        """bf16 weights on the GPU, 3-D convolution kernels channels-last
        (NDHWC), the layout of cuDNN's implicit-GEMM convolutions."""
        self.to(device=device, dtype=dtype)
        for m in self.modules():
            if isinstance(m, _CausalConv):
                m.weight.data = m.weight.data.contiguous(memory_format=torch.channels_last_3d)
            elif isinstance(m, _Upsample):
                m.conv_w.data = m.conv_w.data.contiguous(memory_format=torch.channels_last)
        return self

    def unit_flops(self, h: int, w: int) -> list[float]:
        """Multiply-add FLOPs of each unit per latent frame in steady state
        (4 output frames per latent frame after the two temporal upsamplings),
        for a latent of h x w: the pipeline's balancing weights."""
        out, t, hh, ww = [], 1.0, h, w

        def conv(m: _CausalConv, frames, hs, ws):
            co, ci, kt, kh, kw = m.weight.shape
            return 2.0 * co * ci * kt * kh * kw * frames * hs * ws

        for u in self.units:
            if isinstance(u, _Input):
                out.append(conv(u.pre, t, hh, ww) + conv(u.conv, t, hh, ww))
            elif isinstance(u, _ResBlock):
                f = conv(u.c1, t, hh, ww) + conv(u.c2, t, hh, ww)
                out.append(f + (conv(u.short, t, hh, ww) if u.short is not None else 0.0))
            elif isinstance(u, _FrameAttention):
                c = u.proj.shape[0]
                n = hh * ww
                out.append(t * (2.0 * n * c * 4 * c + 4.0 * n * n * c))
            elif isinstance(u, _Upsample):
                f = conv(u.tconv, t, hh, ww) if u.temporal else 0.0
                if u.temporal:
                    t *= 2
                hh, ww = hh * 2, ww * 2
                co, ci, kh, kw = u.conv_w.shape
                out.append(f + 2.0 * co * ci * kh * kw * t * hh * ww)
            else:
                out.append(conv(u.conv, t, hh, ww))
        return out

    def run_units(self, x: torch.Tensor, state: dict, lo: int = 0, hi: int | None = None) -> torch.Tensor:
        hi = len(self.units) if hi is None else hi
        for i in range(lo, hi):
            x = self.units[i](x, state, self.names[i])
        return x


def _frames_in(z: torch.Tensor) -> torch.Tensor:
    """[C, F, h, w] or [1, C, F, h, w] -> [1, C, F, h, w]."""
    return z if z.dim() == 5 else z.unsqueeze(0)


class DecodeStream:
    """One video's decode, fed chunk by chunk.  ``push(z)`` takes the next
    latent frames [C, F, h, w] and returns their pixels [3, F', 8h, 8w]: the
    stream's first latent frame gives 1 pixel frame, every later one 4.

    Each push runs as one or two calls of the units: the stream's first latent
    frame always alone (its call skips the temporal upsampling convolutions,
    as the reference's first per-frame call does), any other frames of a push
    together.  Every operation is causal in time or per frame, so grouping
    frames after the first changes no result beyond floating-point order."""

    def __init__(self, dec: VAEDecoder, lo: int = 0, hi: int | None = None) -> None:
        self.dec, self.lo, self.hi = dec, lo, hi
        self.state: dict = {}
        self.frames_in = 0

    def split(self, z: torch.Tensor) -> list[torch.Tensor]:
        """The calls a push of latent frames ``z`` makes: [1, C, f, h, w] groups."""
        x = _frames_in(z)
        if self.frames_in == 0 and x.shape[2] > 1:
            groups = [x[:, :, :1], x[:, :, 1:]]
        else:
            groups = [x]
        self.frames_in += x.shape[2]
        return groups

    @torch.no_grad()
    def run(self, x: torch.Tensor) -> torch.Tensor:
        """One call of this stream's units on [1, C, T, H, W] activations."""
        p = next(self.dec.parameters())
        x = x.to(device=p.device, dtype=p.dtype)
        if x.is_cuda:
            x = x.contiguous(memory_format=torch.channels_last_3d)
        return self.dec.run_units(x, self.state, self.lo, self.hi)

    def push(self, z: torch.Tensor) -> torch.Tensor:
        outs = [self.run(g) for g in self.split(z)]
        return torch.cat(outs, 2)[0]


def decode_framewise(dec: VAEDecoder, z: torch.Tensor) -> torch.Tensor:
    """Frame-by-frame decode of a whole latent video, the reference's loop
    (vae.py:621-637): the stream fed one latent frame per call."""
    s = DecodeStream(dec)
    zz = _frames_in(z)
    return torch.cat([s.push(zz[:, :, i:i + 1]) for i in range(zz.shape[2])], 1)


# ---------------------------------------------------------------- pipeline
def partition_units(costs: list[float], n: int) -> list[int]:
    """Cut points [0, c1, ..., len] of a contiguous split of the units into n
    groups minimising the largest group's cost (the reference balances its
    VAE stages the same way, wave_rt/pipelines/vae.py:64-90)."""
    m = len(costs)
    n = max(1, min(n, m))
    pre = [0.0]
    for c in costs:
        pre.append(pre[-1] + c)
    # dp[k][i]: best max-cost splitting units[:i] into k groups
    INF = float("inf")
    dp = [[INF] * (m + 1) for _ in range(n + 1)]
    cut = [[0] * (m + 1) for _ in range(n + 1)]
    dp[0][0] = 0.0
    for k in range(1, n + 1):
        for i in range(k, m + 1):
            for j in range(k - 1, i):
                v = max(dp[k - 1][j], pre[i] - pre[j])
                if v < dp[k][i]:
                    dp[k][i], cut[k][i] = v, j
    cuts = [m]
    i = m
    for k in range(n, 0, -1):
        i = cut[k][i]
        cuts.append(i)
    return cuts[::-1]


class VAEPipelineStage:
    """One rank of a VAE pipeline: units [cuts[k], cuts[k+1]) of the decoder
    (the reference's ``vae_stage``, wave_rt/pipelines/vae.py:42-207).

    Stage 0 turns latent frames into its calls (``DecodeStream.split``) and
    sends each call's output on; later stages run one call per message, in
    order, so every stage sees the same call boundaries (the first latent
    frame alone).  Messages carry the shape first and an all-zero shape means
    the end (wave_rt/pipelines/vae.py:21-39).  Transport: ``torch.distributed``
    send/recv (NCCL between GPUs, gloo in the CPU tests)."""

    def __init__(self, dec: VAEDecoder, cuts: list[int], k: int, ranks: list[int], group=None) -> None:
        self.dec, self.cuts, self.k, self.ranks, self.group = dec, cuts, k, ranks, group
        self.stream = DecodeStream(dec, cuts[k], cuts[k + 1])
        self.first = k == 0
        self.last = k == len(cuts) - 2

    def push_latents(self, z: torch.Tensor) -> list[torch.Tensor]:
        """Stage 0: the outputs of the calls for latent frames z."""
        return [self.stream.run(g) for g in self.stream.split(z)]

    def run(self, x: torch.Tensor) -> torch.Tensor:
        return self.stream.run(x)

    def send_next(self, y: torch.Tensor | None) -> None:
        import torch.distributed as dist

        dst = self.ranks[self.k + 1]
        if y is None:
            dist.send(torch.zeros(5, dtype=torch.int64, device=self._dev()), dst, group=self.group)
            return
        y = y.contiguous()
        dist.send(torch.tensor(list(y.shape), dtype=torch.int64, device=y.device), dst, group=self.group)
        dist.send(y, dst, group=self.group)

    def recv_prev(self) -> torch.Tensor | None:
        import torch.distributed as dist

        src = self.ranks[self.k - 1]
        shp = torch.empty(5, dtype=torch.int64, device=self._dev())
        dist.recv(shp, src, group=self.group)
        if int(shp.abs().sum()) == 0:
            return None
        p = next(self.dec.parameters())
        y = torch.empty(tuple(shp.tolist()), dtype=p.dtype, device=p.device)
        dist.recv(y, src, group=self.group)
        return y

    def _dev(self):
        return next(self.dec.parameters()).device

    def serve(self) -> list[torch.Tensor]:
        """Stages after the first: run every message until the end marker,
        forwarding to the next stage; the last stage returns its pixel calls
        ([3, F', H, W] each)."""
        outs = []
        while True:
            x = self.recv_prev()
            if x is None:
                if not self.last:
                    self.send_next(None)
                return outs
            y = self.run(x)
            if self.last:
                outs.append(y[0])
            else:
                self.send_next(y)
