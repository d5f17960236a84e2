"""Drive the reference's own wavefront engine (SJTU-DENG-Lab/WaveForcing,
``wave_rt.denoiser.engine.WaveDenoiser``) without SGLang.

The reference's engine takes a per-rank backend (``WaveBackend``,
wave_rt/runtime/backend.py:165-520, built on SGLang) and imports three SGLang
RoPE symbols in ``CommonExchangeMixin._init_rope`` (exchange/common.py:32-42).
Neither exists without SGLang.  This module supplies both, so that the
engine's own code -- its tick loop ``_systolic``, its exchange mixins, its
promotion, migration and ``close`` -- runs unchanged:

  * ``install_sglang_stubs``: stand-ins for ``_apply_rotary_emb``,
    ``get_rotary_pos_embed`` and ``current_platform``, restated from the
    vendored naive model's RoPE (naive_rt/rolling_forcing/wan/modules/
    causal_model.py:27-54): per-axis frequencies over (frame, height, width)
    split as ``rope_dim_list``, tables built in float64 and cast to float32,
    interleaved pairs rotated in float32.  SGLang's own versions are not
    vendored; these follow the arithmetic the survey of the reference states.
  * ``StubBackend``: the attributes and methods ``WaveDenoiser`` reads from
    its backend, with a pluggable per-rank ``model(latent_bcthw, step,
    start_frame, exch)`` whose self-attention calls the installed exchange
    closure with the keyword contract of ``patched_forward``
    (backend.py:87-157).

Users: the CPU test that drops this repository's paged mixin into the
reference's WaveDenoiser (tests/test_reference_dropin.py), and the GPU
reference arm of bench.py (``--impl reference-gpu``).  The reference
checkout is located by ``reference_checkout()``; nothing here is imported
by the package.
"""

from __future__ import annotations

import os
import sys
import types
from types import SimpleNamespace

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def reference_checkout() -> str | None:
    """A WaveForcing checkout holding ``wave_rt``: $WF_REFERENCE, then
    baseline/_ref (where the reference's package is laid out for GPU boxes),
    then a ``reference`` directory beside this repository."""
    cands = [os.environ.get("WF_REFERENCE", ""), os.path.join(ROOT, "baseline", "_ref"),
             os.path.join(os.path.dirname(ROOT), "reference")]
    for c in cands:
        if c and os.path.isdir(os.path.join(c, "wave_rt")):
            return os.path.abspath(c)
    return None


# --------------------------------------------------------------- SGLang RoPE
def rope_tables_3d(sizes, head_dim: int, rope_dim_list, start_frame: int, theta: float = 10000.0,
                   dtype=torch.float64, device=None):
    """cos/sin [F*h*w, head_dim/2] for frames [start_frame, start_frame + F):
    each axis a of (frame, height, width) contributes rope_dim_list[a]/2
    angles pos / theta^(2i / rope_dim_list[a]) (causal_model.py:27-54)."""
    F, h, w = sizes
    parts = []
    for a, (n, d) in enumerate(zip((F, h, w), rope_dim_list)):
        pos = torch.arange(n, dtype=dtype, device=device) + (start_frame if a == 0 else 0)
        inv = 1.0 / torch.pow(torch.tensor(theta, dtype=dtype, device=device),
                              torch.arange(0, d, 2, dtype=dtype, device=device) / d)
        parts.append(torch.outer(pos, inv))
    fr, hh, ww = parts
    ang = torch.cat([fr[:, None, None, :].expand(F, h, w, fr.shape[1]),
                     hh[None, :, None, :].expand(F, h, w, hh.shape[1]),
                     ww[None, None, :, :].expand(F, h, w, ww.shape[1])], -1).reshape(F * h * w, -1)
    assert ang.shape[1] * 2 == head_dim
    return torch.cos(ang), torch.sin(ang)


def apply_rotary_interleaved(x, cos, sin, is_neox_style: bool = False):
    """x [..., T, H, D]; cos/sin [T, D/2]: (x0, x1) -> (x0 c - x1 s, x0 s + x1 c)
    on interleaved pairs, in float32; returns float32 (callers cast)."""
    if is_neox_style:
        raise NotImplementedError("the wavefront path uses interleaved (non-neox) RoPE")
    xf = x.float().reshape(*x.shape[:-1], -1, 2)
    c = cos.float()[:, None, :]
    s = sin.float()[:, None, :]
    x0, x1 = xf[..., 0], xf[..., 1]
    return torch.stack([x0 * c - x1 * s, x0 * s + x1 * c], -1).reshape(x.shape)


def install_sglang_stubs() -> None:
    """Register the three SGLang symbols that exchange/common.py:32-42 imports."""
    if "sglang.multimodal_gen.runtime.layers.rotary_embedding.factory" in sys.modules:
        return
    names = ["sglang", "sglang.multimodal_gen", "sglang.multimodal_gen.runtime",
             "sglang.multimodal_gen.runtime.layers", "sglang.multimodal_gen.runtime.layers.rotary_embedding",
             "sglang.multimodal_gen.runtime.layers.rotary_embedding.factory",
             "sglang.multimodal_gen.runtime.platforms"]
    mods = {}
    for n in names:
        m = types.ModuleType(n)
        m.__path__ = []  # importable as a package
        mods[n] = m
        sys.modules[n] = m

    def get_rotary_pos_embed(sizes, hidden_size, heads_num, rope_dim_list, dtype=torch.float32,
                             rope_theta=10000, start_frame=0, device=None, **_):
        return rope_tables_3d(sizes, hidden_size // heads_num, rope_dim_list, start_frame, float(rope_theta),
                              dtype=dtype, device=device)

    mods["sglang.multimodal_gen.runtime.layers.rotary_embedding"]._apply_rotary_emb = apply_rotary_interleaved
    mods["sglang.multimodal_gen.runtime.layers.rotary_embedding.factory"].get_rotary_pos_embed = get_rotary_pos_embed
    mods["sglang.multimodal_gen.runtime.platforms"].current_platform = SimpleNamespace(
        is_float64_supported=lambda: True)


def import_reference():
    """Import the reference's engine module (SGLang stubs installed first)."""
    path = reference_checkout()
    if path is None:
        raise RuntimeError("no WaveForcing checkout found (set WF_REFERENCE)")
    install_sglang_stubs()
    if path not in sys.path:
        sys.path.insert(0, path)
    import wave_rt.denoiser.engine as engine  # noqa: E402

    return engine


# ------------------------------------------------------------------ backend
class FlowScheduler:
    """``add_noise`` of the reference's scheduler as the engine calls it
    (engine.py:221-235): x = (1 - sigma) x0 + sigma n, sigma = t / 1000 (no
    shift; the stub has no trained schedule to reproduce)."""

    def add_noise(self, x0, noise, timestep):
        s = (timestep.float() / 1000.0).view(-1, *([1] * (x0.dim() - 1)))
        return ((1 - s) * x0.float() + s * noise.float()).to(x0.dtype)


class StubBackend:
    """What WaveDenoiser reads from ``self.be`` (engine.py:36-62, :221-235,
    :287-626): geometry, schedule, noise, a barrier, the exchange-closure
    slot and ``forward_chunk``.  ``model(latent_bcthw, step, start_frame,
    exch) -> x0_btchw`` is the per-rank DiT."""

    def __init__(self, *, rank: int, device, dtype, num_layers: int, heads: int, head_dim: int, channels: int,
                 lat_h: int, lat_w: int, tokens_per_frame: int, steps, full_noise, model,
                 sliding_window_num_frames: int = 21, context_noise: float = 0.0) -> None:
        import torch.distributed as dist

        self._dist = dist
        self.rank = rank
        self.device = torch.device(device)
        self.num_layers = num_layers
        self.num_attention_heads = heads
        self.attention_head_dim = head_dim
        self.latent_channels = channels
        self.num_token_per_frame = tokens_per_frame
        self.rf_stage = SimpleNamespace(sliding_window_num_frames=sliding_window_num_frames)
        self.server_args = SimpleNamespace(pipeline_config=SimpleNamespace(context_noise=context_noise))
        self.ctx = SimpleNamespace(target_dtype=dtype, scheduler=FlowScheduler(), height=lat_h, width=lat_w,
                                   latents=full_noise, timesteps=torch.tensor([float(s) for s in steps]))
        self.model = model
        self.exch = None

    @property
    def dsl(self):
        return self.ctx.timesteps

    @property
    def full_noise_bcthw(self):
        return self.ctx.latents

    def set_exchange_fn(self, fn) -> None:
        self.exch = fn

    def forward_chunk(self, noisy_chunk_bcthw, step_value, start_frame):
        return self.model(noisy_chunk_bcthw, float(step_value), int(start_frame), self.exch)

    def barrier(self) -> None:
        if self._dist.is_initialized():
            self._dist.barrier()

    def decode(self, latents):
        return latents


def make_config(engine_mod, *, rf_step: int, steps, num_frames: int, exchange_mode: str):
    """A WaveConfig for ``rf_step`` denoise ranks + the store (wp_size =
    rf_step + 1, config.py:79-83), causal K/V context."""
    from wave_rt.config import WaveConfig

    return WaveConfig(rf_step=rf_step, wp_size=rf_step + 1, denoising_step_list=tuple(steps), num_frames=num_frames,
                      exchange_mode=exchange_mode, kv_context="causal")


# ------------------------------------------------------------ Wan DiT model
def wan_forward(model, *, fused: bool):
    """``model(latent_bcthw, step, start_frame, exch) -> x0_btchw`` over this
    repository's Wan-shaped DiT (waveforcing_b200/wavefront/dit.py, random
    weights).  ``step`` is the warped timestep the engine passes (its dsl,
    backend.py:460-463); x0 = x_t - (step / 1000) * flow, the flow-matching
    inversion of naive_rt/rolling_forcing/utils/wan_wrapper.py:169-193.

    fused=False is the reference's GPU path restated in plain torch: q, k and
    v as three linears, the RoPE stand-in above applied as patched_forward
    does (``apply_rope(q, cos, sin).type_as(v)``, backend.py:119-121), torch
    ops for norms and modulation, and whatever attention backend is selected
    (torch SDPA for the reference).  fused=True is this repository's path
    (libwfk row kernels, fused QKV, the selected backend)."""
    from waveforcing_b200.wavefront.dit import StageTask

    def torch_rope(x, cos, sin):
        return apply_rotary_interleaved(x, cos, sin).to(x.dtype)

    def forward(lat_bcthw, step, start_frame, exch):
        xt = lat_bcthw[0]
        task = StageTask(xt, float(step), int(start_frame), 0, exch)
        if fused:
            flow = model.forward_stages([task])[0]
        else:
            flow = model.forward_stages([task], fused=False, rope_fn=torch_rope, separate_qkv=True)[0]
        x0 = (xt.double() - (float(step) / 1000.0) * flow.double()).to(xt.dtype)  # [C, F, H, W]
        return x0.permute(1, 0, 2, 3).unsqueeze(0).contiguous()

    return forward
