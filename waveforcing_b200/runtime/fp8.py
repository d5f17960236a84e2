"""W8A8 linear hook on the libwfk tcgen05 GEMM.

Mirrors wave_rt/runtime/fp8.py:
  * ``WfW8A8Linear``             ~ ``WaveFp8Linear`` (:21-61): post-load
    replacement owning the quantised weight and its scale as buffers, whose
    ``forward(x)`` returns ``(y, None)`` -- SGLang's linear return contract.
  * ``quantize_transformer_w8a8`` ~ ``quantize_transformer_fp8`` (:93-137):
    walks ``transformer.blocks`` and replaces ``ffn.fc_in``/``ffn.fc_out``
    (scope ``ffn``, default) or every 2-D ``*Linear`` (scope ``all``,
    ``WAVE_FP8_SCOPE``).
Granularity ``tensor`` reproduces the reference (static per-tensor weight
scale, dynamic per-tensor bf16 activation scale, e4m3); ``channel`` (the
default here) uses per-output-channel weight scales and per-token activation
scales, with e4m3 or int8 codes.
"""

from __future__ import annotations

import os

import torch
import torch.nn as nn

from waveforcing_b200 import _lib as L
from waveforcing_b200 import kernels

_QTYPES = {"e4m3": L.WF_DTYPE_E4M3, "fp8": L.WF_DTYPE_E4M3, "int8": L.WF_DTYPE_S8, "s8": L.WF_DTYPE_S8}


class WfW8A8Linear(nn.Module):
    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None, qtype: str = "e4m3",
                 granularity: str = "channel") -> None:
        super().__init__()
        if granularity not in ("channel", "tensor"):
            raise ValueError("granularity must be 'channel' or 'tensor'")
        if granularity == "tensor" and _QTYPES[qtype] != L.WF_DTYPE_E4M3:
            raise ValueError("per-tensor granularity is the reference's e4m3 form only")
        self.qtype = _QTYPES[qtype]
        self.granularity = granularity
        self.out_dtype = weight.dtype
        self.out_features, self.in_features = weight.shape
        w = weight.detach().to(torch.bfloat16).contiguous()
        if granularity == "channel":
            wq, ws = kernels.weight_quant(w, self.qtype)
        else:
            # fp8.py:32-36 verbatim in f32: one scale for the whole matrix
            wf = weight.detach().to(torch.float32)
            s = (wf.abs().amax() / 448.0).clamp(min=1e-8)
            wq = (wf / s).to(torch.float8_e4m3fn).view(torch.uint8)
            ws = s.reshape(1).to(torch.float32)
        self.register_buffer("w_q", wq)
        self.register_buffer("w_scale", ws)
        self.register_buffer("bias", bias.detach().to(torch.bfloat16) if bias is not None else None)
        self._ws = None

    def _raw(self, x2: torch.Tensor, activation: int = L.WF_ACT_NONE,
             input_activation: int = L.WF_ACT_NONE) -> torch.Tensor:
        x2 = x2.to(torch.bfloat16)
        if x2.stride(-1) != 1 or x2.stride(0) % 8:
            x2 = x2.contiguous()
        if self.granularity == "channel":
            xq, xs = kernels.act_quant(x2, self.qtype, activation=input_activation)
            mode = L.WF_SCALE_TOKEN
        else:
            if input_activation != L.WF_ACT_NONE:
                raise ValueError("an input activation is only fused into the per-token quantiser")
            if self._ws is None or self._ws.device != x2.device:
                self._ws = torch.empty(1, dtype=torch.int32, device=x2.device)
            xq, xs = kernels.kv_quant(x2, L.WF_SCALE_TENSOR, workspace=self._ws)
            mode = L.WF_SCALE_TENSOR
        return kernels.gemm_w8a8(xq, xs, self.w_q, self.w_scale, self.bias, self.qtype, mode, activation=activation)

    def gemm_q(self, xq: torch.Tensor, xs: torch.Tensor, activation: int = L.WF_ACT_NONE) -> torch.Tensor:
        """This linear on an input already quantised per token with this
        module's qtype (codes [M, in_features], scales [M]), e.g. by
        kernels.ln_modulate_quant.  Per-channel granularity only."""
        if self.granularity != "channel":
            raise ValueError("pre-quantised input needs per-token scales (granularity 'channel')")
        return kernels.gemm_w8a8(xq, xs, self.w_q, self.w_scale, self.bias, self.qtype, L.WF_SCALE_TOKEN,
                                 activation=activation)

    def forward(self, x: torch.Tensor):
        shape = x.shape
        y = self._raw(x.reshape(-1, shape[-1]))
        return y.reshape(*shape[:-1], self.out_features), None

    def forward_gelu_input(self, x: torch.Tensor) -> torch.Tensor:
        """This linear applied to GELU(approximate="tanh")(x): the activation is
        computed inside the per-token input quantiser, so the bf16 activation
        tensor is never written (the FFN's fc_out after a plain fc_in)."""
        shape = x.shape
        y = self._raw(x.reshape(-1, shape[-1]), input_activation=L.WF_ACT_GELU_TANH)
        return y.reshape(*shape[:-1], self.out_features)

    def forward_gelu(self, x: torch.Tensor) -> torch.Tensor:
        """GELU(approximate="tanh") of this linear's bf16 output, fused into the
        GEMM epilogue (the FFN's fc_in + activation)."""
        shape = x.shape
        y = self._raw(x.reshape(-1, shape[-1]), L.WF_ACT_GELU_TANH)
        return y.reshape(*shape[:-1], self.out_features)


def concat_w8a8(mods: list["WfW8A8Linear"]) -> "WfW8A8Linear":
    """One W8A8 linear whose output is the concatenation of ``mods``' outputs
    (shared input, per-channel scales): q/k/v become one GEMM on one
    activation quantisation."""
    a = mods[0]
    if any(m.granularity != "channel" or m.qtype != a.qtype for m in mods):
        raise ValueError("only per-channel W8A8 linears of one qtype concatenate")
    out = WfW8A8Linear.__new__(WfW8A8Linear)
    nn.Module.__init__(out)
    out.qtype, out.granularity, out.out_dtype = a.qtype, "channel", a.out_dtype
    out.in_features = a.in_features
    out.out_features = sum(m.out_features for m in mods)
    out.register_buffer("w_q", torch.cat([m.w_q for m in mods], 0).contiguous())
    out.register_buffer("w_scale", torch.cat([m.w_scale for m in mods], 0).contiguous())
    biases = [m.bias for m in mods]
    out.register_buffer("bias", torch.cat(biases, 0).contiguous() if all(b is not None for b in biases) else None)
    out._ws = None
    return out


_TARGET_SUFFIXES = ("ffn.fc_in", "ffn.fc_out")


def _is_quantizable_linear(mod: nn.Module) -> bool:
    if isinstance(mod, WfW8A8Linear):
        return False
    w = getattr(mod, "weight", None)
    return isinstance(w, torch.Tensor) and w.dim() == 2 and type(mod).__name__.endswith("Linear")


def quantize_transformer_w8a8(transformer: nn.Module, scope: str | None = None, qtype: str = "e4m3",
                              granularity: str = "channel", verbose: bool = False) -> int:
    """Replace block linears in place; returns the number replaced."""
    if scope is None:
        scope = os.environ.get("WAVE_FP8_SCOPE", "ffn")
    blocks = getattr(transformer, "blocks", None)
    if blocks is None:
        raise ValueError("transformer has no .blocks to quantize")
    n = 0
    for block in blocks:
        if scope == "all":
            targets = [name for name, m in block.named_modules() if name and _is_quantizable_linear(m)]
        else:
            targets = list(_TARGET_SUFFIXES)
        for suffix in targets:
            parent = block
            *path, leaf = suffix.split(".")
            for p in path:
                parent = getattr(parent, p, None)
                if parent is None:
                    break
            if parent is None:
                continue
            mod = getattr(parent, leaf, None)
            if mod is None or not _is_quantizable_linear(mod):
                continue
            b = mod.bias.data if isinstance(getattr(mod, "bias", None), torch.Tensor) else None
            setattr(parent, leaf, WfW8A8Linear(mod.weight.data, b, qtype, granularity))
            n += 1
    if verbose:
        print(f"[wf-w8a8] quantized {n} linears ({qtype}, {granularity}, scope={scope})", flush=True)
    return n
