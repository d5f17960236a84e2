"""Attention plugin surface: the ``wf_b200`` backend.

Mirrors the reference's selection and dispatch:
  * backend registry   -- wave_rt/config.py:18, argparse choices :161-163
  * enable_* functions -- wave_rt/runtime/backend.py:49-62
  * dispatch           -- wave_rt/runtime/backend.py:141-148, one call per
                          layer per tick on the current stream with
                          (roped_query, ctx_k, ctx_v) in NHD layout.
``wf_b200`` runs the tcgen05 flash-attention kernel of libwfk; the other
names are accepted so a config written for the reference parses unchanged,
but only ``wf_b200`` and ``torch_sdpa`` execute here.
"""

from __future__ import annotations

from typing import Callable

import torch

from waveforcing_b200 import kernels

ATTENTION_BACKENDS = ("torch_sdpa", "fa_custom", "sa", "fa", "fa2", "wf_b200")

_WAVE_STATE: dict = {
    "exchange_fn": None,
    "attn": "torch_sdpa",
    "fa_func": None,
    "layer_prof_sink": None,
}


def set_exchange_fn(fn: Callable | None) -> None:
    """wave_rt/runtime/backend.py:26-27."""
    _WAVE_STATE["exchange_fn"] = fn


def wf_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                 softmax_scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """flash_attn_func-compatible call: q [B, Lq, H, D], k/v [B, Lk, H, D] -> [B, Lq, H, D]
    (written into ``out`` when given, e.g. a caller's batched output rows)."""
    if causal:
        raise ValueError("wf_b200 attention is non-causal; block causality comes from the K/V context")
    return kernels.attention(q, k, v, softmax_scale=softmax_scale, out=out)


def enable_wf_b200() -> None:
    """Select the libwfk tcgen05 kernel for the wavefront attention (like enable_fa_custom)."""
    from waveforcing_b200 import _lib

    _lib.lib()  # fail now, loudly, if the extension is missing
    _WAVE_STATE["attn"] = "wf_b200"
    _WAVE_STATE["fa_func"] = wf_attention


def select_backend(name: str) -> None:
    if name not in ATTENTION_BACKENDS:
        raise ValueError(f"unknown --attention-backend {name!r}; choices: {ATTENTION_BACKENDS}")
    if name == "wf_b200":
        enable_wf_b200()
    elif name == "torch_sdpa":
        _WAVE_STATE["attn"] = "torch_sdpa"
        _WAVE_STATE["fa_func"] = None
    else:
        raise ValueError(f"backend {name!r} needs a third-party kernel that this build does not ship")


def _torch_sdpa(q, k, v):
    out = torch.nn.functional.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                                           v.transpose(1, 2))
    return out.transpose(1, 2)


def sdpa_elsewhere(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Attention outside the wavefront path (the text cross-attention).  The
    reference runs only the patched self-attention through its custom kernels
    and leaves SGLang's other attention on torch SDPA for every custom backend
    (wave_rt/runtime/backend.py:215-219); this does the same.  NHD in and out."""
    return _torch_sdpa(q, k, v)


def set_attention_timer(sink: list | None) -> None:
    """When ``sink`` is a list, every dispatched attention appends
    (flops, start_event, end_event, algorithmic_bytes) recorded on the current stream."""
    _WAVE_STATE["attn_timer"] = sink


def dispatch_attention(roped_query: torch.Tensor, ctx_k: torch.Tensor, ctx_v: torch.Tensor,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """The branch of wave_rt/runtime/backend.py:141-148 with wf_b200 added.
    With ``out`` the result lands there: the wf_b200 kernel writes it
    directly, other backends copy into it."""
    sink = _WAVE_STATE.get("attn_timer")
    if sink is not None:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
    if _WAVE_STATE["attn"] == "wf_b200" and _WAVE_STATE["fa_func"] is wf_attention:
        out = wf_attention(roped_query, ctx_k, ctx_v, causal=False, out=out)
    elif _WAVE_STATE["attn"] == "wf_b200":
        res = _WAVE_STATE["fa_func"](roped_query, ctx_k, ctx_v, causal=False)
        out = res if out is None else out.copy_(res)
    elif out is not None:
        out.copy_(_torch_sdpa(roped_query, ctx_k, ctx_v))
    else:
        out = _torch_sdpa(roped_query, ctx_k, ctx_v)
    if sink is not None:
        e1.record()
        B, Lq, H, D = roped_query.shape
        Lk = ctx_k.shape[1]
        nbytes = 2.0 * B * H * D * (2 * Lq + 2 * Lk)  # read Q, K, V and write O once (bf16)
        sink.append((4.0 * B * Lq * Lk * H * D, e0, e1, nbytes))
    return out
