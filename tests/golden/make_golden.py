"""Generate the golden fixtures in this directory by running the REFERENCE's
own code (SJTU-DENG-Lab/WaveForcing, a pure-Python project) on CPU.

Run once in a container where the reference checkout is importable:

    WF_REFERENCE=<path to the WaveForcing checkout> python tests/golden/make_golden.py

What is produced and from which reference code:
  * codec_per_tensor.npz -- CommonExchangeMixin._all_gather_fp8
    (wave_rt/denoiser/exchange/common.py:143-164) run on a 1-rank gloo group;
    the u8 codes are captured from its all_gather call.
  * w8a8_per_tensor.npz  -- WaveFp8Linear (wave_rt/runtime/fp8.py:21-61)
    run on CPU through torch._scaled_mm.
  * rope.npz             -- causal_rope_apply and rope_params of the vendored
    naive model (naive_rt/rolling_forcing/wan/modules/causal_model.py:27-54,
    model.py:29-37, causal_model.py:549-554); ``diffusers`` is stubbed
    because only its base classes are imported there.
  * geometry.json        -- the slot geometry closed over by
    PagedExchangeMixin._make_denoise_exch_paged / _make_store_exch_paged
    (wave_rt/denoiser/exchange/paged.py:156-265) for every (tick, rank) of
    5-step and 4-step wavefronts.
  * sdpa.npz             -- torch CPU SDPA exactly as the reference's
    fallback calls it (naive_rt/rolling_forcing/wan/modules/attention.py:75-89).

The fixtures are small (a few hundred KB in total).  Nothing at test time
reads the reference checkout.
"""

from __future__ import annotations

import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _ref_path() -> str:
    p = os.environ.get("WF_REFERENCE")
    if not p or not os.path.isdir(p):
        raise SystemExit("set WF_REFERENCE to the WaveForcing checkout")
    return p


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def gen_codec():
    import torch.distributed as dist
    from wave_rt.denoiser.exchange.common import CommonExchangeMixin

    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29531")
        dist.init_process_group("gloo", rank=0, world_size=1)

    captured = []
    real_ag = dist.all_gather

    def spy(out, inp, *a, **k):
        if inp.dtype == torch.uint8:
            captured.append(inp.clone())
        return real_ag(out, inp, *a, **k)

    cases = {}
    shapes = [(2, 24, 2, 128), (2, 7, 3, 128), (2, 1, 1, 128)]
    kinds = ["normal", "wide", "tiny", "zeros", "outlier"]
    g = torch.Generator().manual_seed(0)
    ci = 0
    for shp in shapes:
        for kind in kinds:
            if kind == "normal":
                x = torch.randn(shp, generator=g)
            elif kind == "wide":
                x = torch.randn(shp, generator=g) * torch.exp(torch.randn(shp, generator=g) * 4)
            elif kind == "tiny":
                x = torch.randn(shp, generator=g) * 1e-9
            elif kind == "zeros":
                x = torch.zeros(shp)
            else:
                x = torch.randn(shp, generator=g)
                x.view(-1)[7] = 3000.0
            x = x.to(torch.bfloat16)
            obj = object.__new__(CommonExchangeMixin)
            obj._kv_shape = shp
            obj.device = "cpu"
            obj.world = 1
            obj.dtype = torch.bfloat16
            captured.clear()
            dist.all_gather = spy
            try:
                deq = obj._all_gather_fp8(x)[0]
            finally:
                dist.all_gather = real_ag
            codes = captured[0]
            scale = (x.abs().amax() / 448.0).clamp(min=1e-8).to(torch.float32)
            cases[f"c{ci}_x"] = _bits(x)
            cases[f"c{ci}_codes"] = codes.numpy().copy()
            cases[f"c{ci}_scale"] = np.float32(scale.item())
            cases[f"c{ci}_deq"] = deq.to(torch.float32).numpy().copy()
            ci += 1
    cases["n"] = np.int64(ci)
    np.savez_compressed(os.path.join(HERE, "codec_per_tensor.npz"), **cases)
    print("codec cases", ci)


def gen_w8a8():
    from wave_rt.runtime.fp8 import WaveFp8Linear

    g = torch.Generator().manual_seed(1)
    out = {}
    dims = [(64, 128, 96, True), (37, 256, 64, False), (8, 64, 32, True)]
    for i, (M, K, N, has_bias) in enumerate(dims):
        x = (torch.randn(M, K, generator=g) * 2).to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
        b = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16) if has_bias else None
        lin = WaveFp8Linear(w, b, compile_fwd=False)
        y, none = lin(x)
        assert none is None
        out[f"c{i}_x"] = _bits(x)
        out[f"c{i}_w"] = _bits(w)
        if b is not None:
            out[f"c{i}_b"] = _bits(b)
        out[f"c{i}_wq"] = lin.w_fp8.view(torch.uint8).numpy().copy()
        out[f"c{i}_ws"] = np.float32(lin.w_scale.item())
        out[f"c{i}_y"] = _bits(y)
    out["n"] = np.int64(len(dims))
    np.savez_compressed(os.path.join(HERE, "w8a8_per_tensor.npz"), **out)
    print("w8a8 cases", len(dims))


def gen_rope():
    # The naive model imports diffusers only for base classes; stub them.
    for name in ["diffusers", "diffusers.configuration_utils", "diffusers.models",
                 "diffusers.models.modeling_utils"]:
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["diffusers.configuration_utils"].ConfigMixin = object
    sys.modules["diffusers.configuration_utils"].register_to_config = lambda f: f
    sys.modules["diffusers.models.modeling_utils"].ModelMixin = torch.nn.Module
    # Load the modules package by path without running its __init__ (which
    # imports the T5 tokenizer stack that is not needed here).
    import importlib

    pkg = types.ModuleType("_wf_naive_wan")
    pkg.__path__ = [os.path.join(_ref_path(), "naive_rt", "rolling_forcing", "wan", "modules")]
    sys.modules["_wf_naive_wan"] = pkg
    causal_rope_apply = importlib.import_module("_wf_naive_wan.causal_model").causal_rope_apply
    rope_params = importlib.import_module("_wf_naive_wan.model").rope_params

    d = 128
    freqs = torch.cat([rope_params(1024, d - 4 * (d // 6)),
                       rope_params(1024, 2 * (d // 6)),
                       rope_params(1024, 2 * (d // 6))], dim=1)
    g = torch.Generator().manual_seed(2)
    out = {}
    cases = [(3, 4, 6, 0, 2), (3, 4, 6, 9, 3), (2, 3, 5, 57, 1), (1, 30, 52, 12, 1)]
    for i, (f, h, w, sf, n) in enumerate(cases):
        L = f * h * w
        x = torch.randn(1, L, n, d, generator=g).to(torch.bfloat16)
        grid = torch.tensor([[f, h, w]])
        y = causal_rope_apply(x, grid, freqs, start_frame=sf)
        out[f"c{i}_x"] = _bits(x[0])
        out[f"c{i}_y"] = _bits(y[0])
        out[f"c{i}_meta"] = np.array([f, h, w, sf, n], np.int64)
    out["n"] = np.int64(len(cases))
    np.savez_compressed(os.path.join(HERE, "rope.npz"), **out)
    print("rope cases", len(cases))


def gen_geometry():
    from wave_rt.denoiser.exchange.paged import PagedExchangeMixin

    def closure_vars(fn):
        return {n: c.cell_contents for n, c in zip(fn.__code__.co_freevars, fn.__closure__)}

    records = []
    for rf_step in (5, 4, 3, 2, 1):
        world = rf_step + 1
        num_blocks = 12
        npb, T, maf = 3, 4680, 21
        wmax_frames = maf - rf_step * npb - npb
        naw_max = 1 + max(0, wmax_frames // npb)
        for t in range(num_blocks + world - 1):
            act = [n for n in range(rf_step) if 0 <= t - n < num_blocks]
            oldest = (t - max(act)) if act else 0
            store_active = 0 <= t - rf_step < num_blocks
            for r in range(world):
                obj = object.__new__(PagedExchangeMixin)
                obj.store_rank = rf_step
                obj.rank = r
                obj.rf_step = rf_step
                obj._cur_tick = t
                obj._os_gt = 2
                obj.tokens_per_chunk = T
                obj.npb = npb
                obj.max_attn_frames = maf
                obj._pg_naw = naw_max
                obj._pg_wmax = naw_max + 1 + rf_step
                rec = dict(rf_step=rf_step, tick=t, rank=r, act_ranks=act,
                           tick_csf=oldest * npb, tick_qf=len(act) * npb,
                           store_active=store_active, wmax=obj._pg_wmax)
                if r < rf_step and 0 <= t - r < num_blocks:
                    fn = obj._make_denoise_exch_paged([], act, oldest * npb, len(act) * npb, store_active)
                    cv = closure_vars(fn)
                    rec.update(role="denoise", gen=cv["gen"], naw=cv["naw"], live_off=cv["live_off"],
                               self_off=cv["self_off"], active_len=cv["active_len"],
                               recv_srcs=cv["recv_srcs"], send_slots=[list(s) for s in cv["send_slots"]])
                elif r == rf_step and store_active:
                    fn = obj._make_store_exch_paged([], [], t - rf_step, act)
                    cv = closure_vars(fn)
                    rec.update(role="store", gen=cv["gen"],
                               send_slots=[list(s) for s in cv["send_slots"]])
                else:
                    rec.update(role="idle")
                records.append(rec)
    with open(os.path.join(HERE, "geometry.json"), "w") as f:
        json.dump(records, f)
    print("geometry records", len(records))


def gen_sdpa():
    import torch.nn.functional as F

    g = torch.Generator().manual_seed(3)
    out = {}
    cases = [(130, 200, 2), (128, 128, 1), (5, 300, 1), (64, 64, 2)]
    for i, (Lq, Lk, H) in enumerate(cases):
        q = (torch.randn(1, Lq, H, 128, generator=g)).to(torch.bfloat16)
        k = (torch.randn(1, Lk, H, 128, generator=g)).to(torch.bfloat16)
        v = (torch.randn(1, Lk, H, 128, generator=g)).to(torch.bfloat16)
        # attention.py:76-89 (q/k/v already half precision; computed in f32 here
        # for a tight golden, the op the bf16 call approximates)
        o = F.scaled_dot_product_attention(q.float().transpose(1, 2), k.float().transpose(1, 2),
                                           v.float().transpose(1, 2)).transpose(1, 2)
        out[f"c{i}_q"] = _bits(q[0])
        out[f"c{i}_k"] = _bits(k[0])
        out[f"c{i}_v"] = _bits(v[0])
        out[f"c{i}_o"] = o[0].numpy().astype(np.float32)
    out["n"] = np.int64(len(cases))
    np.savez_compressed(os.path.join(HERE, "sdpa.npz"), **out)
    print("sdpa cases", len(cases))


def main():
    sys.path.insert(0, _ref_path())
    torch.manual_seed(0)
    gen_codec()
    gen_w8a8()
    gen_rope()
    gen_geometry()
    gen_sdpa()


if __name__ == "__main__":
    main()
