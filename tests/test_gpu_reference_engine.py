"""Full-wavefront parity on GPUs against the reference's own GPU path.

Both arms run inside the reference's WaveDenoiser (wave_rt/denoiser/engine.py,
driven by baseline/harness.py), one rank per stage on its own GPU: a 2-step
wavefront, ranks 0-1 denoise and rank 2 is the store (with 2 GPUs: a 1-step
wavefront, rank 0 denoises and rank 1 is the store), over a Wan-shaped DiT
of 1.3B width (dim 1536, 12 x 128 heads, FFN 8960; 2 layers) on 60 x 104
latents (4680 tokens per chunk), 10 chunks.

  A. the reference's path: its own PagedExchangeMixin and CUDA-IPC layer, bf16
     K/V, torch SDPA attention, the DiT in plain torch ops; for W8A8 the
     reference's own WaveFp8Linear (wave_rt/runtime/fp8.py:21-61, per-tensor
     scales through torch._scaled_mm) installed by its quantize_transformer_fp8;
  B. this repository's path: its PagedExchangeMixin ahead of the reference's
     bases, libwfk attention, fused row kernels, FP8 K/V transport per token
     or per tensor; for W8A8 its quantize_transformer_w8a8 with per-tensor
     scales (tcgen05 kind::f8f6f4).

Bar: the store's final latents at cosine >= 0.999 (the north-star bar for
full-step latents).  Needs 2 or more GPUs and the reference package
(baseline/_ref or WF_REFERENCE); NVLS is off and the process group has a short
timeout.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from baseline import harness

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs"),
              pytest.mark.skipif(harness.reference_checkout() is None, reason="needs the reference package")]

# 2-step wavefront on 3 GPUs; with 2 GPUs a 1-step wavefront (one denoise
# rank and the store: the store's live-slot publishes, promotion, the anchor)
STEPS = (1000, 500) if torch.cuda.device_count() >= 3 else (1000,)
NUM_FRAMES = 30

VARIANTS = {  # name -> (arm, env for this repository's mixin, W8A8)
    "ref": ("ref", {}, False),
    "wf_bf16": ("wf", {"WAVE_FP8KV_ONESIDED": "0"}, False),
    "wf_fp8_token": ("wf", {"WAVE_FP8KV_ONESIDED": "1", "WAVE_FP8KV_GRAN": "token"}, False),
    "wf_fp8_tensor": ("wf", {"WAVE_FP8KV_ONESIDED": "1", "WAVE_FP8KV_GRAN": "tensor"}, False),
    "ref_w8a8": ("ref", {}, True),
    "wf_w8a8": ("wf", {"WAVE_FP8KV_ONESIDED": "0"}, True),
}


def _run(engine, rank, dev, name):
    from waveforcing_b200 import _lib as L
    from waveforcing_b200.denoiser.exchange.paged import PagedExchangeMixin as WfPaged
    from waveforcing_b200.runtime import backend
    from waveforcing_b200.runtime.fp8 import quantize_transformer_w8a8
    from waveforcing_b200.wavefront.dit import DiTConfig, FlowMatch, WanDiT

    arm, env, w8a8 = VARIANTS[name]
    os.environ.update(env)
    cfg = DiTConfig(dim=1536, heads=12, layers=2, ffn=8960, text_len=64, text_dim=256)
    model = WanDiT.random(cfg, dev, seed=0)
    if w8a8 and arm == "ref":
        from wave_rt.runtime.fp8 import quantize_transformer_fp8

        quantize_transformer_fp8(model, scope="ffn")
    elif w8a8:
        quantize_transformer_w8a8(model, scope="ffn", qtype="e4m3", granularity="tensor")
    g = torch.Generator(device="cpu").manual_seed(1)
    model.set_text(torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(dev))
    backend.select_backend("torch_sdpa" if arm == "ref" else "wf_b200")
    fm = FlowMatch()
    dsl = [fm.timestep(s) for s in STEPS]
    gn = torch.Generator(device="cpu").manual_seed(0)
    noise = torch.randn((1, cfg.in_ch, NUM_FRAMES, cfg.lat_h, cfg.lat_w), generator=gn).to(torch.bfloat16).to(dev)
    be = harness.StubBackend(rank=rank, device=dev, dtype=torch.bfloat16, num_layers=cfg.layers, heads=cfg.heads,
                             head_dim=cfg.head_dim, channels=cfg.in_ch, lat_h=cfg.lat_h, lat_w=cfg.lat_w,
                             tokens_per_frame=cfg.tokens_per_frame, steps=dsl, full_noise=noise,
                             model=harness.wan_forward(model, fused=(arm == "wf")))
    wcfg = harness.make_config(engine, rf_step=len(STEPS), steps=dsl, num_frames=NUM_FRAMES, exchange_mode="paged")
    cls = engine.WaveDenoiser
    if arm == "wf":
        cls = type("SwappedDenoiser", (WfPaged, engine.WaveDenoiser), {})
    den = cls(be, wcfg)
    final, _tick_ms, _ = den._systolic(be.full_noise_bcthw, warmup_pass=False, num_ticks=den.num_ticks)
    torch.cuda.synchronize()
    status = L.status_take()
    if arm == "wf":
        den._pg.check_timeouts()
    den.close()
    # numpy, not tensors: a queued tensor's shared storage dies with its sender
    return {c: x.float().cpu().numpy() for c, x in final.items()}, status


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=90))
    try:
        torch.set_grad_enabled(False)
        engine = harness.import_reference()
        out = {}
        for name in VARIANTS:
            out[name] = _run(engine, rank, dev, name)
            dist.barrier()
        q.put((rank, out))
    except Exception as e:  # report, then leave the group without further collectives
        import traceback

        q.put((rank, {"error": repr(e), "tb": traceback.format_exc()}))
    finally:
        dist.destroy_process_group()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cos(a, b):
    keys = sorted(a)
    assert keys == sorted(b) and keys
    x = torch.cat([torch.as_tensor(a[c]) for c in keys], 1).double().flatten()
    y = torch.cat([torch.as_tensor(b[c]) for c in keys], 1).double().flatten()
    return torch.nn.functional.cosine_similarity(x, y, dim=0).item()


def test_full_wavefront_against_reference_gpu_path():
    world = len(STEPS) + 1
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    try:
        for _ in ps:
            r, out = q.get(timeout=600)
            res[r] = out
    finally:
        for p in ps:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r, out in res.items():
        assert "error" not in out, out.get("tb")
        for name, (_final, st) in out.items():
            assert st == 0, f"rank {r} {name}: a bounded wait gave up"
    store = res[world - 1]
    assert len(store["ref"][0]) == NUM_FRAMES // 3
    cos = {name: _cos(store["ref"][0], store[name][0]) for name in ("wf_bf16", "wf_fp8_token", "wf_fp8_tensor")}
    cos["wf_w8a8"] = _cos(store["ref_w8a8"][0], store["wf_w8a8"][0])
    for name, c in cos.items():
        assert c >= 0.999, (name, cos)
