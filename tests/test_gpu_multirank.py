"""Wavefront over 2 and more GPUs: stages placed on separate ranks exchange K/V
through CUDA IPC peer writes + release flags (bf16) or the fused FP8
quantise-and-publish kernel, latents migrate over NCCL.  The final latents
must match the single-GPU run with every stage merged on one device.

Runs only when at least 2 GPUs are visible; ranks are child processes with a
short process-group timeout, NVLS off.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")]

STEPS = (1000, 750, 500, 250)


def _engine_run(rank, world, fp8, group=None):
    from waveforcing_b200 import _lib as L
    from waveforcing_b200.runtime import backend
    from waveforcing_b200.wavefront.dit import DiTConfig, WanDiT
    from waveforcing_b200.wavefront.engine import EngineConfig, WavefrontEngine

    backend.select_backend("wf_b200")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    cfg = DiTConfig(dim=256, heads=2, layers=2, ffn=512, text_len=16, text_dim=64, lat_h=16, lat_w=24)
    model = WanDiT.random(cfg, dev, seed=0)
    g = torch.Generator(device="cpu").manual_seed(1)
    model.set_text(torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(dev))
    eng = WavefrontEngine(model, EngineConfig(steps=STEPS, num_frames=27, fp8_kv=fp8, timeout_s=20.0),
                          rank=rank, world=world, device=dev, group=group)
    for t in range(eng.num_ticks):
        eng.tick(t)
    torch.cuda.synchronize()
    eng.xport.check_timeouts()
    status = L.status_take()
    final = {c: x.float().cpu() for c, x in eng.final.items()}
    eng.close()
    return final, status


def _worker(rank, world, port, fp8, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    try:
        final, status = _engine_run(rank, world, fp8)
        # numpy, not tensors: a queued tensor's shared storage dies with its sender
        q.put((rank, {c: x.numpy() for c, x in final.items()}, status))
    except Exception as e:  # report, then leave the group without further collectives
        q.put((rank, repr(e), -1))
    finally:
        dist.destroy_process_group()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _multi(world, fp8):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, fp8, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = {}
    for _ in ps:
        r, final, st = q.get(timeout=300)
        out[r] = (final, st)
    for p in ps:
        p.join(timeout=60)
    return out


@pytest.mark.parametrize("fp8", [False, True])
def test_two_gpu_wavefront_matches_single_gpu(fp8):
    single, st1 = _engine_run(0, 1, fp8)
    assert st1 == 0
    multi = _multi(2, fp8)
    for r, (final, st) in multi.items():
        assert not isinstance(final, str), final
        assert st == 0, f"rank {r}: a bounded wait gave up"
    store_final = {}
    for final, _ in multi.values():
        store_final.update({c: torch.from_numpy(x) for c, x in final.items()})
    assert sorted(store_final) == sorted(single)
    a = torch.cat([single[c] for c in sorted(single)], 1).double().flatten()
    b = torch.cat([store_final[c] for c in sorted(single)], 1).double().flatten()
    cos = torch.nn.functional.cosine_similarity(a, b, dim=0).item()
    assert cos >= 0.999, cos
