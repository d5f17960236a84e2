"""Steady-state wavefront throughput of the WaveRT per-layer DiT hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {wf,reference}]
                    [--preset 1.3b] [--kv fp8|bf16] [--w8a8 none|e4m3|int8]

Workload (metric "steady FPS p50"): the 1.3B-shaped 5-step
wavefront (steps 1000,800,600,400,200 + the clean-KV store stage) at 480x832
(60x104 latents, 4680 tokens per 3-frame chunk), random-init bf16 weights,
512-token N(0,1) text context, Gaussian noise from seed 0.  The rf_step+1
stages are placed on the N ranks (merged when N < 6; ranks beyond 6 idle).
One bench step = one steady-state tick (every stage active, anchor + 7 clean
pages); each tick denoises one 3-latent-frame chunk = 12 output frames, so
steady FPS = 12000 / p50(tick ms) over the timed ticks (the reference's
definition, scripts/sweep_matrix.py:34-35,213-228, on the steady window).
Ticks before the timed window fill the pipeline and are untimed.

``value``  device-timed: noise resident in HBM, CUDA events on every rank,
           per-tick max over ranks, p50.
``e2e``    the same ticks driven from pinned HOST noise: each tick copies its
           noise chunk host->device and reads the finished latent chunk back.
``--impl reference``  the reference's torch CPU path (oracle port, all host
           threads): each step is BASELINE config 1 measured in full (FP8
           round trip, 12-head SDPA, one linear); `value` is the steady FPS
           the measured rates give for this tick's work.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

FRAMES_PER_TICK = 12  # 3 latent frames -> 12 output frames per chunk
METRIC = "steady FPS p50 (1.3B 5-step wavefront, 399 latent frames, 480x832)"


def metric_name(args) -> str:
    """The metric of this run: BASELINE's name for its default workload, the
    same form naming the preset and step count otherwise."""
    S = len(args.denoise_steps.split(","))
    if args.preset == "1.3b" and S == 5:
        return METRIC
    return f"steady FPS p50 ({args.preset.upper()} {S}-step wavefront, 399 latent frames, 480x832)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="wf", choices=["wf", "reference", "reference-gpu"],
                    help="reference: the reference's CPU torch path on the host cores (the driver's reference "
                         "arm); reference-gpu: the reference's own wavefront engine and paged exchange on GPUs "
                         "(one rank per stage, torch SDPA, bf16 K/V), for the comparison on the same box")
    ap.add_argument("--preset", default="1.3b")
    ap.add_argument("--kv", default="fp8", choices=["fp8", "bf16"])
    ap.add_argument("--w8a8", default="none", choices=["none", "e4m3", "int8"])
    ap.add_argument("--denoise-steps", default="1000,800,600,400,200")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--vae", action="store_true",
                    help="also run the whole wavefront with streaming VAE decode of every finished chunk "
                         "(on ranks without stages when there are any, else on the store rank)")
    ap.add_argument("--kernel", default=None,
                    choices=["attn", "attn8", "gemm", "actq", "codec", "dequant", "assemble", "publish", "qkpub",
                             "vae"],
                    help="time one hot-path kernel alone at the steady r0 shape (for ncu captures)")
    ap.add_argument("--ctx-chunks", type=int, default=8, help="--kernel attn: K/V length in chunks")
    ap.add_argument("--kv-len", type=int, default=0,
                    help="--kernel attn: K/V length in tokens (overrides --ctx-chunks; 512 = cross-attention)")
    ap.add_argument("--q-len", type=int, default=0,
                    help="--kernel attn: query length in tokens (default one chunk; 28080 = the tick's "
                         "batched cross-attention of six stages)")
    ap.add_argument("--gemm-nk", default="", help="--kernel gemm: N,K (default the FFN fc_in)")
    ap.add_argument("--act-k", type=int, default=0, help="--kernel actq: row length K (default the FFN width)")
    ap.add_argument("--act-gelu", action="store_true",
                    help="--kernel actq: quantise GELU_tanh(x) (fc_out's input); --kernel gemm: GELU epilogue")
    ap.add_argument("--library", action="store_true",
                    help="--kernel attn: also time torch SDPA, the reference's attention call, on the same buffers")
    ap.add_argument("--trace", action="store_true",
                    help="profile two steady ticks with torch.profiler (CUPTI): in-stream kernel time, device idle "
                         "inside the tick, per-kernel shares (one JSON line; no bench line)")
    ap.add_argument("--timeline", default="",
                    help="after the timed ticks, write a cross-rank device timeline of --steps more steady ticks to "
                         "this JSON file: globaltimer stamps at every tick phase, layer entry and remote flag wait, "
                         "aligned at a world all_reduce (no profiler; one extra summary JSON line)")
    ap.add_argument("--forward", action="store_true",
                    help="BASELINE config 2: one full DiT forward of a 3-frame chunk at t=600 with a 6-chunk context")
    return ap.parse_args()


# --------------------------------------------------------------------- util
def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- CPU side
def steady_tick_work(cfg, rf_step: int, max_attn_frames: int = 21, npb: int = 3) -> dict:
    """Algorithmic work of one steady-state tick of the rf_step wavefront + store
    (every stage active, anchor + 7 clean pages).  Stage s < rf_step attends to
    naw + 1 + (rf_step - s) chunks (anchor/working, live store slot, its own
    chunk, the higher stages' in-flight chunks; wave_rt/denoiser/exchange/
    paged.py:160-189); the store attends to anchor + clean pages + its own
    chunk.  Linears per stage and layer: q, k, v, o, cross q, cross o on T
    rows (6 dim^2) and the FFN (2 dim ffn); the cross k/v of the 512 text rows
    are cached once.  FP8 codec: stages 1..rf_step-1 and the store publish
    (quantise) one K and one V chunk per layer; stage s receives (dequantises)
    rf_step - s chunks of K and of V per layer."""
    T, dim, ffn, Ln = cfg.tokens_per_chunk, cfg.dim, cfg.ffn, cfg.layers
    wmax = max(0, (max_attn_frames - rf_step * npb - npb) // npb)
    naw = 1 + wmax
    ctx = [naw + 1 + (rf_step - s) for s in range(rf_step)]
    ctx.append(1 + max(0, (max_attn_frames - 2 * npb) // npb) + 1)
    stages = rf_step + 1
    return {
        "ctx_chunks": ctx,
        "attn_flops": Ln * sum(4.0 * T * c * T * dim for c in ctx),
        "cross_flops": Ln * stages * 4.0 * T * cfg.text_len * dim,
        "linear_flops": Ln * stages * 2.0 * T * (6 * dim * dim + 2 * dim * ffn),
        "quant_elems": Ln * rf_step * 2.0 * T * dim,
        "dequant_elems": Ln * (rf_step * (rf_step + 1) // 2) * 2.0 * T * dim,
    }


def _config1_inputs(cfg, seed: int = 0):
    """q one 3-frame chunk, K/V three chunks (two prior +
    current), fp32 N(0,1)/sqrt(head_dim) from seed 0."""
    T, H, D = cfg.tokens_per_chunk, cfg.heads, cfg.head_dim
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, T, H, D, generator=g) / math.sqrt(D)
    k = torch.randn(1, 3 * T, H, D, generator=g) / math.sqrt(D)
    v = torch.randn(1, 3 * T, H, D, generator=g) / math.sqrt(D)
    return q, k, v


def cpu_config1_sample(cfg, inputs):
    """One measured sample of the reference's CPU torch path
    in full (all heads):
      * the per-tensor FP8 K/V codec of wave_rt/denoiser/exchange/common.py:
        143-164 on stack(K, V) in the runtime dtype (quantise, then dequantise);
      * attention: F.scaled_dot_product_attention in fp32 on the transposed
        [B, H, L, D] views, as naive_rt/rolling_forcing/wan/modules/
        attention.py:76-89, on the dequantised K/V;
      * one T-row linear of the layer (the q projection, dim x dim) in fp32.
    Returns the wall seconds of each part."""
    from oracle import attention as oattn
    from oracle import codec as ocodec

    q, k, v = inputs
    T, H, D = cfg.tokens_per_chunk, cfg.heads, cfg.head_dim
    L = k.shape[1]
    t0 = time.perf_counter()
    kv = torch.stack([k[0], v[0]]).to(torch.bfloat16).reshape(2 * L, H * D)
    codes, scale = ocodec.quant_per_tensor_torch(kv)
    t1 = time.perf_counter()
    deq = ocodec.dequant_torch(codes, scale, per_token=False)
    t2 = time.perf_counter()
    oattn.sdpa_reference_torch(q, deq[:L].reshape(1, L, H, D), deq[L:].reshape(1, L, H, D))
    t3 = time.perf_counter()
    w = torch.randn(cfg.dim, cfg.dim) * 0.02
    t4 = time.perf_counter()
    torch.nn.functional.linear(q.reshape(T, H * D), w)
    t5 = time.perf_counter()
    return {"quant_s": t1 - t0, "dequant_s": t2 - t1, "attn_s": t3 - t2, "linear_s": t5 - t4,
            "codec_elems": float(2 * L * H * D), "attn_flops": 4.0 * T * L * H * D,
            "linear_flops": 2.0 * T * cfg.dim * cfg.dim}


def cpu_tick_model(cfg, rf_step: int, samples: list) -> dict:
    """Steady tick on the host's cores from the measured config-1 rates: the
    tick's attention (self + cross) at the measured SDPA FLOP/s, its linears at
    the measured linear FLOP/s, its FP8 publishes and receives at the measured
    quantise and dequantise element rates (medians over the samples)."""
    med = lambda key: statistics.median(x[key] for x in samples)  # noqa: E731
    s0 = samples[0]
    attn_rate = s0["attn_flops"] / med("attn_s")
    lin_rate = s0["linear_flops"] / med("linear_s")
    q_rate = s0["codec_elems"] / med("quant_s")
    d_rate = s0["codec_elems"] / med("dequant_s")
    w = steady_tick_work(cfg, rf_step)
    parts = {"attention_s": (w["attn_flops"] + w["cross_flops"]) / attn_rate,
             "linears_s": w["linear_flops"] / lin_rate,
             "codec_s": w["quant_elems"] / q_rate + w["dequant_elems"] / d_rate}
    tick_s = sum(parts.values())
    return {"tick_s": tick_s, "fps": FRAMES_PER_TICK / tick_s, "parts": parts,
            "rates": {"sdpa_tflops": attn_rate / 1e12, "linear_tflops": lin_rate / 1e12,
                      "quant_gelem_s": q_rate / 1e9, "dequant_gelem_s": d_rate / 1e9},
            "config1_layer_s": med("quant_s") + med("dequant_s") + med("attn_s")}


def cpu_baseline(cfg, rf_step: int, min_s: float = 10.0, max_samples: int = 64) -> dict:
    """The cpu_baseline object of the bench line: config-1 samples on all host
    threads for about `min_s` seconds, converted to steady FPS by cpu_tick_model."""
    threads = torch.get_num_threads()
    inputs = _config1_inputs(cfg)
    samples = []
    t0 = time.perf_counter()
    while not samples or (time.perf_counter() - t0 < min_s and len(samples) < max_samples):
        samples.append(cpu_config1_sample(cfg, inputs))
    m = cpu_tick_model(cfg, rf_step, samples)
    L = 3 * cfg.tokens_per_chunk
    return {"value": m["fps"], "unit": "FPS", "cores": threads, "nproc": os.cpu_count(), "kind": "port",
            "sample": (f"BASELINE config 1 measured in full on the host: per-tensor FP8 round trip of stack(K,V) "
                       f"[2x{L}x{cfg.dim}] (common.py:143-164), fp32 SDPA q {cfg.tokens_per_chunk} x K/V {L} x "
                       f"{cfg.heads} heads (attention.py:76-89), one {cfg.tokens_per_chunk}x{cfg.dim}x{cfg.dim} "
                       f"linear; {len(samples)} samples; tick = measured rates x the tick's work "
                       f"(attention + cross FLOPs, linear FLOPs, codec elements)"),
            "config1_layer_ms": 1e3 * m["config1_layer_s"], "tick_s_model": m["tick_s"],
            "tick_parts_s": m["parts"], "rates": m["rates"], "samples": len(samples)}


def gpu_config1(cfg, dev, reps: int = 10) -> dict:
    """The GPU time of the same config-1 call as cpu_config1_sample: libwfk's
    per-tensor FP8 round trip of stack(K, V) (wf_kv_quant + wf_kv_dequant) and
    wf_attn_fwd, CUDA-event timed over `reps` calls after warm-up."""
    from waveforcing_b200 import _lib as L
    from waveforcing_b200 import kernels

    q, k, v = _config1_inputs(cfg)
    H, D, Lk = cfg.heads, cfg.head_dim, k.shape[1]
    qd = q.to(dev).bfloat16()
    kv = torch.stack([k[0], v[0]]).to(dev).bfloat16().reshape(2 * Lk, H * D)
    codes = torch.empty(2 * Lk, H * D, device=dev, dtype=torch.uint8)
    scale = torch.empty(1, device=dev)
    ws = torch.empty(1, device=dev, dtype=torch.int32)
    deq = torch.empty(2 * Lk, H * D, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(qd)

    def call():
        kernels.kv_quant(kv, L.WF_SCALE_TENSOR, codes=codes, scales=scale, workspace=ws)
        kernels.kv_dequant(codes, scale, L.WF_SCALE_TENSOR, out=deq)
        d = deq.view(2, 1, Lk, H, D)
        kernels.attention(qd, d[0], d[1], out=out)

    for _ in range(3):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        call()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    return {"gpu_ms": ms, "what": f"BASELINE config 1 layer: per-tensor FP8 round trip of stack(K,V) + attention, "
                                  f"q {cfg.tokens_per_chunk} x K/V {Lk} x {H} heads (bf16 on the GPU, fp32 on the host)"}


def bench_config(args, world: int) -> dict:
    """The `config` object, identical in both arms for the same flags."""
    from waveforcing_b200.wavefront.dit import DiTConfig
    from waveforcing_b200.wavefront.engine import place_stages

    cfg = DiTConfig.preset(args.preset)
    S = len(args.denoise_steps.split(","))
    return {"workload": f"{args.preset} {S}-step wavefront + store, steady tick, stages merged onto "
                        f"{min(world, S + 1)} rank(s)",
            "model": f"Wan2.1-{args.preset}-shape", "tokens_per_chunk": cfg.tokens_per_chunk,
            "denoise_steps": args.denoise_steps, "kv_transport": args.kv, "w8a8": args.w8a8, "world": world,
            "l2": "inputs larger than L2 (K/V slabs and weights, GBs per tick)",
            "parallelism": f"wavefront stages over {min(world, S + 1)} GPU(s)",
            "stage_rank": place_stages(S, world)}


def run_reference_arm(args):
    """The reference's CPU torch path on the host's cores (rank 0 only): each
    step is one measured config-1 sample (cpu_config1_sample), its wall time is
    ms_per_step, and `value` is the steady FPS that the measured rates give for
    this config's tick (cpu_tick_model)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from waveforcing_b200.wavefront.dit import DiTConfig

    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = DiTConfig.preset(args.preset)
    S = len(args.denoise_steps.split(","))
    inputs = _config1_inputs(cfg)
    for _ in range(max(0, args.warmup)):
        cpu_config1_sample(cfg, inputs)
    samples, walls = [], []
    for _ in range(max(1, args.steps)):
        t0 = time.perf_counter()
        samples.append(cpu_config1_sample(cfg, inputs))
        walls.append(time.perf_counter() - t0)
    m = cpu_tick_model(cfg, S, samples)
    threads = torch.get_num_threads()
    desc = (f"each step = BASELINE config 1 in full on the host (per-tensor FP8 K/V round trip, fp32 SDPA "
            f"{cfg.tokens_per_chunk}x{3 * cfg.tokens_per_chunk}x{cfg.heads} heads, one dim x dim linear); value = "
            f"steady FPS of the tick at the measured rates (tick {m['tick_s']:.1f} s)")
    line = {
        "impl": "reference", "metric": metric_name(args), "value": m["fps"], "unit": "FPS", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * statistics.median(walls),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (config 1 inputs, seed 0)", "config": bench_config(args, world),
        "cpu_baseline": {"value": m["fps"], "unit": "FPS", "cores": threads, "nproc": os.cpu_count(), "kind": "port",
                         "sample": desc},
        "e2e": {"value": m["fps"], "unit": "FPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "tick_s_model": m["tick_s"], "tick_parts_s": m["parts"], "rates": m["rates"],
        "config1_layer_ms": 1e3 * m["config1_layer_s"],
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------- reference on GPUs
def run_reference_gpu_arm(args):
    """The reference's own GPU path on this box: wave_rt's WaveDenoiser
    (wave_rt/denoiser/engine.py) in ``paged`` mode with the reference's own
    PagedExchangeMixin and CUDA-IPC layer (wave_rt/distributed/ipc.py), bf16
    K/V, torch SDPA attention, over the Wan-shaped DiT in plain torch ops
    (baseline/harness.py: SGLang's backend and RoPE helpers stood in).  The
    reference needs one rank per stage, rf_step + 1 (wave_rt/config.py:79-83),
    so it runs only at that world size.  Metric as the reference reports it:
    steady FPS = 12000 / p50(per-tick ms [12:-4]) from the engine's own tick
    timer (max over ranks per tick), DiT FPS = 1596 / diffusion seconds
    (scripts/sweep_matrix.py:34-35,137-138,213-228; wave_rt/bench.py:81)."""
    import datetime

    steps_list = tuple(int(x) for x in args.denoise_steps.split(","))
    S = len(steps_list)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != S + 1:
        if rank == 0:
            print(json.dumps({"impl": "reference-gpu", "unavailable":
                              f"the reference runs one rank per stage: world {S + 1} for {S} steps, got {world}"}))
        return
    from baseline import harness

    if harness.reference_checkout() is None:
        if rank == 0:
            print(json.dumps({"impl": "reference-gpu", "unavailable": "no reference package in baseline/_ref "
                                                                      "(python baseline/install_ref.py <checkout>)"}))
        return
    from waveforcing_b200.runtime import backend
    from waveforcing_b200.wavefront.dit import DiTConfig, FlowMatch, WanDiT

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=180))
    torch.set_grad_enabled(False)
    engine = harness.import_reference()
    backend.select_backend("torch_sdpa")
    cfg = DiTConfig.preset(args.preset)
    model = WanDiT.random(cfg, dev, seed=0)
    g = torch.Generator(device="cpu").manual_seed(0)
    model.set_text(torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(dev))
    fm = FlowMatch()
    dsl = [fm.timestep(x) for x in steps_list]
    gn = torch.Generator(device="cpu").manual_seed(0)
    nf = 399
    noise = torch.randn((cfg.in_ch, nf, cfg.lat_h, cfg.lat_w), generator=gn).to(torch.bfloat16)
    be = harness.StubBackend(rank=rank, device=dev, dtype=torch.bfloat16, num_layers=cfg.layers, heads=cfg.heads,
                             head_dim=cfg.head_dim, channels=cfg.in_ch, lat_h=cfg.lat_h, lat_w=cfg.lat_w,
                             tokens_per_frame=cfg.tokens_per_frame, steps=dsl, full_noise=noise[None].to(dev),
                             model=harness.wan_forward(model, fused=False))
    wcfg = harness.make_config(engine, rf_step=S, steps=dsl, num_frames=nf, exchange_mode="paged")
    den = engine.WaveDenoiser(be, wcfg)
    den._warmup(n_iters=max(1, min(3, args.warmup)))
    dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
    t0 = time.perf_counter()
    final, tick_ms, _ = den._systolic(be.full_noise_bcthw, warmup_pass=False, num_ticks=den.num_ticks)
    torch.cuda.synchronize()
    dist.barrier()
    wall = time.perf_counter() - t0
    clocks = sampler.stop() if sampler else None
    t = torch.tensor(tick_ms, device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    tick_ms = t.tolist()
    wt = torch.tensor([wall], device=dev, dtype=torch.float64)
    dist.all_reduce(wt, op=dist.ReduceOp.MAX)
    wall = wt.item()
    den.close()
    if rank == 0:
        steady = tick_ms[12:-4]
        p50 = statistics.median(steady)
        print(json.dumps({
            "impl": "reference-gpu", "metric": metric_name(args), "value": FRAMES_PER_TICK * 1000.0 / p50, "unit": "FPS",
            "n_gpus": world, "tick_ms_p50": p50, "higher_is_better": True,
            "dit_fps": {"value": 4 * nf / wall, "unit": "FPS", "diffusion_s": wall},
            "ticks": len(tick_ms), "steady_ticks": len(steady), "dtype": "bf16", "data": "synthetic",
            "config": dict(bench_config(args, world), kv_transport="bf16", attention="torch SDPA",
                           engine="reference wave_rt WaveDenoiser + PagedExchangeMixin (CUDA IPC)"),
            "timing": "the engine's own per-tick host timer (no per-tick sync), max over ranks; "
                      "DiT FPS from the barrier-bracketed wall time of all ticks",
            "clocks": clocks}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


# ------------------------------------------------------------------ trace
def trace_ticks(args, make_engine, noise_cpu, fill, dev, rank, n_trace: int = 2):
    """Device activity of ``n_trace`` steady ticks from a CUPTI trace
    (torch.profiler): every kernel's in-stream start and end.  Reports the
    union of kernel intervals against the span from the first kernel to the
    last (device idle inside the ticks), the host time to issue the ticks,
    and each kernel family's share of the summed kernel time."""
    from torch.profiler import ProfilerActivity, profile

    eng = make_engine(noise_cpu.to(dev))
    eng_local = eng.local
    for t in range(fill + max(1, args.warmup)):
        eng.tick(t)
    torch.cuda.synchronize()
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
    t0 = fill + max(1, args.warmup)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        h0 = time.perf_counter()
        for i in range(n_trace):
            eng.tick(t0 + i)
        host_ms = (time.perf_counter() - h0) * 1e3
        torch.cuda.synchronize()
    eng.close()
    ivs = []
    by_name: dict = {}
    for e in prof.events():
        if e.device_type != torch.autograd.DeviceType.CUDA:
            continue
        start = e.time_range.start
        end = e.time_range.end
        if end <= start:
            continue
        ivs.append((start, end))
        key = e.name.split("(")[0].split("<")[0].strip()
        by_name[key] = by_name.get(key, 0.0) + (end - start)
    ivs.sort()
    busy, cur_s, cur_e = 0.0, None, None
    for s_, e_ in ivs:
        if cur_e is None or s_ > cur_e:
            if cur_e is not None:
                busy += cur_e - cur_s
            cur_s, cur_e = s_, e_
        else:
            cur_e = max(cur_e, e_)
    if cur_e is not None:
        busy += cur_e - cur_s
    span = (ivs[-1][1] - ivs[0][0]) if ivs else 0.0
    total = sum(by_name.values())
    top = sorted(by_name.items(), key=lambda kv: -kv[1])[:16]
    # every rank's own device activity (stages hosted, kernel-busy time per
    # tick); waits in flag/credit kernels count as busy, so they are listed
    wait_keys = ("wait_flag_kernel",)
    waits = sum(v for k, v in by_name.items() if any(w in k for w in wait_keys))
    mine = {"rank": rank, "stages": list(eng_local), "busy_ms_per_tick": busy / 1e3 / n_trace,
            "flag_wait_ms_per_tick": waits / 1e3 / n_trace,
            "busy_minus_waits_ms_per_tick": (busy - waits) / 1e3 / n_trace,
            "nccl_ms_per_tick": sum(v for k, v in by_name.items() if "nccl" in k.lower()) / 1e3 / n_trace}
    per_rank = [mine]
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        per_rank = [None] * dist.get_world_size()
        dist.all_gather_object(per_rank, mine)
    if rank == 0:
        print(json.dumps({
            "trace": f"{n_trace} steady ticks, rank {rank}", "kernels": len(ivs),
            "kernels_per_tick": len(ivs) / n_trace, "span_ms_per_tick": span / 1e3 / n_trace,
            "busy_ms_per_tick": busy / 1e3 / n_trace, "idle_frac": 1 - busy / span if span else None,
            "kernel_sum_ms_per_tick": total / 1e3 / n_trace, "host_issue_ms_per_tick": host_ms / n_trace,
            "shares": [{"kernel": k, "ms_per_tick": v / 1e3 / n_trace, "share": v / total} for k, v in top],
            "per_rank": per_rank,
            "note": "CUPTI kernel timestamps (profiler overhead on the host side; kernel durations in-stream)"}),
            flush=True)


def timeline_ticks(args, eng, t0, dev, rank, world):
    """Device stamps (``wf_stamp``) of ``args.steps`` further steady ticks of
    ``eng`` (from tick ``t0``) on every rank, aligned at a world all_reduce,
    written to ``args.timeline``.  Per rank and tick they give the stream's
    phase times (begin, slots acquired, forward done, promotion, migration
    received) and per layer the entry and the end of each remote flag wait.
    Run after the timed ticks, so the stamps' launches are not in them."""
    from waveforcing_b200.wavefront.timeline import Timeline

    torch.cuda.synchronize()
    tl = Timeline(dev)
    eng.timeline = tl
    eng.xport.timeline = tl
    tl.align()
    for i in range(args.steps):
        eng.tick(t0 + i)
    rows = tl.rows()
    eng.timeline = eng.xport.timeline = None
    mine = {"rank": rank, "stages": list(eng.local), "rows": rows}
    allr = [mine]
    if world > 1:
        allr = [None] * world
        dist.all_gather_object(allr, mine)
    if rank == 0:
        with open(args.timeline, "w") as f:
            json.dump({"ticks": [t0, t0 + args.steps], "ranks": allr}, f)
        span = {}
        for r in allr:
            d = dict(r["rows"])
            for i in range(args.steps):
                t = t0 + i
                if f"t{t}.begin" in d and f"t{t}.migrated" in d:
                    span.setdefault(t, []).append((r["rank"], d[f"t{t}.begin"], d[f"t{t}.forward"],
                                                   d[f"t{t}.migrated"]))
        ticks = sorted(span)
        period = [(max(x[3] for x in span[b]) - max(x[3] for x in span[a])) / 1e3 for a, b in zip(ticks, ticks[1:])]
        print(json.dumps({"timeline": args.timeline, "ticks": ticks, "stamps_per_rank": [len(r["rows"]) for r in allr],
                          "tick_period_ms": period}), flush=True)


# ---------------------------------------------------------------- GPU side
def run_gpu_arm(args):
    from waveforcing_b200 import kernels
    from waveforcing_b200.runtime import backend
    from waveforcing_b200.runtime.fp8 import quantize_transformer_w8a8
    from waveforcing_b200.wavefront.dit import DiTConfig, WanDiT
    from waveforcing_b200.wavefront.engine import EngineConfig, WavefrontEngine

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=300))
    torch.set_grad_enabled(False)
    backend.select_backend("wf_b200")

    steps_list = tuple(int(s) for s in args.denoise_steps.split(","))
    S = len(steps_list)
    fill = S + 8  # first tick with every stage active and anchor + 7 clean pages
    n_ticks = fill + args.warmup + args.steps * (2 if args.timeline else 1)
    cfg = DiTConfig.preset(args.preset)
    # the 399-frame run; only its first n_ticks ticks are executed (fill, warm-up, timed steady window)
    ecfg = EngineConfig(steps=steps_list, num_frames=399, fp8_kv=(args.kv == "fp8"))
    if n_ticks > ecfg.num_blocks:
        raise SystemExit(f"--steps/--warmup too large: {n_ticks} ticks > {ecfg.num_blocks} chunks")
    model = WanDiT.random(cfg, dev, seed=0)
    if args.w8a8 != "none":
        quantize_transformer_w8a8(model, scope="all", qtype=args.w8a8, granularity="channel")
    g = torch.Generator(device="cpu").manual_seed(0)
    text = torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(dev)
    model.set_text(text)

    def make_engine(noise):
        return WavefrontEngine(model, ecfg, rank=rank, world=world, device=dev, noise=noise)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(vals: list[float]) -> list[float]:
        t = torch.tensor(vals, device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    # ---------------- device-resident run (value)
    gn = torch.Generator(device="cpu").manual_seed(ecfg.seed)
    noise_cpu = torch.randn((cfg.in_ch, ecfg.num_frames, cfg.lat_h, cfg.lat_w), generator=gn).to(torch.bfloat16)
    if args.trace:
        trace_ticks(args, make_engine, noise_cpu, fill, dev, rank)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    eng = make_engine(noise_cpu.to(dev))
    for t in range(fill + args.warmup):
        eng.tick(t)
    barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
    attn_sink: list = []
    wait_sink: list = []
    backend.set_attention_timer(attn_sink)
    eng.xport.wait_timer = wait_sink
    launches0 = kernels.LAUNCHES[0]
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    host_ms = []
    evs[0].record()
    torch.cuda.nvtx.range_push("timed")
    ahead = 0  # ticks whose issue began while the device was still on earlier work
    for i in range(args.steps):
        h0 = time.perf_counter()
        if i > 0:  # evs[i] closes tick i - 1
            ahead += 0 if evs[i].query() else 1
        eng.tick(fill + args.warmup + i)
        host_ms.append((time.perf_counter() - h0) * 1e3)
        evs[i + 1].record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    backend.set_attention_timer(None)
    launches = kernels.LAUNCHES[0] - launches0
    clocks = sampler.stop() if sampler else None
    tick_ms = max_over_ranks([evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)])
    total_ms = max_over_ranks([evs[0].elapsed_time(evs[-1])])[0]
    p50 = statistics.median(tick_ms)
    fps = FRAMES_PER_TICK * 1000.0 / p50
    # attention roofline from the live events of the timed region (rank 0's GPU)
    a_flops = sum(x[0] for x in attn_sink)
    a_ms = sum(x[1].elapsed_time(x[2]) for x in attn_sink)
    n_attn = len(attn_sink)
    a_bytes = sum(x[3] for x in attn_sink) / max(1, n_attn)
    eng.xport.wait_timer = None
    # exposed exchange: device time this rank's compute stream spent in remote flag waits
    wait_ms_rank = sum(e0.elapsed_time(e1) for e0, e1 in wait_sink) / args.steps
    wait_ms = max_over_ranks([wait_ms_rank])[0]
    # Every rank's tick has the same length, so the critical (busiest) rank is
    # the active rank that waits least; its waits are the exchange time exposed
    # on the critical path.  Ranks without stages (N = 8: two) are left out.
    crit = -max_over_ranks([-wait_ms_rank if eng.local else float("-inf")])[0]
    stage0_wait = max_over_ranks([wait_ms_rank if 0 in eng.local else 0.0])[0]
    host_p50 = max_over_ranks([statistics.median(host_ms)])[0]
    # lowest over ranks: 1.0 means the host was ahead at every tick (device-bound)
    host_ahead = -max_over_ranks([-ahead / max(1, args.steps - 1) if eng.local else float("-inf")])[0]
    if args.timeline:
        timeline_ticks(args, eng, fill + args.warmup + args.steps, dev, rank, world)
    eng.close()
    del eng
    torch.cuda.empty_cache()

    # ---------------- host-driven full run (e2e and DiT FPS)
    # The whole 399-frame wavefront (all ticks, fill and drain included), driven
    # from pinned HOST noise: every tick copies its noise chunk host->device and
    # every finished latent chunk is read back to pinned host memory.  e2e =
    # 12000 / p50 of its steady ticks; DiT FPS = 1596 / diffusion seconds
    # (scripts/sweep_matrix.py:463, wave_rt/bench.py:81).
    e2e, dit = None, None
    if not args.no_e2e:
        noise_host = noise_cpu.pin_memory()
        eng = make_engine(noise_host)
        out_host = torch.empty((cfg.in_ch, 3, cfg.lat_h, cfg.lat_w), dtype=torch.bfloat16).pin_memory()
        nt = eng.num_ticks
        barrier()
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(nt + 1)]
        ev[0].record()
        d2h = 0
        for t in range(nt):
            eng.tick(t)  # copies its noise chunk from pinned host memory (engine.noise_chunk)
            c = t - eng.store
            if c in eng.final:
                out_host.copy_(eng.final.pop(c), non_blocking=True)
                d2h += out_host.numel() * out_host.element_size()
            ev[t + 1].record()
        torch.cuda.synchronize()
        barrier()
        tms = max_over_ranks([ev[i].elapsed_time(ev[i + 1]) for i in range(nt)])
        total_s = max_over_ranks([ev[0].elapsed_time(ev[-1]) / 1e3])[0]
        steady = tms[fill:nt - S] if nt - S > fill else tms
        h2d = cfg.in_ch * 3 * cfg.lat_h * cfg.lat_w * 2 if 0 in eng.local else 0
        tot = max_over_ranks([float(h2d), float(d2h) / nt])
        e2e = {"value": FRAMES_PER_TICK * 1000.0 / statistics.median(steady), "unit": "FPS",
               "h2d_bytes_per_step": int(tot[0]), "d2h_bytes_per_step": int(tot[1]),
               "ticks": nt, "steady_ticks": len(steady)}
        dit = {"value": 4 * ecfg.num_frames / total_s, "unit": "FPS", "diffusion_s": total_s,
               "definition": "output frames (4 x 399 latent) / wall time of all ticks incl. fill and drain"}
        eng.close()
        del eng

    vae_e2e = run_vae_e2e(args, make_engine, noise_cpu, cfg, dev, rank, world, barrier, max_over_ranks) \
        if args.vae else None

    peaks, src = _peaks()
    if rank == 0:
        achieved = a_flops / (a_ms * 1e-3) / 1e12 if a_ms > 0 else None
        peak = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops"))
        traffic = None
        tp = os.path.join(ROOT, "profiles", "attention_traffic.json")
        if os.path.exists(tp):
            # DRAM bytes of the captured r0 launch equal its algorithmic bytes (ratio in the
            # profile); scale that ratio to the mean launch of this run
            with open(tp) as f:
                traffic = a_bytes * json.load(f)["ratio_traffic_to_algorithmic"]
        cpu = None
        config1 = None
        if world == 1:
            torch.set_num_threads(os.cpu_count() or 1)
            cpu = cpu_baseline(cfg, S)
            config1 = gpu_config1(cfg, dev)
            config1["cpu_ms"] = cpu["config1_layer_ms"]
            config1["cpu_over_gpu"] = cpu["config1_layer_ms"] / config1["gpu_ms"]
        line = {
            "metric": metric_name(args), "value": fps, "unit": "FPS", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "tick_ms_p50": p50,
            "tick_ms": [round(x, 2) for x in tick_ms],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init N(0,0.02) weights, N(0,1) text, seed-0 Gaussian noise)",
            "config": bench_config(args, world),
            "roofline": {"bound": "tensor",
                         "kernel": "attn_fwd_bf16_kernel (wavefront self-attention; the text cross-attention "
                                   "runs on torch SDPA, as in the reference)",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": (achieved / peak) if achieved else None, "traffic": traffic,
                         "traffic_source": ("not measured in this run: the mean launch's algorithmic bytes x "
                                            "the DRAM/algorithmic ratio of the committed ncu capture "
                                            "(profiles/attention_traffic.json)") if traffic is not None else None,
                         "launches": n_attn, "peak_source": f"{src} bf16_tflops_sustained"},
            "cpu_baseline": cpu,
            "config1": config1,
            "e2e": e2e,
            **({"e2e_with_vae": vae_e2e} if vae_e2e is not None else {}),
            "dit_fps": dit,
            "exchange": {"critical_rank_wait_ms_per_tick": crit,
                         "critical_frac_of_tick": crit / p50 if p50 else None,
                         "max_rank_wait_ms_per_tick": wait_ms,
                         "stage0_rank_wait_ms_per_tick": stage0_wait,
                         "note": "device time consumer streams spent in bounded flag waits for remote K/V; "
                                 "the critical rank is the active rank that waits least (the busiest: its "
                                 "waits are on the critical path); lighter ranks wait for slower producers"},
            "host_issue_ms_per_tick_p50": host_p50,
            "host_ahead_frac": host_ahead,
            "gpu_launches": launches,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_kernel_bench(args):
    """One hot-path kernel alone, CUDA-event timed, at the steady-state r0 shape:
      attn  q [4680, H, 128] vs K/V [ctx*4680, H, 128] bf16 (r0 sees 8 chunks)
      gemm  W8A8 e4m3 FFN fc_in [4680 x dim] x [ffn x dim]^T
      codec per-token FP8 quantise-and-publish of one layer's K and V to 4 slots
      dequant per-token FP8 dequantise of one layer's 5 received K and V slots
              into the bf16 context buffer (one launch for K, one for V)
      assemble one layer's r0 K/V context in one wf_kv_assemble launch: anchor
              key re-RoPEd into slot 0, anchor value, one working page and
              the own chunk copied, 5 received FP8 slots dequantised
    The launches rotate over independent buffer sets whose total footprint
    exceeds L2 (126 MB), so each launch reads its inputs from HBM, and `steps`
    launches are captured in one CUDA graph so that host-side argument
    marshalling stays out of the timed region."""
    from waveforcing_b200 import _lib as L
    from waveforcing_b200 import kernels
    from waveforcing_b200.wavefront.dit import DiTConfig

    cfg = DiTConfig.preset(args.preset)
    dev = torch.device("cuda", 0)
    T, H, D = cfg.tokens_per_chunk, cfg.heads, cfg.head_dim
    g = torch.Generator(device=dev).manual_seed(0)
    l2 = 126e6

    def n_sets(set_bytes):
        return max(2, int(math.ceil(1.5 * l2 / set_bytes)))

    fns = []
    lib_fns = []  # torch SDPA on the same buffers (--library)
    lib_diff = None
    if args.kernel == "attn":
        Lk = args.kv_len if args.kv_len > 0 else args.ctx_chunks * T
        if args.q_len > 0:
            T = args.q_len
        set_bytes = 2 * (2 * T + 2 * Lk) * H * D
        for i in range(n_sets(set_bytes)):
            q = torch.randn(1, T, H, D, device=dev, generator=g).bfloat16()
            k = torch.randn(1, Lk, H, D, device=dev, generator=g).bfloat16()
            v = torch.randn(1, Lk, H, D, device=dev, generator=g).bfloat16()
            o = torch.empty_like(q)
            fns.append(lambda q=q, k=k, v=v, o=o: kernels.attention(q, k, v, out=o))
            if args.library:
                # torch SDPA wants [batch, heads, tokens, dim]; the transposed views share storage.
                qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
                lib_fns.append(lambda qt=qt, kt=kt, vt=vt: torch.nn.functional.scaled_dot_product_attention(qt, kt, vt))
                if i == 0:
                    ref = lib_fns[0]().transpose(1, 2)
                    lib_diff = float((kernels.attention(q, k, v).float() - ref.float()).abs().max())
                    del ref
        work, unit, bound = 4.0 * T * Lk * H * D / 1e12, "TFLOP/s", "tensor"
        name = f"attn_fwd q{T} kv{Lk} h{H}"
    elif args.kernel == "attn8":
        # FP8-input attention: e4m3 K/V codes with per-token scales, expanded
        # to f16 in shared memory; the library leg (--library) times the path
        # it replaces, per-token dequantisation to bf16 + the bf16 kernel
        Lk = args.kv_len if args.kv_len > 0 else args.ctx_chunks * T
        if args.q_len > 0:
            T = args.q_len
        HD = H * D
        set_bytes = 2 * 2 * T * HD + 2 * Lk * (HD + 4)
        for i in range(n_sets(set_bytes)):
            q = torch.randn(1, T, H, D, device=dev, generator=g).bfloat16()
            kx = torch.randn(Lk, HD, device=dev, generator=g).bfloat16()
            vx = torch.randn(Lk, HD, device=dev, generator=g).bfloat16()
            kc, ks = kernels.kv_quant(kx, L.WF_SCALE_TOKEN)
            vc, vs = kernels.kv_quant(vx, L.WF_SCALE_TOKEN)
            o = torch.empty_like(q)
            kc4, vc4 = kc.view(1, Lk, H, D), vc.view(1, Lk, H, D)
            fns.append(lambda q=q, kc4=kc4, vc4=vc4, ks=ks, vs=vs, o=o: kernels.attention_fp8(
                q, kc4, vc4, ks, vs, L.WF_SCALE_TOKEN, out=o))
            if args.library:
                kb = torch.empty(1, Lk, H, D, device=dev, dtype=torch.bfloat16)
                vb = torch.empty_like(kb)

                def deq_attn(q=q, kc=kc, vc=vc, ks=ks, vs=vs, kb=kb, vb=vb, o=o):
                    kernels.kv_dequant(kc, ks, L.WF_SCALE_TOKEN, out=kb.view(Lk, HD))
                    kernels.kv_dequant(vc, vs, L.WF_SCALE_TOKEN, out=vb.view(Lk, HD))
                    kernels.attention(q, kb, vb, out=o)

                lib_fns.append(deq_attn)
                if i == 0:
                    a8 = kernels.attention_fp8(q, kc4, vc4, ks, vs, L.WF_SCALE_TOKEN)
                    deq_attn()
                    lib_diff = float((a8.float() - o.float()).abs().max() / o.float().abs().max())
        work, unit, bound = 4.0 * T * Lk * H * D / 1e12, "TFLOP/s", "tensor"
        name = f"attn_fwd e4m3 K/V (per-token scales) q{T} kv{Lk} h{H}"
    elif args.kernel == "qkpub":
        # the steady tick's QKV row kernel at N=1: six stages' rows (5 denoise
        # + store) in one launch; stages 1..4 publish to the stages below
        # them, the store to all five (per-token FP8, local slots)
        S, dim, hd = 6, cfg.dim, cfg.head_dim
        ndst = [0, 1, 2, 3, 4, 5]
        rows = S * T
        set_bytes = rows * 3 * dim * 2 + 3 * rows * dim * 2 + sum(ndst) * 2 * T * (dim + 4)
        wq = (torch.randn(dim, device=dev, generator=g) * 0.5 + 1).bfloat16()
        wk = (torch.randn(dim, device=dev, generator=g) * 0.5 + 1).bfloat16()
        ang = torch.rand(rows, hd // 2, device=dev, generator=g) * 6.2831853
        cos, sin = torch.cos(ang), torch.sin(ang)
        for _ in range(n_sets(set_bytes)):
            qkv = torch.randn(rows, 3 * dim, device=dev, generator=g).bfloat16()
            slots = [[(torch.empty(T, dim, device=dev, dtype=torch.uint8),
                       torch.empty(T, dim, device=dev, dtype=torch.uint8),
                       torch.empty(T, device=dev), torch.empty(T, device=dev)) for _ in range(n)] for n in ndst]
            pub = [[tuple(t.data_ptr() for t in d) for d in st] for st in slots]
            keep = (qkv, slots)
            fns.append(lambda qkv=qkv, pub=pub, keep=keep: kernels.qk_norm_rope_publish(
                qkv, dim, wq, wk, cos, sin, hd, T, 1e-6, pub))
            if args.library:
                def unfused(qkv=qkv, slots=slots):
                    q, k, ku = kernels.qk_norm_rope(qkv, dim, wq, wk, cos, sin, hd, T, 1e-6)
                    for st, lst in enumerate(slots):
                        if lst:
                            r = slice(st * T, (st + 1) * T)
                            kernels.kv_quant_publish(k[r], qkv[r, 2 * dim:], *[[d[i].data_ptr() for d in lst]
                                                                                for i in range(4)])
                lib_fns.append(unfused)
        # read qkv; write q, k, un-roped k; codes + scales of K and V per destination
        work = (rows * 3 * dim * 2 + 3 * rows * dim * 2 + sum(ndst) * 2 * T * (dim + 4)) / 1e9
        unit, bound = "GB/s", "hbm"
        name = f"qk_norm_rope_publish {rows}x{3 * dim} (6 stages, {sum(ndst)} FP8 destinations)"
    elif args.kernel == "gemm":
        # M = --q-len (default one chunk); N, K = --gemm-nk (default the FFN
        # fc_in); the library leg is the bf16 linear it replaces (cuBLAS)
        M = args.q_len if args.q_len > 0 else T
        N, K = (int(x) for x in args.gemm_nk.split(",")) if args.gemm_nk else (cfg.ffn, cfg.dim)
        set_bytes = M * K + N * K + 2 * M * N + (2 * M * K + 2 * N * K if args.library else 0)
        for i in range(n_sets(set_bytes)):
            x = torch.randn(M, K, device=dev, generator=g).bfloat16()
            w = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()
            wq, ws = kernels.weight_quant(w)
            xq, xs = kernels.act_quant(x)
            out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            gact = L.WF_ACT_GELU_TANH if args.act_gelu else L.WF_ACT_NONE
            fns.append(lambda xq=xq, xs=xs, wq=wq, ws=ws, out=out: kernels.gemm_w8a8(xq, xs, wq, ws, None, out=out,
                                                                                      activation=gact))
            if args.library:
                ob = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                lib_fns.append(lambda x=x, w=w, ob=ob: torch.matmul(x, w.t(), out=ob))
                if i == 0:
                    ref = torch.matmul(x, w.t())
                    lib_diff = float((kernels.gemm_w8a8(xq, xs, wq, ws, None).float() - ref.float()).abs().max()
                                     / ref.float().abs().max())
            else:
                del x, w
        work, unit, bound = 2.0 * M * N * K / 1e12, "TFLOP/s", "tensor"
        name = f"gemm_w8a8 e4m3 {M}x{N}x{K}" + (" + GELU(tanh) epilogue" if args.act_gelu else "")
    elif args.kernel == "actq":
        # per-token activation quantiser: M = --q-len (default the N=1 tick's
        # six stages), K = --act-k; bytes = bf16 read + codes + scales
        M = args.q_len if args.q_len > 0 else 6 * T
        Kq = args.act_k if args.act_k > 0 else cfg.ffn
        act = L.WF_ACT_GELU_TANH if args.act_gelu else L.WF_ACT_NONE
        set_bytes = M * Kq * 3 + 4 * M
        for _ in range(n_sets(set_bytes)):
            x = torch.randn(M, Kq, device=dev, generator=g).bfloat16()
            xq = torch.empty(M, Kq, device=dev, dtype=torch.uint8)
            xs = torch.empty(M, device=dev)
            fns.append(lambda x=x, xq=xq, xs=xs: kernels.act_quant(x, L.WF_DTYPE_E4M3, xq, xs, activation=act))
        work = set_bytes / 1e9
        unit, bound = "GB/s", "hbm"
        name = f"act_quant{' GELU_tanh' if args.act_gelu else ''} e4m3 {M}x{Kq}"
    elif args.kernel == "assemble":
        HD = H * D
        n_deq = 5
        ctx = (3 + n_deq) * T  # anchor, working, own chunk, received slots
        set_bytes = 6 * T * HD * 2 + 2 * n_deq * T * (HD + 4) + 2 * ctx * HD * 2 + 2 * T * (D // 2) * 4
        for _ in range(n_sets(set_bytes)):
            pages = [torch.randn(T, HD, device=dev, generator=g).bfloat16() for _ in range(6)]
            codes = [torch.randint(0, 256, (n_deq * T, HD), device=dev, dtype=torch.uint8, generator=g)
                     for _ in range(2)]
            for c in codes:
                c[(c & 0x7F) == 0x7F] = 0  # no NaN codes
            scales = [torch.rand(n_deq * T, device=dev, generator=g) + 0.5 for _ in range(2)]
            ang = torch.rand(T, D // 2, device=dev, generator=g) * 6.2831853
            cos, sin = torch.cos(ang), torch.sin(ang)
            kb = torch.empty(ctx, HD, device=dev, dtype=torch.bfloat16)
            vb = torch.empty_like(kb)
            kp, vp, rb = kb.data_ptr(), vb.data_ptr(), HD * 2
            segs = [(L.WF_SEG_ROPE, pages[0].data_ptr(), cos.data_ptr(), sin.data_ptr(), kp, T, HD, HD),
                    (L.WF_SEG_COPY, pages[1].data_ptr(), 0, 0, vp, T, HD, HD)]
            for i, base in ((2, T), (4, 2 * T)):  # working page, own chunk
                segs.append((L.WF_SEG_COPY, pages[i].data_ptr(), 0, 0, kp + base * rb, T, HD, HD))
                segs.append((L.WF_SEG_COPY, pages[i + 1].data_ptr(), 0, 0, vp + base * rb, T, HD, HD))
            segs.append((L.WF_SEG_DEQUANT, codes[0].data_ptr(), scales[0].data_ptr(), 0, kp + 3 * T * rb,
                         n_deq * T, HD, HD))
            segs.append((L.WF_SEG_DEQUANT, codes[1].data_ptr(), scales[1].data_ptr(), 0, vp + 3 * T * rb,
                         n_deq * T, HD, HD))
            keep = (pages, codes, scales, cos, sin, kb, vb)
            fns.append(lambda segs=segs, keep=keep: kernels.kv_assemble(segs, HD, D))
        # ROPE: 2+2 B/elem + 512 B of cos/sin per row; COPY: 2+2 B/elem; DEQUANT: 1+2 B/elem + 4 B/row
        work = (T * (4 * HD + 2 * (D // 2) * 4) + 5 * T * HD * 4 + 2 * n_deq * T * (3 * HD + 4)) / 1e9
        unit, bound = "GB/s", "hbm"
        name = f"kv_assemble r0 context {ctx}x{HD} K+V (RoPE anchor, 5 copied pages, {2 * n_deq} FP8 slots)"
    elif args.kernel == "dequant":
        HD = H * D
        R = 5 * T
        set_bytes = 2 * (R * HD * 3 + 4 * R)
        for _ in range(n_sets(set_bytes)):
            kc = torch.randint(0, 256, (R, HD), device=dev, dtype=torch.uint8, generator=g)
            kc[(kc & 0x7F) == 0x7F] = 0  # no NaN codes
            vc = kc.roll(1, 0)
            ks = torch.rand(R, device=dev, generator=g) + 0.5
            vs = ks.flip(0)
            ko = torch.empty(R, HD, device=dev, dtype=torch.bfloat16)
            vo = torch.empty_like(ko)
            fns.append(lambda kc=kc, ks=ks, ko=ko: kernels.kv_dequant(kc, ks, L.WF_SCALE_TOKEN, out=ko))
            fns.append(lambda vc=vc, vs=vs, vo=vo: kernels.kv_dequant(vc, vs, L.WF_SCALE_TOKEN, out=vo))
        work = (R * HD * 3 + 4 * R) / 1e9  # per launch (one of K or V)
        unit, bound = "GB/s", "hbm"
        name = f"kv_dequant {R}x{HD} per launch (K and V alternate)"
    else:
        HD = H * D
        n = 4
        set_bytes = 2 * T * HD * 2 + n * 2 * (T * HD + 4 * T)
        for _ in range(n_sets(set_bytes)):
            kx = torch.randn(T, HD, device=dev, generator=g).bfloat16()
            vx = torch.randn(T, HD, device=dev, generator=g).bfloat16()
            dst = [(torch.empty(T, HD, device=dev, dtype=torch.uint8), torch.empty(T, HD, device=dev, dtype=torch.uint8),
                    torch.empty(T, device=dev), torch.empty(T, device=dev)) for _ in range(n)]
            ptrs = [[d[i].data_ptr() for d in dst] for i in range(4)]
            fns.append(lambda kx=kx, vx=vx, ptrs=ptrs, dst=dst: kernels.kv_quant_publish(kx, vx, *ptrs))
        work = (2 * T * HD * 2 + n * 2 * (T * HD + 4 * T)) / 1e9
        unit, bound = "GB/s", "hbm"
        name = f"kv_quant_publish {T}x{HD} to {n} slots"
    launches = max(args.steps, len(fns))

    def graph_ms(fs):
        for i in range(max(3, args.warmup)):
            fs[i % len(fs)]()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(launches):
                fs[i % len(fs)]()
        graph.replay()  # warm the graph itself
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / launches
        del graph
        return t

    ms = graph_ms(fns)
    library = None
    if lib_fns:
        lms = graph_ms(lib_fns)
        library = {"name": {"attn8": "per-token dequant to bf16 + bf16 wf_attn_fwd",
                            "gemm": "bf16 torch.matmul of the same shape (cuBLAS)",
                            "qkpub": "wf_qk_norm_rope + wf_kv_quant_publish per stage (the unfused pair)"}.get(
                                args.kernel, "torch SDPA, default dispatch (cuDNN on B200)"), "ms": lms,
                   "achieved": work / (lms * 1e-3), "max_abs_diff_vs_wf": lib_diff,
                   # the product kernel once more after the library leg, to expose clock drift
                   "wf_ms_after": graph_ms(fns)}
    peaks, src = _peaks()
    peak = peaks["bf16_tflops"] if bound == "tensor" else peaks["hbm_gbs"]
    if args.kernel == "gemm":
        peak *= 2  # dense FP8 peak = 2x bf16 (nominal ratio; measured peak is bf16 only)
    ach = work / (ms * 1e-3)
    print(json.dumps({"kernel": name, "ms": ms, "achieved": ach, "unit": unit, "peak": peak,
                      "frac": ach / peak, "peak_source": src + (" bf16 burst x2" if args.kernel == "gemm" else ""),
                      "launches": launches, "buffer_sets": len(fns), "status": L.status_take(),
                      **({"library": library} if library else {})}), flush=True)


def run_vae_e2e(args, make_engine, noise_cpu, cfg, dev, rank, world, barrier, max_over_ranks):
    """The whole 399-frame wavefront with streaming VAE decode: every chunk the
    store finishes is decoded to 12 pixel frames (9 for the first chunk) and
    read back to pinned host memory.
    * Ranks that host no stage (2 of 8 GPUs at 5 steps) form a VAE pipeline,
      as the reference runs its VAE on the spare GPUs (wave_rt/pipelines/
      vae.py:42-207).  The store rank sends each finished latent chunk to the
      first of them, and the units are split between them by FLOPs.
    * Without idle ranks the store rank decodes after each tick, on its own
      stream order.
    FPS = pixel frames / wall time from the first tick to the last pixel
    frame on the host, max over ranks."""
    from waveforcing_b200.pipelines import vae as V

    eng = make_engine(noise_cpu.pin_memory())
    stage_ranks = sorted(set(eng.stage_rank))
    vae_ranks = [r for r in range(world) if r not in stage_ranks]
    store_rank = eng.stage_rank[eng.store]
    torch.backends.cudnn.benchmark = True
    dec = V.VAEDecoder.random(V.VAEConfig(), seed=0).for_gpu(dev) if (rank in vae_ranks or (
        not vae_ranks and rank == store_rank)) else None
    cuts = V.partition_units(dec.unit_flops(cfg.lat_h, cfg.lat_w), len(vae_ranks)) if (dec and vae_ranks) else None
    pix_host = torch.empty((3, 12, 8 * cfg.lat_h, 8 * cfg.lat_w), dtype=torch.bfloat16).pin_memory()
    frames = 0
    nt = eng.num_ticks
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    if rank in vae_ranks:
        k = vae_ranks.index(rank)
        st = V.VAEPipelineStage(dec, cuts, k, vae_ranks)
        if k == 0:
            import torch.distributed as dist_

            zbuf = torch.empty((cfg.in_ch, 3, cfg.lat_h, cfg.lat_w), dtype=torch.bfloat16, device=dev)
            for _ in range(ecfg_blocks(eng)):
                dist_.recv(zbuf, store_rank)
                for y in st.push_latents(zbuf):
                    if st.last:
                        pix_host[:, :y.shape[2]].copy_(y[0], non_blocking=True)
                        frames += y.shape[2]
                    else:
                        st.send_next(y)
            if not st.last:
                st.send_next(None)
        else:
            while True:
                x = st.recv_prev()
                if x is None:
                    if not st.last:
                        st.send_next(None)
                    break
                y = st.run(x)
                if st.last:
                    pix_host[:, :y.shape[2]].copy_(y[0], non_blocking=True)
                    frames += y.shape[2]
                else:
                    st.send_next(y)
    else:
        stream = V.DecodeStream(dec) if dec is not None else None
        for t in range(nt):
            eng.tick(t)
            c = t - eng.store
            if c in eng.final:
                z = eng.final.pop(c)
                if stream is not None:
                    y = stream.push(z)
                    pix_host[:, :y.shape[1]].copy_(y, non_blocking=True)
                    frames += y.shape[1]
                elif rank == store_rank:
                    import torch.distributed as dist_

                    dist_.send(z.contiguous(), vae_ranks[0])
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    barrier()
    wall = max_over_ranks([wall])[0]
    frames = int(max_over_ranks([float(frames)])[0])
    eng.close()
    del eng
    return {"value": frames / wall, "unit": "FPS", "pixel_frames": frames, "wall_s": wall,
            "vae_ranks": vae_ranks if vae_ranks else [store_rank],
            "vae_cuts": cuts, "definition": "pixel frames (1 + 4 x (399 - 1)) / wall time from the first tick to "
                                            "the last decoded frame in host memory, max over ranks; host clock",
            "decoder": "Wan2.1-shaped VAE decoder (dim 96, z 16), random-init, bf16 channels-last on cuDNN"}


def ecfg_blocks(eng) -> int:
    return eng.cfg.num_blocks


def run_vae_bench(args):
    """Streaming VAE decode of one finished chunk (3 latent frames at the
    480x832 latent 60x104 -> 12 pixel frames) by the Wan2.1-shaped decoder
    (waveforcing_b200/pipelines/vae.py), bf16 channels-last on cuDNN, in
    steady state: the stream has already decoded frame 0 and earlier chunks.
    CUDA events around each push, ``--steps`` chunks after ``--warmup``."""
    from waveforcing_b200.pipelines import vae as V

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    torch.backends.cudnn.benchmark = True
    cfg = V.VAEConfig()
    dec = V.VAEDecoder.random(cfg, seed=0).for_gpu(dev)
    lh, lw = 60, 104
    g = torch.Generator(device="cpu").manual_seed(0)
    n = 1 + 3 * (args.warmup + args.steps)
    z = torch.randn(cfg.z_dim, n, lh, lw, generator=g).to(dev, torch.bfloat16)
    s = V.DecodeStream(dec)
    s.push(z[:, :1])
    f = 1
    for _ in range(args.warmup):
        s.push(z[:, f:f + 3])
        f += 3
    torch.cuda.synchronize()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    evs[0].record()
    out_frames = 0
    for i in range(args.steps):
        y = s.push(z[:, f:f + 3])
        out_frames += y.shape[1]
        f += 3
        evs[i + 1].record()
    torch.cuda.synchronize()
    ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    p50 = statistics.median(ms)
    flops = 3 * sum(dec.unit_flops(lh, lw))
    shares = None
    if args.trace:
        # kernel families of one more chunk (CUPTI, in-stream durations)
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], record_shapes=True) as prof:
            s.push(z[:, f:f + 3]) if f + 3 <= n else s.push(z[:, 1:4])
            torch.cuda.synchronize()
        ops = []
        for a in prof.key_averages(group_by_input_shape=True):
            dt = getattr(a, "device_time_total", None) or getattr(a, "cuda_time_total", 0)
            if a.key.startswith("aten::") and dt > 0:
                ops.append((dt / 1e3, a.key, str(a.input_shapes)[:120], a.count))
        ops.sort(key=lambda r: -r[0])
        op_shares = [{"op": k, "ms": ms, "shapes": sh, "calls": c} for ms, k, sh, c in ops[:16]]
        by: dict = {}
        for e in prof.events():
            if e.device_type == torch.autograd.DeviceType.CUDA and e.time_range.end > e.time_range.start:
                k = e.name.split("(")[0][:90]
                by[k] = by.get(k, 0.0) + (e.time_range.end - e.time_range.start) / 1e3
        tot = sum(by.values())
        shares = [{"kernel": k, "ms": v, "share": v / tot} for k, v in sorted(by.items(), key=lambda kv: -kv[1])[:14]]
    peaks, src = _peaks()
    ach = flops / (p50 * 1e-3) / 1e12
    print(json.dumps({"kernel": "streaming VAE decode, one 3-latent-frame chunk (60x104 -> 12 frames of 480x832)",
                      "ms": p50, "pixel_fps": 12 * 1000.0 / p50, "achieved": ach, "unit": "TFLOP/s",
                      "peak": peaks["bf16_tflops"], "frac": ach / peaks["bf16_tflops"],
                      "peak_source": src + " bf16_tflops", "flops_per_chunk": flops,
                      "output_frames": out_frames, "steps": args.steps,
                      "note": "cuDNN convolutions and torch SDPA (library calls); FLOPs counted analytically",
                      **({"trace_shares": shares, "trace_ops": op_shares} if shares else {})}),
          flush=True)


def run_publish_bench(args):
    """The exchange's NVLink leg on 2 GPUs (torchrun, 2 ranks): rank 0 runs the
    fused per-token FP8 quantise-and-publish of one layer's K and V (4680 x
    1536 each) with its destination in rank 1's memory (CUDA IPC), and, for
    reference, a copy-engine peer copy of the same number of bytes.  Bytes
    crossing NVLink per launch = codes + scales of K and V.  Both are timed over
    a CUDA graph of `steps` launches; rank 1 only hosts the destination."""
    import datetime

    from waveforcing_b200 import kernels
    from waveforcing_b200.distributed import ipc
    from waveforcing_b200.wavefront.dit import DiTConfig

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world != 2:
        print(json.dumps({"kernel": "kv_quant_publish over NVLink", "unavailable": "needs exactly 2 ranks (torchrun)"}))
        return
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    cfg = DiTConfig.preset(args.preset)
    T, HD = cfg.tokens_per_chunk, cfg.heads * cfg.head_dim
    nsets = 4  # destination sets rotated so the peer's L2 does not absorb the writes
    dst = [(torch.empty(T, HD, device=dev, dtype=torch.uint8), torch.empty(T, HD, device=dev, dtype=torch.uint8),
            torch.empty(T, device=dev), torch.empty(T, device=dev)) for _ in range(nsets)]
    mine = [[ipc.ipc_export(t) for t in d] for d in dst] if rank == 1 else None
    objs = [None, None]
    dist.all_gather_object(objs, mine)
    dist.barrier()
    if rank == 0:
        ipc.enable_peer(1)
        bases, remote = [], []
        for d in objs[1]:
            ptrs = []
            for h, off in d:
                base = ipc.ipc_open_handle(h)
                bases.append(base)
                ptrs.append(base + off)
            remote.append(ptrs)
        g = torch.Generator(device=dev).manual_seed(0)
        kx = torch.randn(T, HD, device=dev, generator=g).bfloat16()
        vx = torch.randn(T, HD, device=dev, generator=g).bfloat16()
        src = torch.empty(2 * T * HD + 8 * T, device=dev, dtype=torch.uint8)
        stream = torch.cuda.current_stream().cuda_stream
        nv_bytes = 2 * T * HD + 2 * 4 * T

        def pub(i):
            p = remote[i % nsets]
            kernels.kv_quant_publish(kx, vx, [p[0]], [p[1]], [p[2]], [p[3]])

        def cpy(i):
            p = remote[i % nsets]
            ipc.memcpy_dtod_async(p[0], src.data_ptr(), T * HD, torch.cuda.current_stream().cuda_stream)
            ipc.memcpy_dtod_async(p[1], src.data_ptr() + T * HD, T * HD, torch.cuda.current_stream().cuda_stream)

        def timed(fn):
            for i in range(max(3, args.warmup)):
                fn(i)
            torch.cuda.synchronize()
            n = max(args.steps, nsets)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(n):
                    fn(i)
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize()
            del graph
            return e0.elapsed_time(e1) / n

        ms_pub = timed(pub)
        ms_cpy = timed(cpy)
        del stream
        for b in bases:
            ipc.ipc_close_handle(b)
        ref_peer = 770.0  # measured peer copy per direction on this pool (nominal NVLink 5: 900)
        ach = nv_bytes / (ms_pub * 1e-3) / 1e9
        print(json.dumps({"kernel": f"kv_quant_publish {T}x{HD} K+V to 1 peer over NVLink", "ms": ms_pub,
                          "achieved": ach, "unit": "GB/s", "peak": ref_peer, "frac": ach / ref_peer,
                          "peak_source": "measured peer copy 770 GB/s per direction (nominal 900)",
                          "nvlink_bytes_per_launch": nv_bytes, "hbm_bytes_read_per_launch": 2 * T * HD * 2,
                          "copy_engine_same_bytes": {"ms": ms_cpy,
                                                     "gbs": 2 * T * HD / (ms_cpy * 1e-3) / 1e9},
                          "launches": max(args.steps, nsets)}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def run_forward_bench(args):
    """BASELINE config 2 on one GPU: the full 30-layer (1.3B) DiT forward of one
    3-frame chunk-stage task at timestep 600 whose self-attention sees a
    6-chunk K/V context (5 earlier chunks, random bf16 per layer, plus its own
    chunk), with the text cross-attention.  CUDA-event timed per forward."""
    from waveforcing_b200.runtime import backend
    from waveforcing_b200.runtime.fp8 import quantize_transformer_w8a8
    from waveforcing_b200.wavefront.dit import DiTConfig, StageTask, WanDiT

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    torch.set_grad_enabled(False)
    backend.select_backend("wf_b200")
    cfg = DiTConfig.preset(args.preset)
    model = WanDiT.random(cfg, dev, seed=0)
    if args.w8a8 != "none":
        quantize_transformer_w8a8(model, scope="all", qtype=args.w8a8, granularity="channel")
    g = torch.Generator(device="cpu").manual_seed(0)
    model.set_text(torch.randn(cfg.text_len, cfg.text_dim, generator=g).to(dev))
    T, H, D = cfg.tokens_per_chunk, cfg.heads, cfg.head_dim
    ctx = 6
    gd = torch.Generator(device=dev).manual_seed(1)
    kctx = [torch.randn(1, ctx * T, H, D, device=dev, generator=gd).bfloat16() for _ in range(cfg.layers)]
    vctx = [torch.randn(1, ctx * T, H, D, device=dev, generator=gd).bfloat16() for _ in range(cfg.layers)]

    def exch(*, layer_idx, roped_query, roped_key, unroped_key, value, **_):
        kctx[layer_idx][0, (ctx - 1) * T:].copy_(roped_key[0])
        vctx[layer_idx][0, (ctx - 1) * T:].copy_(value[0])
        return kctx[layer_idx], vctx[layer_idx]

    lat = torch.randn(cfg.in_ch, cfg.frames_per_block, cfg.lat_h, cfg.lat_w, device=dev, generator=gd)
    task = StageTask(lat, 600.0, (ctx - 1) * cfg.frames_per_block, 0, exch)
    for _ in range(max(3, args.warmup)):
        model.forward_stages([task])
    torch.cuda.synchronize()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    evs[0].record()
    for i in range(args.steps):
        model.forward_stages([task])
        evs[i + 1].record()
    torch.cuda.synchronize()
    ms = statistics.median([evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)])
    dim, ffn = cfg.dim, cfg.ffn
    lin = 2 * T * (6 * dim * dim + 2 * dim * ffn)  # q,k,v,o, cross q,o, FFN in+out (cross K/V are cached)
    flops = cfg.layers * (4 * T * ctx * T * H * D + lin + 4 * T * cfg.text_len * H * D)
    peaks, src = _peaks()
    tf = flops / (ms * 1e-3) / 1e12
    print(json.dumps({"workload": f"config 2: {args.preset} DiT forward, one 3-frame chunk (T={T}) at t=600, "
                                  f"{ctx}-chunk self-attention context, 512-token text",
                      "ms_per_forward_p50": ms, "steps": args.steps, "tflop_per_forward": flops / 1e12,
                      "achieved_tflops": tf, "frac_of_sustained_bf16": tf / peaks["bf16_tflops_sustained"],
                      "peak_source": src, "w8a8": args.w8a8, "data": "synthetic (random-init weights and context)"}),
          flush=True)


def main():
    args = parse()
    if args.forward:
        run_forward_bench(args)
    elif args.kernel == "publish":
        run_publish_bench(args)
    elif args.kernel == "vae":
        run_vae_bench(args)
    elif args.kernel:
        run_kernel_bench(args)
    elif args.impl == "reference":
        run_reference_arm(args)
    elif args.impl == "reference-gpu":
        run_reference_gpu_arm(args)
    else:
        run_gpu_arm(args)


if __name__ == "__main__":
    main()
