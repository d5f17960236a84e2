"""Wavefront tick engine with stage merging (the caller of the hot path).

Schedule and data flow follow wave_rt/denoiser/engine.py:
  * activity       -- _act_denoise/_act_store :214-219, roles :303-311
  * one tick       -- :287-597: denoise/store forwards with the paged exchange
                      closure installed, drain, clean-KV promotion (anchor
                      sent to the stage ranks at cid 0 :449-488, store slot
                      otherwise :489-515), latent migration point to point +
                      deterministic re-noise :221-235, :516-555
  * ticks          -- num_blocks + stages (engine.py:53 with world = stages)
The reference needs one rank per stage (wave_rt/config.py:79-83).  Here
``place_stages`` maps the rf_step denoise stages and the store onto any
number of ranks: a rank may host several stages, runs them layer-interleaved
(highest stage first, so local publishes precede local reads), and batches
their linears.  Ranks beyond the stage count stay idle.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from waveforcing_b200 import kernels
from waveforcing_b200.denoiser.exchange.paged import PagedTransport
from waveforcing_b200.wavefront.dit import FlowMatch, StageTask, WanDiT, rope_tables


@dataclass
class EngineConfig:
    steps: tuple = (1000, 800, 600, 400, 200)
    num_frames: int = 399  # latent frames
    npb: int = 3
    max_attn_frames: int = 21
    fp8_kv: bool = False
    context_noise: float = 0.0
    seed: int = 0
    timeout_s: float = 60.0

    @property
    def rf_step(self) -> int:
        return len(self.steps)

    @property
    def num_blocks(self) -> int:
        return self.num_frames // self.npb


# Relative attention+linear cost of each stage in steady state (K/V context in
# chunks plus the linears), used to balance merged stages across ranks.
def stage_costs(rf_step: int, max_attn_frames: int = 21, npb: int = 3) -> list[float]:
    wmax = max(0, (max_attn_frames - rf_step * npb - npb) // npb)
    naw = 1 + wmax
    ctx = [naw + 1 + (rf_step - s) for s in range(rf_step)]  # live + self + higher stages
    store_ctx = 1 + max(0, (max_attn_frames - 2 * npb) // npb) + 1
    lin = 2.9  # linears ~ 2.9 chunk-equivalents of attention for the 1.3B shape
    return [c + lin for c in ctx] + [store_ctx + lin]


def place_stages(rf_step: int, world: int) -> list[int]:
    """Contiguous, cost-balanced assignment of stages 0..rf_step to ranks."""
    n = rf_step + 1
    ranks = min(world, n)
    if ranks == n:
        return list(range(n))
    cost = stage_costs(rf_step)
    # exact partition of the ordered stages into `ranks` contiguous groups minimising the max load
    best = None

    def rec(start, k, acc):
        nonlocal best
        if k == 1:
            parts = acc + [(start, n)]
            mx = max(sum(cost[a:b]) for a, b in parts)
            if best is None or mx < best[0]:
                best = (mx, parts)
            return
        for end in range(start + 1, n - k + 2):
            rec(end, k - 1, acc + [(start, end)])

    rec(0, ranks, [])
    out = [0] * n
    for r, (a, b) in enumerate(best[1]):
        for s in range(a, b):
            out[s] = r
    return out


def migration_plan(stage_rank: list[int], rf_step: int, num_blocks: int, t: int) -> list[tuple[int, int, int]]:
    """Latent hand-offs after tick ``t``: (receiving stage, source rank,
    destination rank) for every denoise stage s active at t (engine.py:214-219),
    whose result feeds stage s + 1 at t + 1 (s + 1 = rf_step is the store).
    Stage s active at t is exactly stage s + 1 active at t + 1, so every rank
    derives the same list without communicating."""
    out = []
    for s in range(rf_step):
        if 0 <= t - s < num_blocks:
            out.append((s + 1, stage_rank[s], stage_rank[s + 1]))
    return out


class _StoreKV(list):
    """``store_kv`` of one tick for merged stages.  The store closure assigns
    ``(roped_key, unroped_key, value)`` per layer, [1, T, H, D] views that the
    reference keeps as they are (engine.py:449-515).  Here those views point
    into per-layer buffers of every merged stage, so each assignment keeps a
    copy of only the two tensors the promotion reads: the unroped key and the
    value at the anchor tick (cid 0), the roped key and the value otherwise."""

    def __init__(self, n: int, anchor: bool) -> None:
        super().__init__([None] * n)
        self.anchor = anchor

    def __setitem__(self, i, kv) -> None:
        kr, ku, v = kv
        super().__setitem__(i, (None if self.anchor else kr.clone(), ku.clone() if self.anchor else None, v.clone()))


@dataclass
class TickStats:
    tick_ms: list = field(default_factory=list)


class WavefrontEngine:
    def __init__(self, model: WanDiT, cfg: EngineConfig, *, rank: int = 0, world: int = 1, device="cuda",
                 group=None, noise: torch.Tensor | None = None) -> None:
        self.m = model
        self.cfg = cfg
        self.rank, self.world = rank, world
        self.device = torch.device(device)
        self.group = group
        self.S = cfg.rf_step
        self.store = self.S
        self.stage_rank = place_stages(self.S, world)
        self.local = [s for s in range(self.S + 1) if self.stage_rank[s] == rank]
        mc = model.cfg
        self.Ln, self.T, self.H, self.D = mc.layers, mc.tokens_per_chunk, mc.heads, mc.head_dim
        self.fm = FlowMatch()
        self.xport = PagedTransport(device=self.device, rank=rank, world=world, stage_rank=self.stage_rank,
                                    rf_step=self.S, Ln=self.Ln, T=self.T, H=self.H, D=self.D, npb=cfg.npb,
                                    max_attn_frames=cfg.max_attn_frames, fp8=cfg.fp8_kv,
                                    timeout_s=cfg.timeout_s, group=group)
        self.clean = [[] for _ in range(self.Ln)]
        self.inputs: dict = {}  # stage -> latent chunk [C, F, H, W] for the current tick
        self.final: dict = {}  # chunk -> clean latent (store rank)
        self._rope_cache: dict = {}
        C = mc.in_ch
        if noise is None:
            g = torch.Generator(device="cpu").manual_seed(cfg.seed)
            noise = torch.randn((C, cfg.num_frames, mc.lat_h, mc.lat_w), generator=g).to(torch.bfloat16)
        self.noise = noise  # [C, F_total, H, W]; may live on the host (pinned) or the device
        self.mig_shape = (self.S + 1, C, cfg.npb, mc.lat_h, mc.lat_w)
        self.timeline = None  # optional Timeline (diagnostic): stamps of each tick's phases

    # ----------------------------------------------------------------- helpers
    @property
    def num_ticks(self) -> int:
        return self.cfg.num_blocks + self.S

    def act_denoise(self, n, t):
        return 0 <= n < self.S and 0 <= t - n < self.cfg.num_blocks

    def act_store(self, t):
        return 0 <= t - self.store < self.cfg.num_blocks

    def _rope_tables(self, start_frame: int) -> tuple[torch.Tensor, torch.Tensor]:
        tab = self._rope_cache.get(start_frame)
        if tab is None:
            tab = rope_tables(self.m.cfg, self.cfg.npb, start_frame, self.device)
            self._rope_cache[start_frame] = tab
        return tab

    def _rope_tab(self, start_frame: int, *_geometry) -> tuple[torch.Tensor, torch.Tensor]:
        """Anchor RoPE tables for the exchange closures (the chunk geometry the
        closures also pass is fixed by the model config here)."""
        return self._rope_tables(start_frame)

    def _rope(self, ku: torch.Tensor, start_frame: int) -> torch.Tensor:
        tab = self._rope_tables(start_frame)
        return kernels.rope_apply(ku, tab[0], tab[1])

    def _append_clean(self, page: dict) -> None:
        """common.py:110-114 per layer."""
        for L in range(self.Ln):
            cl = self.clean[L]
            cl.append(page[L])
            if len(cl) > 8:
                cl[:] = cl[:1] + cl[-7:]

    # -------------------------------------------------------------------- tick
    def noise_chunk(self, c: int) -> torch.Tensor:
        npb = self.cfg.npb
        ch = self.noise[:, c * npb:(c + 1) * npb]
        return ch.to(self.device, non_blocking=True).contiguous()

    @torch.no_grad()
    def tick(self, t: int) -> dict:
        cfg, S = self.cfg, self.S
        act = [n for n in range(S) if self.act_denoise(n, t)]
        oldest = (t - max(act)) if act else 0
        tick_csf, tick_qf = oldest * cfg.npb, len(act) * cfg.npb
        store_active = self.act_store(t)
        tl = self.timeline
        if tl is not None:
            tl.mark(f"t{t}.begin")
        if 0 in self.local and self.act_denoise(0, t):
            self.inputs[0] = self.noise_chunk(t)
        tasks = []
        store_kv = _StoreKV(self.Ln, anchor=(t - self.store == 0))
        store_slot: dict = {}
        # one stage per rank copies the store's live slot (all hold the same);
        # none when the store is idle or on this rank (_promote then keeps the
        # store's own K/V and never reads the slot)
        slot_sink_given = not store_active or self.store in self.local
        for s in sorted(self.local, reverse=True):
            if s < S and self.act_denoise(s, t):
                c = t - s
                exch = self.xport.make_denoise_exch(s, self.clean, act, tick_csf, tick_qf, store_active, t,
                                                    self._rope, None if slot_sink_given else store_slot,
                                                    rope_tab_fn=self._rope_tab)
                slot_sink_given = True
                tasks.append(StageTask(self.inputs[s], self.fm.timestep(cfg.steps[s]), c * cfg.npb, s, exch))
            elif s == self.store and store_active:
                c = t - self.store
                exch = self.xport.make_store_exch(self.clean, store_kv, c, act, t, self._rope,
                                                  rope_tab_fn=self._rope_tab)
                # the store's flow output is never used (its input chunk is the final latent):
                # only its K/V are needed, so its last layer stops after the publish
                tasks.append(StageTask(self.inputs[s], cfg.context_noise, c * cfg.npb, s, exch, kv_only=True))
        # no publish of this tick may land in a slab generation that a remote
        # consumer is still reading (it read that generation two ticks ago)
        self.xport.acquire_slots(t)
        if tl is not None:
            tl.mark(f"t{t}.acquired")
        flows = self.m.forward_stages(tasks) if tasks else []
        self.xport.drain()
        self.xport.release_slots(t)
        if tl is not None:
            tl.mark(f"t{t}.forward")
        out = {}
        for task, flow in zip(tasks, flows):
            if task.stage < S:
                step = cfg.steps[task.stage]
                out[task.stage] = self.fm.x0(flow, task.latent.float(), step).to(torch.bfloat16)
            else:
                self.final[task.start_frame // cfg.npb] = task.latent
        self._promote(t, store_active, store_kv, store_slot, bool(tasks))
        if tl is not None:
            tl.mark(f"t{t}.promoted")
        self._migrate(t, out)
        if tl is not None:
            tl.mark(f"t{t}.migrated")
        return out

    def _promote(self, t, store_active, store_kv, store_slot, had_task) -> None:
        if not store_active:
            return
        cid = t - self.store
        Ln = self.Ln
        hosts_store = self.store in self.local
        # store_kv[L] = (roped_key, unroped_key, value) as [1, T, H, D] (copies,
        # see _StoreKV); store_slot[L] = [2, T, H, D] copy of the live slot
        if cid == 0:
            # anchor: the store's unroped key and value for every layer
            # (engine.py:449-488, a world broadcast there), sent point to point
            # to the ranks that host stages; a rank without stages keeps no
            # clean pages and is free for other work (the VAE pipeline)
            if not self.local:
                return
            src = self.stage_rank[self.store]
            if hosts_store:
                blob = torch.stack([torch.stack([store_kv[L][1][0] for L in range(Ln)]),
                                    torch.stack([store_kv[L][2][0] for L in range(Ln)])]).contiguous()
            else:
                blob = torch.empty((2, Ln, self.T, self.H, self.D), device=self.device, dtype=torch.bfloat16)
            peers = sorted(set(self.stage_rank) - {src})
            if self.world > 1 and peers:
                if self.rank == src:
                    ops = [dist.P2POp(dist.isend, blob, self._peer(r), group=self.group) for r in peers]
                else:
                    ops = [dist.P2POp(dist.irecv, blob, self._peer(src), group=self.group)]
                for req in dist.batch_isend_irecv(ops):
                    req.wait()
            self._append_clean([dict(ku=blob[0, L], v=blob[1, L], cid=cid) for L in range(Ln)])
        elif hosts_store:
            self._append_clean([dict(kr=store_kv[L][0][0], v=store_kv[L][2][0], cid=cid) for L in range(Ln)])
        elif len(store_slot) == Ln:
            self._append_clean([dict(kr=store_slot[L][0], v=store_slot[L][1], cid=cid) for L in range(Ln)])

    def _renoise(self, x0, stage, chunk):
        """engine.py:221-235: seed 1000*chunk+stage, re-noised to the next step."""
        g = torch.Generator(device=self.device).manual_seed(1000 * chunk + stage)
        nz = torch.randn(x0.shape, generator=g, device=self.device, dtype=torch.float32)
        return self.fm.add_noise(x0.float(), nz, self.cfg.steps[stage + 1]).to(torch.bfloat16)

    def _migrate(self, t, out: dict) -> None:
        """Hand each denoise stage's result to the next stage (engine.py:516-555).

        The reference gathers every rank's payload with a world all_gather per
        tick (engine.py:550).  Here each result goes point to point: kept in
        place when the next stage is on the same rank, otherwise one NCCL
        send/recv between the two ranks (``migration_plan``); ranks without a
        hand-off this tick take no part.  The all_gather also served the
        reference as the credit for reusing a slab generation two ticks later;
        that role is the transport's credit flags (``PagedTransport.
        release_slots`` / ``acquire_slots``)."""
        S = self.S
        payload = {}
        for s, x0 in out.items():
            c = t - s
            payload[s + 1] = self._renoise(x0, s, c) if s < S - 1 else x0
        recv, ops = {}, []
        for dst_stage, src_rank, dst_rank in migration_plan(self.stage_rank, S, self.cfg.num_blocks, t):
            if src_rank == dst_rank:
                if src_rank == self.rank:
                    self.inputs[dst_stage] = payload[dst_stage]
            elif src_rank == self.rank:
                ops.append(dist.P2POp(dist.isend, payload[dst_stage].contiguous(), self._peer(dst_rank),
                                      group=self.group))
            elif dst_rank == self.rank:
                buf = torch.empty(self.mig_shape[1:], device=self.device, dtype=torch.bfloat16)
                ops.append(dist.P2POp(dist.irecv, buf, self._peer(src_rank), group=self.group))
                recv[dst_stage] = buf
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        self.inputs.update(recv)

    def _peer(self, r: int) -> int:
        """Global rank of group rank ``r`` (P2POp addresses global ranks)."""
        return r if self.group is None else dist.get_global_rank(self.group, r)

    def close(self) -> None:
        self.xport.close()
