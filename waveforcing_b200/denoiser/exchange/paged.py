"""Fixed-slot paged K/V exchange with FP8 transport and stage merging.

Semantics follow wave_rt/denoiser/exchange/paged.py:
  * slab sizing (naw, Wmax)        -- paged.py:26-30
  * denoise slot geometry          -- paged.py:160-189
  * publish: payload then flag     -- paged.py:120-145 (copy stream, release write)
  * consumer wait                  -- paged.py:147-154 (here BOUNDED: a timed-out
                                      wait raises instead of hanging the stream)
  * assembled context Kb[:active]  -- paged.py:191-255; store side :257-310
  * anchor re-RoPE + working set   -- wave_rt/denoiser/exchange/common.py:70-108
  * drain                          -- wave_rt/denoiser/exchange/onesided.py:181-187
The closures keep the reference's keyword contract and return (K, V) as
[1, Lk, H, D] views, so ``PagedExchangeMixin`` drops into the reference's
WaveDenoiser (methods ``_init_paged``, ``_make_denoise_exch_paged``,
``_make_store_exch_paged``, ``_publish_paged``, ``_wait_paged_flag``,
``_drain_publish``).

What is new relative to the reference:
  * stages merge onto fewer ranks: one ``PagedTransport`` per process owns the
    slabs of every consumer stage it hosts; a publish to a stage on the same
    GPU is a stream-ordered local write, to another GPU an IPC peer write
    plus a release flag;
  * FP8 e4m3 transport (the reference refuses FP8 with paged, paged.py:36-37):
    slabs hold e4m3 codes + per-row f32 scales, written by one fused
    quantise-and-publish kernel (per-token scales) or by the per-tensor codec;
    the consumer dequantises the received slots into a bf16 assembly buffer
    before attention.  Local pages (anchor, working, self) stay bf16, so
    numerics do not depend on stage placement.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from waveforcing_b200 import _lib as L
from waveforcing_b200 import kernels
from waveforcing_b200.distributed import ipc


def slab_geometry(max_attn_frames: int, rf_step: int, npb: int):
    """paged.py:26-30 -> (naw_max, Wmax)."""
    wmax_frames = max_attn_frames - rf_step * npb - npb
    naw = 1 + max(0, wmax_frames // npb)
    return naw, naw + 1 + rf_step


def tick_geometry(stage, tick, act, store_active, rf_step, max_attn_frames, npb):
    """paged.py:160-189 for consumer ``stage`` (all in chunk-slot units)."""
    store = rf_step
    clean_len = min(8, max(0, tick - store))
    wmax_chunks = max(0, (max_attn_frames - len(act) * npb - npb) // npb)
    naw = 0 if clean_len == 0 else 1 + min(wmax_chunks, clean_len - 1)
    live = 1 if store_active else 0
    base_infl = naw + live
    infl = [n for n in act if n >= stage]
    recv = [n for n in act if n > stage] + ([store] if store_active else [])
    send = []
    for m in act:
        if m >= stage:
            continue
        send.append((m, base_infl + sum(1 for n in act if m <= n < stage)))
    return dict(clean_len=clean_len, naw=naw, live=live, base_infl=base_infl, active_slots=base_infl + len(infl),
                recv=recv, send=send)


class PagedTransport:
    """Slabs, flags and peer pointers for the stages one process hosts."""

    def __init__(self, *, device, rank: int, world: int, stage_rank: list[int], rf_step: int, Ln: int, T: int,
                 H: int, D: int, npb: int = 3, max_attn_frames: int = 21, GT: int = 2, fp8: bool = False,
                 fp8_gran: str = "token", dtype=torch.bfloat16, timeout_s: float = 30.0, group=None,
                 ipc_open=None) -> None:
        """``ipc_open`` (optional) opens peer handles on behalf of a host that
        owns their lifetime -- the reference WaveDenoiser's ``_ipc_open``, which
        records every mapping for its two-barrier close (engine.py:127-212);
        the transport then leaves closing them to the host.  ``fp8_gran`` is
        the FP8 scale granularity: "token" (one scale per token row, fused
        quantise-and-publish) or "tensor" (the reference's per-tensor scale over
        stack(K, V), common.py:143-150, written into every row's scale)."""
        if fp8_gran not in ("token", "tensor"):
            raise ValueError(f"fp8_gran must be 'token' or 'tensor', got {fp8_gran!r}")
        self.fp8_gran = fp8_gran
        self._host_ipc_open = ipc_open
        self.device = torch.device(device)
        self.rank, self.world = rank, world
        self.stage_rank = list(stage_rank)  # stage -> rank, stages 0..rf_step (rf_step = store)
        self.rf_step, self.store = rf_step, rf_step
        self.Ln, self.T, self.H, self.D, self.npb = Ln, T, H, D, npb
        self.max_attn_frames, self.GT, self.fp8, self.dtype = max_attn_frames, GT, fp8, dtype
        self.timeout_s = timeout_s
        self.group = group
        # assemble each layer's context with one wf_kv_assemble launch (when the
        # caller passes RoPE tables); False keeps the per-page copies
        self.fused_assembly = True
        # per-token FP8 publishes may be done by the kernel that produces K
        # (wf_qk_norm_rope_publish): the closures then expose their targets
        # (``exch.fp8_publish_targets(layer)``) and only write the flags.  Off
        # by default: at the 1.3B tick shape the fused kernel moves fewer
        # bytes but runs slower than wf_qk_norm_rope + wf_kv_quant_publish
        self.fused_publish = False
        self.naw_max, self.Wmax = slab_geometry(max_attn_frames, rf_step, npb)
        self.local = [s for s in range(rf_step + 1) if self.stage_rank[s] == rank]
        # a CPU device is accepted only to exercise the host-side bookkeeping in tests
        self.copy_stream = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None
        self._pending: list = []
        self._ipc_bases: list[int] = []
        self._opened: dict = {}
        self.slabs: dict = {}
        self.flags: dict = {}
        self.src_index: dict = {}
        W = self.Wmax * T
        for m in self.local:
            if m >= rf_step:
                continue
            srcs = list(range(m + 1, rf_step)) + [self.store]
            self.src_index[m] = {s: i for i, s in enumerate(srcs)}
            if fp8:
                # FP8 slabs hold only what is received: the live store slot and
                # the higher stages' in-flight chunks, rf_step - m compact slots
                # (fp8_slot); anchor, working and own pages reach the bf16
                # context buffer (kb, vb) from local memory
                W8 = self.slab_rows(m)
                sl = dict(kc=torch.zeros((GT, Ln, W8, H * D), device=self.device, dtype=torch.uint8),
                          vc=torch.zeros((GT, Ln, W8, H * D), device=self.device, dtype=torch.uint8),
                          ks=torch.ones((GT, Ln, W8), device=self.device, dtype=torch.float32),
                          vs=torch.ones((GT, Ln, W8), device=self.device, dtype=torch.float32),
                          kb=torch.zeros((W, H, D), device=self.device, dtype=dtype),
                          vb=torch.zeros((W, H, D), device=self.device, dtype=dtype))
            else:
                sl = dict(k=torch.zeros((GT, Ln, W, H, D), device=self.device, dtype=dtype),
                          v=torch.zeros((GT, Ln, W, H, D), device=self.device, dtype=dtype))
            self.slabs[m] = sl
            self.flags[m] = torch.zeros((len(srcs), GT, Ln), device=self.device, dtype=torch.int32)
        self.store_buf = None
        if self.store in self.local:
            cap = (1 + max(0, (max_attn_frames - 2 * npb) // npb) + 1) * T
            self.store_buf = (torch.zeros((cap, H, D), device=self.device, dtype=dtype),
                              torch.zeros((cap, H, D), device=self.device, dtype=dtype))
        self.timeout_word = torch.zeros(1, device=self.device, dtype=torch.int32)
        # slab-generation credits, indexed by consumer stage: the rank hosting
        # consumer stage m writes tick + 1 into credit[m] of every rank that
        # publishes to m once its tick's reads are done (release_slots); a
        # producer waits on it before reusing that generation (acquire_slots)
        self.credit = torch.zeros(max(1, rf_step), device=self.device, dtype=torch.int32)
        self.credit_dst: dict = {}  # local consumer stage -> [peer address of credit[m]]
        # when a list, every remote flag wait appends its (start, end) CUDA events:
        # the exposed part of the exchange on this rank's compute stream
        self.wait_timer = None
        self.timeline = None  # optional Timeline: stamps at layer entry and after each remote wait
        # destination tables: consumer stage -> dict of base pointers (local or peer)
        self.dst: dict = {}
        self._exchange_handles()

    # ------------------------------------------------------------------ setup
    def _exchange_handles(self) -> None:
        mine = {}
        for m, sl in self.slabs.items():
            ent = {k: (ipc.ipc_export(t) if self.world > 1 else None) for k, t in sl.items()
                   if k in ("k", "v", "kc", "vc", "ks", "vs")}
            ent["flags"] = ipc.ipc_export(self.flags[m]) if self.world > 1 else None
            mine[m] = ent
        credit_h = ipc.ipc_export(self.credit) if self.world > 1 else None
        if self.world > 1:
            gathered = [None] * self.world
            dist.all_gather_object(gathered, (self.rank, mine, credit_h), group=self.group)
        else:
            gathered = [(self.rank, mine, credit_h)]
        for rk, _ents, ch in gathered:
            if rk == self.rank:
                continue
            # consumer stages here that a stage on rank rk publishes to
            for m in self.local:
                if m < self.store and any(self.stage_rank[s] == rk for s in range(m + 1, self.store + 1)):
                    h, off = ch
                    self.credit_dst.setdefault(m, []).append(self._open(h) + off + 4 * m)
        for rk, ents, _ch in gathered:
            for m, ent in ents.items():
                if rk == self.rank:
                    sl = self.slabs[m]
                    self.dst[m] = {k: sl[k].data_ptr() for k in ent if k != "flags"}
                    self.dst[m]["flags"] = self.flags[m].data_ptr()
                    self.dst[m]["local"] = True
                elif any(s > m or s == self.store for s in self.local):
                    d = {"local": False}
                    for k, (h, off) in ent.items():
                        d[k] = self._open(h) + off
                    self.dst[m] = d
        if self.world > 1:
            dist.barrier(group=self.group)

    def _open(self, h) -> int:
        if h not in self._opened:
            if self._host_ipc_open is not None:
                base = self._host_ipc_open(h)  # the host records and closes it
            else:
                base = ipc.ipc_open_handle(h)
                self._ipc_bases.append(base)
            self._opened[h] = base
        return self._opened[h]

    def close(self, coordinated: bool = True) -> None:
        """Release imported mappings (wave_rt/denoiser/engine.py:156-212): drain
        the copy stream and the device, barrier, close every opened handle in
        reverse order, barrier again; on an exception path (coordinated=False)
        no collective is issued.  Idempotent."""
        if getattr(self, "_closed", False):
            return
        self._closed = True
        if self._host_ipc_open is not None:
            # the host closes the mappings it opened (between its own barriers)
            self._opened.clear()
            self.dst.clear()
            return
        if self.copy_stream is not None:
            self.copy_stream.synchronize()
            torch.cuda.synchronize(self.device)
        if coordinated and self.world > 1:
            dist.barrier(group=self.group)
        for base in reversed(self._ipc_bases):
            ipc.ipc_close_handle(base)
        self._ipc_bases.clear()
        self._opened.clear()
        if coordinated and self.world > 1:
            dist.barrier(group=self.group)
        self.dst.clear()

    # ---------------------------------------------------------------- publish
    def slab_rows(self, m: int) -> int:
        """Token rows per (generation, layer) block of consumer stage m's slab:
        Wmax slots of the bf16 context (paged.py:26-30), or the rf_step - m
        compact received slots of an FP8 slab (at most one live slot and the
        in-flight chunks of stages m+1 .. rf_step-1)."""
        return ((self.rf_step - m) if self.fp8 else self.Wmax) * self.T

    @staticmethod
    def fp8_slot(g: dict, slot: int) -> int:
        """The compact FP8 slab slot of context slot ``slot`` of a tick with
        geometry ``g`` (tick_geometry): the live store slot (slot naw) -> 0;
        the in-flight chunk at base_infl + k (k >= 1; base_infl itself is the
        consumer's own chunk) -> live + k - 1."""
        if g["live"] and slot == g["naw"]:
            return 0
        k = slot - g["base_infl"]
        if k < 1:
            raise ValueError(f"context slot {slot} is not received (naw={g['naw']}, base_infl={g['base_infl']})")
        return g["live"] + k - 1

    def _slot_offsets(self, m, gen, layer, slot):
        """Token-row offset of (gen, layer, slot) in consumer m's slabs (slot is
        compact for FP8 slabs, see fp8_slot)."""
        return (gen * self.Ln + layer) * self.slab_rows(m) + slot * self.T

    def fp8_targets(self, s: int, send, layer: int, gen: int):
        """Producer stage ``s``'s FP8 destination slots for (layer, gen): one
        (codes_k, codes_v, scales_k, scales_v) pointer tuple per (stage, slot)
        of ``send``, local or peer."""
        HD = self.H * self.D
        out = []
        for m, slot in send:
            d = self.dst[m]
            tok = self._slot_offsets(m, gen, layer, slot)
            out.append((d["kc"] + tok * HD, d["vc"] + tok * HD, d["ks"] + tok * 4, d["vs"] + tok * 4))
        return out

    def _expose_targets(self, exch, s: int, send, gen: int) -> None:
        """Let the K-producing kernel publish for this closure (per-token FP8)."""
        if self.fp8 and self.fp8_gran == "token" and self.fused_publish and send:
            exch.fp8_publish_targets = lambda layer: self.fp8_targets(s, send, layer, gen)
            exch.prepublished = set()

    def publish(self, s: int, k: torch.Tensor, v: torch.Tensor, send, layer: int, gen: int, tick: int,
                prepublished: bool = False) -> None:
        """Producer stage ``s`` publishes one layer's K, V [T, H, D] into each
        consumer slot of ``send`` [(stage, slot)] (paged.py:120-145).  With
        ``prepublished`` the codes and scales are already in place (written
        earlier on this stream by wf_qk_norm_rope_publish) and only the
        release flags remain."""
        if not send:
            return
        T, HD = self.T, self.H * self.D
        src_i = {m: self.src_index_of(m, s) for m, _ in send}
        cur_h = self._cur_stream_handle()
        if self.fp8:
            ck, cv, sk, sv = (list(x) for x in zip(*self.fp8_targets(s, send, layer, gen)))
            if prepublished:
                pass
            elif self.fp8_gran == "token":
                kernels.kv_quant_publish(k.reshape(T, HD), v.reshape(T, HD), ck, cv, sk, sv)
            else:
                self._publish_tensor_scaled(k, v, ck, cv, sk, sv, cur_h)
            for m, _slot in send:
                d = self.dst[m]
                if not d["local"]:
                    fl = d["flags"] + ((src_i[m] * self.GT + gen) * self.Ln + layer) * 4
                    ipc.stream_write_u32(cur_h, fl, tick)
            return
        remote = []
        for m, slot in send:
            d = self.dst[m]
            if d["local"]:
                sl = self.slabs[m]
                sl["k"][gen, layer, slot * T:(slot + 1) * T].copy_(k)
                sl["v"][gen, layer, slot * T:(slot + 1) * T].copy_(v)
            else:
                remote.append((m, slot))
        if not remote:
            return
        if self.copy_stream is not None:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self.copy_stream.wait_event(ev)
            sh = self.copy_stream.cuda_stream
        else:
            sh = 0  # host bookkeeping mode (CPU tensors; the IPC layer is the host's)
        nb = k.numel() * k.element_size()
        for m, slot in remote:
            d = self.dst[m]
            off = self._slot_offsets(m, gen, layer, slot) * self.H * self.D * k.element_size()
            ipc.memcpy_dtod_async(d["k"] + off, k.data_ptr(), nb, sh)
            ipc.memcpy_dtod_async(d["v"] + off, v.data_ptr(), nb, sh)
            fl = d["flags"] + ((src_i[m] * self.GT + gen) * self.Ln + layer) * 4
            ipc.stream_write_u32(sh, fl, tick)
        if self.copy_stream is not None:
            k.record_stream(self.copy_stream)
            v.record_stream(self.copy_stream)
        self._pending += [k, v]

    def _cur_stream_handle(self) -> int:
        if self.device.type != "cuda":
            return 0
        return torch.cuda.current_stream(self.device).cuda_stream

    def _publish_tensor_scaled(self, k, v, ck, cv, sk, sv, stream) -> None:
        """FP8 publish with the reference's per-tensor scale: one scale over
        stack(K, V) (common.py:143-150), codes copied to every destination and
        the scale written into each destination's per-row scales, so consumers
        dequantise every slot the same way."""
        T, HD = self.T, self.H * self.D
        kv = torch.stack([k.reshape(T, HD), v.reshape(T, HD)]).view(2 * T, HD)
        codes, scale = kernels.kv_quant(kv, L.WF_SCALE_TENSOR)
        rows = scale.expand(T).contiguous()
        for a, b, c, d in zip(ck, cv, sk, sv):
            ipc.memcpy_dtod_async(a, codes.data_ptr(), T * HD, stream)
            ipc.memcpy_dtod_async(b, codes.data_ptr() + T * HD, T * HD, stream)
            ipc.memcpy_dtod_async(c, rows.data_ptr(), 4 * T, stream)
            ipc.memcpy_dtod_async(d, rows.data_ptr(), 4 * T, stream)
        self._pending += [codes, rows]

    def src_index_of(self, m: int, s: int) -> int:
        srcs = list(range(m + 1, self.rf_step)) + [self.store]
        return srcs.index(s)

    def wait(self, m: int, src: int, layer: int, gen: int, tick: int) -> None:
        """Bounded device-side acquire on src's flag for (gen, layer) (paged.py:147-154)."""
        if self.stage_rank[src] == self.rank:
            return  # same GPU: the publish precedes this read on the stream
        i = self.src_index[m][src]
        addr = self.flags[m][i, gen, layer].data_ptr()
        sink = self.wait_timer if self.device.type == "cuda" else None
        if sink is not None:
            cur = torch.cuda.current_stream(self.device)
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record(cur)
        ipc.wait_flag_bounded(self._cur_stream_handle(), addr, tick, self.timeout_s, self.timeout_word.data_ptr())
        if self.timeline is not None:
            self.timeline.mark(f"s{m}.L{layer}.w{src}")
        if sink is not None:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record(cur)
            sink.append((e0, e1))

    def wait_all(self, m: int, srcs, layer: int, gen: int, tick: int) -> None:
        """``wait`` for every producer in ``srcs`` of (gen, layer), the remote
        ones in one bounded launch (``wf_wait_flags``)."""
        addrs = [self.flags[m][self.src_index[m][src], gen, layer].data_ptr()
                 for src in srcs if self.stage_rank[src] != self.rank]
        if not addrs:
            return
        sink = self.wait_timer if self.device.type == "cuda" else None
        if sink is not None:
            cur = torch.cuda.current_stream(self.device)
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record(cur)
        ipc.wait_flags_bounded(self._cur_stream_handle(), addrs, tick, self.timeout_s, self.timeout_word.data_ptr())
        if self.timeline is not None:
            self.timeline.mark(f"s{m}.L{layer}.w")
        if sink is not None:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record(cur)
            sink.append((e0, e1))

    def remote_consumers(self) -> list[int]:
        """Consumer stages on other ranks that a stage on this rank publishes to."""
        return [m for m in range(self.store) if self.stage_rank[m] != self.rank
                and any(s > m for s in self.local)]

    def acquire_slots(self, tick: int) -> None:
        """Before the first publish of ``tick``: wait (bounded, on the device)
        until every remote consumer has finished tick - GT, the last tick that
        read the slab generation this tick writes.  A consumer on this rank
        needs no wait: its reads precede these writes on the stream."""
        if self.world == 1 or tick < self.GT:
            return
        h = self._cur_stream_handle()
        for m in self.remote_consumers():
            ipc.wait_flag_bounded(h, self.credit[m].data_ptr(), tick - self.GT + 1, self.timeout_s,
                                  self.timeout_word.data_ptr())

    def release_slots(self, tick: int) -> None:
        """After the last read of this tick's slabs (the tick's attention and
        assembly, on the compute stream): tell every remote producer of each
        consumer stage hosted here that ``tick``'s generation is free.  Written
        every tick, active or not, so producers never wait on an idle stage."""
        if self.world == 1:
            return
        h = self._cur_stream_handle()
        for _m, addrs in sorted(self.credit_dst.items()):
            for a in addrs:
                ipc.stream_write_u32(h, a, tick + 1)

    def drain(self) -> None:
        """onesided.py:181-187: order later work after this tick's publications."""
        if self.copy_stream is not None:
            ev = torch.cuda.Event()
            ev.record(self.copy_stream)
            torch.cuda.current_stream(self.device).wait_event(ev)
        self._pending = []

    def check_timeouts(self) -> None:
        """Raise if any bounded wait gave up (reads a device word; syncs)."""
        if int(self.timeout_word.item()) != 0:
            raise TimeoutError("paged exchange: a producer flag did not arrive within the timeout")

    # ---------------------------------------------------------------- context
    def anchor_working_parts(self, clean_L, csf, qf):
        """common.py:70-91 before the RoPE: (anchor page, working pages,
        anchor rope start frame), or None when the clean list is empty."""
        if not clean_L:
            return None
        npb = self.npb
        wmax_chunks = max(0, (self.max_attn_frames - qf - npb) // npb)
        anchor, rest = clean_L[0], clean_L[1:]
        working = rest[-wmax_chunks:] if wmax_chunks > 0 else []
        return anchor, working, csf - len(working) * npb - npb

    def anchor_working(self, clean_L, csf, qf, rope_fn):
        """common.py:70-91 -> (list of K pages, list of V pages) as [T, H, D]."""
        parts = self.anchor_working_parts(clean_L, csf, qf)
        if parts is None:
            return [], []
        anchor, working, rope_start = parts
        ak = rope_fn(anchor["ku"], rope_start)
        return [ak] + [w["kr"] for w in working], [anchor["v"]] + [w["v"] for w in working]

    @staticmethod
    def _rows(t: torch.Tensor) -> tuple[int, int]:
        """(data pointer, token-row stride in elements) of a [.., T, H, D] page
        whose (H, D) rows are contiguous."""
        if t.stride(-1) != 1 or t.stride(-2) != t.shape[-1]:
            raise ValueError("context page rows must be contiguous over (H, D)")
        return t.data_ptr(), t.stride(-3)

    def assemble(self, Kb, Vb, parts, rope_tab_fn, self_kv, self_off, deq=()):
        """The stage's K/V context of one layer in one launch (wf_kv_assemble):
        the anchor re-RoPEd straight into slot 0, working pages and the own
        chunk copied, received FP8 rows dequantised.  ``deq`` lists (rows
        slice of the context, K codes, K scales, V codes, V scales)."""
        T, HD = self.T, self.H * self.D
        kp, kst = self._rows(Kb)
        vp, vst = self._rows(Vb)
        esz = Kb.element_size()
        segs = []
        off = 0
        if parts is not None:
            anchor, working, rs = parts
            cos, sin = rope_tab_fn(rs)
            src, ss = self._rows(anchor["ku"])
            segs.append((L.WF_SEG_ROPE, src, cos.data_ptr(), sin.data_ptr(), kp, T, ss, kst))
            src, ss = self._rows(anchor["v"])
            segs.append((L.WF_SEG_COPY, src, 0, 0, vp, T, ss, vst))
            off = T
            for w in working:
                src, ss = self._rows(w["kr"])
                segs.append((L.WF_SEG_COPY, src, 0, 0, kp + off * kst * esz, T, ss, kst))
                src, ss = self._rows(w["v"])
                segs.append((L.WF_SEG_COPY, src, 0, 0, vp + off * vst * esz, T, ss, vst))
                off += T
        k, v = self_kv
        src, ss = self._rows(k)
        segs.append((L.WF_SEG_COPY, src, 0, 0, kp + self_off * kst * esz, T, ss, kst))
        src, ss = self._rows(v)
        segs.append((L.WF_SEG_COPY, src, 0, 0, vp + self_off * vst * esz, T, ss, vst))
        for rows, kc, ks, vc, vs in deq:
            n = rows.stop - rows.start
            segs.append((L.WF_SEG_DEQUANT, kc.data_ptr(), ks.data_ptr(), 0, kp + rows.start * kst * esz, n, HD, kst))
            segs.append((L.WF_SEG_DEQUANT, vc.data_ptr(), vs.data_ptr(), 0, vp + rows.start * vst * esz, n, HD, vst))
        kernels.kv_assemble(segs, HD, self.D)
        return off

    @staticmethod
    def _lp_mark(prof):
        """A CUDA event for the optional per-layer profile of the host
        (WaveDenoiser._lp_cur, wave_rt/denoiser/exchange/paged.py:206-254)."""
        if prof is None:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return ev

    def make_denoise_exch(self, m: int, clean, act, tick_csf, tick_qf, store_active, tick, rope_fn=None,
                          store_slot_sink: dict | None = None, rope_tab_fn=None, prof=None):
        """The denoise closure of stage ``m`` for one tick (paged.py:156-255).

        ``rope_tab_fn(start_frame, pph, ppw, dim, heads) -> (cos, sin)`` gives
        the anchor's RoPE tables (f32 [T, head_dim/2]); with it every layer's
        context is one wf_kv_assemble launch.  Without it, ``rope_fn(ku,
        start_frame)`` rotates the anchor and the pages are copied one by one.
        ``store_slot_sink[layer]`` receives a [2, T, H, D] copy of the store's
        live slot (the reference's ``_exch_store_slot``, promoted to a clean
        page after the tick).  ``prof()`` returns the host's per-layer profile
        record (or None)."""
        g = tick_geometry(m, tick, act, store_active, self.rf_step, self.max_attn_frames, self.npb)
        if g["active_slots"] > self.Wmax:
            raise RuntimeError(f"[paged stage {m}] active_slots={g['active_slots']} > Wmax={self.Wmax}")
        if rope_tab_fn is None and rope_fn is None:
            raise ValueError("make_denoise_exch needs rope_tab_fn or rope_fn for the anchor re-RoPE")
        T = self.T
        gen = tick % self.GT
        naw, base_infl, act_slots = g["naw"], g["base_infl"], g["active_slots"]
        self_off, live_off, active_len = base_infl * T, naw * T, act_slots * T
        recv, send = g["recv"], g["send"]
        if self.fp8:  # FP8 slabs are addressed by compact slot; consumers share this tick's geometry
            send = [(mm, self.fp8_slot(g, slot)) for mm, slot in send]
        live = g["live"]
        n_in = act_slots - base_infl - 1  # in-flight chunks of higher stages
        # received FP8 rows: (context rows, compact slab rows) of the live slot and the in-flight chunks
        recv_rows = [(slice(naw * T, base_infl * T), slice(0, live * T)),
                     (slice((base_infl + 1) * T, act_slots * T), slice(live * T, (live + n_in) * T))]
        sl = self.slabs[m]

        def exch(*, layer_idx, roped_query, roped_key, unroped_key, value, current_start, tokens_per_frame,
                 post_patch_height, post_patch_width, dim, rope_num_heads, num_frames_per_block):
            Lh = layer_idx
            k = roped_key[0]
            v = value[0]
            lp = prof() if prof is not None else None
            e_en = self._lp_mark(lp)
            if self.timeline is not None:
                self.timeline.mark(f"s{m}.L{Lh}.in")
            self.publish(m, k, v, send, Lh, gen, tick, prepublished=Lh in getattr(exch, "prepublished", ()))
            e_pub = self._lp_mark(lp)
            if self.fp8:
                Kb, Vb = sl["kb"], sl["vb"]
            else:
                Kb, Vb = sl["k"][gen, Lh], sl["v"][gen, Lh]
            if rope_tab_fn is not None and self.fused_assembly:
                parts = self.anchor_working_parts(clean[Lh], tick_csf, tick_qf)
                if (0 if parts is None else 1 + len(parts[1])) != naw:
                    raise RuntimeError(f"[paged stage {m}] anchor+working != naw={naw} (t={tick})")
                self.wait_all(m, recv, Lh, gen, tick)
                e_wt = self._lp_mark(lp)
                deq = []
                if self.fp8:
                    for rows, src in recv_rows:
                        if rows.stop > rows.start:
                            deq.append((rows, sl["kc"][gen, Lh, src], sl["ks"][gen, Lh, src],
                                        sl["vc"][gen, Lh, src], sl["vs"][gen, Lh, src]))
                tabs = (lambda start: rope_tab_fn(start, post_patch_height, post_patch_width, dim,
                                                  rope_num_heads))
                self.assemble(Kb, Vb, parts, tabs, (k, v), self_off, deq)
            else:
                aK, aV = self.anchor_working(clean[Lh], tick_csf, tick_qf, rope_fn)
                if len(aK) != naw:
                    raise RuntimeError(f"[paged stage {m}] anchor+working={len(aK)} != naw={naw} (t={tick})")
                off = 0
                for ak, av in zip(aK, aV):
                    Kb[off:off + T].copy_(ak.reshape(T, self.H, self.D))
                    Vb[off:off + T].copy_(av.reshape(T, self.H, self.D))
                    off += T
                Kb[self_off:self_off + T].copy_(k)
                Vb[self_off:self_off + T].copy_(v)
                self.wait_all(m, recv, Lh, gen, tick)
                e_wt = self._lp_mark(lp)
                if self.fp8:
                    HD = self.H * self.D
                    for rows, src in recv_rows:
                        if rows.stop <= rows.start:
                            continue
                        kernels.kv_dequant(sl["kc"][gen, Lh, src], sl["ks"][gen, Lh, src], L.WF_SCALE_TOKEN,
                                           out=Kb[rows].view(-1, HD))
                        kernels.kv_dequant(sl["vc"][gen, Lh, src], sl["vs"][gen, Lh, src], L.WF_SCALE_TOKEN,
                                           out=Vb[rows].view(-1, HD))
            if store_active and store_slot_sink is not None:
                # torch.stack copies: the live slot outlives this layer's buffers
                store_slot_sink[Lh] = torch.stack([Kb[live_off:live_off + T], Vb[live_off:live_off + T]])
            if lp is not None:
                lp["layers"].append(dict(layer=Lh, enter=e_en, pub=e_pub, wait=e_wt, cat=self._lp_mark(lp)))
            return Kb[:active_len].unsqueeze(0), Vb[:active_len].unsqueeze(0)

        self._expose_targets(exch, m, send, gen)
        return exch

    def make_store_exch(self, clean, store_kv: list, chunk: int, act, tick, rope_fn=None, rope_tab_fn=None,
                        prof=None):
        """The store closure for one tick (paged.py:257-310).  ``store_kv[layer]``
        receives (roped_key, unroped_key, value) as passed, [1, T, H, D] each,
        as the reference keeps them for promotion (engine.py:449-515)."""
        if rope_tab_fn is None and rope_fn is None:
            raise ValueError("make_store_exch needs rope_tab_fn or rope_fn for the anchor re-RoPE")
        clean_len = min(8, max(0, tick - self.store))
        wmax_chunks = max(0, (self.max_attn_frames - len(act) * self.npb - self.npb) // self.npb)
        naw = 0 if clean_len == 0 else 1 + min(wmax_chunks, clean_len - 1)
        # the live slot of every active denoise stage; compact slot 0 of an FP8 slab
        send = [(m, 0 if self.fp8 else naw) for m in act]
        gen = tick % self.GT
        T = self.T
        Kbuf, Vbuf = self.store_buf

        def exch(*, layer_idx, roped_query, roped_key, unroped_key, value, current_start, tokens_per_frame,
                 post_patch_height, post_patch_width, dim, rope_num_heads, num_frames_per_block):
            k = roped_key[0]
            v = value[0]
            lp = prof() if prof is not None else None
            e_en = self._lp_mark(lp)
            if self.timeline is not None:
                self.timeline.mark(f"s{self.store}.L{layer_idx}.in")
            self.publish(self.store, k, v, send, layer_idx, gen, tick,
                         prepublished=layer_idx in getattr(exch, "prepublished", ()))
            e_pub = self._lp_mark(lp)
            if rope_tab_fn is not None and self.fused_assembly:
                parts = self.anchor_working_parts(clean[layer_idx], chunk * self.npb, self.npb)
                n_aw = 0 if parts is None else 1 + len(parts[1])
                tabs = (lambda start: rope_tab_fn(start, post_patch_height, post_patch_width, dim,
                                                  rope_num_heads))
                self.assemble(Kbuf, Vbuf, parts, tabs, (k, v), n_aw * T)
                off = n_aw * T
            else:
                aK, aV = self.anchor_working(clean[layer_idx], chunk * self.npb, self.npb, rope_fn)
                off = 0
                for ak, av in zip(aK, aV):
                    Kbuf[off:off + T].copy_(ak.reshape(T, self.H, self.D))
                    Vbuf[off:off + T].copy_(av.reshape(T, self.H, self.D))
                    off += T
                Kbuf[off:off + T].copy_(k)
                Vbuf[off:off + T].copy_(v)
            store_kv[layer_idx] = (roped_key, unroped_key, value)
            if lp is not None:
                lp["layers"].append(dict(layer=layer_idx, enter=e_en, pub=e_pub, wait=e_pub,
                                         cat=self._lp_mark(lp)))
            return Kbuf[:off + T].unsqueeze(0), Vbuf[:off + T].unsqueeze(0)

        self._expose_targets(exch, self.store, send, gen)
        return exch


def _env_flag(name: str) -> bool:
    import os

    return os.environ.get(name, "").strip().lower() not in ("", "0", "false", "no", "off")


class PagedExchangeMixin:
    """The reference's paged-mode entry points (wave_rt/denoiser/exchange/
    paged.py) over ``PagedTransport``, for the reference's WaveDenoiser, one
    stage per rank (wave_rt/config.py:79-83).  Placed ahead of the reference
    mixins in WaveDenoiser's bases, it needs nothing from its host beyond what
    the reference's classes already provide:

      * ``_init_paged`` is called by ``_init_transport_state`` (engine.py:
        147-148) after ``_ipc_handles`` exists.  It sets what the reference's
        ``_init_onesided`` sets for the paged mode and what ``close()`` reads:
        ``_p2p`` (the IPC module, whose ``ipc_close_handle`` the close uses),
        ``_os_scopy`` (the copy stream, synchronised by the close), ``_os_gt``,
        ``_os_src_index``, ``_os_in_srcs`` and ``_pg_naw`` / ``_pg_wmax`` /
        ``_pg_dst`` / ``_pg_k`` / ``_pg_v``.  Every peer mapping is opened
        through the host's ``_ipc_open``, so the host's close (engine.py:
        156-212) closes them in reverse order between its two barriers.
      * the anchor re-RoPE tables come from the host's ``_anchor_rope``
        (common.py:45-68); the rotation runs inside the one-launch context
        assembly;
      * FP8 transport is switched by the reference's own flag,
        ``WAVE_FP8KV_ONESIDED`` (settings.py:21), which the reference's paged
        mode refuses (paged.py:36-37); ``WAVE_FP8KV_GRAN`` = ``token``
        (default) or ``tensor`` picks the scale granularity;
      * the closures store ``store_kv[L] = (roped_key, unroped_key, value)``
        and ``_exch_store_slot[L]`` as a [2, T, H, D] tensor, the shapes the
        host's promotion reads (engine.py:449-515), and fill ``_lp_cur``.
    """

    def _init_paged(self) -> None:
        self._p2p = ipc
        fp8 = _env_flag("WAVE_FP8KV_ONESIDED")
        gran = __import__("os").environ.get("WAVE_FP8KV_GRAN", "token").strip() or "token"
        self._os_fp8 = False  # the reference's onesided FP8 cast is not used by this transport
        self._paged_fp8 = fp8
        self._pg = PagedTransport(device=self.device, rank=self.rank, world=self.world,
                                  stage_rank=list(range(self.rf_step + 1)), rf_step=self.rf_step, Ln=self.Ln,
                                  T=self.tokens_per_chunk, H=self._kv_shape[2], D=self._kv_shape[3], npb=self.npb,
                                  max_attn_frames=self.max_attn_frames, fp8=fp8, fp8_gran=gran, dtype=self.dtype,
                                  ipc_open=self._ipc_open)
        pg = self._pg
        self._pg_naw, self._pg_wmax = pg.naw_max, pg.Wmax
        self._os_gt = pg.GT
        self._os_scopy = pg.copy_stream
        self._os_src_index = dict(pg.src_index.get(self.rank, {}))
        self._os_in_srcs = sorted(self._os_src_index, key=self._os_src_index.get)
        self._pg_dst = {m: d for m, d in pg.dst.items() if m != self.rank}
        sl = pg.slabs.get(self.rank)
        if sl is not None:
            self._pg_k = sl.get("k", sl.get("kc"))
            self._pg_v = sl.get("v", sl.get("vc"))

    def _wf_rope_tables(self, start_frame, pph, ppw, dim, heads):
        """The host's anchor RoPE tables (common.py:45-68) as f32 [T, head_dim/2]
        interleaved-pair tables, the form wf_kv_assemble reads.  A table of
        head_dim columns (each angle repeated for its pair) is reduced to one
        column per pair."""
        cos, sin = self._anchor_rope(self.npb, pph, ppw, start_frame, dim, heads, self.device)
        hd = dim // heads
        T = self.tokens_per_chunk
        out = []
        for t in (cos, sin):
            t = t.reshape(T, -1)
            if t.shape[1] == hd:
                if not torch.equal(t[:, 0::2], t[:, 1::2]):
                    raise ValueError("anchor RoPE table: head_dim columns that are not pair-repeated")
                t = t[:, 0::2]
            if t.shape[1] != hd // 2:
                raise ValueError(f"anchor RoPE table has {t.shape[1]} columns; expected {hd // 2}")
            out.append(t.float().contiguous())
        return out[0], out[1]

    def _publish_paged(self, k, v, dst_slots, layer: int, gen: int, tick: int) -> None:
        """paged.py:120-145.  ``dst_slots`` are (stage, slot) pairs; with FP8
        transport the slots are compact slab slots (PagedTransport.fp8_slot)."""
        self._pg.publish(self.rank, k, v, dst_slots, layer, gen, tick)

    def _wait_paged_flag(self, src: int, layer: int, gen: int, tick: int) -> None:
        self._pg.wait(self.rank, src, layer, gen, tick)

    def _make_denoise_exch_paged(self, clean, act_ranks, tick_csf, tick_qf, store_active):
        return self._pg.make_denoise_exch(self.rank, clean, act_ranks, tick_csf, tick_qf, store_active,
                                          self._cur_tick, store_slot_sink=self._exch_store_slot,
                                          rope_tab_fn=self._wf_rope_tables, prof=lambda: self._lp_cur)

    def _make_store_exch_paged(self, clean, store_kv, c, act_ranks):
        return self._pg.make_store_exch(clean, store_kv, c, act_ranks, self._cur_tick,
                                        rope_tab_fn=self._wf_rope_tables, prof=lambda: self._lp_cur)

    def _drain_publish(self) -> None:
        self._pg.drain()
