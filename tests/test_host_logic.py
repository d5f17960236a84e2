"""Host-side logic of the wavefront path on CPU: stage placement, slot
geometry (against the reference-generated golden), and the multi-process IPC
handle exchange / close ordering over gloo with a fake IPC layer (the
reference tests its close ordering the same way, tests/test_ipc_lifecycle.py)."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from waveforcing_b200.denoiser.exchange import paged
from waveforcing_b200.wavefront.engine import place_stages, stage_costs


def test_place_stages_contiguous_and_balanced():
    assert place_stages(5, 8) == [0, 1, 2, 3, 4, 5]
    assert place_stages(5, 6) == [0, 1, 2, 3, 4, 5]
    assert place_stages(5, 1) == [0] * 6
    for world in (2, 3, 4, 5):
        pl = place_stages(5, world)
        assert pl[0] == 0 and pl[-1] == world - 1
        assert all(b - a in (0, 1) for a, b in zip(pl, pl[1:])), pl  # contiguous, ordered
        cost = stage_costs(5)
        loads = [sum(c for c, r in zip(cost, pl) if r == k) for k in range(world)]
        assert max(loads) <= sum(cost) / world * 1.6, (world, loads)
    assert place_stages(4, 2) == place_stages(4, 2)


def test_tick_geometry_matches_reference_golden(golden):
    recs = golden("geometry.json")
    for r in recs:
        if r["role"] != "denoise":
            continue
        g = paged.tick_geometry(r["rank"], r["tick"], r["act_ranks"], r["store_active"], r["rf_step"], 21, 3)
        T = 4680
        assert g["naw"] == r["naw"]
        assert g["base_infl"] * T == r["self_off"] and g["naw"] * T == r["live_off"]
        assert g["active_slots"] * T == r["active_len"]
        assert g["recv"] == r["recv_srcs"]
        assert [list(x) for x in g["send"]] == r["send_slots"]


def test_slab_geometry_matches_reference():
    # paged.py:26-30 for 5-step and 4-step, max_attn_frames 21
    assert paged.slab_geometry(21, 5, 3) == (2, 8)
    assert paged.slab_geometry(21, 4, 3) == (3, 8)


# ------------------------------------------------------------- 2-rank gloo
class _FakeIPC:
    def __init__(self, rank, log):
        self.rank, self.log, self.n = rank, log, 0

    def ipc_export(self, t):
        self.n += 1
        return (bytes([self.rank, self.n]) + bytes(62), 0)

    def ipc_open_handle(self, h):
        ptr = 0x10000 * (h[0] + 1) + h[1] * 0x100
        self.log.append(("open", ptr))
        return ptr

    def ipc_close_handle(self, ptr):
        self.log.append(("close", ptr))


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    log = []
    paged.ipc = _FakeIPC(rank, log)
    try:
        # 3-step wavefront (stages 0,1,2 + store 3) on 2 ranks: {0,1} on rank 0, {2,3} on rank 1
        xp = paged.PagedTransport(device="cpu", rank=rank, world=world, stage_rank=[0, 0, 1, 1], rf_step=3, Ln=2,
                                  T=4, H=1, D=8, fp8=False)
        dst = {m: dict(d) for m, d in xp.dst.items()}
        credit = ({m: len(a) for m, a in xp.credit_dst.items()}, xp.remote_consumers())
        xp.close()
        xp.close()  # idempotent
        q.put((rank, sorted(dst), {m: d["local"] for m, d in dst.items()}, log, credit))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_two_rank_handle_exchange_and_close_order():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, stages, local, log, credit = q.get(timeout=120)
        res[r] = (stages, local, log, credit)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # rank 0 hosts consumer stages 0,1 (local); it publishes only from 0/1 to lower stages, so its one
    # remote mapping is rank 1's credit word array, which it signals for both stages (release_slots)
    assert res[0][0] == [0, 1] and all(res[0][1].values())
    assert [op for op, _ in res[0][2]] == ["open", "close"]
    assert res[0][3] == ({0: 1, 1: 1}, [])
    # rank 1's producers (stage 2, store) publish to stages 0 and 1 on rank 0: it waits on their
    # credits (acquire_slots); its own consumer stage 2 is fed locally, so it signals no one
    assert res[1][3] == ({}, [0, 1])
    # rank 1 hosts stage 2 (consumer, local) and the store, which publishes to stages 0,1 on rank 0
    assert res[1][0] == [0, 1, 2] and res[1][1] == {0: False, 1: False, 2: True}
    opens = [p for op, p in res[1][2] if op == "open"]
    closes = [p for op, p in res[1][2] if op == "close"]
    assert opens and closes == list(reversed(opens))
    assert len(set(opens)) == len(opens)  # every handle opened once


def test_context_assembly_segments(monkeypatch):
    """PagedTransport.assemble's segment list (host logic of wf_kv_assemble):
    the anchor re-RoPE into slot 0, working pages after it, the own chunk at
    self_off and received FP8 ranges, with byte offsets and row strides taken
    from the tensors (one page has strided rows)."""
    from waveforcing_b200 import _lib as L

    T, H, D = 4, 2, 8
    HD = H * D
    xp = paged.PagedTransport(device="cpu", rank=0, world=1, stage_rank=[0, 0, 0, 0], rf_step=3, Ln=2,
                              T=T, H=H, D=D, fp8=False)
    page = lambda: {"ku": torch.randn(T, H, D).bfloat16(), "kr": torch.randn(T, H, D).bfloat16(),  # noqa: E731
                    "v": torch.randn(T, H, D).bfloat16()}
    clean = [page() for _ in range(4)]
    clean[2]["kr"] = torch.randn(2 * T, H, D).bfloat16()[::2]  # strided token rows
    parts = xp.anchor_working_parts(clean, csf=30, qf=3)
    anchor, working, rs = parts
    tabs = {}

    def rope_tab(start):
        tabs[start] = (torch.zeros(T, D // 2), torch.zeros(T, D // 2))
        return tabs[start]

    Kb = torch.empty(8 * T, H, D).bfloat16()
    Vb = torch.empty(8 * T, H, D).bfloat16()
    k, v = torch.randn(T, H, D).bfloat16(), torch.randn(T, H, D).bfloat16()
    kc, vc = torch.zeros(2 * T, HD, dtype=torch.uint8), torch.zeros(2 * T, HD, dtype=torch.uint8)
    ks, vs = torch.ones(2 * T), torch.ones(2 * T)
    got = []
    monkeypatch.setattr(paged.kernels, "kv_assemble", lambda segs, cols, hd: got.append((segs, cols, hd)))
    self_off = (1 + len(working)) * T
    n_aw = xp.assemble(Kb, Vb, parts, rope_tab, (k, v), self_off, [(slice(5 * T, 7 * T), kc, ks, vc, vs)])
    assert n_aw == (1 + len(working)) * T
    (segs, cols, hd), = got
    assert (cols, hd) == (HD, D)
    row = HD * 2  # bytes per bf16 context row
    cos, sin = tabs[rs]
    exp = [(L.WF_SEG_ROPE, anchor["ku"].data_ptr(), cos.data_ptr(), sin.data_ptr(), Kb.data_ptr(), T, HD, HD),
           (L.WF_SEG_COPY, anchor["v"].data_ptr(), 0, 0, Vb.data_ptr(), T, HD, HD)]
    for i, w in enumerate(working):
        exp.append((L.WF_SEG_COPY, w["kr"].data_ptr(), 0, 0, Kb.data_ptr() + (1 + i) * T * row, T,
                    w["kr"].stride(0), HD))
        exp.append((L.WF_SEG_COPY, w["v"].data_ptr(), 0, 0, Vb.data_ptr() + (1 + i) * T * row, T, HD, HD))
    exp += [(L.WF_SEG_COPY, k.data_ptr(), 0, 0, Kb.data_ptr() + self_off * row, T, HD, HD),
            (L.WF_SEG_COPY, v.data_ptr(), 0, 0, Vb.data_ptr() + self_off * row, T, HD, HD),
            (L.WF_SEG_DEQUANT, kc.data_ptr(), ks.data_ptr(), 0, Kb.data_ptr() + 5 * T * row, 2 * T, HD, HD),
            (L.WF_SEG_DEQUANT, vc.data_ptr(), vs.data_ptr(), 0, Vb.data_ptr() + 5 * T * row, 2 * T, HD, HD)]
    assert segs == exp
    assert any(w["kr"].stride(0) == 2 * HD for w in working)  # the strided page is among the working set


def test_dit_routes_only_self_attention_through_the_backend(monkeypatch):
    """The reference sends only the patched self-attention through a custom
    kernel and leaves SGLang's other attention on torch SDPA
    (wave_rt/runtime/backend.py:215-219).  A tiny DiT forward on CPU (plain
    torch ops, RoPE restated in torch) must call the backend dispatch once per
    stage and layer and the SDPA path once per layer for the text
    cross-attention."""
    from waveforcing_b200 import kernels
    from waveforcing_b200.runtime import backend
    from waveforcing_b200.wavefront import dit as D

    def rope_torch(x, cos, sin, out=None):
        xf = x.float().reshape(*x.shape[:-1], -1, 2)
        re, im = xf[..., 0], xf[..., 1]
        c, s = cos[:, None, :], sin[:, None, :]
        return torch.stack([re * c - im * s, re * s + im * c], -1).flatten(-2).to(x.dtype)

    calls = {"self": 0, "cross": 0}
    orig_self, orig_cross = D.dispatch_attention, D.sdpa_elsewhere

    def count_self(*a, **kw):
        calls["self"] += 1
        return orig_self(*a, **kw)

    def count_cross(*a):
        calls["cross"] += 1
        return orig_cross(*a)

    monkeypatch.setattr(kernels, "rope_apply", rope_torch)
    monkeypatch.setitem(backend._WAVE_STATE, "attn", "torch_sdpa")
    monkeypatch.setattr(D, "dispatch_attention", count_self)
    monkeypatch.setattr(D, "sdpa_elsewhere", count_cross)
    cfg = D.DiTConfig(dim=256, heads=2, layers=2, ffn=512, text_len=16, text_dim=64, lat_h=4, lat_w=4)
    torch.manual_seed(0)
    m = D.WanDiT.random(cfg, torch.device("cpu"), seed=0)
    m.set_text(torch.randn(cfg.text_len, cfg.text_dim))
    tasks = [D.StageTask(torch.randn(cfg.in_ch, cfg.frames_per_block, cfg.lat_h, cfg.lat_w), 600.0, 3 * s, s)
             for s in (1, 0)]
    out = m.forward_stages(tasks, fused=False)
    assert [tuple(o.shape) for o in out] == [(cfg.in_ch, cfg.frames_per_block, cfg.lat_h, cfg.lat_w)] * 2
    assert all(torch.isfinite(o).all() for o in out)
    assert calls == {"self": cfg.layers * len(tasks), "cross": cfg.layers}


def test_fp8_compact_slots_cover_received_chunks(golden):
    """FP8 slabs keep only received chunks: for every tick of the reference's
    5- and 4-step geometry, each consumer's producers (higher stages, then
    the store's live slot) land on distinct compact slots below rf_step - m,
    and the consumer's read ranges cover exactly those slots."""
    recs = golden("geometry.json")
    seen = 0
    for r in recs:
        if r["role"] != "denoise":
            continue
        S, t, act, live = r["rf_step"], r["tick"], r["act_ranks"], r["store_active"]
        for m in act:
            gm = paged.tick_geometry(m, t, act, live, S, 21, 3)
            got = []
            for s in act:
                if s <= m:
                    continue
                gs = paged.tick_geometry(s, t, act, live, S, 21, 3)
                slot = dict(gs["send"])[m]
                got.append(paged.PagedTransport.fp8_slot(gm, slot))
            if live:
                got.append(0)  # the store's live slot
            n_in = gm["active_slots"] - gm["base_infl"] - 1
            assert sorted(got) == list(range(gm["live"] + n_in)), (S, t, m, got)
            assert all(0 <= c < S - m for c in got)
            seen += 1
    assert seen > 50


def test_kv_only_task_leaves_the_other_stages_unchanged(monkeypatch):
    """The store stage's flow output is never read (its input chunk is the
    final latent), so its task is K/V-only: the last layer stops after the
    K/V publish.  The other stages' outputs must equal a forward where every
    task runs to the head, the K/V-only task returns None, its last-layer
    self-attention is skipped, and a batch of K/V-only tasks returns all None.
    Tiny DiT on CPU with plain torch ops."""
    from waveforcing_b200 import kernels
    from waveforcing_b200.runtime import backend
    from waveforcing_b200.wavefront import dit as D

    def rope_torch(x, cos, sin, out=None):
        xf = x.float().reshape(*x.shape[:-1], -1, 2)
        re, im = xf[..., 0], xf[..., 1]
        c, s = cos[:, None, :], sin[:, None, :]
        return torch.stack([re * c - im * s, re * s + im * c], -1).flatten(-2).to(x.dtype)

    calls = {"self": 0}
    orig_self = D.dispatch_attention

    def count_self(*a, **kw):
        calls["self"] += 1
        return orig_self(*a, **kw)

    monkeypatch.setattr(kernels, "rope_apply", rope_torch)
    monkeypatch.setitem(backend._WAVE_STATE, "attn", "torch_sdpa")
    monkeypatch.setattr(D, "dispatch_attention", count_self)
    cfg = D.DiTConfig(dim=256, heads=2, layers=2, ffn=512, text_len=16, text_dim=64, lat_h=4, lat_w=4)
    m = D.WanDiT.random(cfg, torch.device("cpu"), seed=0)
    g = torch.Generator().manual_seed(1)
    m.set_text(torch.randn(cfg.text_len, cfg.text_dim, generator=g))
    lat = [torch.randn(cfg.in_ch, cfg.frames_per_block, cfg.lat_h, cfg.lat_w, generator=g) for _ in range(3)]

    def tasks(kv_only):
        return [D.StageTask(lat[i], t, 3 * i, i, kv_only=k)
                for i, (t, k) in enumerate(zip((900.0, 0.0, 500.0), kv_only))]

    full = m.forward_stages(tasks((False, False, False)), fused=False)
    calls["self"] = 0
    part = m.forward_stages(tasks((False, True, False)), fused=False)
    assert part[1] is None
    assert calls["self"] == cfg.layers * 3 - 1
    for i in (0, 2):
        torch.testing.assert_close(part[i], full[i], rtol=1e-5, atol=1e-5)  # fewer GEMM rows only
    assert m.forward_stages(tasks((True, True, True))[:1], fused=False) == [None]

