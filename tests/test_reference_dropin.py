"""This repository's paged exchange dropped into the reference's own engine.

The reference's ``WaveDenoiser`` (wave_rt/denoiser/engine.py) is imported
from a WaveForcing checkout and driven by baseline/harness.py (SGLang's RoPE
helpers and backend stood in; the engine's tick loop, exchange mixins,
promotion, migration and close run unchanged).  Three gloo ranks on CPU run
a 2-step wavefront (denoise ranks 0 and 1, store rank 2) twice:

  A. the reference's ``sync`` exchange (all_gather per layer,
     exchange/common.py:255-310) -- the mode its paged mode is verified
     against bit for bit (scripts/paged_verify.sh);
  B. ``paged`` mode with ``waveforcing_b200``'s ``PagedExchangeMixin`` placed
     ahead of the reference's bases, exactly the swap INTEGRATION.md shows.

B's peer mappings go through a CPU stand-in for CUDA IPC: exported tensors
live in shared memory, "device" copies are memmoves between processes, flags
are polled words.  The one-launch context assembly (wf_kv_assemble) is
emulated on the host with the same float32 rotation as the RoPE stand-in;
its CUDA numerics are covered by the GPU tests.

Checked, per rank and tick: every (K, V) context the closures return, every
clean page the engine promotes (keys, shapes, values -- a store_kv entry
without its batch dim would give the wrong page shape), the final latents,
and that ``close()`` returns cleanly having closed, in reverse order, every
mapping the mixin opened through the engine's ``_ipc_open``.
"""

import ctypes
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from baseline import harness

pytestmark = pytest.mark.skipif(harness.reference_checkout() is None,
                                reason="needs a WaveForcing checkout (WF_REFERENCE)")

RF_STEP, LN, H, D, C, NPB, LH, LW = 2, 2, 2, 8, 2, 3, 2, 2
T = NPB * LH * LW
NUM_FRAMES = 3 * 8  # 8 chunks: fill, steady state with anchor + working pages, drain


class ShmIPC:
    """CPU stand-in for wave_rt/distributed/ipc.py over shared memory."""

    def __init__(self, log):
        self.log = log
        self.maps = {}

    def ipc_export(self, t):
        t.share_memory_()
        return t.untyped_storage()._share_filename_cpu_(), t.storage_offset() * t.element_size()

    def ipc_open_handle(self, h):
        st = torch.UntypedStorage._new_shared_filename_cpu(*h)
        ptr = st.data_ptr()
        self.maps[ptr] = st
        self.log.append(("open", ptr))
        return ptr

    def ipc_close_handle(self, ptr):
        self.maps.pop(ptr)
        self.log.append(("close", ptr))

    def memcpy_dtod_async(self, dst, src, nbytes, stream):
        ctypes.memmove(dst, src, nbytes)

    def stream_write_u32(self, stream, addr, value):
        ctypes.c_uint32.from_address(addr).value = value

    def wait_flags_bounded(self, stream, addrs, value, timeout_s, word_ptr):
        for a in addrs:
            self.wait_flag_bounded(stream, a, value, timeout_s, word_ptr)

    def wait_flag_bounded(self, stream, addr, value, timeout_s, word_ptr):
        t0 = time.monotonic()
        while ctypes.c_int32.from_address(addr).value < value:
            if time.monotonic() - t0 > timeout_s:
                ctypes.c_int32.from_address(word_ptr).value = 1
                return
            time.sleep(1e-4)

    def enable_peer(self, peer):
        pass


def _rows(ptr, rows, stride, cols, dtype):
    esz = torch.empty(0, dtype=dtype).element_size()
    n = (rows - 1) * stride + cols if rows else 0
    buf = (ctypes.c_byte * max(1, n * esz)).from_address(ptr)
    flat = torch.frombuffer(buf, dtype=dtype, count=n) if n else torch.empty(0, dtype=dtype)
    return flat.as_strided((rows, cols), (stride, 1))


def emulate_assemble(segs, cols, head_dim):
    """Host emulation of wf_kv_assemble's three segment kinds (include/wfk.h)."""
    from waveforcing_b200 import _lib as L

    for kind, src, aux0, aux1, dst, rows, sst, dstst in segs:
        out = _rows(dst, rows, dstst, cols, torch.bfloat16)
        if kind == L.WF_SEG_COPY:
            out.copy_(_rows(src, rows, sst, cols, torch.bfloat16))
        elif kind == L.WF_SEG_ROPE:
            x = _rows(src, rows, sst, cols, torch.bfloat16).view(rows, cols // head_dim, head_dim)
            cos = _rows(aux0, rows, head_dim // 2, head_dim // 2, torch.float32)
            sin = _rows(aux1, rows, head_dim // 2, head_dim // 2, torch.float32)
            out.copy_(harness.apply_rotary_interleaved(x, cos, sin).to(torch.bfloat16).view(rows, cols))
        else:
            codes = _rows(src, rows, sst, cols, torch.uint8).view(torch.float8_e4m3fn)
            sc = _rows(aux0, rows, 1, 1, torch.float32)
            out.copy_((codes.float() * sc).to(torch.bfloat16))


class ToyDiT:
    """A per-rank model with the self-attention contract of patched_forward
    (wave_rt/runtime/backend.py:87-157): RoPE q/k, call the exchange closure,
    attend over the returned context."""

    def __init__(self, seed=0):
        g = torch.Generator().manual_seed(seed)
        dim = H * D
        self.emb = torch.randn(C, dim, generator=g)
        self.w = [[torch.randn(dim, dim, generator=g) / dim ** 0.5 for _ in range(4)] for _ in range(LN)]
        self.out = torch.randn(dim, C, generator=g) * 0.3
        self.calls = []
        self.tick = lambda: -1

    def __call__(self, lat, step, start_frame, exch):
        x = lat[0].permute(1, 2, 3, 0).reshape(T, C).float() @ self.emb
        rdims = [D - 4 * (D // 6), 2 * (D // 6), 2 * (D // 6)]
        cos, sin = harness.rope_tables_3d((NPB, LH, LW), D, rdims, start_frame)
        cos, sin = cos.float(), sin.float()
        for li in range(LN):
            wq, wk, wv, wo = self.w[li]
            q, k, v = ((x @ m).to(torch.bfloat16).view(1, T, H, D) for m in (wq, wk, wv))
            rq = harness.apply_rotary_interleaved(q, cos, sin).to(torch.bfloat16)
            rk = harness.apply_rotary_interleaved(k, cos, sin).to(torch.bfloat16)
            K, V = exch(layer_idx=li, roped_query=rq, roped_key=rk, unroped_key=k, value=v,
                        current_start=start_frame * LH * LW, tokens_per_frame=LH * LW, post_patch_height=LH,
                        post_patch_width=LW, dim=H * D, rope_num_heads=H, num_frames_per_block=NPB)
            self.calls.append((self.tick(), li, K.clone(), V.clone()))
            o = torch.nn.functional.scaled_dot_product_attention(rq.float().transpose(1, 2), K.float().transpose(1, 2),
                                                                 V.float().transpose(1, 2))
            x = x + o.transpose(1, 2).reshape(T, H * D) @ wo
        x0 = (x @ self.out).view(NPB, LH, LW, C).permute(0, 3, 1, 2)[None]
        return (lat.permute(0, 2, 1, 3, 4).float() - 0.1 * x0).to(lat.dtype)


def _run(engine, rank, mode, cls, ipc_log):
    steps = (1000, 500)
    g = torch.Generator().manual_seed(0)
    noise = torch.randn(1, C, NUM_FRAMES, LH, LW, generator=g).to(torch.bfloat16)
    model = ToyDiT()
    be = harness.StubBackend(rank=rank, device="cpu", dtype=torch.bfloat16, num_layers=LN, heads=H, head_dim=D,
                             channels=C, lat_h=LH, lat_w=LW, tokens_per_frame=LH * LW, steps=steps,
                             full_noise=noise, model=model)
    cfg = harness.make_config(engine, rf_step=RF_STEP, steps=steps, num_frames=NUM_FRAMES, exchange_mode=mode)
    den = cls(be, cfg)
    model.tick = lambda: den._cur_tick
    pages = []
    base = engine.CommonExchangeMixin
    orig = base.__dict__["_append_clean_page"]

    def rec(clean_layer, page):
        pages.append((den._cur_tick, sorted(page), {k: v.clone() for k, v in page.items() if k != "cid"}))
        orig.__func__(clean_layer, page)

    base._append_clean_page = staticmethod(rec)
    try:
        final, _tick_ms, _tl = den._systolic(be.full_noise_bcthw, warmup_pass=False, num_ticks=den.num_ticks)
    finally:
        base._append_clean_page = orig
    opened = list(den._ipc_handles)
    den.close()
    return dict(calls=model.calls, pages=pages, final=final, opened=opened, left=list(den._ipc_handles))


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.synchronize = lambda *a, **k: None  # CPU ranks: nothing is in flight on a device
        engine = harness.import_reference()
        from waveforcing_b200.denoiser.exchange import paged
        from waveforcing_b200.denoiser.exchange.paged import PagedExchangeMixin as WfPaged

        log = []
        paged.ipc = ShmIPC(log)
        paged.kernels.kv_assemble = emulate_assemble

        class SwappedDenoiser(WfPaged, engine.WaveDenoiser):
            pass

        a = _run(engine, rank, "sync", engine.WaveDenoiser, log)
        b = _run(engine, rank, "paged", SwappedDenoiser, log)
        res = dict(n_calls=(len(a["calls"]), len(b["calls"])), mismatch=[], page_mismatch=[],
                   page_shapes=sorted({(k, tuple(t.shape)) for _, _, d in b["pages"] for k, t in d.items()}),
                   n_pages=(len(a["pages"]), len(b["pages"])), final=sorted(b["final"]),
                   final_equal=all(torch.equal(a["final"][c], b["final"][c]) for c in a["final"])
                   and sorted(a["final"]) == sorted(b["final"]),
                   opened=b["opened"], left=b["left"], log=log)
        for (ta, la, ka, va), (tb, lb, kb, vb) in zip(a["calls"], b["calls"]):
            if (ta, la) != (tb, lb) or ka.shape != kb.shape or not (torch.equal(ka, kb) and torch.equal(va, vb)):
                res["mismatch"].append((ta, la, tuple(ka.shape), tuple(kb.shape)))
        for pa, pb in zip(a["pages"], b["pages"]):
            if pa[0] != pb[0] or pa[1] != pb[1] or any(not torch.equal(pa[2][k], pb[2][k]) for k in pa[2]):
                res["page_mismatch"].append((pa[0], pa[1], pb[1]))
        q.put((rank, res))
    except Exception as e:  # report instead of hanging the parent
        import traceback

        q.put((rank, {"error": repr(e), "tb": traceback.format_exc()}))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_paged_mixin_drops_into_reference_waveDenoiser():
    world = RF_STEP + 1
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in procs:
            r, out = q.get(timeout=240)
            res[r] = out
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert "error" not in res[r], res[r].get("tb")
    for r in range(world):
        out = res[r]
        assert out["n_calls"][0] == out["n_calls"][1] > 0, (r, out["n_calls"])
        assert out["mismatch"] == [], (r, out["mismatch"][:4])
        assert out["n_pages"][0] == out["n_pages"][1] > 0
        assert out["page_mismatch"] == [], (r, out["page_mismatch"][:4])
        # clean pages are [1, T, H, D]: anchor (ku, v) then promoted (kr, v)
        assert {s for _, s in out["page_shapes"]} == {(1, T, H, D)}
        assert out["final_equal"]
        # every mapping opened through the engine's _ipc_open was closed, in reverse order
        opens = [p for op, p in out["log"] if op == "open"]
        closes = [p for op, p in out["log"] if op == "close"]
        assert opens == out["opened"] and closes == list(reversed(opens)) and out["left"] == []
    assert res[RF_STEP]["final"] == list(range(NUM_FRAMES // NPB))  # the store finished every chunk
    assert res[RF_STEP]["opened"]  # the store publishes into both denoise ranks' slabs
