"""Latent migration point to point, and the slab-generation credits that
replace the reference's per-tick all_gather as the reuse guard.

The reference hands every denoise stage's result to the next stage with a
world ``all_gather`` per tick (wave_rt/denoiser/engine.py:516-555); the same
collective keeps every rank within a tick of the others, so a producer never
overwrites slab generation ``tick % 2`` while a consumer still reads it.
``WavefrontEngine._migrate`` sends each result only from the rank that made it
to the rank of the next stage, and ``PagedTransport.acquire_slots`` /
``release_slots`` carry the reuse guard as device-side credit words (here
shared-memory words on gloo ranks, the CPU stand-in for CUDA IPC).
"""

import ctypes
import os
import socket
import time
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from waveforcing_b200.denoiser.exchange import paged
from waveforcing_b200.wavefront import engine as E

STEPS = (1000, 750, 500)  # stages 0, 1, 2 and the store (3)
NUM_FRAMES = 3 * 6


class ShmIPC:
    """CUDA IPC stand-in: exported tensors live in shared memory, device
    writes are stores into it, flag waits poll it."""

    def ipc_export(self, t):
        t.share_memory_()
        return t.untyped_storage()._share_filename_cpu_(), t.storage_offset() * t.element_size()

    def ipc_open_handle(self, h):
        st = torch.UntypedStorage._new_shared_filename_cpu(*h)
        self.keep = getattr(self, "keep", []) + [st]
        return st.data_ptr()

    def ipc_close_handle(self, ptr):
        pass

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


def _gather_semantics(stage_rank, S, nb, t):
    """What the all_gather form delivers after tick t: stage -> source rank for
    every stage s >= 1 that is active at t + 1 (engine.py:516-555)."""
    out = {}
    for s in range(1, S + 1):
        nxt = (0 <= t + 1 - s < nb) if s < S else (0 <= t + 1 - S < nb)
        if nxt:
            out[s] = stage_rank[s - 1]
    return out


@pytest.mark.parametrize("S", [4, 5])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 6, 8])
def test_migration_plan_matches_the_gather(S, world):
    stage_rank = E.place_stages(S, world)
    nb = 12
    for t in range(nb + S):
        plan = E.migration_plan(stage_rank, S, nb, t)
        assert {d: src for d, src, _ in plan} == _gather_semantics(stage_rank, S, nb, t)
        assert all(dst == stage_rank[d] for d, _, dst in plan)


def _model():
    return SimpleNamespace(cfg=SimpleNamespace(layers=2, tokens_per_chunk=4, heads=1, head_dim=8, in_ch=2,
                                               lat_h=2, lat_w=2))


def _result(s, t, shape):
    g = torch.Generator().manual_seed(100 * t + s)
    return torch.randn(shape, generator=g).to(torch.bfloat16)


def _worker(rank, world, port, q, delay_release):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    paged.ipc = ShmIPC()
    try:
        cfg = E.EngineConfig(steps=STEPS, num_frames=NUM_FRAMES, timeout_s=10.0)
        eng = E.WavefrontEngine(_model(), cfg, rank=rank, world=world, device="cpu")
        S, nb = eng.S, cfg.num_blocks
        shape = eng.mig_shape[1:]
        got, waited = {}, {}
        for t in range(eng.num_ticks):
            t0 = time.monotonic()
            eng.xport.acquire_slots(t)
            waited[t] = time.monotonic() - t0
            out = {s: _result(s, t, shape) for s in eng.local if s < S and eng.act_denoise(s, t)}
            if delay_release and t == 1 and 0 in eng.local:
                time.sleep(1.0)  # a slow consumer: its producers' tick 3 must wait for this
            eng.xport.release_slots(t)
            if delay_release:
                continue  # the credits alone (migration would pass the delay down the chain)
            eng.inputs.clear()
            eng._migrate(t, out)
            for s, x in eng.inputs.items():
                # numpy, not tensors: a queued tensor's shared storage dies with its sender
                got[(t, s)] = x.float().numpy().copy()
        q.put((rank, eng.local, got, waited, int(eng.xport.timeout_word.item()),
               eng.xport.remote_consumers(), eng.stage_rank))
        eng.close()
    except Exception as e:
        q.put((rank, repr(e), None, None, -1, None, None))
    finally:
        dist.destroy_process_group()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(world, delay_release=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, delay_release)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        r = q.get(timeout=180)
        res[r[0]] = r[1:]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


@pytest.mark.parametrize("world", [2, 3])
def test_p2p_migration_delivers_every_hand_off(world):
    res = _run(world)
    for r, (local, got, _w, tw, _rc, _sr) in res.items():
        assert not isinstance(local, str), local
        assert tw == 0, f"rank {r}: a credit wait timed out"
    stage_rank = res[0][5]
    S = len(STEPS)
    nb = NUM_FRAMES // 3
    # reference results for the receiving side: the producer's x0, re-noised
    # to the next step except into the store (engine.py:221-235)
    ref_eng = E.WavefrontEngine.__new__(E.WavefrontEngine)
    ref_eng.device = torch.device("cpu")
    ref_eng.cfg = E.EngineConfig(steps=STEPS, num_frames=NUM_FRAMES)
    ref_eng.fm = E.FlowMatch()
    shape = (2, 3, 2, 2)
    n_checked = 0
    for t in range(nb + S):
        for d, _src, dst in E.migration_plan(stage_rank, S, nb, t):
            s = d - 1
            x0 = _result(s, t, shape)
            want = ref_eng._renoise(x0, s, t - s) if s < S - 1 else x0
            got = torch.from_numpy(res[dst][1][(t, d)])
            assert torch.equal(got, want.float()), (t, d)
            n_checked += 1
        # nothing else arrived anywhere
        arrived = sum(1 for r in res for (tt, _d) in res[r][1] if tt == t)
        assert arrived == len(E.migration_plan(stage_rank, S, nb, t))
    assert n_checked > 0


def test_slot_credit_holds_a_producer_until_the_consumer_is_done():
    """3 ranks: the stage-0 rank (a consumer of every other stage) releases
    tick 1 a second late; a producer publishing to it may not start tick 3
    (which rewrites tick 1's slab generation) before that release."""
    res = _run(3, delay_release=True)
    for r, (local, _got, waited, tw, rc, _sr) in res.items():
        assert not isinstance(local, str), local
        assert tw == 0
        if rc:  # this rank publishes to a consumer elsewhere
            assert waited[3] > 0.5, (r, waited)
        assert all(w < 0.5 for t, w in waited.items() if t != 3), (r, waited)
    assert any(rc for _l, _g, _w, _t, rc, _s in res.values())
