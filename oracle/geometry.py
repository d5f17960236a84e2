"""Wavefront activity and paged-slot geometry restated in plain Python
(test infrastructure only).

Sources:
  * rank activity         -- wave_rt/denoiser/engine.py:214-219, 303-311
  * ticks                 -- wave_rt/denoiser/engine.py:53
  * paged slab sizing     -- wave_rt/denoiser/exchange/paged.py:26-30
  * denoise slot geometry -- wave_rt/denoiser/exchange/paged.py:160-189
  * store slot geometry   -- wave_rt/denoiser/exchange/paged.py:257-265
  * anchor/working window -- wave_rt/denoiser/exchange/common.py:70-91
  * clean-page retention  -- wave_rt/denoiser/exchange/common.py:110-114
"""

from __future__ import annotations

from dataclasses import dataclass, field


def act_denoise(n: int, t: int, rf_step: int, num_blocks: int) -> bool:
    c = t - n
    return (0 <= n < rf_step) and (0 <= c < num_blocks)


def act_store(t: int, store_rank: int, num_blocks: int) -> bool:
    return 0 <= (t - store_rank) < num_blocks


def num_ticks(num_blocks: int, world: int) -> int:
    return num_blocks + world - 1


def paged_slab(max_attn_frames: int, rf_step: int, npb: int):
    """paged.py:26-30 -> (naw_max, Wmax)."""
    wmax_frames = max_attn_frames - rf_step * npb - npb
    wmax_chunks = max(0, wmax_frames // npb)
    naw = 1 + wmax_chunks
    return naw, naw + 1 + rf_step


@dataclass
class DenoiseGeom:
    clean_len: int
    wmax_chunks: int
    naw: int
    live: int
    base_infl: int
    infl_ranks: list
    active_slots: int
    self_off: int
    live_off: int
    active_len: int
    recv_srcs: list
    send_slots: list = field(default_factory=list)


def denoise_geometry(r, tick, act_ranks, store_active, rf_step, max_attn_frames, npb, T):
    """paged.py:160-189 for denoise rank ``r`` at ``tick``."""
    store_rank = rf_step
    clean_len = min(8, max(0, tick - store_rank))
    wmax_chunks = max(0, (max_attn_frames - len(act_ranks) * npb - npb) // npb)
    naw = 0 if clean_len == 0 else 1 + min(wmax_chunks, clean_len - 1)
    live = 1 if store_active else 0
    base_infl = naw + live
    infl_ranks = [n for n in act_ranks if n >= r]
    active_slots = base_infl + len(infl_ranks)
    recv_srcs = [n for n in act_ranks if n > r] + ([store_rank] if store_active else [])
    send_slots = []
    for m in act_ranks:
        if m >= r:
            continue
        idx = sum(1 for n in act_ranks if m <= n < r)
        send_slots.append((m, base_infl + idx))
    return DenoiseGeom(
        clean_len, wmax_chunks, naw, live, base_infl, infl_ranks, active_slots,
        base_infl * T, naw * T, active_slots * T, recv_srcs, send_slots,
    )


def store_geometry(tick, act_ranks, rf_step, max_attn_frames, npb):
    """paged.py:257-265 -> (naw, send_slots)."""
    store_rank = rf_step
    clean_len = min(8, max(0, tick - store_rank))
    wmax_chunks = max(0, (max_attn_frames - len(act_ranks) * npb - npb) // npb)
    naw = 0 if clean_len == 0 else 1 + min(wmax_chunks, clean_len - 1)
    return naw, [(m, naw) for m in act_ranks]


def anchor_working(clean_ids: list, csf: int, qf: int, max_attn_frames: int, npb: int):
    """common.py:70-91 -> (anchor id, working ids, rope_start frame)."""
    if not clean_ids:
        return None, [], None
    wmax_frames = max_attn_frames - qf - npb
    wmax_chunks = max(0, wmax_frames // npb)
    anchor, rest = clean_ids[0], clean_ids[1:]
    working = rest[-wmax_chunks:] if wmax_chunks > 0 else []
    rope_start = csf - len(working) * npb - npb
    return anchor, working, rope_start


def append_clean_page(clean: list, page) -> None:
    """common.py:110-114: keep the anchor and the 7 newest pages."""
    clean.append(page)
    if len(clean) > 8:
        clean[:] = clean[:1] + clean[-7:]


def tick_roles(t, rf_step, num_blocks, npb):
    """engine.py:303-311 -> (act_ranks, tick_csf, tick_qf, store_active)."""
    act = [n for n in range(rf_step) if act_denoise(n, t, rf_step, num_blocks)]
    oldest_c = (t - max(act)) if act else 0
    return act, oldest_c * npb, len(act) * npb, act_store(t, rf_step, num_blocks)
