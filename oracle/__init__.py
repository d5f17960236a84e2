"""CPU oracle for the WaveRT per-layer DiT hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``waveforcing_b200`` imports this
package; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` use it, and only as the checker (or, for the baseline,
as the timed CPU restatement of the reference's torch path).

Every function cites the reference file:line whose arithmetic it restates
(paths are relative to the SJTU-DENG-Lab/WaveForcing project root).

Parity pins:
  * ``codec``   -- pinned against golden vectors produced by running the
    reference's own ``CommonExchangeMixin._all_gather_fp8`` and torch's
    e4m3 cast (tests/golden/make_golden.py) and exhaustively over all
    65536 bf16 bit patterns.
  * ``w8a8``    -- pinned against the reference's ``WaveFp8Linear`` run on
    CPU through ``torch._scaled_mm`` (tests/golden/make_golden.py).
  * ``attention`` / ``rope`` / ``geometry`` -- the reference's attention
    and RoPE live in un-vendored SGLang; parity is anchored on the
    vendored naive model (naive_rt/rolling_forcing/wan/modules) and on
    the reference's own call sites.  The attention restatement is
    cross-checked against torch's CPU SDPA, the very call the reference
    falls back to (naive_rt/rolling_forcing/wan/modules/attention.py:75-89).
"""
