"""Model check of the W8A8 GEMM kernel's synchronisation protocol (CPU).

`waveforcing_b200/csrc/gemm_w8a8.cu` is persistent and has three roles:
* a TMA producer, which fills a ring of NS k-block slots;
* one MMA-issuing thread, with two TMEM accumulators;
* four epilogue warps, which:
  * read an accumulator and hand it back;
  * scale each 64-column group into one of two shared-memory staging buffers;
  * store the group with TMA, one thread issuing, behind a named barrier.

This test transcribes each role's waits, arrivals, loads, MMA issues, commits
and bulk-store waits with the kernel's phase formulas.  It runs the roles
under random interleavings:
* TMA loads land in any order;
* the tensor pipe executes in issue order;
* TMA stores finish reading their staging buffer at random later times.

It checks:
* no deadlock;
* no ring slot is overwritten before its MMA has executed;
* no accumulator is read before its tile is complete, or overwritten before
  the epilogue read it;
* no staging buffer is rewritten while a store still reads it.

The transcription must follow any change to the kernel's protocol."""
import random

import pytest

from test_attn_protocol import Bar

NS = 4          # k-block ring depth
GROUPS = 4      # 64-column output groups per 256-column tile


class NamedBarrier:
    def __init__(self, n):
        self.n, self.count, self.gen = n, 0, 0

    def arrive(self):
        self.count += 1
        if self.count == self.n:
            self.count = 0
            self.gen += 1


class GemmSim:
    store_wait = True  # the issuing thread waits for earlier stores' reads before the named barrier

    def __init__(self, tiles, nk, seed, epi_warps=4):
        self.rnd = random.Random(seed)
        self.tiles, self.nk, self.E = tiles, nk, epi_warps
        self.b = {f"full{s}": Bar(1) for s in range(NS)}
        self.b.update({f"empty{s}": Bar(1) for s in range(NS)})
        self.b.update({"acc_full0": Bar(1), "acc_full1": Bar(1), "acc_empty0": Bar(epi_warps),
                       "acc_empty1": Bar(epi_warps), "fin": Bar(1)})
        self.named = NamedBarrier(epi_warps)
        self.slot = {}            # ring slot -> (tile, k-block)
        self.slot_reads = {}      # ring slot -> pending MMAs reading it
        self.acc = [None, None]   # accumulator -> (tile, k-blocks accumulated)
        self.acc_pending = [0, 0]
        self.acc_read = [set(), set()]  # epilogue warps that have read the accumulator's current tile
        self.staging = [None, None]
        self.store_reads = []     # staging buffers read by stores in flight
        self.tma, self.pipe = [], []

    def wait(self, bar, parity):
        while not self.b[bar].done(parity):
            yield

    def producer(self):
        it = 0
        for t in range(self.tiles):
            for kb in range(self.nk):
                s = it % NS
                if it >= NS:
                    yield from self.wait(f"empty{s}", ((it // NS) - 1) & 1)
                self.b[f"full{s}"].arrive(expect_tx=2)
                self.tma += [(s, (t, kb)), (s, (t, kb))]
                it += 1
                yield

    def mma(self):
        it = 0
        for local in range(self.tiles):
            buf = local & 1
            if local >= 2:
                yield from self.wait(f"acc_empty{buf}", ((local >> 1) - 1) & 1)
            for kb in range(self.nk):
                s = it % NS
                yield from self.wait(f"full{s}", (it // NS) & 1)
                self.slot_reads[s] = self.slot_reads.get(s, 0) + 1
                self.acc_pending[buf] += 1
                self.pipe.append(("mma", s, (local, kb), buf))
                self.pipe.append(("commit", f"empty{s}"))
                it += 1
                yield
            self.pipe.append(("commit", f"acc_full{buf}"))
        self.pipe.append(("commit", "fin"))
        yield from self.wait("fin", 0)

    def epilogue(self, w):
        grp = 0
        for local in range(self.tiles):
            buf = local & 1
            yield from self.wait(f"acc_full{buf}", (local >> 1) & 1)
            gen = self.named.gen
            self.named.arrive()
            while self.named.gen == gen:
                yield
            for g in range(GROUPS):
                assert self.acc[buf] == (local, self.nk) and not self.acc_pending[buf], \
                    f"epilogue read accumulator {buf}={self.acc[buf]} for tile {local}"
                if g == GROUPS - 1:
                    self.acc_read[buf].add(w)
                    self.b[f"acc_empty{buf}"].arrive()
                yield
                sb = grp & 1
                assert sb not in self.store_reads, f"staging buffer {sb} rewritten while a store reads it"
                self.staging[sb] = (local, g)
                yield
                if w == 0 and self.store_wait:
                    while self.store_reads:  # cp.async.bulk.wait_group.read 0
                        yield
                gen = self.named.gen
                self.named.arrive()
                while self.named.gen == gen:
                    yield
                if w == 0:
                    assert self.staging[sb] == (local, g)
                    self.store_reads.append(sb)
                grp += 1

    def run(self):
        agents = [self.producer(), self.mma()] + [self.epilogue(w) for w in range(self.E)]
        alive = list(range(len(agents)))
        idle = 0
        while alive:
            r = self.rnd.random()
            if self.tma and r < 0.2:
                s, tag = self.tma.pop(self.rnd.randrange(len(self.tma)))
                assert not self.slot_reads.get(s), f"TMA overwrote ring slot {s} before its MMA ran"
                self.slot[s] = tag
                self.b[f"full{s}"].complete_tx(1)
                idle = 0
            elif self.pipe and r < 0.4:
                op = self.pipe.pop(0)
                if op[0] == "commit":
                    self.b[op[1]].arrive()
                else:
                    _, s, (local, kb), buf = op
                    assert self.slot.get(s) == (local, kb), f"MMA read slot {s}={self.slot.get(s)}"
                    self.slot_reads[s] -= 1
                    if kb == 0:
                        assert self.acc[buf] is None or len(self.acc_read[buf]) == self.E, \
                            f"accumulator {buf} overwritten before the epilogue drained it"
                        self.acc_read[buf] = set()
                    else:
                        assert self.acc[buf] == (local, kb)
                    self.acc[buf] = (local, kb + 1)
                    self.acc_pending[buf] -= 1
                idle = 0
            elif self.store_reads and r < 0.5:
                self.store_reads.pop(0)
                idle = 0
            else:
                i = self.rnd.choice(alive)
                try:
                    next(agents[i])
                except StopIteration:
                    alive.remove(i)
                idle += 1
            assert idle < 100000, "deadlock: no role can make progress"
        assert not self.tma and not self.pipe


@pytest.mark.parametrize("tiles,nk", [(1, 1), (1, 6), (3, 2), (5, 5), (6, 1)])
def test_gemm_protocol_random_interleavings(tiles, nk):
    for seed in range(60):
        GemmSim(tiles, nk, seed * 1000 + tiles * 10 + nk).run()


def test_model_detects_a_missing_store_wait():
    """Without the wait for in-flight stores before the named barrier, a
    staging buffer can be rewritten while a store still reads it."""

    class NoWait(GemmSim):
        store_wait = False

    with pytest.raises(AssertionError, match="staging buffer"):
        for seed in range(200):
            NoWait(4, 2, seed).run()


def test_model_detects_a_missing_accumulator_handback():
    """Without the MMA thread's acc_empty wait, an accumulator is reused before
    the epilogue has read it."""

    class NoHandback(GemmSim):
        def wait(self, bar, parity):
            if bar.startswith("acc_empty"):
                return iter(())
            return super().wait(bar, parity)

    with pytest.raises(AssertionError, match="accumulator"):
        for seed in range(200):
            NoHandback(5, 2, seed).run()
