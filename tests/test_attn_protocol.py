"""Model check of the attention kernel's synchronisation protocol (CPU).

`waveforcing_b200/csrc/attn_fwd.cu` coordinates four roles through mbarriers
with parity waits:
* a TMA producer;
* one MMA-issuing thread;
* two softmax warpgroups.

A parity wait is only correct while the waiter is at most one phase behind.
This test transcribes each role's sequence of waits, arrivals, TMA loads, MMA
issues and commits, in the kernel's order and with the kernel's phase
formulas.  It runs the roles under many random interleavings:
* TMA copies land independently, in random order;
* the tensor pipe executes MMAs and commits in issue order.

Every run must finish without deadlock.  Every data access must see the tile
it expects:
* Q, K and V slots are not overwritten before the MMAs that read them have
  executed;
* S is not overwritten before both warpgroups have read it;
* P is not overwritten before PV has read it;
* O is not read or rescaled while a PV is pending;
* the row-max and row-sum exchanges read the partner's value of the same
  exchange.

The transcription must follow any change to the kernel's protocol."""
import random

import pytest

NSK = 2  # K ring depth (256-key tiles)


class Bar:
    """mbarrier: `count` arrivals plus transaction bytes complete a phase."""

    def __init__(self, count):
        self.count, self.pend, self.tx, self.phase = count, count, 0, 0

    def _maybe_complete(self):
        if self.pend == 0 and self.tx == 0:
            self.phase += 1
            self.pend = self.count

    def arrive(self, expect_tx=0):
        assert self.pend > 0
        self.pend -= 1
        self.tx += expect_tx
        self._maybe_complete()

    def complete_tx(self, n):
        self.tx -= n
        self._maybe_complete()

    def done(self, parity):  # mbarrier.try_wait.parity
        return (self.phase & 1) != parity


class Sim:
    early_sfree = False  # the kernel releases S only after the row-max exchange

    def __init__(self, nk, n_items, seed, warps_per_wg=2):
        self.rnd = random.Random(seed)
        self.nk, self.n_items, self.W = nk, n_items, warps_per_wg
        n_soft = 2 * warps_per_wg
        self.b = {
            "q": Bar(1), "s": Bar(1), "sfree": Bar(n_soft), "p": Bar(n_soft), "pv": Bar(1), "xch": Bar(n_soft),
            "last": Bar(1), "q_empty": Bar(1), "o_free": Bar(n_soft), "fin": Bar(1),
        }
        for s in range(NSK):
            self.b[f"full_k{s}"], self.b[f"empty_k{s}"] = Bar(1), Bar(1)
        for h in range(2):
            self.b[f"full_v{h}"], self.b[f"empty_v{h}"] = Bar(1), Bar(1)
        self.smem = {}       # buffer -> tag of the tile it holds
        self.reads = {}      # buffer -> MMAs issued but not yet executed that read it
        self.tmem = {"S": None, "O": None, "P0": {}, "P1": {}}
        self.pending_pv = 0
        self.xch = {}        # (wg, warp) -> exchange index of the value written
        self.tma = []        # in-flight copies: (buffer, tag, barrier, bytes)
        self.pipe = []       # tensor pipe, in issue order

    # ------------------------------------------------------------ TMA
    def load(self, buf, tag, bar, nbytes):
        self.tma.append((buf, tag, bar, nbytes))

    def land(self, i):
        buf, tag, bar, nbytes = self.tma.pop(i)
        assert not self.reads.get(buf), f"TMA overwrote {buf} while an MMA still reads it"
        self.smem[buf] = tag
        self.b[bar].complete_tx(nbytes)

    # ------------------------------------------------------------ MMA
    def issue(self, op, **kw):
        for buf in kw.get("bufs", ()):
            self.reads[buf] = self.reads.get(buf, 0) + 1
        if op == "PV":
            self.pending_pv += 1
        self.pipe.append((op, kw))

    def execute(self):
        op, kw = self.pipe.pop(0)
        if op == "commit":
            self.b[kw["bar"]].arrive()
            return
        for buf, want in zip(kw["bufs"], kw["want"]):
            assert self.smem.get(buf) == want, f"{op} read {buf}={self.smem.get(buf)}, expected {want}"
            self.reads[buf] -= 1
        if op == "QK":
            self.tmem["S"] = kw["tag"]
        else:  # PV over one 128-key half: P half and V slot half
            h, tag = kw["half"], kw["tag"]
            p = self.tmem[f"P{h}"]
            assert all(p.get(w) == tag for w in range(self.W)), f"PV read P{h}={p}, expected {tag}"
            item, j = tag
            done = 2 * j + h  # PV halves this item has accumulated into O so far
            if done > 0:
                assert self.tmem["O"] == (item, done), ("O accumulation order", self.tmem["O"], (item, done))
            self.tmem["O"] = (item, done + 1)  # the item's first PV overwrites O
            self.pending_pv -= 1

    def commit(self, bar):
        self.pipe.append(("commit", {"bar": bar}))

    # ---------------------------------------------------------- roles
    def wait(self, bar, parity):
        while not self.b[bar].done(parity):
            yield

    def producer(self):
        kt = vt = 0
        nk = self.nk

        def load_k(item, j):
            nonlocal kt
            s = kt % NSK
            if kt >= NSK:
                yield from self.wait(f"empty_k{s}", ((kt // NSK) - 1) & 1)
            self.b[f"full_k{s}"].arrive(expect_tx=4)
            for part in range(4):
                self.load(f"K{s}.{part}", (item, j), f"full_k{s}", 1)
            kt += 1

        for n_it in range(self.n_items):
            if n_it > 0:
                yield from self.wait("q_empty", (n_it - 1) & 1)
            self.b["q"].arrive(expect_tx=2)
            for part in range(2):
                self.load(f"Q.{part}", n_it, "q", 1)
            yield
            yield from load_k(n_it, 0)
            for j in range(nk):
                if j + 1 < nk:
                    yield from load_k(n_it, j + 1)
                for half in range(2):
                    if vt >= 1:
                        yield from self.wait(f"empty_v{half}", (vt - 1) & 1)
                    self.b[f"full_v{half}"].arrive(expect_tx=2)
                    for part in range(2):
                        self.load(f"V{half}.{part}", (n_it, j, half), f"full_v{half}", 1)
                    yield
                vt += 1

    def mma(self):
        kt = st = 0
        nk = self.nk
        for n_it in range(self.n_items):
            yield from self.wait("q", n_it & 1)
            for j in range(nk + 1):
                if j < nk:
                    s = kt % NSK
                    yield from self.wait(f"full_k{s}", (kt // NSK) & 1)
                    if st + j >= 1:
                        yield from self.wait("sfree", (st + j - 1) & 1)
                    bufs = ["Q.0", "Q.1"] + [f"K{s}.{p}" for p in range(4)]
                    self.issue("QK", bufs=bufs, want=[n_it] * 2 + [(n_it, j)] * 4, tag=(n_it, j))
                    self.commit(f"empty_k{s}")
                    self.commit("s")
                    if j == nk - 1:
                        self.commit("q_empty")
                    kt += 1
                if j >= 1:
                    g = st + j - 1
                    yield from self.wait("p", g & 1)
                    if j == 1 and n_it > 0:
                        yield from self.wait("o_free", (n_it - 1) & 1)
                    for half in range(2):
                        yield from self.wait(f"full_v{half}", g & 1)
                        bufs = [f"V{half}.{p}" for p in range(2)]
                        self.issue("PV", bufs=bufs, want=[(n_it, j - 1, half)] * 2, half=half, tag=(n_it, j - 1))
                        self.commit(f"empty_v{half}")
                    self.commit("pv")
                yield
            st += nk
            self.commit("last")
        self.commit("fin")
        yield from self.wait("fin", 0)

    def softmax(self, wg, w):
        st = xc = 0
        nk = self.nk
        for n_it in range(self.n_items):
            for j in range(nk):
                yield from self.wait("s", st & 1)
                assert self.tmem["S"] == (n_it, j), f"softmax read S={self.tmem['S']}, expected {(n_it, j)}"
                yield
                if self.early_sfree:
                    self.b["sfree"].arrive()
                self.xch[(wg, w)] = xc
                self.b["xch"].arrive()
                yield from self.wait("xch", xc & 1)
                assert self.xch.get((wg ^ 1, w)) == xc, "row-max exchange read a stale value"
                if not self.early_sfree:
                    self.b["sfree"].arrive()
                yield
                if j > 0:
                    yield from self.wait("pv", (st - 1) & 1)
                assert self.pending_pv == 0, "O rescaled or P written while a PV is pending"
                self.tmem[f"P{wg}"][w] = (n_it, j)
                yield
                self.b["p"].arrive()
                st += 1
                xc += 1
            yield from self.wait("last", n_it & 1)
            assert self.pending_pv == 0
            self.tmem[f"P{wg}"][w] = ("l", n_it)
            self.b["xch"].arrive()
            yield from self.wait("xch", xc & 1)
            xc += 1
            assert self.tmem[f"P{wg ^ 1}"].get(w) == ("l", n_it), "row-sum exchange read a stale value"
            assert self.tmem["O"] == (n_it, 2 * nk) and self.pending_pv == 0, "epilogue read an unfinished O"
            yield
            self.b["o_free"].arrive()

    def run(self):
        agents = [self.producer(), self.mma()] + [self.softmax(wg, w) for wg in range(2) for w in range(self.W)]
        alive = list(range(len(agents)))
        idle = 0
        while alive:
            r = self.rnd.random()
            if self.tma and r < 0.25:
                self.land(self.rnd.randrange(len(self.tma)))
                idle = 0
            elif self.pipe and r < 0.5:
                self.execute()
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


@pytest.mark.parametrize("nk,n_items", [(1, 1), (1, 3), (2, 1), (2, 4), (3, 3), (5, 2)])
def test_attention_protocol_random_interleavings(nk, n_items):
    for seed in range(60):
        Sim(nk, n_items, seed * 1000 + nk * 10 + n_items).run()


def test_model_detects_a_parity_error():
    """A wrong phase formula must trip the model: here the softmax waits for
    PV_{j-1} with the parity of PV_{j-2}."""

    class Broken(Sim):
        def wait(self, bar, parity):
            if bar == "pv":
                parity ^= 1
            yield from super().wait(bar, parity)

    with pytest.raises(AssertionError):
        for seed in range(60):
            Broken(3, 2, seed).run()


def test_model_detects_the_exchange_race():
    """Releasing S before the row-max exchange lets a warpgroup reach the next
    tile's exchange while its partner has not read this one.  With one slot
    and one barrier for the exchange, the model must catch the race."""

    class Early(Sim):
        early_sfree = True

    with pytest.raises(AssertionError):
        for seed in range(200):
            Early(4, 2, seed).run()


class SimFP8(Sim):
    """The FP8 K/V variant (attn_fwd_e4m3_kernel): TMA lands raw tiles (Q in
    bf16, K/V as e4m3 codes in the upper half of their slots) on q_raw /
    raw_k / raw_v; two converter warps, each owning half of every tile's rows,
    rewrite the tiles in place as f16 and arrive on the operand barriers the
    MMA waits on (q, full_k, full_v; two arrivals per phase here, one per
    converter warp).  A raw tile aliases the converted tile of its slot: a
    copy that lands while an MMA still reads the slot, or a conversion that
    writes it then, is a race."""

    def __init__(self, nk, n_items, seed, warps_per_wg=2):
        super().__init__(nk, n_items, seed, warps_per_wg)
        self.b["q"] = Bar(2)
        self.b["q_raw"] = Bar(1)
        for s in range(NSK):
            self.b[f"full_k{s}"], self.b[f"raw_k{s}"] = Bar(2), Bar(1)
        for h in range(2):
            self.b[f"full_v{h}"], self.b[f"raw_v{h}"] = Bar(2), Bar(1)

    def land(self, i):
        buf, tag, bar, nbytes = self.tma.pop(i)
        alias = buf.replace(".raw", ".")
        assert not self.reads.get(alias), f"TMA overwrote {alias} while an MMA still reads it"
        self.smem[buf] = tag
        self.smem[alias] = "clobbered"
        self.b[bar].complete_tx(nbytes)

    def producer(self):
        kt = vt = 0
        nk = self.nk

        def load_k(item, j):
            nonlocal kt
            s = kt % NSK
            if kt >= NSK:
                yield from self.wait(f"empty_k{s}", ((kt // NSK) - 1) & 1)
            self.b[f"raw_k{s}"].arrive(expect_tx=2)
            for w in range(2):
                self.load(f"K{s}.raw{w}", ("raw", (item, j)), f"raw_k{s}", 1)
            kt += 1

        for n_it in range(self.n_items):
            if n_it > 0:
                yield from self.wait("q_empty", (n_it - 1) & 1)
            self.b["q_raw"].arrive(expect_tx=2)
            for w in range(2):
                self.load(f"Q.raw{w}", ("raw", n_it), "q_raw", 1)
            yield
            yield from load_k(n_it, 0)
            for j in range(nk):
                if j + 1 < nk:
                    yield from load_k(n_it, j + 1)
                for half in range(2):
                    if vt >= 1:
                        yield from self.wait(f"empty_v{half}", (vt - 1) & 1)
                    self.b[f"raw_v{half}"].arrive(expect_tx=2)
                    for w in range(2):
                        self.load(f"V{half}.raw{w}", ("raw", (n_it, j, half)), f"raw_v{half}", 1)
                    yield
                vt += 1

    def _convert(self, raw, out, tag):
        assert self.smem.get(raw) == ("raw", tag), f"converter read {raw}={self.smem.get(raw)}, expected raw {tag}"
        assert not self.reads.get(out), f"converter overwrote {out} while an MMA still reads it"
        self.smem[out] = ("f16", tag)
        self.smem[raw] = None

    def converter(self, w):
        kt = vt = 0
        nk = self.nk

        def conv_k(item, j):
            nonlocal kt
            s = kt % NSK
            yield from self.wait(f"raw_k{s}", (kt // NSK) & 1)
            yield
            self._convert(f"K{s}.raw{w}", f"K{s}.{w}", (item, j))
            self.b[f"full_k{s}"].arrive()
            kt += 1

        for n_it in range(self.n_items):
            yield from self.wait("q_raw", n_it & 1)
            yield
            self._convert(f"Q.raw{w}", f"Q.{w}", n_it)
            self.b["q"].arrive()
            yield from conv_k(n_it, 0)
            for j in range(nk):
                if j + 1 < nk:
                    yield from conv_k(n_it, j + 1)
                for half in range(2):
                    yield from self.wait(f"raw_v{half}", vt & 1)
                    yield
                    self._convert(f"V{half}.raw{w}", f"V{half}.{w}", (n_it, j, half))
                    self.b[f"full_v{half}"].arrive()
                vt += 1

    def mma(self):
        kt = st = 0
        nk = self.nk
        for n_it in range(self.n_items):
            yield from self.wait("q", n_it & 1)
            for j in range(nk + 1):
                if j < nk:
                    s = kt % NSK
                    yield from self.wait(f"full_k{s}", (kt // NSK) & 1)
                    if st + j >= 1:
                        yield from self.wait("sfree", (st + j - 1) & 1)
                    bufs = ["Q.0", "Q.1", f"K{s}.0", f"K{s}.1"]
                    self.issue("QK", bufs=bufs, want=[("f16", n_it)] * 2 + [("f16", (n_it, j))] * 2, tag=(n_it, j))
                    self.commit(f"empty_k{s}")
                    self.commit("s")
                    if j == nk - 1:
                        self.commit("q_empty")
                    kt += 1
                if j >= 1:
                    g = st + j - 1
                    yield from self.wait("p", g & 1)
                    if j == 1 and n_it > 0:
                        yield from self.wait("o_free", (n_it - 1) & 1)
                    for half in range(2):
                        yield from self.wait(f"full_v{half}", g & 1)
                        bufs = [f"V{half}.0", f"V{half}.1"]
                        self.issue("PV", bufs=bufs, want=[("f16", (n_it, j - 1, half))] * 2, half=half,
                                   tag=(n_it, j - 1))
                        self.commit(f"empty_v{half}")
                    self.commit("pv")
                yield
            st += nk
            self.commit("last")
        self.commit("fin")
        yield from self.wait("fin", 0)

    def run(self):
        agents = ([self.producer(), self.mma(), self.converter(0), self.converter(1)]
                  + [self.softmax(wg, w) for wg in range(2) for w in range(self.W)])
        alive = list(range(len(agents)))
        idle = 0
        while alive:
            r = self.rnd.random()
            if self.tma and r < 0.25:
                self.land(self.rnd.randrange(len(self.tma)))
                idle = 0
            elif self.pipe and r < 0.5:
                self.execute()
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


@pytest.mark.parametrize("nk,n_items", [(1, 1), (1, 3), (2, 1), (2, 4), (3, 3), (5, 2)])
def test_fp8_attention_protocol_random_interleavings(nk, n_items):
    for seed in range(60):
        SimFP8(nk, n_items, seed * 1000 + nk * 10 + n_items + 7).run()


def test_fp8_model_detects_early_operand_release():
    """Arriving on the operand barrier before the conversion is written must
    trip the model (the MMA would read raw codes)."""

    class Early(SimFP8):
        def _convert(self, raw, out, tag):
            pass  # the converted tile is never written

    with pytest.raises(AssertionError):
        for seed in range(20):
            Early(2, 2, seed).run()
