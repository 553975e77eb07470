"""A model of the barrier protocol of the int4 tensor-core kernel (byteprof_b200/csrc/skinny_i4tc.cu), run
on the CPU under random schedules: mbarriers with phase counts and parity waits (a parity wait is
satisfied by the last completed phase of that parity, so a waiter two phases ahead is let through), copies
that land in any order, MMA commits that complete in issue order, and every buffer tagged with the unit
and group it holds so that a stale read or an early overwrite fails an assertion. The roles and ring sizes
are the kernel's: weight stages (packed codes, scale, zero) of GB groups, digit stages of GB groups, the
unpacked-tile slots filled round-robin by the unpack warps, two TMEM unit buffers and the epilogue.

The rule the kernel relies on: no more unpack warps than unpacked-tile slots. With four warps on three
slots a warp can wait for a slot release two uses old; the last test shows the model catching that."""

import random

import pytest

GROUP_PACKED = 8192
PACKED_REGION = 3 * 4 * GROUP_PACKED  # 96 KB: 12 group slots of weight stages


def a_slots(nb):
    return 5 if nb <= 32 else 3


def digit_slots(nb):
    return (32 * 1024 if nb <= 32 else 64 * 1024) // (nb * 128)


class MBar:
    def __init__(self, count):
        self.count, self.pending, self.tx, self.phase = count, count, 0, 0

    def arrive(self, n=1):
        self.pending -= n
        self._check()

    def expect_tx(self, n):
        self.tx += n
        self.pending -= 1
        self._check()

    def complete_tx(self, n):
        self.tx -= n
        self._check()

    def _check(self):
        assert self.pending >= 0 and self.tx >= 0, "more arrivals or bytes than the phase expects"
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def done(self, parity):
        return (self.phase & 1) != parity


class Deadlock(RuntimeError):
    pass


def run(G, GB, u0, n_units, nb, seed, unpack_warps=None):
    rng = random.Random(seed)
    kas = a_slots(nb)
    W = unpack_warps if unpack_warps is not None else min(4, kas)
    wsu = PACKED_REGION // (GB * GROUP_PACKED)
    dsu = digit_slots(nb) // GB
    UG = (G + GB - 1) // GB
    full = [MBar(1) for _ in range(wsu)]
    empty = [MBar(GB + 4) for _ in range(wsu)]
    afull = [MBar(32) for _ in range(kas)]
    aempty = [MBar(1) for _ in range(kas)]
    dfull = [MBar(1) for _ in range(dsu)]
    dempty = [MBar(1 + 4) for _ in range(dsu)]
    tfull = [MBar(1) for _ in range(2)]
    tempty = [MBar(128) for _ in range(2)]
    wstage, dstage, aslot, tbuf = [None] * wsu, [None] * dsu, [None] * kas, [None] * 2
    events, now, last_commit = [], [0], [0]

    def later(fn):
        events.append((now[0] + rng.randint(1, 40), fn))

    def commit(fn):  # tcgen05.commit arrivals complete in issue order
        t = max(now[0] + rng.randint(1, 40), last_commit[0] + 1)
        last_commit[0] = t
        events.append((t, fn))

    def units():
        for i in range(n_units):
            g0 = ((u0 + i) % UG) * GB
            yield i, min(GB, G - g0)

    def producer():
        for i, ng in units():
            st = i % wsu
            while i >= wsu and not empty[st].done(((i // wsu) + 1) & 1):
                yield
            full[st].expect_tx(3)

            def land(st=st, i=i):
                wstage[st] = i
                for _ in range(3):
                    full[st].complete_tx(1)
            later(land)

    def digits():
        for i, ng in units():
            ds = i % dsu
            while i >= dsu and not dempty[ds].done(((i // dsu) + 1) & 1):
                yield
            dfull[ds].expect_tx(2)

            def land(ds=ds, i=i):
                dstage[ds] = i
                dfull[ds].complete_tx(2)
            later(land)

    def unpack(uw):
        j = 0
        for i, ng in units():
            st, have = i % wsu, False
            for gg in range(ng):
                if j % W != uw:
                    j += 1
                    continue
                if not have:
                    while not full[st].done((i // wsu) & 1):
                        yield
                    have = True
                slot = j % kas
                while j >= kas and not aempty[slot].done(((j // kas) + 1) & 1):
                    yield
                assert wstage[st] == i, "unpack reads a stale weight stage"
                yield
                assert wstage[st] == i, "weight stage refilled during the unpack"
                aslot[slot] = (j, i, gg)
                afull[slot].arrive(32)
                empty[st].arrive(GB - ng + 1 if gg == ng - 1 else 1)
                j += 1

    def mma():
        j = 0
        for i, ng in units():
            ds, ub = i % dsu, i & 1
            while not dfull[ds].done((i // dsu) & 1):
                yield
            while i >= 2 and not tempty[ub].done(((i >> 1) + 1) & 1):
                yield
            for gg in range(ng):
                slot = j % kas
                while not afull[slot].done((j // kas) & 1):
                    yield
                assert aslot[slot] == (j, i, gg), "MMA reads a stale unpacked tile"
                assert dstage[ds] == i, "MMA reads a stale digit stage"

                def release(slot=slot, tag=(j, i, gg)):
                    assert aslot[slot] == tag, "unpacked tile overwritten before the MMA read it"
                    aempty[slot].arrive()
                commit(release)
                j += 1

            def unit_done(ub=ub, i=i, ds=ds):
                tbuf[ub] = i
                tfull[ub].arrive()
                dempty[ds].arrive()
            commit(unit_done)

    def epilogue():
        for i, ng in units():
            st, ds, ub = i % wsu, i % dsu, i & 1
            while not full[st].done((i // wsu) & 1):
                yield
            assert wstage[st] == i, "epilogue reads stale scale rows"
            empty[st].arrive(4)
            while not dfull[ds].done((i // dsu) & 1):
                yield
            while not tfull[ub].done((i >> 1) & 1):
                yield
            assert tbuf[ub] == i and dstage[ds] == i, "epilogue reads a stale accumulator or group sums"
            yield
            tempty[ub].arrive(128)
            dempty[ds].arrive(4)

    alive = [producer(), digits(), mma(), epilogue()] + [unpack(w) for w in range(W)]
    for _ in range(3_000_000):
        if not alive and not events:
            return
        if events and (not alive or rng.random() < 0.3):
            events.sort(key=lambda e: e[0])
            t, fn = events.pop(0)
            now[0] = max(now[0], t)
            fn()
            continue
        role = rng.choice(alive)
        try:
            next(role)
        except StopIteration:
            alive.remove(role)
        now[0] += 1
    raise Deadlock("no progress")


@pytest.mark.parametrize("nb", [16, 32, 48, 64])
@pytest.mark.parametrize("G,GB", [(16, 1), (16, 2), (16, 4), (64, 2), (9, 4), (3, 2)])
def test_the_kernel_ring_configurations_neither_deadlock_nor_read_stale_data(nb, G, GB):
    if digit_slots(nb) // GB < 1:
        pytest.skip("fewer digit slots than groups per unit")
    for u0, n_units in [(0, 3), (5, 7), (3, 20), (1, 40)]:
        for seed in range(8):
            run(G, GB, u0, n_units, nb, seed)


def test_more_unpack_warps_than_slots_is_caught():
    failures = 0
    for seed in range(20):
        try:
            run(16, 2, 3, 20, 48, seed, unpack_warps=4)
        except (AssertionError, Deadlock):
            failures += 1
    assert failures > 0
