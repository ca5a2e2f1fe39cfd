"""Model check of k_gemm_q8's synchronization (csrc/l3g_gemm.cuh), on the CPU.

The kernel's three roles are replayed as programs over mbarriers with the
hardware's phase semantics, under random interleavings and with the
asynchronous parts (bulk copies landing, MMAs completing, tcgen05.commit
arrivals) as separate events that fire at any later time:
- producer (warp 0): the weight copies of the first `ns` stages, then their
  activation copies, then for every later chunk: wait empty[s] (parity
  ((c / ns) - 1) & 1), arrive.expect_tx on full[s], both copies;
- MMA issuer (warp 1): per chunk wait full[s] (parity (c / ns) & 1); per
  block wait tempty[buf] (parity (use - 1) & 1 from its second use), issue
  the MMA into buf, commit to tfull[buf]; after the chunk's 4 blocks commit
  to empty[s];
- the rescale warps (4, 8 or 16 by token tile): per chunk wait full[s]; per group of GB blocks wait
  tfull[buf] of each block in order (parity use & 1) and read the buffer,
  then arrive tempty[buf] of each; after the chunk arrive empty[s].
mbarrier model: a phase completes when its pending arrivals reach zero and
its transaction count is zero; try_wait.parity(P) succeeds when the current
phase's parity differs from P.  tcgen05.commit arrives once every MMA the
thread issued before it has completed.  Checked: no deadlock; a stage is read
(by an MMA or for its scales) only while it holds the chunk the reader
expects; a copy never lands in a stage an unfinished reader still uses; a
TMEM buffer is read only while it holds the expected block and is never
overwritten before every rescale warp read it.
"""
import random

import pytest

EPI = 16
BPC = 4


class Model:
    """Shared state of one replay; `version` counts state changes (a role
    that only polls a barrier changes nothing)."""

    def __init__(self):
        self.version = 0

    def bump(self):
        self.version += 1


class Bar:
    def __init__(self, mdl, count):
        self.m, self.count, self.pending, self.tx, self.phase = mdl, count, count, 0, 0

    def _maybe_complete(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def arrive(self):
        assert self.pending > 0, "arrival beyond the expected count"
        self.pending -= 1
        self.m.bump()
        self._maybe_complete()

    def arrive_expect_tx(self, n):  # mbarrier.arrive.expect_tx: count first, then arrive
        self.tx += n
        self.arrive()

    def complete_tx(self, n):
        self.tx -= n
        assert self.tx >= 0
        self.m.bump()
        self._maybe_complete()

    def ready(self, parity):  # try_wait.parity: the phase of that parity has completed
        return (self.phase & 1) != parity


def run(ns, nb, nchunks, seed, skip_tempty_wait=False, gb=1, epi=EPI):
    """One replay (gb: blocks per rescale group); skip_tempty_wait plants a
    protocol bug (in the model) for the negative test."""
    rng = random.Random(seed)
    mdl = Model()
    full = [Bar(mdl, 1) for _ in range(ns)]
    empty = [Bar(mdl, 1 + epi) for _ in range(ns)]
    tfull = [Bar(mdl, 1) for _ in range(nb)]
    tempty = [Bar(mdl, epi) for _ in range(nb)]
    stage = [None] * ns        # chunk whose two copies have landed in stage s
    landed = [0] * ns
    readers = [set() for _ in range(ns)]  # unfinished readers of the stage's chunk
    tmem = [None] * nb         # block the buffer holds
    unread = [0] * nb          # rescale warps yet to read it
    copies = []                # copies in flight: (stage, chunk)
    commits = []               # commits in flight: (MMAs issued before it, barrier)
    issued = []                # MMAs in issue order: (block, buffer, stage)
    done = [0]                 # MMAs completed (they complete in issue order)

    def producer():
        pre = min(ns, nchunks)
        for c in range(pre):           # weight copies before griddepcontrol.wait
            full[c].arrive_expect_tx(2)
            copies.append((c, c))
            yield
        for c in range(pre):           # then the activation copies
            copies.append((c, c))
            mdl.bump()
            yield
        for c in range(pre, nchunks):
            s = c % ns
            while not empty[s].ready(((c // ns) - 1) & 1):
                yield
            assert not readers[s], "refill while the stage is still read"
            full[s].arrive_expect_tx(2)
            copies.append((s, c))
            copies.append((s, c))
            yield

    def mma():
        blk = 0
        for c in range(nchunks):
            s = c % ns
            while not full[s].ready((c // ns) & 1):
                yield
            assert stage[s] == c, "MMA reads the wrong chunk"
            for _ in range(BPC):
                buf, use = blk % nb, blk // nb
                if use > 0 and not skip_tempty_wait:
                    while not tempty[buf].ready((use - 1) & 1):
                        yield
                assert unread[buf] == 0, "MMA issued into an unread buffer"
                readers[s].add(("mma", blk))
                issued.append((blk, buf, s))
                commits.append((len(issued), tfull[buf]))
                mdl.bump()
                blk += 1
                yield
            commits.append((len(issued), empty[s]))
            mdl.bump()
            yield

    def rescale(w):
        blk = 0
        for c in range(nchunks):
            s = c % ns
            while not full[s].ready((c // ns) & 1):
                yield
            assert stage[s] == c, "scales read from the wrong chunk"
            readers[s].add(("epi", w))
            for _ in range(BPC // gb):
                group = []
                for _ in range(gb):
                    buf, use = blk % nb, blk // nb
                    while not tfull[buf].ready(use & 1):
                        yield
                    assert tmem[buf] == blk, ("stale TMEM buffer", tmem[buf], blk)
                    group.append(buf)
                    blk += 1
                    yield
                for buf in group:
                    unread[buf] -= 1
                    assert unread[buf] >= 0
                    tempty[buf].arrive()
                yield
            readers[s].discard(("epi", w))
            empty[s].arrive()
            yield

    def async_events():
        ev = [("copy", i) for i in range(len(copies))]
        ev += [("commit", i) for i, (n, _) in enumerate(commits) if done[0] >= n]
        if done[0] < len(issued):
            ev.append(("mma", 0))
        return ev

    def fire(e):
        kind, i = e
        if kind == "mma":
            blk, buf, s = issued[done[0]]
            assert unread[buf] == 0, "MMA result overwrites an unread buffer"
            tmem[buf] = blk
            unread[buf] = epi
            readers[s].discard(("mma", blk))
            done[0] += 1
            mdl.bump()
        elif kind == "copy":
            s, c = copies.pop(i)
            assert not readers[s], "a copy lands in a stage still being read"
            landed[s] += 1
            if landed[s] == 2:
                landed[s] = 0
                stage[s] = c
            full[s].complete_tx(1)
        else:
            _, bar = commits.pop(i)
            bar.arrive()

    roles = {0: producer(), 1: mma()}
    roles.update({2 + w: rescale(w) for w in range(epi)})
    idle = 0
    while roles or copies or commits or done[0] < len(issued):
        v = mdl.version
        ev = async_events()
        if ev and (not roles or rng.random() < 0.3):
            fire(rng.choice(ev))
        elif roles:
            r = rng.choice(list(roles))
            try:
                next(roles[r])
            except StopIteration:
                del roles[r]
                mdl.bump()
        idle = idle + 1 if mdl.version == v else 0
        assert idle < 5000, "deadlock"
    assert done[0] == nchunks * BPC
    assert all(u == 0 for u in unread)
    assert all(b.pending == b.count and b.tx == 0 for b in full + empty + tfull + tempty)


# (stages, TMEM buffers, blocks per rescale group): the kernel's pairs are
# NB = 32 / 16 / 8 / 4 buffers with groups of 4 / 4 / 2 / 1 blocks at 16 /
# 32 / 64 / 128 tokens; smaller rings and buffer counts stress the waits
@pytest.mark.parametrize("ns,nb,gb,epi", [(1, 4, 1, 16), (2, 4, 2, 16), (3, 8, 4, 4), (5, 4, 1, 16),
                                          (7, 4, 2, 8), (8, 8, 4, 4), (8, 32, 4, 4), (8, 16, 4, 8),
                                          (8, 8, 2, 16), (6, 4, 1, 16)])
def test_gemm_barrier_protocol(ns, nb, gb, epi):
    for trial in range(30):
        nchunks = random.Random(trial).randint(1, 3 * ns + 5)
        run(ns, nb, nchunks, seed=ns * 1000 + nb * 100 + gb * 10 + trial, gb=gb, epi=epi)


def test_model_catches_a_parity_slip():
    """The replay is not vacuous: an MMA issuer that does not wait for the
    rescale warps to release a buffer is caught (a buffer overwritten while
    unread, or read holding the wrong block)."""
    caught = 0
    for trial in range(30):
        try:
            run(2, 4, 9, seed=trial, skip_tempty_wait=True)
        except AssertionError as e:
            assert "buffer" in str(e) or "stale" in str(e), e
            caught += 1
    assert caught > 0
