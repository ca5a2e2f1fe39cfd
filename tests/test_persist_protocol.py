"""Model check of the persistent layer kernel's synchronization
(csrc/l3g_persist.cuh k_layers), on the CPU.

The kernel's roles are replayed as programs under random interleavings, with
bulk copies landing at any later time, for a few CTAs with random per-CTA
tile counts per phase (the round-robin deal gives CTAs unequal shares):
- producer (one per CTA): every tile of the CTA in consumption order,
  layer by layer (QKV tiles, attention stages, Wo, up/gate and down tiles);
  before tile t >= ns it waits empty[t % ns] (parity ((t / ns) - 1) & 1);
  before the attention stage holding this step's own K/V it waits until the
  step's barrier counters show the layer's QKV barrier complete; it stops
  when its CTA aborts or, in that wait, when the step's abort word is set;
- consumer warps (NW per CTA): per phase, per tile wait full[t % ns]
  (parity (t / ns) & 1), read, arrive empty; after a failed wait (abort)
  the warp skips its remaining waits and arrivals but keeps walking the
  phases; at each grid barrier: CTA sync, thread 0 adds one arrival to
  counter b % nsub (unless aborting: it sets the abort word) and spins until
  every counter i holds (index + 1) * its CTAs, or abort, CTA sync, and every warp reads the
  CTA's decision; after the loop thread 0 waits for the producer to stop and
  for the last copy into each slot.
mbarrier model as in test_gemm_protocol.  Checked: no deadlock (with and
without an injected timeout); a consumer only reads a slot holding the tile
it expects; a copy never lands in a slot being read; the stage holding this
step's K/V is copied only after every CTA appended its rows (finished the
layer's QKV phase); every phase starts only after every CTA finished the
previous phase (the reads and writes the barriers order); no copy is in
flight when a CTA exits.
"""
import random

import pytest

from test_gemm_protocol import Bar, Model

PHASES = 7  # QKV, ATT, MERGE, WO, UPGATE, QUANT, DOWN
TILED = {0: "qkv", 1: "att", 3: "wo", 4: "upgate", 6: "down"}  # phases with ring tiles


def sub_count(grid, nsub, i):
    """CTAs that arrive on counter i (l3g_persist_plan.h sub_count)."""
    return grid // nsub + (1 if i < grid % nsub else 0)


def run(G, NW, ns, layers, seed, inject_abort=False, skip_pos_wait=False, nsub=1, fuse=False):
    rng = random.Random(seed)
    mdl = Model()
    # phases run per layer (the fused act-quant drops QUANT) and barriers per layer
    phs = [0, 1, 2, 3, 4, 6] if fuse else list(range(PHASES))
    bpl = len(phs)
    # per CTA, per layer, per tiled phase: its tile count; the attention
    # phase's last stage of a CTA with stages is the one holding the step's K/V
    # (only some CTAs hold it: the last split of each kv head)
    tiles = [[{ph: rng.randint(0, 3) for ph in TILED} for _ in range(layers)] for _ in range(G)]
    # up/gate: 2 * nblk row groups of nsl tiles, dealt round-robin; groups 2j
    # and 2j + 1 hold the two halves of SwiGLU block j
    nblk = [rng.randint(1, 4) for _ in range(layers)]
    nsl_up = [rng.randint(1, 2) for _ in range(layers)]
    ups = [[list(range(b, 2 * nblk[l], G)) for l in range(layers)] for b in range(G)]
    for b in range(G):
        for l in range(layers):
            tiles[b][l][4] = len(ups[b][l]) * nsl_up[l]
    holds_pos = [[tiles[b][l][1] > 0 and rng.random() < 0.5 for l in range(layers)] for b in range(G)]
    seq = []  # per CTA: [(layer, phase, index, is_pos_stage)]
    for b in range(G):
        s = []
        for l in range(layers):
            for ph in (0, 1, 3, 4, 6):
                n = tiles[b][l][ph]
                for i in range(n):
                    s.append((l, ph, i, ph == 1 and holds_pos[b][l] and i == n - 1))
        seq.append(s)

    counter = [0] * nsub  # CTA b arrives on counter b % nsub
    abort_word = [0]

    def complete(k):
        """Barrier k is complete: every counter holds (k + 1) * its CTAs."""
        return all(counter[i] >= (k + 1) * sub_count(G, nsub, i) for i in range(nsub))
    # fused act-quant state
    GSL = ns + 2                                   # the kernel's MAX_STAGES + 2 for ns <= MAX_STAGES
    act_written = [[[False] * NW for _ in range(2 * nblk[l])] for l in range(layers)]
    gcnt = [[0] * GSL for _ in range(G)]           # shared-memory group counts per CTA
    gown = [[None] * GSL for _ in range(G)]        # (layer, group) a slot counts
    qcnt = [[0] * nblk[l] for l in range(layers)]  # global per-block counts
    quantized = [[False] * nblk[l] for l in range(layers)]
    qkv_done = [[False] * G for _ in range(layers)]  # CTA b appended its K/V rows of layer l
    done_phase = [-1] * G  # highest (layer * PHASES + phase) every warp of CTA b finished
    warp_done = [[-1] * NW for _ in range(G)]
    exited = [False] * G

    class Cta:
        def __init__(self, b):
            self.b = b
            self.full = [Bar(mdl, 1) for _ in range(ns)]
            self.empty = [Bar(mdl, NW) for _ in range(ns)]
            self.slot = [None] * ns
            self.readers = [set() for _ in range(ns)]
            self.abort = False
            self.issued = 0
            self.producer_done = False
            self.sync_gen = [0, 0]  # CTA-sync instance counter, arrivals in it
            self.stop = False

    ctas = [Cta(b) for b in range(G)]
    copies = []  # (cta, slot, tile index)

    def producer(c):
        b = c.b
        t = 0
        for (l, ph, i, pos) in seq[b]:
            if c.abort:
                break
            if pos and not skip_pos_wait:
                while not complete(l * bpl + 0):
                    if c.abort or abort_word[0]:
                        c.abort = True
                        break
                    yield
                if c.abort:
                    break
            if pos:  # the copy reads the rows the QKV phase appended
                assert all(qkv_done[l]), "K/V stage copied before every CTA appended its rows"
            s = t % ns
            if t >= ns:
                ok = True
                while not c.empty[s].ready(((t // ns) - 1) & 1):
                    if c.abort:
                        ok = False
                        break
                    yield
                if not ok:
                    break
                assert not c.readers[s], "refill while the slot is read"
            c.full[s].arrive_expect_tx(1)
            copies.append((c, s, t))
            t += 1
            c.issued = t
            yield
        c.producer_done = True
        mdl.bump()

    def cta_sync(c):
        """bar.sync over the CTA's NW consumer warps (a generator)."""
        gen = c.sync_gen[0]
        c.sync_gen[1] += 1
        mdl.bump()
        if c.sync_gen[1] == NW:
            c.sync_gen[0] += 1
            c.sync_gen[1] = 0
        while c.sync_gen[0] == gen:
            yield

    def consumer(c, w, abort_at):
        b = c.b
        t = 0
        alive = True
        k = 0  # waits so far (for the injected timeout)
        bi = 0  # barriers passed
        for l in range(layers):
            for j, ph in enumerate(phs):
                # every CTA finished the previous phase (what the barrier orders)
                lin = l * bpl + j
                assert min(done_phase) >= lin - 1 or c.stop, ("phase started early", b, lin, done_phase)
                if fuse and ph == 6:
                    assert all(quantized[l]) or c.stop, "down phase before every block was quantized"
                n = tiles[b][l][ph] if ph in TILED else 0
                for i in range(n):
                    if alive:
                        s = t % ns
                        k += 1
                        if abort_at is not None and k == abort_at:
                            c.abort = True  # an injected timeout: the wait gives up
                            alive = False
                            mdl.bump()
                        while alive and not c.full[s].ready((t // ns) & 1):
                            if c.abort:
                                alive = False
                                break
                            yield
                        if alive:
                            assert c.slot[s] == t, ("wrong tile in slot", c.slot[s], t)
                            c.readers[s].add(w)
                            mdl.bump()
                            yield
                            c.readers[s].discard(w)
                            c.empty[s].arrive()
                    t += 1
                    if fuse and ph == 4 and alive and (i + 1) % nsl_up[l] == 0:
                        # the group's epilogue, then ps_swiglu_quant
                        kk = i // nsl_up[l]
                        g = ups[b][l][kk]
                        act_written[l][g][w] = True
                        mdl.bump()
                        yield
                        slot = kk % GSL
                        assert gown[b][slot] in (None, (l, g)), ("group count slot aliased", gown[b][slot], g)
                        gown[b][slot] = (l, g)
                        gcnt[b][slot] += 1
                        mdl.bump()
                        if gcnt[b][slot] == NW:
                            gcnt[b][slot] = 0
                            gown[b][slot] = None
                            yield
                            blk = g // 2
                            old = qcnt[l][blk]
                            qcnt[l][blk] += 1
                            mdl.bump()
                            if old == 1:
                                yield
                                assert all(act_written[l][2 * blk]) and all(act_written[l][2 * blk + 1]), \
                                    "block quantized before both halves were written"
                                quantized[l][blk] = True
                                qcnt[l][blk] = 0
                                mdl.bump()
                        yield
                warp_done[b][w] = lin
                if l == layers - 1 and j == bpl - 1:
                    break  # the last layer's down phase has no barrier
                # grid barrier
                yield from cta_sync(c)
                done_phase[b] = min(warp_done[b])
                if ph == 0:
                    qkv_done[l][b] = True  # every warp's epilogues appended their K/V rows
                if w == 0:
                    stop = c.abort
                    if stop:
                        abort_word[0] = 1
                        mdl.bump()
                    else:
                        counter[b % nsub] += 1
                        mdl.bump()
                        while not complete(bi):
                            if c.abort or abort_word[0]:
                                stop = True
                                break
                            yield
                    if stop:
                        c.abort = True
                    c.stop = stop
                bi += 1
                yield from cta_sync(c)
                if c.stop:
                    break
            if c.stop:
                break
        # drain (thread 0 of warp 0), then exit
        yield from cta_sync(c)
        if w == 0:
            if c.abort:
                while not c.producer_done:
                    yield
                while any(cc is c for cc, _, _ in copies):
                    yield
            else:
                assert c.producer_done or not copies
            assert not any(cc is c for cc, _, _ in copies), "exit with a copy in flight"
            exited[b] = True

    roles = {}
    victim = (rng.randrange(G), rng.randrange(NW), rng.randint(1, 6)) if inject_abort else None
    for c in ctas:
        roles[("p", c.b)] = producer(c)
        for w in range(NW):
            at = victim[2] if victim and victim[0] == c.b and victim[1] == w else None
            roles[("c", c.b, w)] = consumer(c, w, at)
    idle = 0
    while roles or copies:
        v = mdl.version
        if copies and (not roles or rng.random() < 0.3):
            c, s, t = copies.pop(rng.randrange(len(copies)))
            assert not c.readers[s], "a copy lands in a slot being read"
            c.slot[s] = t
            c.full[s].complete_tx(1)
        elif roles:
            r = rng.choice(list(roles))
            try:
                next(roles[r])
            except StopIteration:
                del roles[r]
                mdl.bump()
        idle = idle + 1 if mdl.version == v else 0
        assert idle < 20000, "deadlock"
    assert all(exited)
    if not inject_abort:
        assert abort_word[0] == 0
        assert sum(counter) == (layers * bpl - 1) * G
        if fuse:
            assert all(all(q) for q in quantized) and not any(any(q) for q in qcnt)
    return abort_word[0]


@pytest.mark.parametrize("G,NW,ns,nsub", [(1, 2, 2, 1), (3, 2, 2, 1), (4, 3, 3, 1), (5, 2, 6, 1),
                                          (2, 4, 1, 1), (5, 2, 3, 2), (7, 2, 2, 3), (4, 2, 3, 4)])
def test_persistent_protocol(G, NW, ns, nsub):
    """One barrier counter, or arrivals spread over nsub counters
    (L3G_PERSIST_BAR_SPREAD), including grids that do not divide evenly;
    with and without the fused SwiGLU act-quant (L3G_PERSIST_FUSE_QUANT)."""
    for trial in range(25):
        for fuse in (False, True):
            run(G, NW, ns, layers=2, seed=G * 1000 + NW * 100 + ns * 10 + trial, nsub=nsub, fuse=fuse)


@pytest.mark.parametrize("G,NW,ns,nsub", [(3, 2, 2, 1), (4, 3, 3, 1), (5, 2, 3, 2)])
def test_persistent_protocol_with_a_timeout(G, NW, ns, nsub):
    """One consumer wait gives up (a bounded wait running out): every CTA
    still reaches its exit, with no copy in flight."""
    aborted = sum(run(G, NW, ns, layers=2, seed=7 * trial + G, inject_abort=True, nsub=nsub,
                      fuse=trial % 2 == 1)
                  for trial in range(40))
    assert aborted >= 10  # the abort path ran, not just clean steps


def test_model_catches_a_missing_kv_wait():
    """The replay is not vacuous: a producer that copies the stage holding
    this step's K/V without waiting for the QKV barrier is caught."""
    caught = 0
    for trial in range(40):
        try:
            run(4, 2, 3, layers=2, seed=trial, skip_pos_wait=True)
        except AssertionError as e:
            assert "K/V stage" in str(e), e
            caught += 1
    assert caught > 0


def test_model_catches_a_small_group_count_ring():
    """The replay is not vacuous for the fused act-quant either: with fewer
    shared-memory count slots than the warps' drift (one slot), a fast warp
    reuses a slot another group still counts, and the replay reports it."""
    caught = 0
    for trial in range(60):
        try:
            _run_with_gsl(trial)
        except AssertionError as e:
            assert "aliased" in str(e) or "before both halves" in str(e), e
            caught += 1
    assert caught > 0


def _run_with_gsl(trial):
    """run() with the count ring cut to one slot (a planted bug, in the model)."""
    import inspect
    import test_persist_protocol as mod
    code = inspect.getsource(mod.run).replace("GSL = ns + 2", "GSL = 1")
    ns_ = {}
    exec(compile(code, "<planted>", "exec"), mod.__dict__, ns_)
    ns_["run"](3, 3, 4, layers=2, seed=trial, fuse=True)

