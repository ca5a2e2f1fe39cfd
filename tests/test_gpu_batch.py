"""Batched decode (l3g_batch_step) against the single-session path and the
host restatement of the sampler, through the C ABI.

Sessions with different prompt lengths (so different positions and, across
256-position splits, different attention split counts) step together.  Per
session:
- the logits equal the single-session l3g_forward logits on a clone of the
  state within the parity tolerance (1e-2 relative L2; both compute the
  same quantized arithmetic, the batched path with fp32 sums in another
  order; at depth the bar is max(1e-2, 1.5 x the band by which the
  reference's own cgo and pure-Go builds differ on the longest session's
  last tokens), and the K/V rows the step appends match within 1e-4 at
  layer 0 (2e-3 with the f16 cache) and within that bar deeper, where an
  fp32 order difference can flip an int8 activation rounding;
- the sampled id equals SampleTopK restated on the host (tests/sampler_ref)
  over the top-K of the returned logits, with the Philox draw keyed by the
  session's seed and counted by its position;
- the position advances by one per step.
Covered: head dims 32 / 64 / 128, a group of 3, the f16 cache, argument
errors.
"""
import numpy as np
import pytest

from conftest import synthetic_model
from refspread import LOGIT_TOL, ReferenceRuns, rel_l2
from sampler_ref import sample_topk

pytestmark = pytest.mark.gpu


def _topk(logits, k):
    order = np.lexsort((np.arange(logits.size), -logits.astype(np.float64)))[:k]
    return order, logits[order]


@pytest.mark.parametrize("name,lens,ctx,kv,split", [
    ("tiny-g3", [1, 5, 40, 90], 128, 0, ""),
    ("small", [3, 17, 100, 300, 511 - 4], 512, 0, ""),
    ("mid", [2, 255, 256, 600], 1024, 0, ""),
    ("small", [7, 120, 260], 512, 1, ""),
    # attention splits of 512 positions (the host picks longer splits when
    # the sessions' positions fill several waves of CTAs)
    ("mid", [2, 511, 512, 600], 1024, 0, "512"),
])
def test_batch_step_matches_single_session(gpu_lib, oracle_mod, monkeypatch, name, lens, ctx, kv,
                                           split):
    import synthetic
    if split:
        monkeypatch.setenv("L3G_BD_SPLIT", split)
    cfg, T = synthetic_model(name)
    # the reference builds' own spread on the longest session's last tokens
    longest = int(np.argmax(lens))
    ids_l = synthetic.prompt_ids(cfg, lens[longest], seed=100 + longest)
    tail = min(3, len(ids_l) - 1)
    R = ReferenceRuns(oracle_mod, cfg, T, ids_l[-tail:], ctx, with_f64=False,
                      prefix_ids=ids_l[:-tail]) if tail > 0 else None
    bar = R.tol() if R is not None else LOGIT_TOL
    opts = gpu_lib.default_options(device=0, kv_dtype=kv)
    m = gpu_lib.LoadModelFromTensors(gpu_lib.hparams_for(cfg), T, opts)
    ws = m.NewWorkspace(ctx, 40)
    n = len(lens)
    states, clones = [], []
    for i, L in enumerate(lens):
        ids = synthetic.prompt_ids(cfg, L, seed=100 + i)
        s = m.NewState(ctx)
        m.Prefill(s, ids, ws)
        c = m.NewState(ctx)
        c.Restore(s.Snapshot())
        states.append(s)
        clones.append(c)
    batch = gpu_lib.Batch(m, 8)
    rng = np.random.default_rng(7)
    seeds = [int(x) for x in rng.integers(1, 2**62, n)]
    tokens = [int(t) for t in rng.integers(0, cfg.vocab, n)]
    for step in range(3):
        pos = [s.Pos for s in states]
        nxt, logits = batch.step(states, tokens, seeds, top_k=40, temperature=1.3, want_logits=True)
        buf = np.empty(cfg.vocab, np.float32)
        for i in range(n):
            assert states[i].Pos == pos[i] + 1
            m.ForwardIntoWorkspace(clones[i], tokens[i], buf, ws)
            assert rel_l2(logits[i], buf) < bar, (step, i, rel_l2(logits[i], buf), bar)
            for layer in range(cfg.n_layers):
                kb, vb = states[i].read_kv(layer, pos[i], 1)
                kc, vc = clones[i].read_kv(layer, pos[i], 1)
                tol = 2e-3 if kv else 1e-4
                if layer > 0:
                    tol = max(tol, bar)
                assert rel_l2(kb, kc) < tol and rel_l2(vb, vc) < tol, (step, i, layer)
            ids, lg = _topk(logits[i], 40)
            assert nxt[i] == sample_topk(ids, lg, 1.3, seeds[i], pos[i]), (step, i)
        tokens = [int(t) for t in nxt]
    batch.Close()
    for s in states + clones:
        s.Close()
    ws.Close()
    m.Close()


def test_batch_argument_errors(gpu_lib):
    import synthetic
    cfg, T = synthetic_model("small")
    m = gpu_lib.LoadModelFromTensors(gpu_lib.hparams_for(cfg), T, gpu_lib.default_options(device=0))
    ws = m.NewWorkspace(64, 40)
    s1, s2 = m.NewState(64), m.NewState(64)
    m.Prefill(s1, synthetic.prompt_ids(cfg, 4, seed=1), ws)
    batch = gpu_lib.Batch(m, 2)
    with pytest.raises(gpu_lib.L3GError, match="appears twice"):
        batch.step([s1, s1], [1, 2], [3, 4])
    with pytest.raises(gpu_lib.L3GError, match="outside"):
        batch.step([s1, s2, s1], [1, 2, 3], [3, 4, 5])
    with pytest.raises(gpu_lib.L3GError, match="token out of range"):
        batch.step([s1, s2], [1, cfg.vocab], [3, 4])
    s2.Pos = 64
    with pytest.raises(gpu_lib.L3GError, match="context length exceeded"):
        batch.step([s1, s2], [1, 2], [3, 4])
    assert s1.Pos == 4
    with pytest.raises(gpu_lib.L3GError, match="max_seqs"):
        gpu_lib.Batch(m, 0)
    batch.Close()
    s1.Close()
    s2.Close()
    ws.Close()
    m.Close()
