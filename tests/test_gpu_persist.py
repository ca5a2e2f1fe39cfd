"""Persistent layer kernel (k_layers: every layer of a decode step in one
launch of one CTA per SM, phases separated by grid barriers) through the C
ABI, against the per-kernel step and the oracle.

- Same model and tokens: logits, every layer's KV cache and the hidden state
  are bit-identical to the per-kernel step's when that step uses the same
  tile layout (four rows per warp, L3G_RPW=4) and the same split merge
  (global partials, L3G_ATT_CLUSTER=0): both compute the same Q8_0 block
  products, norms, RoPE, attention partials and merges in the same order.
  Covered: head sizes 32, 64 and 128, query heads per kv head 2, 3 and 4,
  f32 and f16 caches, short contexts (most splits empty) and 1500 positions
  (every split busy).
- Against the cgo reference (the oracle linked to the reference's simd.c)
  within the band of test_gpu_parity, and greedy ids under teacher forcing.
- The device-fed greedy loop gives the per-token loop's tokens; the traced
  step stamps every CTA at every grid barrier.
"""

import numpy as np
import pytest

from conftest import synthetic_model
from refspread import ReferenceRuns, rel_l2

pytestmark = pytest.mark.gpu


def _fusions(fuse):
    """fuse: "0" none, "1" the SwiGLU act-quant, "m" the split merge, "1m" both."""
    return "1" in fuse, "m" in fuse


def _load(gpu_lib, monkeypatch, cfg, T, persistent, fuse="0", spread="1", **kw):
    fq, fm = _fusions(fuse)
    monkeypatch.setenv("L3G_RPW", "4")
    monkeypatch.setenv("L3G_ATT_CLUSTER", "0")
    monkeypatch.setenv("L3G_PERSIST_FUSE_QUANT", "1" if fq else "0")
    monkeypatch.setenv("L3G_PERSIST_FUSE_MERGE", "1" if fm else "0")
    monkeypatch.setenv("L3G_PERSIST_BAR_SPREAD", spread)
    if persistent:
        monkeypatch.setenv("L3G_PERSIST", "1")
    else:
        monkeypatch.delenv("L3G_PERSIST", raising=False)
    m = gpu_lib.LoadModelFromTensors(gpu_lib.hparams_for(cfg), T, gpu_lib.default_options(**kw))
    monkeypatch.delenv("L3G_PERSIST", raising=False)
    return m


def _run(gpu_lib, m, cfg, ids, ctx, prefill=0):
    s = m.NewState(ctx)
    ws = m.NewWorkspace(ctx, 40)
    if prefill:
        m.Prefill(s, ids[:prefill], ws)
    out = []
    logits = np.empty(cfg.vocab, np.float32)
    for t in ids[prefill:]:
        m.ForwardIntoWorkspace(s, int(t), logits, ws)
        out.append(logits.copy())
    kv = [s.read_kv(layer, 0, len(ids)) for layer in range(cfg.n_layers)]
    hidden = ws.read(gpu_lib.BUF_HIDDEN, cfg.n_emb)
    return ws, out, kv, hidden


@pytest.mark.parametrize("name,n_tok,prefill,kv,fuse,spread", [
    ("tiny", 24, 0, "f32", "0", "1"), ("tiny-gqa", 24, 0, "f32", "0", "1"),
    ("small", 40, 0, "f32", "0", "1"), ("small-hd128", 24, 0, "f32", "0", "1"),
    ("small-hd128", 24, 0, "f16", "0", "1"), ("tiny-g3", 24, 0, "f32", "0", "1"),
    ("mid", 16, 0, "f32", "0", "1"), ("llama3.2-1b-2l", 12, 0, "f32", "0", "1"),
    ("small-hd128", 1500, 1496, "f32", "0", "1"),
    # the SwiGLU act-quant fused into up/gate, barrier arrivals spread over counters
    ("tiny", 24, 0, "f32", "1", "3"), ("mid", 16, 0, "f32", "1", "16"),
    ("llama3.2-1b-2l", 12, 0, "f32", "1", "1"), ("small", 40, 0, "f32", "0", "16"),
    # the split merge in the attention phase, alone and with the act-quant fold
    ("small-hd128", 1500, 1496, "f32", "m", "1"), ("mid", 16, 0, "f32", "1m", "4"),
    ("tiny-g3", 24, 0, "f32", "m", "1"),
])
def test_bit_identical_to_per_kernel_step(gpu_lib, monkeypatch, name, n_tok, prefill, kv, fuse,
                                          spread):
    import synthetic
    cfg, T = synthetic_model(name)
    ctx = max(64, n_tok + 8)
    ids = synthetic.prompt_ids(cfg, n_tok, seed=13)
    kw = {"kv_dtype": gpu_lib.L3G_KV_F16} if kv == "f16" else {}
    base = _load(gpu_lib, monkeypatch, cfg, T, False, **kw)
    ws0, l0, kv0, h0 = _run(gpu_lib, base, cfg, ids, ctx, prefill)
    assert not ws0.persistent()
    pers = _load(gpu_lib, monkeypatch, cfg, T, True, fuse, spread, **kw)
    ws1, l1, kv1, h1 = _run(gpu_lib, pers, cfg, ids, ctx, prefill)
    assert ws1.persistent()
    lay = ws1.persist_layout()
    fq, fm = _fusions(fuse)
    assert lay["barriers_per_layer"] == 7 - fq - fm
    assert lay["barrier_counters"] == int(spread)
    for i, (a, b) in enumerate(zip(l0, l1)):
        assert np.array_equal(a, b), (i, rel_l2(b, a))
    for layer, ((k0, v0), (k1, v1)) in enumerate(zip(kv0, kv1)):
        assert np.array_equal(k0, k1) and np.array_equal(v0, v1), layer
    assert np.array_equal(h0, h1)


@pytest.mark.parametrize("name,n_tok,fuse", [("mid", 16, "0"), ("llama3.2-1b-2l", 12, "0"),
                                            ("mid", 16, "1")])
def test_logits_vs_reference(gpu_lib, oracle_mod, monkeypatch, name, n_tok, fuse):
    import synthetic
    cfg, T = synthetic_model(name)
    ctx = min(cfg.ctx_len, 256)
    ids = synthetic.prompt_ids(cfg, n_tok, seed=11)
    R = ReferenceRuns(oracle_mod, cfg, T, ids, ctx, with_f64=False)
    m = _load(gpu_lib, monkeypatch, cfg, T, True, fuse)
    s = m.NewState(ctx)
    ws = m.NewWorkspace(ctx, 40)
    assert ws.persistent()
    logits = np.empty(cfg.vocab, np.float32)
    errs = []
    for i, t in enumerate(ids):
        m.ForwardIntoWorkspace(s, int(t), logits, ws)
        errs.append(rel_l2(logits, R.cgo[i]))
    assert max(errs) < R.tol(), (errs, R.band())
    for layer in range(cfg.n_layers):
        K, V = s.read_kv(layer, 0, n_tok)
        K0, V0 = R.cgo_model.kv(layer, 0, n_tok)
        assert rel_l2(K, K0) < R.tol() and rel_l2(V, V0) < R.tol()


def test_greedy_ids_vs_reference(gpu_lib, oracle_mod, monkeypatch):
    """Teacher-forced greedy decode on the persistent step: argmax ids equal
    the cgo reference's except inside its top-2 band."""
    import synthetic
    from test_gpu_parity import _greedy_teacher
    cfg, T = synthetic_model("small")
    n_prompt, n_gen = 8, 48
    ctx = n_prompt + n_gen + 1
    prompt = synthetic.prompt_ids(cfg, n_prompt, seed=21)
    fed = _greedy_teacher(oracle_mod, cfg, T, prompt, n_gen, ctx)
    R = ReferenceRuns(oracle_mod, cfg, T, fed, ctx, prefix_ids=prompt[:-1])
    m = _load(gpu_lib, monkeypatch, cfg, T, True)
    s = m.NewState(ctx)
    ws = m.NewWorkspace(ctx, 40)
    m.Prefill(s, prompt[:-1], ws)
    bad = []
    for i, tok in enumerate(fed):
        got, _ = m.ForwardArgmax(s, tok, ws)
        ref = R.cgo[i]
        top2 = np.sort(ref)[-2:]
        if got != int(np.argmax(ref)) and float(top2[1] - top2[0]) >= R.gap_exempt(i):
            bad.append((i, int(np.argmax(ref)), got))
    assert not bad, bad


def test_device_loop_and_barrier_stamps(gpu_lib, monkeypatch):
    """l3g_decode_greedy on the persistent step gives the per-token loop's
    tokens; a traced step stamps every CTA's arrival and release at every
    grid barrier (release after arrival, every CTA released after the last
    arrival)."""
    import synthetic
    cfg, T = synthetic_model("mid")
    m = _load(gpu_lib, monkeypatch, cfg, T, True)
    prompt = synthetic.prompt_ids(cfg, 6, seed=3)
    s1, s2 = m.NewState(64), m.NewState(64)
    ws = m.NewWorkspace(64, 40)
    m.Prefill(s1, prompt[:-1], ws)
    toks_dev, _ = m.DecodeGreedy(s1, int(prompt[-1]), 12, ws)
    m.Prefill(s2, prompt[:-1], ws)
    tok, toks = int(prompt[-1]), []
    for _ in range(12):
        tok, _ = m.ForwardArgmax(s2, tok, ws)
        toks.append(tok)
    assert list(toks_dev) == toks
    m.TraceStep(s2, tok, ws)
    st = ws.persist_stamps()
    nb = ws.persist_layout()["barriers_per_layer"] * cfg.n_layers - 1  # the last down ends the kernel
    arr, rel = st[:nb, :, 0], st[:nb, :, 1]
    assert (arr > 0).all() and (rel >= arr).all()
    assert (rel.min(axis=1) >= arr.max(axis=1)).all()
    assert (st[nb:] == 0).all()
