"""The paged KV cache through the C ABI: states whose pages come from a
shared pool (l3g_kvpool_new, l3g_state_new_in_pool) against states with a
private pool (l3g_state_new, every page mapped at once).

A page holds 256 positions of one (layer, kv head); the kernels find every
K|V row through the state's page table, so a pooled state whose pages are
scattered over the pool computes exactly what a private state computes:
- logits, the KV cache and sampled ids are bit-identical between the two,
  over positions that cross page boundaries, with pages interleaved with
  another session's (per-token steps, the device-fed loop, batched prefill
  and the batched decode step), f32 and f16 caches;
- a pool that runs out of pages fails the step with "KV pool exhausted"
  and leaves the state where it was; freeing a state returns its pages;
- snapshots move sessions between pooled and private states.
(The reference keeps one contiguous KVCache per State, state.go:3-23; it
has no pages.)
"""
import numpy as np
import pytest

from conftest import synthetic_model

pytestmark = pytest.mark.gpu


def _load(gpu_lib, name, kv=0):
    cfg, T = synthetic_model(name)
    opts = gpu_lib.default_options(device=0, kv_dtype=kv)
    return cfg, gpu_lib.LoadModelFromTensors(gpu_lib.hparams_for(cfg), T, opts)


def _heads(cfg):
    return cfg.n_layers * cfg.n_heads_kv


@pytest.mark.parametrize("name,kv", [("small-hd128", 0), ("small-hd128", 1), ("tiny-gqa", 0)])
def test_pooled_state_matches_private(gpu_lib, name, kv):
    import synthetic
    cfg, m = _load(gpu_lib, name, kv)
    ctx = min(cfg.ctx_len, 700)
    n = ctx - 40
    ids = synthetic.prompt_ids(cfg, n + 8, seed=9)
    other = synthetic.prompt_ids(cfg, n, seed=10)
    pps = -(-ctx // gpu_lib.KV_PAGE)
    pool = m.NewKvPool(2 * _heads(cfg) * pps)
    ws = m.NewWorkspace(ctx, 40)
    priv, a, b = m.NewState(ctx), m.NewStateInPool(pool, ctx), m.NewStateInPool(pool, ctx)
    m.Prefill(priv, ids[:n], ws)
    # a and b take pages in turn, so a's pages are not consecutive in the pool
    for i in range(n):
        m.Prefill(a, ids[i:i + 1], ws)
        m.Prefill(b, other[i:i + 1], ws)
    assert a.Pages == b.Pages == _heads(cfg) * -(-n // gpu_lib.KV_PAGE)
    assert pool.FreePages == 2 * _heads(cfg) * pps - a.Pages - b.Pages
    for layer in range(cfg.n_layers):
        kp, vp = priv.read_kv(layer, 0, n)
        ka, va = a.read_kv(layer, 0, n)
        assert np.array_equal(kp, ka) and np.array_equal(vp, va), layer
    lp = np.empty(cfg.vocab, np.float32)
    la = np.empty(cfg.vocab, np.float32)
    for t in ids[n:n + 4]:
        m.ForwardIntoWorkspace(priv, int(t), lp, ws)
        m.ForwardIntoWorkspace(a, int(t), la, ws)
        assert np.array_equal(lp, la)
    tp, _ = m.DecodeGreedy(priv, int(ids[n + 4]), 4, ws)
    ta, _ = m.DecodeGreedy(a, int(ids[n + 4]), 4, ws)
    assert np.array_equal(tp, ta)
    for s in (priv, a, b):
        s.Close()
    assert pool.FreePages == 2 * _heads(cfg) * pps
    ws.Close()
    pool.Close()
    m.Close()


def test_pool_exhaustion_and_release(gpu_lib):
    import synthetic
    cfg, m = _load(gpu_lib, "tiny")
    h = _heads(cfg)
    pool = m.NewKvPool(h)  # one page per (layer, kv head): 256 positions of one state
    ws = m.NewWorkspace(cfg.ctx_len, 40)
    s1 = m.NewStateInPool(pool, cfg.ctx_len)
    ids = synthetic.prompt_ids(cfg, 8, seed=2)
    m.Prefill(s1, ids, ws)
    assert s1.Pages == h and pool.FreePages == 0
    s2 = m.NewStateInPool(pool, cfg.ctx_len)
    with pytest.raises(gpu_lib.L3GError, match="KV pool exhausted"):
        m.Prefill(s2, ids[:1], ws)
    assert s2.Pos == 0 and s2.Pages == 0
    s1.Close()
    assert pool.FreePages == h
    m.Prefill(s2, ids, ws)  # the freed pages serve the next session
    assert s2.Pages == h
    with pytest.raises(gpu_lib.L3GError, match="a KV pool needs at least one page"):
        m.NewKvPool(0)
    s2.Close()
    ws.Close()
    pool.Close()
    m.Close()


def test_snapshot_moves_sessions_between_pooled_and_private(gpu_lib):
    import synthetic
    cfg, m = _load(gpu_lib, "small")
    ctx = 512
    ids = synthetic.prompt_ids(cfg, 300, seed=4)
    pool = m.NewKvPool(_heads(cfg) * 4)
    ws = m.NewWorkspace(ctx, 40)
    a = m.NewStateInPool(pool, ctx)
    m.Prefill(a, ids[:290], ws)
    priv = m.NewState(ctx)
    priv.Restore(a.Snapshot())
    b = m.NewStateInPool(pool, ctx)
    b.Restore(priv.Snapshot())
    assert priv.Pos == b.Pos == 290 and b.Pages == _heads(cfg) * 2
    la, lp, lb = (np.empty(cfg.vocab, np.float32) for _ in range(3))
    for t in ids[290:]:
        m.ForwardIntoWorkspace(a, int(t), la, ws)
        m.ForwardIntoWorkspace(priv, int(t), lp, ws)
        m.ForwardIntoWorkspace(b, int(t), lb, ws)
        assert np.array_equal(la, lp) and np.array_equal(la, lb)
    for s in (a, priv, b):
        s.Close()
    ws.Close()
    pool.Close()
    m.Close()


def test_batched_prefill_and_batch_step_on_pooled_states(gpu_lib):
    import synthetic
    cfg, m = _load(gpu_lib, "small")
    ctx = 512
    lens = [20, 257, 300]
    pool = m.NewKvPool(_heads(cfg) * 2 * len(lens))
    ws = m.NewWorkspace(ctx, 40)
    pooled, privs = [], []
    for i, L in enumerate(lens):
        ids = synthetic.prompt_ids(cfg, L, seed=40 + i)
        p, q = m.NewStateInPool(pool, ctx), m.NewState(ctx)
        m.PrefillBatched(p, ids, ws)
        m.PrefillBatched(q, ids, ws)
        pooled.append(p)
        privs.append(q)
    for p, q in zip(pooled, privs):
        for layer in range(cfg.n_layers):
            kp, vp = p.read_kv(layer, 0, p.Pos)
            kq, vq = q.read_kv(layer, 0, q.Pos)
            assert np.array_equal(kp, kq) and np.array_equal(vp, vq)
    batch = gpu_lib.Batch(m, 4)
    seeds = [11, 12, 13]
    tp = tq = [5, 6, 7]
    for _ in range(3):
        tp, lp = batch.step(pooled, tp, seeds, want_logits=True)
        tq, lq = batch.step(privs, tq, seeds, want_logits=True)
        assert np.array_equal(np.asarray(tp), np.asarray(tq))
        assert np.array_equal(lp, lq)
    batch.Close()
    for s in pooled + privs:
        s.Close()
    ws.Close()
    pool.Close()
    m.Close()
