"""The reference top-K path's attention on the GPU
(l3g_workspace_set_topk_fast_exp: weights fastExp(score - max) with the
maximum over all positions, infer.go:376-423, 520-525) through the C ABI,
against the oracle's ForwardTopKIntoWorkspace restatement.

- The last layer's attention output and the top-K items of a top-K step
  match the cgo reference's top-K path (oracle + simd.c) within the band of
  test_gpu_parity (max(1e-2, 1.5 x the distance of the pure-Go build)).
- The mode switches only the top-K and sampled calls: with it on, the full
  logits are still the exact-exp path's; turning it off gives back the exact
  top-K bit for bit; turning it on again repeats the fast items bit for bit.
"""

import numpy as np
import pytest

from conftest import synthetic_model
from refspread import BAND_MARGIN, LOGIT_TOL, rel_l2

pytestmark = pytest.mark.gpu


def _load_gpu(gpu_lib, cfg, T, **kw):
    return gpu_lib.LoadModelFromTensors(gpu_lib.hparams_for(cfg), T, gpu_lib.default_options(**kw))


def _oracle_topk(oracle_mod, cfg, T, ids, ctx, use_ref):
    """The reference's ingest (ForwardIntoWorkspace without logits) of
    ids[:-1], then ForwardTopKIntoWorkspace on ids[-1]: (items as {id: logit},
    the last layer's attention output)."""
    om = oracle_mod.OracleModel(cfg, T)
    om.new_state(ctx)
    for t in ids[:-1]:
        om.forward(int(t), logits=False, use_ref=use_ref)
    tid, tlg = om.forward_topk(int(ids[-1]), 40, use_ref=use_ref)
    attn = om.buffer("attn").copy()
    om.close()
    return dict(zip(tid.tolist(), tlg.tolist())), attn


@pytest.mark.parametrize("name,n,kv", [("small", 40, "f32"), ("small-hd128", 700, "f32"),
                                       ("tiny-g3", 30, "f32"), ("tiny-gqa", 1, "f32"),
                                       ("small", 300, "f16")])
def test_fast_topk_matches_reference_topk_path(gpu_lib, oracle_mod, name, n, kv):
    import synthetic
    cfg, T = synthetic_model(name)
    ids = synthetic.prompt_ids(cfg, n, seed=13)
    ctx = n + 8
    cgo, attn_cgo = _oracle_topk(oracle_mod, cfg, T, ids, ctx, use_ref=True)
    pure, attn_pure = _oracle_topk(oracle_mod, cfg, T, ids, ctx, use_ref=False)
    kw = {"kv_dtype": gpu_lib.L3G_KV_F16} if kv == "f16" else {}
    m = _load_gpu(gpu_lib, cfg, T, **kw)
    s = m.NewState(ctx)
    ws = m.NewWorkspace(ctx, 40)
    ws.SetTopKFastExp(True)
    if n > 1:
        m.Prefill(s, ids[:-1], ws)
    items = m.ForwardTopKIntoWorkspace(s, int(ids[-1]), 40, ws)
    assert len(items) == 40 and s.Pos == n
    # f16 storage rounds every K/V value: twice the bar, as in test_gpu_parity
    widen = 2.0 if kv == "f16" else 1.0
    attn = ws.read(gpu_lib.BUF_ATTN, cfg.n_heads * cfg.head_dim)
    tol_attn = widen * max(LOGIT_TOL, BAND_MARGIN * rel_l2(attn_pure, attn_cgo))
    assert rel_l2(attn, attn_cgo) < tol_attn, (rel_l2(attn, attn_cgo), rel_l2(attn_pure, attn_cgo))
    got = {it.ID: it.Logit for it in items}
    common = sorted(set(got) & set(cgo))
    common_pure = sorted(set(pure) & set(cgo))
    assert len(common) >= 36, (len(common), len(common_pure))
    g = np.array([got[i] for i in common])
    c = np.array([cgo[i] for i in common])
    band = rel_l2([pure[i] for i in common_pure], [cgo[i] for i in common_pure])
    assert rel_l2(g, c) < widen * max(LOGIT_TOL, BAND_MARGIN * band), (rel_l2(g, c), band)
    m.Close()


def test_fast_mode_switches_only_the_topk_calls(gpu_lib):
    import synthetic
    cfg, T = synthetic_model("small-hd128")
    n = 600
    ids = synthetic.prompt_ids(cfg, n, seed=17)
    m = _load_gpu(gpu_lib, cfg, T)
    s = m.NewState(n + 4)
    ws = m.NewWorkspace(n + 4, 40)
    m.Prefill(s, ids[:-1], ws)
    last = int(ids[-1])

    def step_topk(fast):
        ws.SetTopKFastExp(fast)
        s.Pos = n - 1
        items = m.ForwardTopKIntoWorkspace(s, last, 40, ws)
        return [it.ID for it in items], np.array([it.Logit for it in items], np.float32)

    fast_ids, fast_lg = step_topk(True)
    # the full-logits call keeps the exact exp with the mode on
    s.Pos = n - 1
    logits = np.empty(cfg.vocab, np.float32)
    m.ForwardIntoWorkspace(s, last, logits, ws)
    exact_ids, exact_lg = step_topk(False)
    order = np.lexsort((np.arange(cfg.vocab), -logits))[:40]
    assert exact_ids == order.tolist()
    assert np.array_equal(exact_lg, logits[order])
    # the fast items came from the other softmax
    got = dict(zip(fast_ids, fast_lg.tolist()))
    assert any(got.get(i, None) != float(v) for i, v in zip(exact_ids, exact_lg))
    # back on: the same fast items, bit for bit (the captured graph is keyed by the mode)
    again_ids, again_lg = step_topk(True)
    assert again_ids == fast_ids and np.array_equal(again_lg, fast_lg)
    # the sampled call runs the same attention: its pick is one of the fast items
    s.Pos = n - 1
    pick = m.ForwardSample(s, last, ws, top_k=40, temperature=0.8, seed=3)
    assert pick in fast_ids
    assert gpu_lib.lib().l3g_workspace_set_topk_fast_exp(ws._h, 2) == gpu_lib.L3G_E_INVALID
    m.Close()
