"""Batched prefill (l3g_prefill_batched) against token-by-token prefill and
the reference, through the C ABI.

The batched path computes the same per-token arithmetic (same activation
quantization, exact int32 block sums) with fp32 sums in another order, so:
- the KV cache it writes for layer 0 matches the token-by-token path's
  within 1e-4 relative L2; from layer 1 on, an fp32 summation-order
  difference can round an activation onto the other side of an int8
  boundary (QuantizeQ8_0Into before every matvec), and the deeper layers'
  rows are held to max(1e-2, 1.5 x the band by which the reference's own
  cgo and pure-Go builds differ on the same tokens) instead;
- the logits of the tokens decoded after it match the token-by-token run's
  and, within the reference's own band, the cgo reference's (the oracle with
  the reference's simd.c, teacher-forced on the same ids).
Covered: head dims 32 / 64 / 128, a group of 3, several passes (more than
512 tokens), a start position above zero (two batched calls in a row), and
the f16 KV cache.
"""
import numpy as np
import pytest

from conftest import synthetic_model
from refspread import LOGIT_TOL, ReferenceRuns, rel_l2

pytestmark = pytest.mark.gpu


def _kv_close(gpu_lib, cfg, s_a, s_b, npos, tol=1e-4, deep_tol=LOGIT_TOL):
    """Layer 0 within tol; deeper layers (past the first int8 re-quantization
    of the stream) within deep_tol: the fixed 1e-2 bar, or the reference
    builds' own band where that is wider."""
    for layer in range(cfg.n_layers):
        ka, va = s_a.read_kv(layer, 0, npos)
        kb, vb = s_b.read_kv(layer, 0, npos)
        t = tol if layer == 0 else max(tol, deep_tol)
        assert rel_l2(ka, kb) < t, (layer, rel_l2(ka, kb))
        assert rel_l2(va, vb) < t, (layer, rel_l2(va, vb))


@pytest.mark.parametrize("name,n_prompt,split,ctx", [
    ("tiny", 40, None, 64),
    ("tiny-g3", 100, 37, 128),
    ("small", 300, None, 512),
    ("small-hd128", 700, 100, 1024),
    ("mid", 600, 513, 1024),
])
def test_batched_prefill_matches_token_by_token(gpu_lib, oracle_mod, name, n_prompt, split, ctx):
    import synthetic
    cfg, T = synthetic_model(name)
    ids = synthetic.prompt_ids(cfg, n_prompt + 4, seed=23)
    prompt, tail = ids[:n_prompt], ids[n_prompt:]
    m = gpu_lib.LoadModelFromTensors(gpu_lib.hparams_for(cfg), T, gpu_lib.default_options(device=0))
    ws = m.NewWorkspace(ctx, 40)
    s_tok, s_bat = m.NewState(ctx), m.NewState(ctx)
    m.Prefill(s_tok, prompt, ws)
    if split is None:
        m.PrefillBatched(s_bat, prompt, ws)
    else:  # two calls: the second starts at position `split`
        m.PrefillBatched(s_bat, prompt[:split], ws)
        assert s_bat.Pos == split
        m.PrefillBatched(s_bat, prompt[split:], ws)
    assert s_bat.Pos == s_tok.Pos == n_prompt
    R = ReferenceRuns(oracle_mod, cfg, T, tail, ctx, with_f64=False, prefix_ids=prompt)
    _kv_close(gpu_lib, cfg, s_tok, s_bat, n_prompt, deep_tol=R.tol())
    # decode the tail from both states
    logits_tok, logits_bat = [], []
    buf = np.empty(cfg.vocab, np.float32)
    for t in tail:
        m.ForwardIntoWorkspace(s_tok, int(t), buf, ws)
        logits_tok.append(buf.copy())
        m.ForwardIntoWorkspace(s_bat, int(t), buf, ws)
        logits_bat.append(buf.copy())
    for i in range(len(tail)):
        assert rel_l2(logits_bat[i], logits_tok[i]) < R.tol()
        assert rel_l2(logits_bat[i], R.cgo[i]) < R.tol(), (i, R.band())
    s_tok.Close()
    s_bat.Close()
    ws.Close()
    m.Close()


def test_batched_prefill_f16_cache_and_errors(gpu_lib):
    import synthetic
    cfg, T = synthetic_model("small")
    opts = gpu_lib.default_options(device=0, kv_dtype=gpu_lib.L3G_KV_F16)
    m = gpu_lib.LoadModelFromTensors(gpu_lib.hparams_for(cfg), T, opts)
    ws = m.NewWorkspace(256, 40)
    s_tok, s_bat = m.NewState(256), m.NewState(256)
    ids = synthetic.prompt_ids(cfg, 200, seed=5)
    m.Prefill(s_tok, ids, ws)
    m.PrefillBatched(s_bat, ids, ws)
    _kv_close(gpu_lib, cfg, s_tok, s_bat, 200, tol=2e-3)  # f16 rounding of nearby values
    with pytest.raises(gpu_lib.L3GError, match="context length exceeded"):
        m.PrefillBatched(s_bat, synthetic.prompt_ids(cfg, 57, seed=6), ws)
    with pytest.raises(gpu_lib.L3GError, match="token out of range"):
        m.PrefillBatched(s_bat, np.array([1, cfg.vocab], np.int32), ws)
    assert s_bat.Pos == 200
    s_tok.Close()
    s_bat.Close()
    ws.Close()
    m.Close()
