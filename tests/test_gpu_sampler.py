"""The device sampler (l3g_forward_sample, l3g_decode_sample) against the
host restatement of SampleTopK with the same Philox draws, and the chat
loop's stop rule."""
import numpy as np
import pytest

from conftest import synthetic_model
from sampler_ref import sample_topk

pytestmark = pytest.mark.gpu


def _load(gpu_lib, name):
    cfg, T = synthetic_model(name)
    return cfg, gpu_lib.LoadModelFromTensors(gpu_lib.hparams_for(cfg), T, gpu_lib.default_options())


def test_device_sample_equals_restatement(gpu_lib):
    import synthetic
    cfg, m = _load(gpu_lib, "small")
    ids = synthetic.prompt_ids(cfg, 6, seed=41)
    s = m.NewState(64)
    ws_items = m.NewWorkspace(64, 64)
    m.Prefill(s, ids[:-1], ws_items)
    p0 = s.Pos
    ws = m.NewWorkspace(64, 64)  # fresh: its draw index starts at 0
    picks = set()
    for draw, (k, temp, seed) in enumerate([(40, 0.8, 7), (8, 1.5, 123456789), (64, 3.0, 2**40 + 3),
                                            (1, 0.8, 5), (40, 2.0, 11), (40, 2.0, 12)]):
        s.Pos = p0
        items = m.ForwardTopKIntoWorkspace(s, int(ids[-1]), k, ws_items)
        s.Pos = p0
        got = m.ForwardSample(s, int(ids[-1]), ws, top_k=k, temperature=temp, seed=seed)
        want = sample_topk([it.ID for it in items], [it.Logit for it in items], temp, seed, draw)
        assert got == want, (k, temp, seed)
        picks.add(got)
    assert len(picks) > 1  # high temperatures do not always pick the argmax
    m.Close()


def test_device_sampled_loop_and_stop_rule(gpu_lib):
    import synthetic
    cfg, m = _load(gpu_lib, "small")
    ids = synthetic.prompt_ids(cfg, 6, seed=43)
    s = m.NewState(96)
    m.Prefill(s, ids[:-1], m.NewWorkspace(96, 40))
    p0 = s.Pos
    toks, _ = m.DecodeSample(s, int(ids[-1]), 10, m.NewWorkspace(96, 40), top_k=40, temperature=1.2,
                             seed=99)
    assert len(toks) == 10 and s.Pos == p0 + 10
    # the same draws one call at a time (a fresh workspace: draw indices 0..9)
    s.Pos = p0
    ws = m.NewWorkspace(96, 40)
    tok, host = int(ids[-1]), []
    for _ in range(10):
        tok = m.ForwardSample(s, tok, ws, top_k=40, temperature=1.2, seed=99)
        host.append(tok)
    assert host == toks.tolist()
    # stop rule: samples through the first stop id; the position covers the
    # stop token's ingestion
    stop = int(toks[3])
    j = toks.tolist().index(stop)
    s.Pos = p0
    out, _ = m.DecodeSample(s, int(ids[-1]), 10, m.NewWorkspace(96, 40), top_k=40, temperature=1.2,
                            seed=99, stop_ids=[stop])
    assert out.tolist() == toks[:j + 1].tolist()
    assert s.Pos == p0 + j + 2
    m.Close()
