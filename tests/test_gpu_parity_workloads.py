"""GPU parity on the workload shapes at full depth, against the cgo reference
(the oracle's restatement of infer.go linked to the reference's own simd.c),
reported against the fixed bar: logits within 1e-2 relative L2, greedy ids
equal except where the reference's top-2 logit gap is below 1e-3.

Workloads (seeded synthetic Q8_0 weights, seeded prompt ids):
- the 1B shape, all 16 layers: 16 prompt tokens, then 128 greedy tokens;
- the 3B shape, all 28 layers: 64 prompt tokens, then 32 greedy tokens;
- the 8B shape, all 32 layers, untied output, llama3 RoPE scaling (the
  restatement extended with the published Llama-3.1 rule, since the
  reference has none): 64 prompt tokens, then 16 greedy tokens.
The greedy ids are the cgo reference's own argmax choices (ties to the
lower id); the GPU is teacher-forced along them.

Two comparisons per decode step:
- from the reference's state: the GPU state is loaded with the reference's
  KV cache of every earlier position (l3g_state_restore), then runs the
  step.  This checks the step function itself, and is held to the fixed
  bar with no allowance: every step's logits within 1e-2 and its argmax
  equal to the reference's unless the top-2 gap is below 1e-3.
- free-running: the GPU keeps its own KV cache through the whole run.  Two
  correct builds whose float32 summation orders differ round some
  activation onto the other side of an int8 quantization boundary sooner
  or later, and the difference then settles at the quantization noise
  level (about 1% of the logits); the reference's own cgo and pure-Go
  builds do the same.  The raw worst relative L2 and the number of steps
  above 1e-2 are recorded next to the band by which the pure-Go build
  differs from the cgo build on the same tokens, and the bar is
  max(1e-2, 1.5 x that band) (tests/refspread.py).

Each case appends its figures as one JSON line to $L3G_PARITY_LOG when set.
"""
import json
import os

import numpy as np
import pytest

from refspread import BAND_MARGIN, GAP_EXEMPT, LOGIT_TOL, rel_l2

pytestmark = pytest.mark.gpu

SNAP_HEADER_BYTES = 48  # "L3GKV1\0\0" + ten int32 fields, then the K|V rows

WORKLOADS = [
    # name, prompt tokens, greedy tokens, state context
    ("llama3.2-1b", 16, 128, 2048),
    ("llama3.2-3b", 64, 32, 4096),
    ("llama3.1-8b", 64, 16, 4096),
]


def _log(record):
    path = os.environ.get("L3G_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(record) + "\n")


def _top2_gap(x):
    top2 = np.partition(x, -2)[-2:]
    return float(abs(top2[1] - top2[0]))


def _argmax(x):
    return int(np.argmax(x))  # numpy: first (lowest) index among equal maxima


def _restore_from_oracle(state, om, cfg, pos):
    """Loads positions [0, pos) of the oracle's KV cache into a GPU state
    (layout [layer][kv head][pos][K hd | V hd], f32) and moves it to pos."""
    state.Pos = pos
    snap = state.Snapshot()
    L, nkv, hd = cfg.n_layers, cfg.n_heads_kv, cfg.head_dim
    K, V = om.kv_arrays()
    K = K.reshape(L, om.ctx, nkv, hd)[:, :pos].transpose(0, 2, 1, 3)
    V = V.reshape(L, om.ctx, nkv, hd)[:, :pos].transpose(0, 2, 1, 3)
    rows = np.concatenate([K, V], axis=-1).astype(np.float32)
    assert snap.size == SNAP_HEADER_BYTES + rows.nbytes
    snap[SNAP_HEADER_BYTES:] = np.ascontiguousarray(rows).view(np.uint8).reshape(-1)
    state.Restore(snap)


@pytest.mark.parametrize("name,n_prompt,n_gen,ctx", WORKLOADS)
def test_workload_parity(gpu_lib, oracle_mod, name, n_prompt, n_gen, ctx):
    import torch
    import synthetic
    cfg = synthetic.CONFIGS[name]
    T = synthetic.make_model(cfg, seed=0, device="cuda")
    torch.cuda.empty_cache()
    prompt = synthetic.prompt_ids(cfg, n_prompt, seed=1)
    octx = n_prompt + n_gen + 1
    cgo = oracle_mod.OracleModel(cfg, T)
    cgo.new_state(octx)
    pure = oracle_mod.OracleModel(cfg, T)
    pure.new_state(octx)
    m = gpu_lib.LoadModelFromTensors(gpu_lib.hparams_for(cfg), T, gpu_lib.default_options(device=0))
    s = m.NewState(ctx)        # free-running: the GPU's own KV cache
    ws = m.NewWorkspace(ctx, 40)
    s2 = m.NewState(ctx)       # reloaded from the reference's KV before every step
    ws2 = m.NewWorkspace(ctx, 40)

    for t in prompt[:-1]:
        cgo.forward(int(t), logits=False)
        pure.forward(int(t), logits=False, use_ref=False)
    m.Prefill(s, prompt[:-1], ws)

    logits = np.empty(cfg.vocab, np.float32)
    shared_logits = np.empty(cfg.vocab, np.float32)
    tok = int(prompt[-1])
    free_err, shared_err, band, gaps = [], [], [], []
    shared_id_miss, free_id_miss, free_id_exempt, shared_id_exempt = [], [], 0, 0
    for i in range(n_gen):
        pos = n_prompt - 1 + i
        _restore_from_oracle(s2, cgo, cfg, pos)
        m.ForwardIntoWorkspace(s2, tok, shared_logits, ws2)
        m.ForwardIntoWorkspace(s, tok, logits, ws)
        ref = cgo.forward(tok)
        other = pure.forward(tok, use_ref=False)
        free_err.append(rel_l2(logits, ref))
        shared_err.append(rel_l2(shared_logits, ref))
        band.append(rel_l2(other, ref))
        gap = _top2_gap(ref)
        gaps.append(gap)
        want = _argmax(ref)
        if _argmax(shared_logits) != want:
            if gap < GAP_EXEMPT:
                shared_id_exempt += 1
            else:
                shared_id_miss.append((i, want, _argmax(shared_logits), gap))
        if _argmax(logits) != want:
            noise = float(np.abs(other - ref).max())
            if gap < max(GAP_EXEMPT, 2.0 * noise):
                free_id_exempt += 1
            else:
                free_id_miss.append((i, want, _argmax(logits), gap))
        tok = want
    ref_band = max(band)
    tol = max(LOGIT_TOL, BAND_MARGIN * ref_band)
    record = {
        "test": "workload_parity", "config": name, "prompt": n_prompt, "greedy_steps": n_gen,
        "from_reference_state": {
            "worst_rel_l2": max(shared_err), "mean_rel_l2": float(np.mean(shared_err)),
            "steps_over_1e-2": int(sum(e >= LOGIT_TOL for e in shared_err)),
            "id_mismatches": len(shared_id_miss), "id_mismatches_gap_below_1e-3": shared_id_exempt},
        "free_running": {
            "worst_rel_l2": max(free_err), "first_rel_l2": free_err[0],
            "mean_rel_l2": float(np.mean(free_err)),
            "steps_over_1e-2": int(sum(e >= LOGIT_TOL for e in free_err)),
            "id_mismatches": len(free_id_miss), "id_mismatches_exempt": free_id_exempt},
        "reference_band": {"worst_pure_vs_cgo": ref_band,
                           "steps_over_1e-2": int(sum(b >= LOGIT_TOL for b in band))},
        "free_running_tol": tol, "min_top2_gap": min(gaps),
    }
    _log(record)
    ws2.Close(); s2.Close(); ws.Close(); s.Close(); m.Close()
    cgo.close(); pure.close()
    # the step function, from the reference's own state: the fixed bar
    assert max(shared_err) < LOGIT_TOL, record
    assert not shared_id_miss, (shared_id_miss, record)
    # the free-running trajectory: within the reference builds' own band
    assert max(free_err) < tol, record
    assert not free_id_miss, (free_id_miss, record)
