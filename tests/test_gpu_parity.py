"""GPU parity tests: the CUDA library (through its C ABI) against the oracle.

Tolerances: matvec and logits within 1e-2 relative L2 of
the reference's CGO_ENABLED=1 path (the oracle with the reference's own
simd.c), greedy ids identical except where the reference's top-2 logit gap is
below 1e-3.  Activation quantization is compared bit for bit.
"""
import numpy as np
import pytest

from conftest import synthetic_model

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2      # relative L2, north star
GAP_EXEMPT = 1e-3     # top-2 gap below which a greedy mismatch is allowed


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


def test_quantize_bit_exact(gpu_lib, oracle_mod):
    import torch
    rng = np.random.default_rng(1)
    for n, scale in ((32, 1.0), (4096, 3.0), (14336, 0.01), (100, 50.0), (33, 1e-4)):
        x = (rng.standard_normal(n) * scale).astype(np.float32)
        x[: min(n, 32)][::7] = 0.0
        xd = torch.from_numpy(x).cuda()
        nb = (n + 31) // 32
        d = torch.empty(nb, dtype=torch.float32, device="cuda")
        qs = torch.empty(nb * 32, dtype=torch.int8, device="cuda")
        gpu_lib.quantize_q8_0_device(xd.data_ptr(), n, d.data_ptr(), qs.data_ptr())
        torch.cuda.synchronize()
        d0, q0 = oracle_mod.quantize_q8_0(x)
        assert np.array_equal(d.cpu().numpy(), d0)
        assert np.array_equal(qs.cpu().numpy(), q0)


MATVEC_SHAPES = [  # (rows, cols): the 8B microbench shapes plus ragged ones
    (4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (128256, 4096),
    (37, 96), (1, 32), (2050, 1792), (513, 512),
]


@pytest.mark.parametrize("rows,cols", MATVEC_SHAPES)
def test_matvec_vs_reference_simd(gpu_lib, oracle_mod, rows, cols):
    """l3g_matvec_q8 against the reference's own matvec_q8_c (simd.c)."""
    import synthetic
    import torch
    if not oracle_mod.have_ref_simd():
        pytest.fail("oracle/_ref/libref_simd.so (the reference's simd.c) is missing")
    g = torch.Generator().manual_seed(rows * 7 + cols)
    w = synthetic.quantize_q8_0_rows(torch.randn(rows, cols, generator=g) * 0.02, torch).numpy()
    x = np.random.default_rng(rows).standard_normal(cols).astype(np.float32)
    d0, q0 = oracle_mod.quantize_q8_0(x)
    ref = oracle_mod.ref_matvec_q8(w, d0, q0, rows, cols)
    M = gpu_lib.Matrix(w, rows, cols)
    xd = torch.from_numpy(d0).cuda()
    xq = torch.from_numpy(q0).cuda()
    out = torch.full((rows,), 12345.0, device="cuda")
    M.matvec(xd.data_ptr(), xq.data_ptr(), out.data_ptr())
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert rel_l2(got, ref) < 1e-5
    assert np.allclose(got, ref, rtol=1e-4, atol=1e-5 * float(np.abs(ref).max()))
    # a row sub-range writes exactly [start, end) like matvec_q8_c's loop
    if rows >= 3:
        s, e = rows // 3, rows // 3 + max(1, rows // 4)
        out.fill_(7.0)
        M.matvec(xd.data_ptr(), xq.data_ptr(), out.data_ptr(), s, e)
        torch.cuda.synchronize()
        part = out.cpu().numpy()
        assert np.array_equal(part[s:e], got[s:e])
        assert (part[:s] == 7.0).all() and (part[e:] == 7.0).all()
    M.Close()


def _load_gpu(gpu_lib, cfg, T, **kw):
    return gpu_lib.LoadModelFromTensors(gpu_lib.hparams_for(cfg), T, gpu_lib.default_options(**kw))


@pytest.mark.parametrize("name,n_tok", [("tiny", 24), ("tiny-gqa", 24), ("small", 40),
                                        ("small-hd128", 24), ("mid", 16)])
def test_forward_logits_and_kv_parity(gpu_lib, oracle_mod, name, n_tok):
    import synthetic
    cfg, T = synthetic_model(name)
    ctx = min(cfg.ctx_len, 256)
    om = oracle_mod.OracleModel(cfg, T)
    om.new_state(ctx)
    m = _load_gpu(gpu_lib, cfg, T)
    s = m.NewState(ctx)
    ws = m.NewWorkspace(ctx, 40)
    logits = np.empty(cfg.vocab, np.float32)
    worst = 0.0
    for t in synthetic.prompt_ids(cfg, n_tok, seed=11):
        ref = om.forward(int(t))
        m.ForwardIntoWorkspace(s, int(t), logits, ws)
        worst = max(worst, rel_l2(logits, ref))
    assert worst < LOGIT_TOL, worst
    assert s.Pos == n_tok
    # every layer's KV cache: roped K and V at every position
    for layer in range(cfg.n_layers):
        K, V = s.read_kv(layer, 0, n_tok)
        K0, V0 = om.kv(layer, 0, n_tok)
        assert rel_l2(K, K0) < LOGIT_TOL and rel_l2(V, V0) < LOGIT_TOL
    # final hidden state and the last layer's attention / SwiGLU outputs
    assert rel_l2(ws.read(gpu_lib.BUF_HIDDEN, cfg.n_emb), om.buffer("hidden")) < LOGIT_TOL
    assert rel_l2(ws.read(gpu_lib.BUF_ATTN, cfg.n_emb), om.buffer("attn")) < LOGIT_TOL
    assert rel_l2(ws.read(gpu_lib.BUF_FFN_ACT, cfg.n_ff), om.buffer("ffn_act")) < LOGIT_TOL


@pytest.mark.parametrize("name,n_prompt,n_gen", [("small", 8, 48), ("mid", 8, 32)])
def test_greedy_ids_match(gpu_lib, oracle_mod, name, n_prompt, n_gen):
    """Teacher-forced greedy decode: at each step both sides see the same
    token; argmax ids must agree unless the oracle's top-2 gap < 1e-3."""
    import synthetic
    cfg, T = synthetic_model(name)
    ctx = n_prompt + n_gen + 1
    om = oracle_mod.OracleModel(cfg, T)
    om.new_state(ctx)
    m = _load_gpu(gpu_lib, cfg, T)
    s = m.NewState(ctx)
    ws = m.NewWorkspace(ctx, 40)
    prompt = synthetic.prompt_ids(cfg, n_prompt, seed=21)
    for t in prompt[:-1]:
        om.forward(int(t), logits=False)
    m.Prefill(s, prompt[:-1], ws)
    tok = int(prompt[-1])
    mismatches = []
    for step in range(n_gen):
        ref = om.forward(tok)
        got_id, got_logit = m.ForwardArgmax(s, tok, ws)
        ref_id = int(np.argmax(ref))
        top2 = np.sort(ref)[-2:]
        if got_id != ref_id and top2[1] - top2[0] >= GAP_EXEMPT:
            mismatches.append((step, ref_id, got_id, float(top2[1] - top2[0])))
        tok = ref_id
    assert not mismatches, mismatches


def test_long_context_split_attention(gpu_lib, oracle_mod):
    """Positions spread over many attention splits (hd 128, llama3 RoPE
    scaling, a single kv head group of 4)."""
    import synthetic
    cfg, T = synthetic_model("small-hd128")
    n = 1500
    om = oracle_mod.OracleModel(cfg, T)
    om.new_state(n + 8)
    m = _load_gpu(gpu_lib, cfg, T)
    s = m.NewState(n + 8)
    ws = m.NewWorkspace(n + 8, 40)
    ids = synthetic.prompt_ids(cfg, n, seed=4)
    for t in ids[:-4]:
        om.forward(int(t), logits=False)
    m.Prefill(s, ids[:-4], ws)
    logits = np.empty(cfg.vocab, np.float32)
    for t in ids[-4:]:
        ref = om.forward(int(t))
        m.ForwardIntoWorkspace(s, int(t), logits, ws)
        assert rel_l2(logits, ref) < LOGIT_TOL
    K, V = s.read_kv(1, n - 64, 64)
    K0, V0 = om.kv(1, n - 64, 64)
    assert rel_l2(K, K0) < LOGIT_TOL and rel_l2(V, V0) < LOGIT_TOL


def test_fp16_kv_cache(gpu_lib, oracle_mod):
    import synthetic
    cfg, T = synthetic_model("small")
    om = oracle_mod.OracleModel(cfg, T)
    om.new_state(64)
    m = _load_gpu(gpu_lib, cfg, T, kv_dtype=gpu_lib.L3G_KV_F16)
    s = m.NewState(64)
    ws = m.NewWorkspace(64, 40)
    logits = np.empty(cfg.vocab, np.float32)
    for t in synthetic.prompt_ids(cfg, 20, seed=8):
        ref = om.forward(int(t))
        m.ForwardIntoWorkspace(s, int(t), logits, ws)
        assert rel_l2(logits, ref) < LOGIT_TOL


def test_topk_matches_full_logits(gpu_lib, oracle_mod):
    import synthetic
    cfg, T = synthetic_model("small")
    m = _load_gpu(gpu_lib, cfg, T)
    s1, s2 = m.NewState(32), m.NewState(32)
    ws = m.NewWorkspace(32, 40)
    ids = synthetic.prompt_ids(cfg, 6, seed=3)
    logits = np.empty(cfg.vocab, np.float32)
    for t in ids:
        m.ForwardIntoWorkspace(s1, int(t), logits, ws)
    for t in ids[:-1]:
        m.ForwardIntoWorkspace(s2, int(t), None, ws)
    for k in (1, 40, 64):
        s2.Pos = len(ids) - 1
        items = m.ForwardTopKIntoWorkspace(s2, int(ids[-1]), k, ws)
        assert len(items) == k
        order = np.lexsort((np.arange(cfg.vocab), -logits))[:k]
        assert [it.ID for it in items] == order.tolist()
        assert np.array_equal(np.array([it.Logit for it in items], np.float32), logits[order])
    s2.Pos = len(ids) - 1
    nid, nlg = m.ForwardArgmax(s2, int(ids[-1]), ws)
    assert nid == int(np.argmax(logits)) and nlg == logits.max()


def test_determinism_and_rewind(gpu_lib):
    import synthetic
    cfg, T = synthetic_model("tiny-gqa")
    m = _load_gpu(gpu_lib, cfg, T)
    s = m.NewState(32)
    ws = m.NewWorkspace(32, 40)
    ids = synthetic.prompt_ids(cfg, 8, seed=6)
    runs = []
    for _ in range(2):
        s.Pos = 0
        out = np.empty(cfg.vocab, np.float32)
        for t in ids:
            m.ForwardIntoWorkspace(s, int(t), out, ws)
        runs.append(out.copy())
    assert np.array_equal(runs[0], runs[1])


def test_gguf_file_load_matches_tensor_load(gpu_lib, tmp_path):
    import synthetic
    cfg, T = synthetic_model("tiny-gqa")
    path = str(tmp_path / "m.gguf")
    synthetic.write_gguf(path, cfg, T)
    m1 = gpu_lib.LoadModel(path)
    m2 = _load_gpu(gpu_lib, cfg, T)
    assert m1.HP.NEmb == cfg.n_emb and m1.HP.VocabSize == cfg.vocab
    outs = []
    for m in (m1, m2):
        s = m.NewState(16)
        ws = m.NewWorkspace(16, 40)
        lg = np.empty(cfg.vocab, np.float32)
        for t in synthetic.prompt_ids(cfg, 5, seed=1):
            m.ForwardIntoWorkspace(s, int(t), lg, ws)
        outs.append(lg.copy())
    assert np.array_equal(outs[0], outs[1])


def test_error_paths(gpu_lib):
    import synthetic
    cfg, T = synthetic_model("tiny")
    m = _load_gpu(gpu_lib, cfg, T)
    s = m.NewState(3)
    ws = m.NewWorkspace(3, 40)
    with pytest.raises(gpu_lib.L3GError, match="token out of range: 97") as e:
        m.ForwardIntoWorkspace(s, cfg.vocab, None, ws)
    assert e.value.code == gpu_lib.L3G_E_TOKEN
    for t in (1, 2, 3):
        m.ForwardIntoWorkspace(s, t, None, ws)
    with pytest.raises(gpu_lib.L3GError, match=r"context length exceeded \(3\)") as e:
        m.ForwardIntoWorkspace(s, 1, None, ws)
    assert e.value.code == gpu_lib.L3G_E_CTX
    big = m.NewState(8)
    small_ws = m.NewWorkspace(4, 40)
    with pytest.raises(gpu_lib.L3GError, match="workspace ctxLen=4 < state ctxLen=8"):
        m.ForwardIntoWorkspace(big, 1, None, small_ws)
    with pytest.raises(gpu_lib.L3GError, match="logitsOut len"):
        m.ForwardIntoWorkspace(big, 1, np.empty(5, np.float32), m.NewWorkspace(8, 40))
    # missing tensor
    T2 = dict(T)
    del T2["blk.1.ffn_down.weight"]
    with pytest.raises(gpu_lib.L3GError, match='missing tensor "blk.1.ffn_down.weight"'):
        _load_gpu(gpu_lib, cfg, T2)


def test_bounded_wait_reports_and_context_survives(gpu_lib):
    """A wait that nothing completes gives up after its limit, reports an
    error status, and the CUDA context stays usable."""
    import torch
    assert gpu_lib.selftest_bounded_wait(-1, 2000) == gpu_lib.L3G_E_DEVICE
    x = torch.ones(64, device="cuda")
    d = torch.empty(2, device="cuda")
    q = torch.empty(64, dtype=torch.int8, device="cuda")
    gpu_lib.quantize_q8_0_device(x.data_ptr(), 64, d.data_ptr(), q.data_ptr())
    torch.cuda.synchronize()
    assert (q.cpu().numpy() == 127).all()
