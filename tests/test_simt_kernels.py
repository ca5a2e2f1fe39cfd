"""Device kernels run on the CPU under the SIMT emulator (tests/simt/): the
kernels' own source, built for the host with software versions of the
inline-PTX helpers, every CUDA thread a coroutine (tests/simt/simt.h).

Covered here, against the oracle and the reference's loops:
- the persistent decode step (k_layers: every layer of a token in one
  launch, grid barriers between the phases, one producer warp per CTA
  streaming weight tiles and K|V stages through a bulk-copy ring): hidden
  state, last-layer attention output and the appended K/V of every layer
  against the oracle (the reference's Go forward restated, linked to its
  simd.c), for head sizes 32, 64 and 128, query heads per kv head 2 and 3,
  1 to 4 attention splits with several stages each, f32 and f16 caches;
  bit-identical across random schedules and copy delays, with and without
  the fused SwiGLU act-quant, with spread barrier counters and a two-slot
  ring; and the abort path when a CTA never arrives;
- the top-K path's fastExp attention (k_attf_scores / values / merge)
  against the reference's loop (infer.go:376-423);
- the batched Q8_0 product on the tensor cores (k_gemm_quantize, k_gemm_q8,
  k_gemm_reduce) on a software model of tcgen05 (tests/simt/simt_tcgen05.h:
  tensor memory, asynchronous kind::i8 MMAs reading canonical K-major
  shared-memory operands through their descriptors, commits to mbarriers,
  32x32b loads): every token's row against the reference's own matvec_q8_c
  (simd.c), for ragged rows and columns, one to two token tiles of 16 to
  128, K split over 2 to 4 CTAs, short rings and random schedules;
- batched prefill (every kernel of a pass, launched in the runtime's order)
  against the oracle's token-by-token ingest, and batched decode of
  sessions at different positions against the oracle's forward per session
  and the host restatement of SampleTopK.

What the emulator does not check: the hardware memory model (one OS thread
runs every coroutine, so memory is sequentially consistent), timing, and
whether the hardware reads the tensor-core descriptors as the model does
(the encodings themselves are checked against CUTLASS in test_gemm_layout).
"""
import dataclasses
import os

import numpy as np
import pytest

from conftest import synthetic_model
from refspread import rel_l2


@pytest.fixture(scope="module")
def S():
    import simt_lib
    simt_lib.lib()
    simt_lib.lib().emu_schedule(0, 0, 0)
    return simt_lib


def _model(name, ctx):
    cfg, T = synthetic_model(name)
    if ctx > cfg.ctx_len:
        cfg = dataclasses.replace(cfg, ctx_len=ctx)
    return cfg, T


def _oracle_after(oracle_mod, cfg, T, ids, ctx):
    om = oracle_mod.OracleModel(cfg, T)
    om.new_state(ctx)
    for t in ids:
        om.forward(int(t), logits=False)
    return om


# (config, prefix positions, tokens stepped, grid, kv f16, step options)
CASES = [
    ("tiny-gqa", 0, 3, 4, False, {}),                       # hd 32, G 2, one split
    ("tiny-gqa", 600, 2, 8, False, {}),                     # 4 splits x 2 stages
    ("tiny-g3", 300, 2, 5, False, {}),                      # G 3 (padded to 4)
    ("small", 200, 2, 6, False, {"fuse_quant": 1}),         # hd 64, fused act-quant
    ("tiny-gqa", 600, 2, 8, False, {"fuse_merge": 1}),      # merge in the attention phase
    ("small", 200, 2, 6, False, {"fuse_quant": 1, "fuse_merge": 1}),
    ("small-hd128", 100, 2, 3, False, {}),                  # hd 128, one kv head
    ("tiny-gqa", 260, 2, 7, False, {"max_stages": 2, "nsub": 4}),
    ("small", 100, 2, 6, True, {}),                         # f16 cache
]


@pytest.mark.parametrize("name,prefix,n,grid,f16,kw", CASES)
def test_persistent_step_matches_oracle(S, oracle_mod, name, prefix, n, grid, f16, kw):
    import synthetic
    ctx = prefix + n + 3
    cfg, T = _model(name, ctx)
    ids = synthetic.prompt_ids(cfg, prefix + n, seed=3)
    om = _oracle_after(oracle_mod, cfg, T, ids[:prefix], ctx)
    pm = S.PersistentModel(cfg, T, ctx, grid, kv_f16=f16)
    if prefix:
        K, V = om.kv_arrays()
        pm.load_kv(K, V, prefix)
    # f16 storage rounds every K/V value: the bar of the GPU tests for it
    tol = 2e-2 if f16 else 1e-5
    for pos in range(prefix, prefix + n):
        hidden, rec = pm.step(ids[pos], pos, **kw)
        assert rec.err == 0, (rec.err, rec.where)
        om.forward(int(ids[pos]), logits=False)
        assert rel_l2(hidden, om.buffer("hidden")) < tol
        assert rel_l2(pm.attn.read(np.float32), om.buffer("attn")) < max(tol, 2e-3 if f16 else 0)
        K, V = om.kv_arrays()
        K = K.reshape(cfg.n_layers, ctx, cfg.n_heads_kv, cfg.head_dim)[:, pos]
        V = V.reshape(cfg.n_layers, ctx, cfg.n_heads_kv, cfg.head_dim)[:, pos]
        kv = pm.read_kv()[:, :, pos]
        assert rel_l2(kv[:, :, 0], K) < tol
        assert rel_l2(kv[:, :, 1], V) < tol
    if "max_splits" not in kw and prefix >= 200:
        assert rec.splits > 1  # the split merge is exercised
    pm.close()
    om.close()


def _run_steps(S, cfg, T, ctx, grid, ids, prefix_kv, **kw):
    pm = S.PersistentModel(cfg, T, ctx, grid)
    pm.load_kv(*prefix_kv)
    out = [pm.step(ids[p], p, **kw)[0] for p in range(prefix_kv[2], len(ids))]
    kv = pm.read_kv()
    pm.close()
    return np.array(out), kv


def test_persistent_step_is_bit_identical_across_schedules(S, oracle_mod):
    """Random thread orders and bulk-copy delays, the fused act-quant, the
    fused merge, spread barrier counters and a short ring change no bit of
    the result."""
    import synthetic
    cfg, T = _model("tiny-g3", 160)
    ctx = 160
    ids = synthetic.prompt_ids(cfg, 152, seed=9)
    om = _oracle_after(oracle_mod, cfg, T, ids[:150], ctx)
    K, V = om.kv_arrays()
    prefix_kv = (K.copy(), V.copy(), 150)
    om.close()
    try:
        S.lib().emu_schedule(0, 0, 0)
        base_h, base_kv = _run_steps(S, cfg, T, ctx, 5, ids, prefix_kv)
        variants = [(1, {"fuse_quant": 1}), (2, {"nsub": 3, "max_stages": 3}),
                    (3, {"fuse_quant": 1, "nsub": 2, "max_stages": 2}),
                    (4, {"fuse_merge": 1}), (5, {"fuse_quant": 1, "fuse_merge": 1, "max_stages": 2})]
        for seed, kw in variants:
            S.lib().emu_schedule(1, seed, 64)
            h, kv = _run_steps(S, cfg, T, ctx, 5, ids, prefix_kv, **kw)
            assert np.array_equal(h, base_h), (seed, kw)
            assert np.array_equal(kv, base_kv), (seed, kw)
    finally:
        S.lib().emu_schedule(0, 0, 0)


def test_persistent_step_abort_when_a_cta_never_arrives(S):
    """One CTA of the plan's grid is not launched: the others' bounded grid
    barrier waits give up, the step reports a timeout, and every CTA exits
    with no bulk copy in flight (the emulator fails the launch otherwise)."""
    import synthetic
    cfg, T = _model("tiny-gqa", 40)
    pm = S.PersistentModel(cfg, T, 40, 4)
    ids = synthetic.prompt_ids(cfg, 2, seed=1)
    _, rec = pm.step(ids[0], 0, launch_grid=3, wait_ns=200000)
    assert rec.err == 1  # ERR_TIMEOUT
    # the next step, with every CTA present, is unaffected by the aborted one
    # (the barrier words start from zero each step, as k_embed leaves them)
    _, rec = pm.step(ids[0], 0)
    assert rec.err == 0
    pm.close()


@pytest.mark.parametrize("G,hd,hkv,n,splits,f16", [(4, 64, 2, 37, 5, False), (1, 32, 3, 100, 7, False),
                                                   (3, 128, 1, 260, 4, False), (8, 64, 1, 9, 3, True),
                                                   (2, 128, 2, 1, 6, False)])
def test_fast_exp_attention_kernels(S, G, hd, hkv, n, splits, f16):
    from test_topk_fast_attention import fast_exp_kernel, reference_head
    rng = np.random.default_rng(G * 1000 + n)
    ctx = S.kv_len(n + 4)  # a whole number of KV pages
    q = rng.standard_normal((hkv * G, hd)).astype(np.float32)
    kv = rng.standard_normal((hkv, ctx, 2, hd)).astype(np.float32)
    if f16:
        kv = kv.astype(np.float16).astype(np.float32)
    dq = S.Dev(q)
    dkv = S.Dev(kv.astype(np.float16) if f16 else kv)
    io = S.Dev(np.array([0, n - 1, 0, 0], np.int32))
    bufs = [S.Dev(hkv * G * ctx * 4), S.Dev(hkv * splits * G * 4), S.Dev(hkv * splits * G * 4),
            S.Dev(hkv * splits * G * hd * 4), S.Dev(hkv * G * hd * 4), S.Dev(hkv * G * hd // 32 * 4),
            S.Dev(hkv * G * hd)]
    S.check(S.lib().emu_attf(dq.ptr, dkv.ptr, ctx, hd, G, hkv, splits, 1 if f16 else 0, io.ptr,
                             *[b.ptr for b in bufs]))
    got = bufs[4].read(np.float32).reshape(hkv * G, hd)
    scale = np.float32(1.0 / np.sqrt(hd))
    for h in range(hkv * G):
        g = h // G
        want = reference_head(q[h], kv[g, :n, 0], kv[g, :n, 1], scale, fast_exp_kernel)
        assert rel_l2(got[h], want) < 2e-6, h
    # the act-quant for Wo is QuantizeQ8_0Into of the output, bit for bit
    import oracle
    d0, q0 = oracle.quantize_q8_0(bufs[4].read(np.float32))
    assert np.array_equal(bufs[5].read(np.float32), d0)
    assert np.array_equal(bufs[6].read(np.int8), q0)
    for b in [dq, dkv, io] + bufs:
        b.free()


@pytest.mark.parametrize("world,grid,prefix", [(2, 4, 0), (4, 5, 150)])
def test_persistent_step_tensor_parallel(S, oracle_mod, world, grid, prefix):
    """`world` ranks of the persistent step in one emulated launch: each holds
    its shard as the library's shard plan cuts it, pushes its Wo / down rows
    into every rank's receive buffer with the step's epochs and sums the
    ranks' rows in rank order.  Every rank ends with the same hidden state,
    within 1e-5 of the oracle; a random schedule with both fusions gives the
    same bits."""
    import synthetic
    ctx = prefix + 2 + 3
    # 8 query heads over 4 kv heads, so that 4 ranks hold one kv head each
    cfg = synthetic.Config("tp-4kv", 256, 2, 8, 4, 512, 300, tied=True, ctx_len=max(64, ctx))
    T = synthetic.make_model(cfg, seed=0)
    ids = synthetic.prompt_ids(cfg, prefix + 2, seed=4)
    om = _oracle_after(oracle_mod, cfg, T, ids[:prefix], ctx)
    K, V = om.kv_arrays()
    K, V = K.copy(), V.copy()

    def run(**kw):
        ms = [S.PersistentModel(cfg, T, ctx, grid, world=world, rank=r) for r in range(world)]
        for m in ms:
            m.load_kv(K, V, prefix)
        out = []
        for i, pos in enumerate(range(prefix, prefix + 2)):
            hs, recs = S.step_tp(ms, ids[pos], pos, step_count=i + 1, **kw)
            assert all(r.err == 0 for r in recs), [(r.err, r.where) for r in recs]
            assert all(np.array_equal(hs[0], h) for h in hs)
            out.append(hs[0])
        for m in ms:
            m.close()
        return np.array(out)

    try:
        S.lib().emu_schedule(0, 0, 0)
        got = run()
        for i, pos in enumerate(range(prefix, prefix + 2)):
            om.forward(int(ids[pos]), logits=False)
            assert rel_l2(got[i], om.buffer("hidden")) < 1e-5, i
        S.lib().emu_schedule(1, 11, 64)
        assert np.array_equal(run(fuse_merge=1, fuse_quant=1), got)
    finally:
        S.lib().emu_schedule(0, 0, 0)
        om.close()


GEMM_CASES = [  # rows, cols, tokens, K split, grid (0: one CTA per unit), ring stages (0: full)
    (200, 96, 1, 1, 0, 0), (384, 160, 17, 1, 0, 0), (130, 512, 40, 2, 0, 0),
    (256, 1024, 64, 4, 3, 0), (129, 256, 65, 1, 0, 0), (256, 384, 100, 3, 0, 0),
    (128, 128, 128, 1, 0, 0), (300, 256, 130, 2, 2, 2),
]


def _gemm(S, w, x, rows, cols, ksplit, grid, nstages):
    import ctypes as C
    import l3g
    n_tok = x.shape[0]
    A = S.Dev(l3g.gemm_repack(w, rows, cols))
    X = S.Dev(x)
    act = S.Dev(l3g.gemm_act_bytes(n_tok, cols))
    out = S.Dev(n_tok * rows * 4)
    part = S.Dev(max(1, ksplit) * n_tok * rows * 4)
    S.check(S.lib().emu_gemm_quantize(X.ptr, n_tok, cols, act.ptr))
    err, where = C.c_int(), C.c_int()
    S.check(S.lib().emu_gemm(A.ptr, rows, cols, act.ptr, n_tok, out.ptr, ksplit, part.ptr, grid,
                             nstages, C.byref(err), C.byref(where)))
    got = out.read(np.float32).reshape(n_tok, rows)
    for d in (A, X, act, out, part):
        d.free()
    return got, err.value


@pytest.mark.parametrize("rows,cols,n_tok,ksplit,grid,nstages", GEMM_CASES)
def test_tensor_core_product_matches_reference_simd(S, oracle_mod, rows, cols, n_tok, ksplit, grid,
                                                    nstages):
    import synthetic
    import torch
    if not oracle_mod.have_ref_simd():
        pytest.fail("oracle/_ref/libref_simd.so (the reference's simd.c) is missing")
    g = torch.Generator().manual_seed(rows * 7 + cols)
    w = synthetic.quantize_q8_0_rows(torch.randn(rows, cols, generator=g) * 0.02, torch).numpy()
    x = np.random.default_rng(n_tok).standard_normal((n_tok, cols)).astype(np.float32)
    got, err = _gemm(S, w, x, rows, cols, ksplit, grid, nstages)
    assert err == 0
    for n in range(n_tok):
        d0, q0 = oracle_mod.quantize_q8_0(x[n])
        ref = oracle_mod.ref_matvec_q8(w, d0, q0, rows, cols)
        assert rel_l2(got[n], ref) < 1e-6, n


def test_tensor_core_product_is_bit_identical_across_schedules(S):
    import synthetic
    import torch
    rows, cols = 256, 512
    g = torch.Generator().manual_seed(3)
    w = synthetic.quantize_q8_0_rows(torch.randn(rows, cols, generator=g) * 0.02, torch).numpy()
    x = np.random.default_rng(4).standard_normal((33, cols)).astype(np.float32)
    try:
        S.lib().emu_schedule(0, 0, 0)
        base, _ = _gemm(S, w, x, rows, cols, 2, 0, 2)
        for seed in (5, 6):
            S.lib().emu_schedule(1, seed, 64)
            assert np.array_equal(_gemm(S, w, x, rows, cols, 2, 0, 2)[0], base)
    finally:
        S.lib().emu_schedule(0, 0, 0)



PREFILL_CASES = [  # config, first pass, second pass, rows per warp of the decode tiles, f16 cache
    ("tiny-gqa", 40, 25, 1, False),
    ("tiny-g3", 130, 0, 2, False),   # two token tiles of 128
    ("small", 70, 30, 8, False),
    ("small-hd128", 33, 20, 4, True),
]


@pytest.mark.parametrize("name,p1,p2,rpw,f16", PREFILL_CASES)
def test_batched_prefill_matches_token_by_token_ingest(S, oracle_mod, name, p1, p2, rpw, f16):
    """Batched prefill (one or two passes, launched as the runtime's
    enqueue_prefill_pass launches them: embedding, RMSNorm + act-quant rows,
    tensor-core products on weight chunks built by k_gemm_from_tiles from the
    decode tiles, RoPE + KV append, causal attention over the cache, SwiGLU
    + act-quant) leaves the KV cache the oracle's token-by-token ingest
    leaves: layer 0 within 1e-6 (the same quantization and exact block
    sums; fp32 sums in another order), deeper layers within the band of
    int8 rounding flips."""
    import synthetic
    ctx = p1 + p2 + 4
    cfg, T = _model(name, ctx)
    ids = synthetic.prompt_ids(cfg, p1 + p2, seed=5)
    om = _oracle_after(oracle_mod, cfg, T, ids, ctx)
    K, V = om.kv_arrays()
    K = K.reshape(cfg.n_layers, ctx, cfg.n_heads_kv, cfg.head_dim).copy()
    V = V.reshape(cfg.n_layers, ctx, cfg.n_heads_kv, cfg.head_dim).copy()
    om.close()  # its K, V views die with it: copied above
    pm = S.PrefillModel(cfg, T, ctx, rpw=rpw, kv_f16=f16)
    assert pm.prefill(ids[:p1], 0).err == 0
    if p2:
        assert pm.prefill(ids[p1:], p1).err == 0
    kv = pm.read_kv()
    pm.close()
    n = p1 + p2
    for l in range(cfg.n_layers):
        tol = (2e-3 if l == 0 else 3e-2) if f16 else (1e-6 if l == 0 else 5e-3)
        assert rel_l2(kv[l, :, :n, 0].transpose(1, 0, 2), K[l, :n]) < tol, l
        assert rel_l2(kv[l, :, :n, 1].transpose(1, 0, 2), V[l, :n]) < tol, l


BATCH_CASES = [  # config, session prompt lengths, context, f16 cache
    ("tiny-g3", [1, 5, 40, 90], 128, False),
    ("small", [3, 17, 100, 300, 507], 512, False),   # 1 and 2 attention splits of 256
    ("small", [7, 120, 260], 512, True),
]


@pytest.mark.parametrize("name,lens,ctx,f16", BATCH_CASES)
def test_batched_decode_step_matches_oracle_and_sampler(S, oracle_mod, name, lens, ctx, f16):
    """Batched decode of sessions at different positions (launched as the
    runtime's l3g_batch_step launches it): each session's logits equal the
    oracle's ForwardIntoWorkspace on that session's cache, and each sampled id
    is SampleTopK restated on the host (tests/sampler_ref.py) over the top-K
    of those logits with the Philox draw keyed by the session's seed and
    counted by its position; two steps, the second fed the first's picks."""
    import synthetic
    from sampler_ref import sample_topk
    cfg, T = _model(name, ctx)
    bm = S.BatchModel(cfg, T, ctx, kv_f16=f16)
    oms, caches = [], []
    for i, L in enumerate(lens):
        om = _oracle_after(oracle_mod, cfg, T, synthetic.prompt_ids(cfg, L, seed=100 + i), ctx)
        K, V = om.kv_arrays()
        c = bm.new_cache()
        S.load_session_kv(c, cfg, ctx, K, V, L, f16)
        oms.append(om)
        caches.append(c)
    rng = np.random.default_rng(7)
    seeds = [int(x) for x in rng.integers(1, 2**62, len(lens))]
    tokens = [int(t) for t in rng.integers(0, cfg.vocab, len(lens))]
    pos = list(lens)
    tol = 3e-2 if f16 else 1e-3
    for _ in range(2):
        lg, nxt, rec = bm.step(caches, pos, tokens, seeds, top_k=40, temperature=1.3)
        assert rec.err == 0
        for i in range(len(lens)):
            assert rel_l2(lg[i], oms[i].forward(tokens[i])) < tol, i
            order = np.lexsort((np.arange(cfg.vocab), -lg[i].astype(np.float64)))[:40]
            assert nxt[i] == sample_topk(order, lg[i][order], 1.3, seeds[i], pos[i]), i
        tokens, pos = nxt, [p + 1 for p in pos]
    for om in oms:
        om.close()
    bm.close()


@pytest.mark.skipif(os.environ.get("L3G_SIMT_SLOW") != "1",
                    reason="about 3 minutes and 6 GB of host memory (set L3G_SIMT_SLOW=1)")
@pytest.mark.parametrize("fuse", [0, 1])
def test_persistent_step_at_the_8b_layer_shapes(S, oracle_mod, fuse):
    """The persistent step at the Llama-3.1-8B layer shapes (two layers),
    planned for 148 SMs as on a B200: multi-slice tiles, 8 kv heads of 4
    query heads, 10 attention splits of 32-position stages over 300 cached
    positions.  The hidden state and the appended K/V lie within the band by
    which the reference's own builds (cgo simd.c and pure Go) differ on the
    same step."""
    import synthetic
    cfg, T = synthetic_model("llama3.1-8b-2l")
    prefix, ctx = 300, 304
    ids = synthetic.prompt_ids(cfg, prefix + 1, seed=3)
    cgo = _oracle_after(oracle_mod, cfg, T, ids[:prefix], ctx)
    K, V = cgo.kv_arrays()
    K, V = K.copy(), V.copy()
    pure = oracle_mod.OracleModel(cfg, T)
    pure.new_state(ctx)
    Kp, Vp = pure.kv_arrays()
    Kp[:], Vp[:] = K, V
    pure.pos = prefix
    pm = S.PersistentModel(cfg, T, ctx, 148)
    pm.load_kv(K, V, prefix)
    hidden, rec = pm.step(ids[prefix], prefix, fuse_quant=fuse, fuse_merge=fuse)  # both folds or none
    assert rec.err == 0 and rec.splits == 10
    cgo.forward(int(ids[prefix]), logits=False)
    pure.forward(int(ids[prefix]), logits=False, use_ref=False)
    band = rel_l2(pure.buffer("hidden"), cgo.buffer("hidden"))
    assert rel_l2(hidden, cgo.buffer("hidden")) <= max(1e-5, 1.5 * band)
    kv = pm.read_kv()
    Kc = cgo.kv_arrays()[0].reshape(cfg.n_layers, ctx, cfg.n_heads_kv, cfg.head_dim)
    Kq = pure.kv_arrays()[0].reshape(cfg.n_layers, ctx, cfg.n_heads_kv, cfg.head_dim)
    for l in range(cfg.n_layers):
        kband = rel_l2(Kq[l, prefix], Kc[l, prefix])
        assert rel_l2(kv[l, :, prefix, 0], Kc[l, prefix]) <= max(1e-5, 1.5 * kband), l
    pm.close()
    cgo.close()
    pure.close()


def test_persistent_step_multi_slice_tiles(S, oracle_mod):
    """The 1B layer shapes (two layers): rows of 2048 and 8192 columns are
    cut into 2 and 8 column slices of 1024 per tile, so every row group
    takes several tiles of the ring.  On a step where no int8 rounding flips
    between the builds (checked: the reference's cgo and pure-Go builds
    agree to 1e-6 there) the hidden state and the appended K/V match the
    oracle within 1e-5."""
    import synthetic
    cfg, T = synthetic_model("llama3.2-1b-2l")
    assert S.tile_geometry(cfg.n_emb, cfg.n_ff)["nslices"] == 8
    prefix, ctx = 33, 37
    ids = synthetic.prompt_ids(cfg, prefix + 1, seed=prefix)
    cgo = _oracle_after(oracle_mod, cfg, T, ids[:prefix], ctx)
    K, V = cgo.kv_arrays()
    K, V = K.copy(), V.copy()
    pure = oracle_mod.OracleModel(cfg, T)
    pure.new_state(ctx)
    Kp, Vp = pure.kv_arrays()
    Kp[:], Vp[:] = K, V
    pure.pos = prefix
    pm = S.PersistentModel(cfg, T, ctx, 12)
    pm.load_kv(K, V, prefix)
    hidden, rec = pm.step(ids[prefix], prefix)
    assert rec.err == 0
    cgo.forward(int(ids[prefix]), logits=False)
    pure.forward(int(ids[prefix]), logits=False, use_ref=False)
    assert rel_l2(pure.buffer("hidden"), cgo.buffer("hidden")) < 1e-6  # a flip-free step
    assert rel_l2(hidden, cgo.buffer("hidden")) < 1e-5
    kv = pm.read_kv()
    Kc = cgo.kv_arrays()[0].reshape(cfg.n_layers, ctx, cfg.n_heads_kv, cfg.head_dim)
    for l in range(cfg.n_layers):
        assert rel_l2(kv[l, :, prefix, 0], Kc[l, prefix]) < 1e-5, l
    pm.close()
    cgo.close()
    pure.close()


@pytest.mark.parametrize("rows,cols,rpw,lo,hi", [(4096, 512, 4, 0, 4096), (37, 96, 1, 0, 37),
                                                 (2050, 1792, 2, 0, 2050), (513, 2048, 8, 100, 400)])
def test_decode_matvec_matches_reference_simd(S, oracle_mod, rows, cols, rpw, lo, hi):
    """The decode step's k_matvec (the kernel measured on the B200, and
    tested there against the same reference) under the emulator: rows
    [lo, hi) equal the reference's matvec_q8_c (simd.c) within 1e-6, the
    other rows untouched -- a check of the emulator on a kernel whose GPU
    results are known."""
    import synthetic
    import torch
    g = torch.Generator().manual_seed(rows * 7 + cols)
    w = synthetic.quantize_q8_0_rows(torch.randn(rows, cols, generator=g) * 0.02, torch).numpy()
    x = np.random.default_rng(rows).standard_normal(cols).astype(np.float32)
    d0, q0 = oracle_mod.quantize_q8_0(x)
    ref = oracle_mod.ref_matvec_q8(w, d0, q0, rows, cols)
    raw = S.Dev(w)
    tiles = S.repack([(raw, 0, rows)], cols, rows, rpw=rpw)
    xd, xq = S.Dev(d0), S.Dev(q0)
    out = S.Dev(np.full(rows, 7.0, np.float32))
    S.check(S.lib().emu_matvec(tiles.ptr, rows, cols, rpw, xd.ptr, xq.ptr, out.ptr, lo, hi, 148))
    got = out.read(np.float32)
    assert rel_l2(got[lo:hi], ref[lo:hi]) < 1e-6
    assert (got[:lo] == 7.0).all() and (got[hi:] == 7.0).all()
    for d in (raw, tiles, xd, xq, out):
        d.free()


@pytest.mark.parametrize("n,threads", [(2048, 256), (2048, 512), (4096, 1024), (4096, 256),
                                       (64, 256), (512, 1024), (256, 256), (1024, 64)])
def test_bitonic_sort_of_topk_keys(S, n, threads):
    """bitonic_desc, the sort of every top-K kernel, under the emulator: n
    unique keys (ordered logit bits, inverted id, as the top-K kernels build
    them) come out in descending order, whether warps sort their own
    segments between block barriers (n a multiple of the block, 32 or more
    keys per warp) or every step is block-wide (the others)."""
    rng = np.random.default_rng(n * 7 + threads)
    ids = rng.permutation(n).astype(np.uint64)
    vals = rng.integers(0, 2**31, n, dtype=np.uint64)
    vals[: n // 8] = vals[0]  # ties in value, broken by the id
    keys = (vals << np.uint64(32)) | (~ids & np.uint64(0xFFFFFFFF))
    d = S.Dev(keys)
    S.check(S.lib().emu_bitonic(d.ptr, n, threads))
    got = d.read(np.uint64)
    assert np.array_equal(got, np.sort(keys)[::-1])
    d.free()


@pytest.mark.parametrize("G,hd,hkv,n,f16,nsm,ns", [
    (4, 128, 2, 700, False, 148, 4), (3, 64, 2, 37, False, 148, 4), (2, 32, 3, 300, False, 148, 6),
    (4, 128, 1, 90, True, 148, 4), (4, 128, 2, 700, False, 8, 4), (2, 64, 2, 600, False, 2, 6),
    (4, 128, 2, 500, False, 4, 3)])
def test_decode_attention_matches_exact_softmax(S, G, hd, hkv, n, f16, nsm, ns):
    """The decode step's k_attention (measured on the B200) under the
    emulator: split-K over the cache with the distributed global merge (the
    CTAs of a kv head wait on each other's arrival counters, which must come
    back to zero), against the reference's exact-exp loop (infer.go:130-175)
    in float64, and its act-quant for Wo bit for bit; rings of 3, 4 (the
    one-GPU default) and 6 stages (the tensor-parallel default), with few
    SMs so that a split streams many stages through the ring."""
    import oracle
    rng = np.random.default_rng(G * 100 + n)
    ctx = S.kv_len(n + 5)  # a whole number of KV pages
    q = rng.standard_normal((hkv * G, hd)).astype(np.float32)
    kv = rng.standard_normal((hkv, ctx, 2, hd)).astype(np.float32)
    if f16:
        kv = kv.astype(np.float16).astype(np.float32)
    dq, dkv = S.Dev(q), S.Dev(kv.astype(np.float16) if f16 else kv)
    io = S.Dev(np.array([0, n - 1, 0, 0], np.int32))
    out, od, oq = S.Dev(hkv * G * hd * 4), S.Dev(hkv * G * hd // 32 * 4), S.Dev(hkv * G * hd)
    import ctypes as C
    splits = C.c_int()
    S.check(S.lib().emu_attention(dq.ptr, dkv.ptr, ctx, hd, G, hkv, 1 if f16 else 0, io.ptr, out.ptr,
                                  od.ptr, oq.ptr, nsm, ns, C.byref(splits)))
    if nsm < 148:  # every split streams more stages than its ring holds
        P = 8
        while P * 2 <= min(S.KV_PAGE, 32768 // (2 * hd * (2 if f16 else 4))):
            P *= 2
        assert -(-n // splits.value) > ns * P
    got = out.read(np.float32).reshape(hkv * G, hd)
    scale = np.float32(1.0 / np.sqrt(hd))
    for h in range(hkv * G):
        g = h // G
        s = (kv[g, :n, 0].astype(np.float64) @ q[h].astype(np.float64)) * float(scale)
        w = np.exp(s - s.max())
        want = (w / w.sum()) @ kv[g, :n, 1].astype(np.float64)
        assert rel_l2(got[h], want) < 1e-5, h
    d0, q0 = oracle.quantize_q8_0(out.read(np.float32))
    assert np.array_equal(od.read(np.float32), d0) and np.array_equal(oq.read(np.int8), q0)
    for d in (dq, dkv, io, out, od, oq):
        d.free()
