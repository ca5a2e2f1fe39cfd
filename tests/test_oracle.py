"""CPU tests of the oracle (the C restatement of llama3.go's decode path and
the reference's own simd.c): known answers for the scalar pieces, agreement of
the restatement with the reference kernels, and a cross-check of the whole
forward against an independent float64 numpy implementation."""
import math
import struct

import numpy as np
import pytest

from conftest import synthetic_model


def f32(x):
    return np.float32(x)


def quant_f32_restated(x):
    """QuantizeQ8_0Into (q8_0.go:22-79) in numpy float32, operation by
    operation, for bit-exact comparison."""
    x = np.asarray(x, np.float32)
    n = x.size
    nb = (n + 31) // 32
    d = np.empty(nb, np.float32)
    q = np.zeros(nb * 32, np.int8)
    for b in range(nb):
        blk = x[b * 32:(b + 1) * 32]
        m = np.float32(0)
        for v in blk:
            av = -v if v < 0 else v
            if av > m:
                m = av
        s = np.float32(m / np.float32(127.0))
        if s == 0:
            s = np.float32(1e-8)
        d[b] = s
        inv = np.float32(np.float32(1.0) / s)
        for i in range(32):
            v = blk[i] if i < blk.size else np.float32(0)
            fv = np.float32(v * inv)
            qi = int(np.float32(fv + f32(0.5))) if fv >= 0 else int(np.float32(fv - f32(0.5)))
            q[b * 32 + i] = max(-128, min(127, qi))
    return d, q


def test_quantize_known_answers(oracle_mod):
    # all-zero block -> scale 1e-8, q = 0 (q8_0.go:53-55)
    d, q = oracle_mod.quantize_q8_0(np.zeros(32, np.float32))
    assert d[0] == np.float32(1e-8) and not q.any()
    # maxabs maps to +-127; exact halves round away from zero
    x = np.zeros(32, np.float32)
    x[0], x[1], x[2], x[3] = 127.0, -127.0, 63.5, -63.5
    d, q = oracle_mod.quantize_q8_0(x)
    assert d[0] == 1.0
    assert list(q[:4]) == [127, -127, 64, -64]
    # ragged tail: the last block is padded with zeros (q8_0.go:58-63)
    d, q = oracle_mod.quantize_q8_0(np.arange(1, 41, dtype=np.float32))
    assert d.size == 2 and q.size == 64 and not q[40:].any()


def test_quantize_matches_float32_restatement(oracle_mod):
    rng = np.random.default_rng(0)
    for scale in (1.0, 1e-3, 40.0):
        x = (rng.standard_normal(320) * scale).astype(np.float32)
        d0, q0 = oracle_mod.quantize_q8_0(x)
        d1, q1 = quant_f32_restated(x)
        assert np.array_equal(d0, d1) and np.array_equal(q0, q1)


def test_f16_decode_known_answers(oracle_mod):
    f = oracle_mod.f16_to_f32
    assert f(0x3C00) == 1.0
    assert f(0xC000) == -2.0
    assert f(0x0001) == pytest.approx(2.0 ** -24)          # subnormal, float16.go:20-29
    assert f(0x03FF) == pytest.approx(1023 * 2.0 ** -24)
    assert math.isinf(f(0x7C00)) and f(0x7C00) > 0
    assert math.isinf(f(0xFC00)) and f(0xFC00) < 0
    assert math.isnan(f(0x7E00))
    assert math.copysign(1.0, f(0x8000)) == -1.0
    for bits in range(0, 0x7C00, 97):
        assert f(bits) == float(np.array([bits], np.uint16).view(np.float16)[0])


def _fast_exp_emulated(x):
    prod = np.float32(np.float32(x) * np.float32(12102203))
    t = int(prod)  # truncation toward zero through int64
    bits = ((t & 0xFFFFFFFF) + 1064866816) & 0xFFFFFFFF
    return struct.unpack("<f", struct.pack("<I", bits))[0]


def test_fast_exp_formula(oracle_mod):
    for x in (0.0, -0.5, -1.0, -3.25, -10.0, -50.0, -87.0):
        assert oracle_mod.fast_exp(x) == _fast_exp_emulated(x)
        assert abs(oracle_mod.fast_exp(x) - math.exp(x)) <= 0.07 * math.exp(x) + 1e-30
    # below about -88 the Go conversion wraps the bits (infer.go:520-525)
    assert oracle_mod.fast_exp(-100.0) == _fast_exp_emulated(-100.0)


def test_silu_and_rmsnorm(oracle_mod):
    for x in (-8.0, -1.0, 0.0, 0.3, 5.0):
        want = np.float32(np.float32(x) / (np.float32(1.0) + np.float32(math.exp(-x))))
        assert oracle_mod.silu(x) == want
    x = np.linspace(-2, 3, 64).astype(np.float32)
    w = np.linspace(0.5, 1.5, 64).astype(np.float32)
    got = oracle_mod.rmsnorm(x, w, 1e-5)
    want = x / np.sqrt(np.mean(x.astype(np.float64) ** 2) + 1e-5) * w
    assert np.allclose(got, want, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("rows,cols", [(8, 64), (37, 256), (64, 4096)])
def test_restated_row_dot_vs_reference_simd(oracle_mod, rows, cols):
    """dotQ8_0Row (pure Go path) vs the reference's matvec_q8_c (cgo path)."""
    if not oracle_mod.have_ref_simd():
        pytest.skip("reference simd.c not built")
    import synthetic
    import torch
    rng = np.random.default_rng(rows)
    g = torch.Generator().manual_seed(rows * 131 + cols)
    w = synthetic.quantize_q8_0_rows(torch.randn(rows, cols, generator=g) * 0.02, torch).numpy()
    d, qs = oracle_mod.quantize_q8_0(rng.standard_normal(cols).astype(np.float32))
    ref = oracle_mod.ref_matvec_q8(w, d, qs, rows, cols)
    pure = np.array([oracle_mod.dot_q8_0_row(w[r], d, qs) for r in range(rows)], np.float32)
    # the two builds add the same fp32 block terms in different orders: the
    # difference is bounded by a few ulps of the sum of the terms' magnitudes
    wq = w.reshape(rows, cols // 32, 34)
    dw = wq[:, :, :2].copy().view(np.float16)[:, :, 0].astype(np.float64)
    isum = (wq[:, :, 2:].view(np.int8).astype(np.int64) * qs.reshape(1, -1, 32)).sum(-1)
    mag = (np.abs(dw * d.astype(np.float64)[None, :] * isum)).sum(-1)
    assert (np.abs(ref.astype(np.float64) - pure) <= 4 * np.finfo(np.float32).eps * mag * np.log2(cols)).all()
    # row sub-range semantics of matvec_q8_c(start_row, end_row)
    part = oracle_mod.ref_matvec_q8(w, d, qs, rows, cols, start=rows // 3, end=rows // 2)
    assert np.array_equal(part[rows // 3:rows // 2], ref[rows // 3:rows // 2])
    assert not part[: rows // 3].any()


@pytest.mark.parametrize("name", ["tiny", "tiny-gqa"])
def test_oracle_forward_vs_float64_numpy(oracle_mod, name):
    import npref
    import synthetic
    cfg, T = synthetic_model(name)
    factors = synthetic.llama3_freq_factors(cfg) if cfg.rope_scaling else None
    om = oracle_mod.OracleModel(cfg, T, threads=2)
    om.new_state(32)
    npm = npref.NpModel(cfg, T, 32, factors)
    for t in synthetic.prompt_ids(cfg, 10, seed=5):
        a = om.forward(int(t))
        b = npm.forward(int(t))
        rel = np.linalg.norm(a - b) / np.linalg.norm(b)
        assert rel < 2e-3, rel
    # the KV cache holds roped K and raw V in the reference layout
    K, V = om.kv(cfg.n_layers - 1, 0, 10)
    assert np.allclose(K, npm.K[-1, :10], rtol=1e-3, atol=1e-4)
    assert np.allclose(V, npm.V[-1, :10], rtol=1e-3, atol=1e-4)


def test_oracle_thread_count_does_not_change_results(oracle_mod):
    import synthetic
    cfg, T = synthetic_model("tiny-gqa")
    outs = []
    for th in (1, 3, 8):
        om = oracle_mod.OracleModel(cfg, T, threads=th)
        om.new_state(16)
        for t in synthetic.prompt_ids(cfg, 4, seed=2):
            lg = om.forward(int(t))
        outs.append(lg)
    assert all(np.array_equal(outs[0], o) for o in outs[1:])


def test_oracle_topk_path(oracle_mod):
    """ForwardTopKIntoWorkspace: K items, distinct ids, unsorted merge order;
    with K = vocab every id appears once."""
    import synthetic
    cfg, T = synthetic_model("tiny")
    om = oracle_mod.OracleModel(cfg, T, threads=3)
    om.new_state(16)
    ids = synthetic.prompt_ids(cfg, 3, seed=9)
    for t in ids[:-1]:
        om.forward(int(t), logits=False)
    got_ids, got_lg = om.forward_topk(int(ids[-1]), cfg.vocab)
    assert sorted(got_ids.tolist()) == list(range(cfg.vocab))
    om.pos = 2
    i5, l5 = om.forward_topk(int(ids[-1]), 5)
    order = np.argsort(-got_lg, kind="stable")
    assert set(i5.tolist()) == set(got_ids[order[:5]].tolist())


def test_oracle_context_exceeded(oracle_mod):
    import synthetic
    cfg, T = synthetic_model("tiny")
    om = oracle_mod.OracleModel(cfg, T, threads=1)
    om.new_state(2)
    om.forward(1, logits=False)
    om.forward(2, logits=False)
    with pytest.raises(RuntimeError, match="context length exceeded"):
        om.forward(3)
    om.pos = 0
    with pytest.raises(RuntimeError, match="token out of range"):
        om.forward(cfg.vocab)


def test_sampler_restatement(oracle_mod):
    ids = np.array([7, 3, 9], np.int32)
    lg = np.array([1.0, 2.0, 0.5], np.float32)
    # cumulative pick in item order over exp((l - max)/T) (sampling.go:115-142)
    T = 0.8
    invT = 1.0 / float(np.float32(T))  # Sampler.Temperature is a float32
    e = np.exp((lg.astype(np.float64) - 2.0) * invT)
    c = np.cumsum(e) / e.sum()
    for r in (0.0, c[0] - 1e-7, c[0] + 1e-7, c[1] + 1e-7, 0.999999):
        want = ids[np.searchsorted(c, r)]
        assert oracle_mod.sample_topk(ids, lg, T, r) == want


def test_reference_builds_disagree_by_quantization_noise(oracle_mod):
    """The reference's CGO_ENABLED=1 (simd.c) and CGO_ENABLED=0 (pure Go)
    builds differ only in float32 summation order, yet once a per-block
    activation rounding flips, the difference cascades to the quantization
    noise level (about 1% of the logits).  This band, not float rounding, is
    what separates any two correct implementations of this decode step."""
    from refspread import ReferenceRuns
    import synthetic
    cfg, T = synthetic_model("mid")
    R = ReferenceRuns(oracle_mod, cfg, T, synthetic.prompt_ids(cfg, 8, seed=11), 16)
    assert 5e-3 < R.band() < 5e-2
