"""The oracle against the committed golden fixtures (tests/golden/): outputs
of the reference's own simd.c, the input of its BenchmarkMatVecQ8, and the
oracle's forward logits (drift check).  tests/golden/make_golden.py made
them."""
import os
import sys

import numpy as np
import pytest

from refspread import rel_l2

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLDEN)
import make_golden  # noqa: E402


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def _cases():
    z = _load("ref_simd_matvec.npz")
    return [(i, *z[f"c{i}_shape"].tolist()) for i in range(len(make_golden.MATVEC_CASES))]


@pytest.mark.parametrize("i,rows,cols,seed", _cases())
def test_matvec_fixture(oracle_mod, i, rows, cols, seed):
    z = _load("ref_simd_matvec.npz")
    w = make_golden.q8_matrix(rows, cols, seed)
    assert make_golden.sha(w) == str(z[f"c{i}_w_sha256"])
    # activation quantization, bit for bit
    d, qs = oracle_mod.quantize_q8_0(make_golden.activation(cols, seed))
    assert np.array_equal(d, z[f"c{i}_xd"]) and np.array_equal(qs, z[f"c{i}_xq"])
    want = z[f"c{i}_out"]
    # the reference's own kernel reproduces its recorded output exactly
    if oracle_mod.have_ref_simd():
        assert np.array_equal(oracle_mod.ref_matvec_q8(w, d, qs, rows, cols), want)
    # the restated pure-Go row dot (q8_0.go:87-105) agrees to f32 rounding
    got = np.array([oracle_mod.dot_q8_0_row(w[r], d, qs) for r in range(rows)], np.float32)
    assert rel_l2(got, want) < 1e-6


def test_dot_fixture(oracle_mod):
    z = _load("ref_simd_dot.npz")
    lib = oracle_mod.lib()
    for n in make_golden.DOT_LENGTHS:
        a, b, want = z[f"n{n}_a"], z[f"n{n}_b"], float(z[f"n{n}_out"])
        assert abs(float(np.dot(a.astype(np.float64), b.astype(np.float64))) - want) <= 1e-5 * max(1.0, abs(want))
        if oracle_mod.have_ref_simd():
            assert np.float32(lib.orc_ref_dot(oracle_mod.fp(a), oracle_mod.fp(b), n)) == np.float32(want)


def test_reference_benchmark_input(oracle_mod):
    """BenchmarkMatVecQ8's x[i] = (i % 10) * 0.1 quantizes to the recorded
    blocks, and its all-zero matrix gives zeros."""
    z = _load("ref_benchmark_matvec.npz")
    d, qs = oracle_mod.quantize_q8_0(z["x"])
    assert np.array_equal(d, z["xd"]) and np.array_equal(qs, z["xq"])
    assert not z["out"].any()
    # every block holds 0.0 .. 0.9: scale 0.9/127, and 0.9 maps to 127
    assert np.allclose(d, np.float32(0.9) / np.float32(127.0))
    assert qs.reshape(-1, 32).max(1).tolist() == [127] * d.size


@pytest.mark.parametrize("name,n,pseed", make_golden.FORWARD_CASES)
def test_oracle_forward_fixture(oracle_mod, name, n, pseed):
    from conftest import synthetic_model
    import synthetic
    z = _load("oracle_forward.npz")
    cfg, T = synthetic_model(name)
    assert make_golden.model_sha(T) == str(z[f"{name}_model_sha256"])
    ids = synthetic.prompt_ids(cfg, n, seed=pseed)
    assert np.array_equal(ids, z[f"{name}_ids"])
    if not oracle_mod.have_ref_simd():
        pytest.skip("oracle/_ref/libref_simd.so absent")
    om = oracle_mod.OracleModel(cfg, T)
    om.new_state(64)
    got = np.stack([om.forward(int(t)).copy() for t in ids])
    om.close()
    assert np.array_equal(got, z[f"{name}_logits"])
