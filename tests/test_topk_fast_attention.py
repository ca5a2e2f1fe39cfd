"""CPU checks of the top-K path's fastExp attention (csrc/l3g_attention_fast.cuh).

The reference's ForwardTopKIntoWorkspace weights position t of a head by
fastExp(score_t - max) with max over ALL positions (infer.go:376-423,
520-525).  The kernels split the positions over CTAs in three passes
(scores and split maxima; the head maximum, weights and per-split sums;
merge in split order).  These tests replay those passes index by index in
numpy, with the per-warp position assignment and the summation orders of
the kernels, and compare them with the reference's loop restated directly,
so that the decomposition is shown equal to the reference before it runs on
a GPU.  They also pin the kernel's fastExp bit formula (int64 truncation,
low 32 bits) against the oracle's restatement, including the wrapping region
below x ~ -88.
"""
import numpy as np
import pytest

NW = 8       # warps per CTA (ATTF_THREADS / 32)
MAXG = 8


def fast_exp_kernel(x: np.float32) -> np.float32:
    """fast_exp_ref of the kernel: prod = fl(x * 12102203), bits =
    uint32(int64(prod)) + 1064866816 (mod 2^32)."""
    prod = np.float32(np.float32(x) * np.float32(12102203.0))
    bits = (int(np.int64(np.trunc(np.float64(prod)))) + 1064866816) & 0xFFFFFFFF
    return np.array([bits], np.uint32).view(np.float32)[0]


def attf_range(n, splits, s):
    chunk = (n + splits - 1) // splits
    t0 = min(n, s * chunk)
    return t0, min(n, t0 + chunk)


def reference_head(q, K, V, scale, fexp, weights=None):
    """infer.go:376-423 for one query head: scores, max (init -1e30),
    e = fastExp(score - max), sumExp, out += (e * invSumExp) * V, all f32
    in position order."""
    n = K.shape[0]
    scores = np.empty(n, np.float32)
    mx = np.float32(-1e30)
    for t in range(n):
        sc = np.float32(np.float32(np.dot(q, K[t])) * scale)
        scores[t] = sc
        if sc > mx:
            mx = sc
    sum_exp = np.float32(0.0)
    for t in range(n):
        e = fexp(np.float32(scores[t] - mx))
        scores[t] = e
        sum_exp = np.float32(sum_exp + e)
    if weights is not None:
        weights[:] = scores
    inv = np.float32(np.float32(1.0) / sum_exp)
    out = np.zeros(q.shape[0], np.float32)
    for t in range(n):
        out = (out + np.float32(scores[t] * inv) * V[t]).astype(np.float32)
    return out


def kernel_replay(q, K, V, scale, splits, fexp, weights=None):
    """The three kernels for one kv head: q [G][hd], K/V [n][hd].
    Returns out [G][hd]; weights [G][n], when given, receives every e."""
    G, hd = q.shape
    n = K.shape[0]
    ctx = n + 5  # the scores rows are ctx long; only [0, n) is written
    scores = np.full((G, ctx), np.nan, np.float32)
    pmax = np.empty((splits, G), np.float32)
    # pass 0: k_attf_scores, CTA (g, s); warp w takes t0 + w, t0 + w + NW, ...
    for s in range(splits):
        t0, t1 = attf_range(n, splits, s)
        wmax = np.full((NW, MAXG), np.float32(-1e30), np.float32)
        for w in range(NW):
            for t in range(t0 + w, t1, NW):
                for h in range(G):
                    sc = np.float32(np.float32(np.dot(q[h], K[t])) * scale)
                    scores[h, t] = sc
                    wmax[w, h] = max(wmax[w, h], sc)
        for h in range(G):
            m = np.float32(-1e30)
            for w in range(NW):
                m = max(m, wmax[w, h])
            pmax[s, h] = m
    # pass 1: k_attf_values
    psum = np.empty((splits, G), np.float32)
    po = np.empty((splits, G, hd), np.float32)
    for s in range(splits):
        t0, t1 = attf_range(n, splits, s)
        M = [max([np.float32(-1e30)] + [pmax[s2, h] for s2 in range(splits)]) for h in range(G)]
        wl = np.zeros((NW, G), np.float32)
        wo = np.zeros((NW, G, hd), np.float32)
        for w in range(NW):
            for t in range(t0 + w, t1, NW):
                for h in range(G):
                    e = fexp(np.float32(scores[h, t] - M[h]))
                    if weights is not None:
                        weights[h, t] = e
                    wl[w, h] = np.float32(wl[w, h] + e)
                    wo[w, h] = (wo[w, h] + e * V[t]).astype(np.float32)
        for h in range(G):
            acc = np.zeros(hd, np.float32)
            ls = np.float32(0.0)
            for w in range(NW):
                acc = (acc + wo[w, h]).astype(np.float32)
                ls = np.float32(ls + wl[w, h])
            po[s, h] = acc
            psum[s, h] = ls
    # pass 2: k_attf_merge (one warp per 32 outputs; here per head)
    out = np.empty((G, hd), np.float32)
    for h in range(G):
        L = np.float32(0.0)
        O = np.zeros(hd, np.float32)
        for s in range(splits):
            L = np.float32(L + psum[s, h])
            O = (O + po[s, h]).astype(np.float32)
        out[h] = (O * np.float32(np.float32(1.0) / L)).astype(np.float32)
    assert not np.isnan(scores[:, :n]).any()  # every position scored exactly once
    return out


def test_fast_exp_bits_match_the_oracle(oracle_mod):
    xs = [0.0, -1e-7, -0.5, -1.0, -2.75, -10.0, -31.4, -87.0, -88.5, -89.0, -100.0,
          -150.0, -177.4, -1000.0, 0.25]
    rng = np.random.default_rng(11)
    xs += list(-rng.exponential(20.0, 300)) + list(-rng.uniform(80, 200, 100))
    for x in xs:
        x = np.float32(x)
        got = int(fast_exp_kernel(x).view(np.uint32))
        want = int(np.float32(oracle_mod.fast_exp(float(x))).view(np.uint32))
        if np.isnan(np.uint32(got).view(np.float32)):
            # a NaN returned through ctypes (float -> double -> float) comes
            # back quieted: compare with the quiet bit set on both sides
            got |= 1 << 22
        assert got == want, (x, hex(got), hex(want))


def test_split_ranges_cover_every_position_once():
    for n in list(range(1, 70)) + [127, 128, 129, 4097, 4352, 8320]:
        for splits in (1, 2, 3, 7, 8, 37, 64):
            seen = np.zeros(n, np.int32)
            for s in range(splits):
                t0, t1 = attf_range(n, splits, s)
                assert 0 <= t0 <= t1 <= n
                seen[t0:t1] += 1
            assert (seen == 1).all(), (n, splits)


@pytest.mark.parametrize("n,G,hd,splits", [(1, 4, 64, 37), (5, 1, 32, 2), (37, 4, 64, 3),
                                           (130, 3, 64, 8), (261, 8, 32, 17)])
def test_passes_equal_the_reference_loop(oracle_mod, n, G, hd, splits):
    rng = np.random.default_rng(1000 * n + G)
    q = rng.standard_normal((G, hd)).astype(np.float32)
    K = rng.standard_normal((n, hd)).astype(np.float32)
    V = rng.standard_normal((n, hd)).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(hd))
    fexp = fast_exp_kernel
    got = kernel_replay(q, K, V, scale, splits, fexp)
    for h in range(G):
        want = reference_head(q[h], K, V, scale, fexp)
        err = np.linalg.norm(got[h] - want) / max(np.linalg.norm(want), 1e-30)
        assert err < 2e-6, (h, err)


def test_passes_follow_fast_exp_not_exp(oracle_mod):
    """The decomposition keeps the reference's weights: with the exact exp in
    its place the outputs move by the approximation's few percent, far above
    the decomposition's rounding."""
    rng = np.random.default_rng(5)
    G, hd, n = 4, 64, 200
    q = (3 * rng.standard_normal((G, hd))).astype(np.float32)
    K = rng.standard_normal((n, hd)).astype(np.float32)
    V = rng.standard_normal((n, hd)).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(hd))
    got = kernel_replay(q, K, V, scale, 7, fast_exp_kernel)
    exact = lambda x: np.float32(np.exp(np.float64(x)))
    for h in range(G):
        want = reference_head(q[h], K, V, scale, fast_exp_kernel)
        other = reference_head(q[h], K, V, scale, exact)
        e_same = np.linalg.norm(got[h] - want) / np.linalg.norm(want)
        e_other = np.linalg.norm(got[h] - other) / np.linalg.norm(other)
        assert e_same < 2e-6 and e_other > 100 * e_same, (e_same, e_other)


def test_wrapped_weights_are_reproduced(oracle_mod):
    """Scores more than ~88 below the maximum give the reference's wrapped
    (garbage: huge, infinite or NaN) fastExp bits; the passes form exactly
    the reference's weights, bit for bit, wrapped ones included."""
    G, hd, n = 2, 32, 64
    q = np.zeros((G, hd), np.float32)
    q[0, 0] = 1.0
    q[1, 1] = 1.0
    K = np.zeros((n, hd), np.float32)
    K[:, 0] = np.linspace(0.0, -1200.0, n).astype(np.float32)  # scores 0 .. -212
    K[:, 1] = np.linspace(3.0, -3.0, n).astype(np.float32)     # an ordinary head
    V = np.random.default_rng(2).standard_normal((n, hd)).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(hd))
    assert np.float32(K[-1, 0] * scale) < -88  # the wrapping region is exercised
    got_w = np.empty((G, n), np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        got = kernel_replay(q, K, V, scale, 5, fast_exp_kernel, got_w)
        ref_exp = lambda x: np.float32(oracle_mod.fast_exp(float(x)))
        for h in range(G):
            want_w = np.empty(n, np.float32)
            want = reference_head(q[h], K, V, scale, ref_exp, want_w)
            a = got_w[h].view(np.uint32).copy()
            b = want_w.view(np.uint32).copy()
            nan = np.isnan(got_w[h])
            a[nan] |= np.uint32(1 << 22)  # ctypes quiets NaNs (see above)
            assert (a == b).all(), h
            if h == 1:
                assert np.linalg.norm(got[h] - want) / np.linalg.norm(want) < 2e-6
