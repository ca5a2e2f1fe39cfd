"""Index math of the batched kernels, replayed on the CPU (no GPU).

Each replay transcribes a kernel's index expressions and loop structure
literally into numpy and checks it against an independent statement of what
it must compute:
- k_gemm_from_tiles (csrc/l3g_prefill.cuh): weight chunks built from the
  decode kernels' tile layout (k_repack's layout, for every rows-per-warp
  choice and several column slicings) equal the library's own host repack
  (l3g_gemm_repack) of the same GGUF rows, byte for byte;
- k_bd_attention + k_bd_merge (csrc/l3g_batch.cuh): 256-position splits,
  warps striding over positions, per-warp online softmax, the CTA's merge of
  8 warps and the merge across splits give softmax attention over positions
  0..pos (float64 restatement of infer.go:130-175) within 1e-5;
- k_pf_attention (csrc/l3g_prefill.cuh): query blocks of 64 / group
  positions, key tiles of 32 with the causal limit of each row, online
  softmax, for a pass starting above position zero;
- k_gemm_q8's work units with a split K (gemm_ksplit, the producer's and the
  rescale warps' chunk sequences): every (row tile, token tile, chunk) is
  visited exactly once, both roles walk the same sequence per CTA, and each
  unit owns one partial-sum slot.
"""
import numpy as np
import pytest

TILE_TARGET = 32 * 1024
NW = 8


def make_tiles(rows, cols, rpw):
    """The decode matrices' tile plan (l3g_model.cu make_tiles)."""
    wr = NW * rpw
    nb = cols // 32
    nsl = max(1, -(-(cols * wr) // TILE_TARGET))
    while nb % nsl:
        nsl += 1
    ck = cols // nsl
    tile_bytes = -(-(wr * ck + wr * (ck // 32) * 2) // 16) * 16
    n_groups = -(-rows // wr)
    return dict(rows=rows, cols=cols, wr=wr, ck=ck, nslices=nsl, tile_bytes=tile_bytes,
                n_groups=n_groups)


def repack_tiles(q8, t):
    """k_repack (l3g_kernels.cuh) for one row segment: GGUF rows -> tiles."""
    out = np.zeros(t["n_groups"] * t["nslices"] * t["tile_bytes"], np.uint8)
    nbc = t["cols"] // 32
    rows = q8.reshape(t["rows"], nbc, 34)
    bpt = t["ck"] // 32
    for r in range(t["n_groups"] * t["wr"]):
        g, i = divmod(r, t["wr"])
        for b in range(nbc):
            s, bb = divmod(b, bpt)
            tile = ((g * t["nslices"]) + s) * t["tile_bytes"]
            qd = tile + i * t["ck"] + bb * 32
            dd = tile + t["wr"] * t["ck"] + (i * bpt + bb) * 2
            if r < t["rows"]:
                out[dd:dd + 2] = rows[r, b, :2]
                out[qd:qd + 32] = rows[r, b, 2:]
    return out


def gemm_from_tiles(tiles, t):
    """k_gemm_from_tiles, transcribed."""
    TILE_M, A_Q, A_CHUNK, KC, BPC, QBLK = 128, 16384, 17408, 128, 4, 32
    nbc = t["cols"] // 32
    nk = -(-t["cols"] // KC)
    n_rt = -(-t["rows"] // TILE_M)
    dst = np.zeros(n_rt * nk * A_CHUNK, np.uint8)

    def q_offset(rows, m, k):
        return (k // 16) * rows * 16 + m * 16 + (k % 16)

    for e in range(t["rows"] * nbc):
        r, b = divmod(e, nbc)
        g, i = divmod(r, t["wr"])
        bpt = t["ck"] // 32
        s, bb = divmod(b, bpt)
        tile = (g * t["nslices"] + s) * t["tile_bytes"]
        q = tile + i * t["ck"] + bb * 32
        d = tile + t["wr"] * t["ck"] + (i * bpt + bb) * 2
        rt, m = divmod(r, TILE_M)
        c, j = divmod(b, BPC)
        ch = (rt * nk + c) * A_CHUNK
        o0 = ch + q_offset(TILE_M, m, j * QBLK)
        o1 = ch + q_offset(TILE_M, m, j * QBLK + 16)
        dst[o0:o0 + 16] = tiles[q:q + 16]
        dst[o1:o1 + 16] = tiles[q + 16:q + 32]
        od = ch + A_Q + (j * TILE_M + m) * 2
        dst[od:od + 2] = tiles[d:d + 2]
    return dst


@pytest.mark.parametrize("rows,cols,rpw", [(200, 288, 1), (130, 4096, 4), (300, 1024, 2),
                                           (64, 8192, 8), (1000, 128, 4)])
def test_gemm_from_tiles_equals_host_repack(rows, cols, rpw):
    import l3g
    rng = np.random.default_rng(rows + cols + rpw)
    q8 = rng.integers(0, 256, rows * cols // 32 * 34).astype(np.uint8)
    t = make_tiles(rows, cols, rpw)
    tiles = repack_tiles(q8, t)
    assert np.array_equal(gemm_from_tiles(tiles, t), l3g.gemm_repack(q8, rows, cols))


def _attention_f64(q, K, V, scale):
    """softmax(q . K_t * scale) . V over the given positions, float64."""
    s = (K.astype(np.float64) @ q.astype(np.float64)) * scale
    e = np.exp(s - s.max())
    return (e / e.sum()) @ V.astype(np.float64)


def _expf(x):
    return np.float32(np.exp(np.float64(x))) if np.isfinite(x) else np.float32(0.0)


def bd_attention(Q, K, V, pos, group, scale, split=256):
    """k_bd_attention + k_bd_merge for one sequence and kv head (float32)."""
    hd = K.shape[1]
    ns = -(-(pos + 1) // split)
    parts = []
    for sp in range(ns):
        p0, p1 = sp * split, min(pos + 1, sp * split + split)
        wm = np.full((8, group), -np.inf, np.float32)
        wl = np.zeros((8, group), np.float32)
        wo = np.zeros((8, group, hd), np.float32)
        for w in range(8):
            for p in range(p0 + w, p1, 8):
                for g in range(group):
                    s = np.float32(np.dot(Q[g], K[p]) * np.float32(scale))
                    mn = max(wm[w, g], s)
                    corr = _expf(wm[w, g] - mn) if wm[w, g] != -np.inf else np.float32(0.0)
                    pe = _expf(s - mn)
                    wl[w, g] = wl[w, g] * corr + pe
                    wo[w, g] = wo[w, g] * corr + pe * V[p]
                    wm[w, g] = mn
        M = wm.max(axis=0)
        f = np.where(wm == -np.inf, 0.0, np.exp(wm - M)).astype(np.float32)
        parts.append((M, (wl * f).sum(0), (wo * f[..., None]).sum(0)))
    M = np.max([p[0] for p in parts], axis=0)
    L = np.zeros(group, np.float32)
    O = np.zeros((group, hd), np.float32)
    for m, l, o in parts:
        f = np.where(m == -np.inf, 0.0, np.exp(m - M)).astype(np.float32)
        L += l * f
        O += o * f[:, None]
    return O / L[:, None]


@pytest.mark.parametrize("pos,group,hd", [(0, 4, 128), (9, 3, 32), (255, 4, 64), (256, 1, 128),
                                          (700, 8, 64)])
def test_split_decode_attention_replay(pos, group, hd):
    rng = np.random.default_rng(pos * 10 + group)
    K = rng.normal(0, 1, (pos + 1, hd)).astype(np.float32)
    V = rng.normal(0, 1, (pos + 1, hd)).astype(np.float32)
    Q = rng.normal(0, 1, (group, hd)).astype(np.float32)
    scale = float(np.float32(1.0 / np.sqrt(hd)))
    got = bd_attention(Q, K, V, pos, group, scale)
    for g in range(group):
        want = _attention_f64(Q[g], K, V, scale)
        assert np.abs(got[g] - want).max() < 1e-5 * max(1.0, np.abs(want).max())


def pf_attention(Q, K, V, P, pos0, group, scale):
    """k_pf_attention for one kv head: Q [P][group][hd] -> out [P][group][hd]."""
    hd = K.shape[1]
    bq = max(1, 64 // group)
    out = np.zeros((P, group, hd), np.float32)
    for blk in range(-(-P // bq)):
        tok0 = blk * bq
        ntok = min(bq, P - tok0)
        R = group * ntok
        last = pos0 + tok0 + ntok - 1
        m = np.full(R, -np.inf, np.float32)
        l = np.zeros(R, np.float32)
        o = np.zeros((R, hd), np.float32)
        for kb in range(0, last + 1, 32):
            keys = np.arange(kb, kb + 32)
            kt = np.where((keys <= last)[:, None], K[np.minimum(keys, last)], 0.0).astype(np.float32)
            vt = np.where((keys <= last)[:, None], V[np.minimum(keys, last)], 0.0).astype(np.float32)
            for r in range(R):
                t, g = divmod(r, group)
                limit = pos0 + tok0 + t
                s = (kt @ Q[tok0 + t, g]).astype(np.float32) * np.float32(scale)
                valid = keys <= limit
                s = np.where(valid, s, -np.inf).astype(np.float32)
                mn = max(m[r], s.max())
                pe = np.where(valid, np.exp(s - mn), 0.0).astype(np.float32)
                corr = np.float32(0.0) if m[r] == -np.inf else _expf(m[r] - mn)
                l[r] = l[r] * corr + pe.sum()
                m[r] = mn
                o[r] = o[r] * corr + pe @ vt
        for r in range(R):
            t, g = divmod(r, group)
            out[tok0 + t, g] = o[r] / l[r]
    return out


@pytest.mark.parametrize("P,pos0,group,hd", [(5, 0, 4, 64), (40, 13, 3, 32), (70, 100, 1, 128),
                                             (33, 0, 8, 32)])
def test_causal_prefill_attention_replay(P, pos0, group, hd):
    rng = np.random.default_rng(P + pos0 + group)
    n = pos0 + P
    K = rng.normal(0, 1, (n, hd)).astype(np.float32)
    V = rng.normal(0, 1, (n, hd)).astype(np.float32)
    Q = rng.normal(0, 1, (P, group, hd)).astype(np.float32)
    scale = float(np.float32(1.0 / np.sqrt(hd)))
    got = pf_attention(Q, K, V, P, pos0, group, scale)
    for p in range(P):
        for g in range(group):
            lim = pos0 + p + 1
            want = _attention_f64(Q[p, g], K[:lim], V[:lim], scale)
            assert np.abs(got[p, g] - want).max() < 1e-5 * max(1.0, np.abs(want).max()), (p, g)


def gemm_ksplit(n_rt, nk, n_tok, rows, nsm, part_floats):
    """gemm_ksplit (l3g_batched.cu), transcribed."""
    nt = 16 if n_tok <= 16 else 32 if n_tok <= 32 else 64 if n_tok <= 64 else 128
    tiles = n_rt * (-(-n_tok // nt))
    if part_floats == 0 or tiles >= nsm:
        return 1
    want = nsm // tiles
    best = 1
    for d in range(2, nk + 1):
        if d > want:
            break
        if nk % d == 0 and d * n_tok * rows <= part_floats:
            best = d
    return best


@pytest.mark.parametrize("rows,cols,n_tok,nsm", [(768, 4096, 64, 148), (4096, 1792, 64, 148),
                                                 (4096, 512, 5, 148), (3584, 4096, 64, 148),
                                                 (6144, 4096, 512, 148), (200, 288, 17, 8)])
def test_split_k_units_cover_every_chunk_once(rows, cols, n_tok, nsm):
    """k_gemm_q8's work units: the producer's and the rescale warps' chunk
    sequences (transcribed) visit every (row tile, token tile, chunk) exactly
    once, in the same order per CTA, and each unit's partial sums go to its
    own K range slot."""
    nt = 16 if n_tok <= 16 else 32 if n_tok <= 32 else 64 if n_tok <= 64 else 128
    n_rt, n_tt, nk = -(-rows // 128), -(-n_tok // nt), -(-cols // 128)
    ks = gemm_ksplit(n_rt, nk, n_tok, rows, nsm, part_floats=10**9)
    assert nk % ks == 0
    nku = nk // ks
    n_units = n_rt * n_tt * ks
    G = max(1, min(nsm, n_units))
    seen = {}
    for cta in range(G):
        my_units = -(-(n_units - cta) // G) if cta < n_units else 0
        prod = []
        for c in range(my_units * nku):  # producer (a_src / b_src)
            u = cta + (c // nku) * G
            tile, kc = u // ks, (u % ks) * nku + c % nku
            prod.append((tile % n_rt, tile // n_rt, kc))
        epi = []
        for ui in range(my_units):       # rescale warps
            u = cta + ui * G
            tile, k = u // ks, u % ks
            for kc in range(nku):
                epi.append((tile % n_rt, tile // n_rt, k * nku + kc))
            slot = (tile, k)
            assert slot not in seen
            seen[slot] = cta
        assert prod == epi
    cover = {}
    for cta in range(G):
        my_units = -(-(n_units - cta) // G) if cta < n_units else 0
        for c in range(my_units * nku):
            u = cta + (c // nku) * G
            tile, kc = u // ks, (u % ks) * nku + c % nku
            cover[(tile, kc)] = cover.get((tile, kc), 0) + 1
    assert len(cover) == n_rt * n_tt * nk and set(cover.values()) == {1}
    want = nsm // (n_rt * n_tt)
    if any(nk % d == 0 for d in range(2, min(nk, want) + 1)):
        assert ks > 1  # few tiles: the K range is split when a divisor fits
