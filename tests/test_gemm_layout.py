"""Batched Q8_0 product on the tensor cores: host-side checks (no GPU).

- The kind::i8 instruction descriptor and the shared-memory matrix
  descriptors equal CUTLASS's sm100 definitions (tests/gemm_layout_check.cu,
  compiled host-only by nvcc against the CUTLASS headers in the image).
- A replay of what the MMAs read: the library's own host repack of the
  weights (l3g_gemm_repack), the activation chunks as l3g_gemm_quantize lays
  them out, and each block's descriptors decoded by the PTX rule for K-major
  operands without swizzle (element (row, k) at start + (row % 8) * 16 +
  (row / 8) * SBO + k % 16 + (k / 16) * LBO).  The per-block int32 products,
  rescaled by fp16(d_w) * d_x in fp32 as the kernel does, match the
  reference's own matvec_q8_c (simd.c:33-110) for every token.
"""
import importlib.util
import os
import subprocess

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

A_Q_BYTES, A_CHUNK, KC, TILE_M = 16384, 17408, 128, 128


def _cutlass_include():
    for pkg, sub in (("flashinfer", ("data", "cutlass", "include")),
                     ("tilelang", ("3rdparty", "cutlass", "include"))):
        try:
            spec = importlib.util.find_spec(pkg)
        except (ImportError, ValueError):
            spec = None
        if spec is None or not spec.submodule_search_locations:
            continue
        p = os.path.join(list(spec.submodule_search_locations)[0], *sub)
        if os.path.exists(os.path.join(p, "cute", "arch", "mma_sm100_desc.hpp")):
            return p
    return None


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    import build
    inc = _cutlass_include()
    if inc is None:
        pytest.skip("CUTLASS headers not found")
    exe = str(tmp_path_factory.mktemp("gemm") / "gemm_layout_check")
    subprocess.run([build.nvcc(), "-std=c++17", "-Wno-deprecated-gpu-targets", "-I", inc,
                    "-I", os.path.join(ROOT, "llama3.go_b200", "csrc"),
                    os.path.join(HERE, "gemm_layout_check.cu"), "-o", exe],
                   check=True, capture_output=True)
    r = subprocess.run([exe], capture_output=True, text=True)
    lines = [ln.split() for ln in r.stdout.splitlines()]
    return r.returncode, lines


def test_descriptors_match_cutlass(harness):
    rc, lines = harness
    idesc = [ln for ln in lines if ln and ln[0] == "idesc"]
    sdesc = [ln for ln in lines if ln and ln[0] == "sdesc"]
    assert len(idesc) == 4 and len(sdesc) == 4
    for _, nt, c, o in idesc:
        assert c == o, (nt, c, o)
    for _, nt, ca, oa, cb, ob in sdesc:
        start = 0x3FFF
        assert int(ca, 16) & ~start == int(oa, 16) & ~start, (nt, ca, oa)
        assert int(cb, 16) & ~start == int(ob, 16) & ~start, (nt, cb, ob)
        assert int(oa, 16) & start == 0x400 >> 4
    assert rc == 0 and ["result", "0"] in lines


def _blocks(lines, nt):
    out = [ln for ln in lines if ln and ln[0] == "block" and int(ln[1]) == nt]
    assert [int(ln[2]) for ln in out] == [0, 1, 2, 3]
    return [(int(ln[3]), int(ln[4]), int(ln[5], 16), int(ln[6], 16)) for ln in out]


def _decode(desc):
    start = (desc & 0x3FFF) << 4
    lbo = ((desc >> 16) & 0x3FFF) << 4
    sbo = ((desc >> 32) & 0x3FFF) << 4
    assert (desc >> 46) & 3 == 1, "sm_100 descriptor version"
    assert (desc >> 49) & 7 == 0 and (desc >> 52) & 1 == 0
    assert (desc >> 61) & 7 == 0, "no swizzle"
    return start, lbo, sbo


def _operand_offsets(desc, rows, base):
    """Byte offsets (from base) of the rows x 32 K-major int8 operand."""
    start, lbo, sbo = _decode(desc)
    m = np.arange(rows)[:, None]
    k = np.arange(32)[None, :]
    return start - base + (m % 8) * 16 + (m // 8) * sbo + (k % 16) + (k // 16) * lbo


@pytest.mark.parametrize("nt", [16, 32, 64, 128])
def test_block_descriptors_cover_each_chunk_once(harness, nt):
    """The four MMAs of a chunk read every int8 of the weight and activation
    chunks exactly once, and nothing outside them."""
    _, lines = harness
    seen_a = np.zeros(A_Q_BYTES, np.int32)
    seen_b = np.zeros(nt * KC, np.int32)
    for a0, b0, ad, bd in _blocks(lines, nt):
        assert b0 == a0 + A_CHUNK
        oa = _operand_offsets(ad, TILE_M, a0)
        ob = _operand_offsets(bd, nt, b0)
        assert oa.min() >= 0 and oa.max() < A_Q_BYTES
        assert ob.min() >= 0 and ob.max() < nt * KC
        np.add.at(seen_a, oa.ravel(), 1)
        np.add.at(seen_b, ob.ravel(), 1)
    assert (seen_a == 1).all() and (seen_b == 1).all()


def _random_q8(rng, rows, cols):
    nb = cols // 32
    d = (np.abs(rng.normal(0, 0.02, (rows, nb))) * 3 / 127 + 1e-4).astype(np.float16)
    q = rng.integers(-127, 128, (rows, nb, 32)).astype(np.int8)
    out = np.empty((rows, nb, 34), np.uint8)
    out[..., :2] = d.view(np.uint8).reshape(rows, nb, 2)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(-1)


def _token_tile(n):
    return 16 if n <= 16 else 32 if n <= 32 else 64 if n <= 64 else 128


def act_chunks(oracle, x, cols):
    """The activation chunks l3g_gemm_quantize writes: per token tile and
    128-column chunk, int8 q [8 slabs][nt][16] then fp32 d [4][nt]; each row
    quantized by QuantizeQ8_0Into; padding zero."""
    n_tok = x.shape[0]
    nt = _token_tile(n_tok)
    nk = -(-cols // KC)
    cb = nt * KC + 4 * nt * 4
    buf = np.zeros(-(-n_tok // nt) * nk * cb, np.uint8)
    for n in range(n_tok):
        d, qs = oracle.quantize_q8_0(x[n])
        ti, nn = divmod(n, nt)
        for b in range(cols // 32):
            c, j = divmod(b, 4)
            base = (ti * nk + c) * cb
            for h in (0, 1):
                off = base + (2 * j + h) * nt * 16 + nn * 16
                buf[off:off + 16] = qs[b * 32 + h * 16:b * 32 + h * 16 + 16].view(np.uint8)
            o = base + nt * KC + (j * nt + nn) * 4
            buf[o:o + 4] = np.float32(d[b]).reshape(1).view(np.uint8)
    return buf, nt, cb


def replay(lines, wpack, act, rows, cols, n_tok):
    """What k_gemm_q8 computes, from the bytes and descriptors alone."""
    nt = _token_tile(n_tok)
    blocks = _blocks(lines, nt)
    nk = -(-cols // KC)
    n_rt, n_tt = -(-rows // TILE_M), -(-n_tok // nt)
    cb = nt * KC + 4 * nt * 4
    out = np.zeros((n_tok, rows), np.float32)
    for rt in range(n_rt):
        for tt in range(n_tt):
            acc = np.zeros((TILE_M, nt), np.float32)
            for c in range(nk):
                a0 = blocks[0][0]
                stage = np.zeros(A_CHUNK + cb, np.uint8)
                ach = wpack[(rt * nk + c) * A_CHUNK:(rt * nk + c + 1) * A_CHUNK]
                stage[:A_CHUNK] = ach
                stage[A_CHUNK:] = act[(tt * nk + c) * cb:(tt * nk + c + 1) * cb]
                dw = stage[A_Q_BYTES:A_CHUNK].view(np.float16).astype(np.float32).reshape(4, TILE_M)
                dx = stage[A_CHUNK + nt * KC:].view(np.float32).reshape(4, nt)
                for j, (ba0, _, ad, bd) in enumerate(blocks):
                    assert ba0 == a0
                    A = stage[_operand_offsets(ad, TILE_M, a0)].view(np.int8).astype(np.int64)
                    B = stage[_operand_offsets(bd, nt, a0)].view(np.int8).astype(np.int64)
                    D = (A @ B.T).astype(np.float64)  # exact int32 block sums
                    s = (dw[j][:, None] * dx[j][None, :]).astype(np.float32)
                    acc = (D * s.astype(np.float64) + acc.astype(np.float64)).astype(np.float32)
            r0 = rt * TILE_M
            nr = min(TILE_M, rows - r0)
            nn = min(nt, n_tok - tt * nt)
            out[tt * nt:tt * nt + nn, r0:r0 + nr] = acc[:nr, :nn].T
    return out


@pytest.mark.parametrize("rows,cols,n_tok", [(200, 288, 5), (128, 256, 17), (130, 512, 40),
                                             (256, 128, 130)])
def test_replayed_mma_matches_reference_matvec(harness, oracle_mod, rows, cols, n_tok):
    import l3g
    _, lines = harness
    rng = np.random.default_rng(rows * 7919 + cols + n_tok)
    w = _random_q8(rng, rows, cols)
    x = rng.normal(0, 1, (n_tok, cols)).astype(np.float32)
    wpack = l3g.gemm_repack(w, rows, cols)
    act, nt, _ = act_chunks(oracle_mod, x, cols)
    assert act.size == l3g.gemm_act_bytes(n_tok, cols)
    got = replay(lines, wpack, act, rows, cols, n_tok)
    for n in range(n_tok):
        d, qs = oracle_mod.quantize_q8_0(x[n])
        ref = oracle_mod.ref_matvec_q8(w, d, qs, rows, cols)
        err = np.linalg.norm(got[n] - ref) / np.linalg.norm(ref)
        assert err < 1e-5, (n, err)


def test_repack_and_size_errors():
    import l3g
    assert l3g.gemm_matrix_bytes(200, 288) == 2 * 3 * A_CHUNK
    assert l3g.gemm_act_bytes(5, 288) == 3 * (16 * 144)
    assert l3g.gemm_act_bytes(200, 4096) == 2 * 32 * (128 * 144)
    for rows, cols in ((0, 32), (4, 0), (4, 48)):
        with pytest.raises(l3g.L3GError, match="Q8_0 matrix"):
            l3g.gemm_matrix_bytes(rows, cols)
    with pytest.raises(l3g.L3GError):
        l3g.gemm_act_bytes(0, 128)
    with pytest.raises(l3g.L3GError, match="do not match"):
        l3g.gemm_repack(np.zeros(10, np.uint8), 1, 32)


def test_bias_conversion_is_exact():
    """k_gemm_q8 turns each int32 block sum v into fp32 as the bits of
    1.5 * 2^23 + v minus 1.5 * 2^23; every |v| < 2^22 (a Q8_0 block sum is at
    most 32 * 128 * 128 = 2^19) comes back exactly."""
    v = np.arange(-(1 << 22) + 1, 1 << 22, dtype=np.int32)
    f = (v + np.int32(0x4B400000)).view(np.float32) - np.float32(12582912.0)
    assert np.array_equal(f, v.astype(np.float32))
    assert 32 * 128 * 128 < (1 << 22)
