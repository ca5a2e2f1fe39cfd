"""l3g_matvec_q8_argmax_static: the matvec fused with an argmax over its rows,
reducing across CTAs in the library's static device scratch instead of any
allocation.  Checked against the existing entry point l3g_matvec_q8 (same
tiles, same accumulation) plus a host argmax, on consecutive calls (the
scratch's arrival counter must come back to zero after every launch).
The cross-CTA merge itself (k_matvec with the EPI_LOGITS epilogue on a
static-style scratch) also runs on the CPU under the SIMT emulator.

The file name sorts last so that, in a full run, it executes after every
other GPU test; it passes alone as well.
"""
import numpy as np
import pytest


def _matrix(gpu_lib, rows, cols, seed):
    import synthetic
    import torch
    g = torch.Generator().manual_seed(seed)
    w = synthetic.quantize_q8_0_rows(torch.randn(rows, cols, generator=g) * 0.02, torch).numpy()
    return gpu_lib.Matrix(w, rows, cols)


def _activation(cols, seed):
    import torch
    x = torch.from_numpy(np.random.default_rng(seed).standard_normal(cols).astype(np.float32)).cuda()
    d = torch.empty(cols // 32, dtype=torch.float32, device="cuda")
    q = torch.empty(cols, dtype=torch.int8, device="cuda")
    return x, d, q


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(32000, 4096), (2050, 1792), (37, 96)])
def test_static_argmax_matches_matvec_on_consecutive_calls(gpu_lib, rows, cols):
    import torch
    M = _matrix(gpu_lib, rows, cols, rows + cols)
    res = torch.zeros(4, dtype=torch.int32, device="cuda")
    for call in range(2):  # two calls in a row, different inputs
        x, d, q = _activation(cols, 100 * call + rows)
        gpu_lib.quantize_q8_0_device(x.data_ptr(), cols, d.data_ptr(), q.data_ptr())
        ref = torch.empty(rows, device="cuda")
        M.matvec(d.data_ptr(), q.data_ptr(), ref.data_ptr())
        out = torch.full((rows,), 7.0, device="cuda")
        M.matvec_argmax_static(d.data_ptr(), q.data_ptr(), out.data_ptr(), res.data_ptr())
        torch.cuda.synchronize()
        r = ref.cpu().numpy()
        o = out.cpu().numpy()
        assert np.allclose(o, r, rtol=1e-6, atol=1e-6 * float(np.abs(r).max()))
        idx, status = int(res[0]), int(res[2])
        value = float(res[1:2].view(torch.float32).item())
        assert status == 0
        assert idx == int(np.argmax(o)) and value == float(o[idx])
        assert abs(float(r[idx]) - float(r.max())) <= 1e-6 * float(np.abs(r).max())
    M.Close()


@pytest.mark.gpu
def test_static_argmax_without_logits_and_capped_grid(gpu_lib):
    import torch
    rows, cols = 4099, 512
    M = _matrix(gpu_lib, rows, cols, 5)
    x, d, q = _activation(cols, 6)
    gpu_lib.quantize_q8_0_device(x.data_ptr(), cols, d.data_ptr(), q.data_ptr())
    ref = torch.empty(rows, device="cuda")
    M.matvec(d.data_ptr(), q.data_ptr(), ref.data_ptr())
    torch.cuda.synchronize()
    want = int(np.argmax(ref.cpu().numpy()))
    res = torch.zeros(4, dtype=torch.int32, device="cuda")
    for max_ctas in (0, 1, 7, gpu_lib.ARGMAX_STATIC_MAX_CTAS):
        M.matvec_argmax_static(d.data_ptr(), q.data_ptr(), 0, res.data_ptr(), max_ctas=max_ctas)
        torch.cuda.synchronize()
        assert int(res[0]) == want and int(res[2]) == 0, max_ctas
    M.Close()


@pytest.mark.gpu
def test_static_argmax_rejects_more_ctas_than_slots(gpu_lib):
    import torch
    M = _matrix(gpu_lib, 64, 64, 9)
    _, d, q = _activation(64, 10)
    res = torch.zeros(4, dtype=torch.int32, device="cuda")
    with pytest.raises(gpu_lib.L3GError, match="static argmax scratch holds"):
        M.matvec_argmax_static(d.data_ptr(), q.data_ptr(), 0, res.data_ptr(),
                               max_ctas=gpu_lib.ARGMAX_STATIC_MAX_CTAS + 1)
    M.Close()


@pytest.mark.gpu
def test_static_argmax_against_reference_simd_fixture(gpu_lib):
    """The entry's logits and argmax against the committed outputs of the
    reference's own matvec_q8_c (tests/golden/ref_simd_matvec.npz), with
    the recorded quantized activations."""
    import os
    import sys
    import torch
    from refspread import rel_l2
    golden = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    sys.path.insert(0, golden)
    import make_golden
    z = np.load(os.path.join(golden, "ref_simd_matvec.npz"))
    res = torch.zeros(4, dtype=torch.int32, device="cuda")
    for i in range(len(make_golden.MATVEC_CASES)):
        rows, cols, seed = z[f"c{i}_shape"].tolist()
        w = make_golden.q8_matrix(rows, cols, seed)
        M = gpu_lib.Matrix(w, rows, cols)
        xd = torch.from_numpy(z[f"c{i}_xd"]).cuda()
        xq = torch.from_numpy(z[f"c{i}_xq"]).cuda()
        ref = z[f"c{i}_out"]
        for _ in range(2):
            out = torch.full((rows,), 12345.0, device="cuda")
            M.matvec_argmax_static(xd.data_ptr(), xq.data_ptr(), out.data_ptr(), res.data_ptr())
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            assert rel_l2(got, ref) < 1e-5, (rows, cols)
            idx = int(res[0])
            assert int(res[2]) == 0 and idx == int(np.argmax(got))
            # the reference's own largest row, unless another row is within
            # the matvec's rounding of it
            top = float(ref.max())
            assert idx == int(np.argmax(ref)) or ref[idx] >= top - 1e-5 * float(np.abs(ref).max())
        M.Close()


@pytest.mark.gpu
def test_static_argmax_keeps_callers_device(gpu_lib):
    """With the matrix on another device, the caller's current device is
    the same after the call as before it (needs two GPUs)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import synthetic
    rows, cols = 300, 256
    g = torch.Generator().manual_seed(3)
    w = synthetic.quantize_q8_0_rows(torch.randn(rows, cols, generator=g) * 0.02, torch).numpy()
    M = gpu_lib.Matrix(w, rows, cols, device=1)
    with torch.cuda.device(1):
        x = torch.from_numpy(np.random.default_rng(4).standard_normal(cols).astype(np.float32)).cuda()
        d = torch.empty(cols // 32, dtype=torch.float32, device="cuda")
        q = torch.empty(cols, dtype=torch.int8, device="cuda")
        res = torch.zeros(4, dtype=torch.int32, device="cuda")
        gpu_lib.quantize_q8_0_device(x.data_ptr(), cols, d.data_ptr(), q.data_ptr())
        torch.cuda.synchronize()
    torch.cuda.set_device(0)
    M.matvec_argmax_static(d.data_ptr(), q.data_ptr(), 0, res.data_ptr())
    assert torch.cuda.current_device() == 0
    with torch.cuda.device(1):
        torch.cuda.synchronize()
    assert int(res[2].cpu()) == 0 and int(res[0].cpu()) >= 0
    M.Close()


@pytest.mark.parametrize("rpw", [1, 4])
def test_static_argmax_merge_under_the_emulator(oracle_mod, rpw):
    """The kernel the entry launches (k_matvec, EPI_LOGITS, pre-quantized
    activation) run on the CPU under the SIMT emulator against one
    static-style scratch of 1024 per-CTA slots and one arrival counter,
    with back-to-back launches of 1, 5 (not dividing the row groups), 7 and
    all-groups CTAs and random schedules: each launch's index is the
    lowest row among equal maxima (the top row is planted three times, in
    row groups that land on different CTAs), its value the kernel's logit of
    that row, the logits equal the reference's matvec_q8_c within 1e-6, and the arrival counter is zero after every launch, with no host
    reset between launches."""
    import simt_lib as S
    import synthetic
    import torch
    from refspread import rel_l2
    rows, cols = 400, 256
    g = torch.Generator().manual_seed(11)
    w = synthetic.quantize_q8_0_rows(torch.randn(rows, cols, generator=g) * 0.02, torch).numpy()
    x = np.random.default_rng(12).standard_normal(cols).astype(np.float32)
    d0, q0 = oracle_mod.quantize_q8_0(x)
    ref = oracle_mod.ref_matvec_q8(w, d0, q0, rows, cols)
    # plant the largest row at rows 130, 270 and 390 (row groups of 8 or 32
    # rows: different groups, dealt to different CTAs)
    rb = w.reshape(rows, -1)
    top = int(np.argmax(ref))
    for r in (270, 130, 390):
        rb[r] = rb[top]
    ref = oracle_mod.ref_matvec_q8(w, d0, q0, rows, cols)
    assert ref[130] == ref[270] == ref[390] == ref.max()
    raw = S.Dev(w)
    tiles = S.repack([(raw, 0, rows)], cols, rows, rpw=rpw)
    xd, xq = S.Dev(d0), S.Dev(q0)
    am_val = S.Dev(np.zeros(1024, np.float32))
    am_idx = S.Dev(np.zeros(1024, np.int32))
    counter = S.Dev(np.zeros(1, np.uint32))
    ng = S.tile_geometry(rows, cols, rpw)["n_groups"]
    try:
        for i, grid in enumerate((1, 5, 7, ng, 5)):
            S.lib().emu_schedule(1, 7 * grid + rpw, 2)
            out = S.Dev(np.full(rows, 9.0, np.float32))
            res = S.Dev(np.array([-1, 0, 0, 0], np.int32))
            S.check(S.lib().emu_matvec_epi(tiles.ptr, rows, cols, rpw, xd.ptr, xq.ptr,
                                           out.ptr if i % 2 == 0 else None, 3, am_val.ptr,
                                           am_idx.ptr, counter.ptr, res.ptr, grid))
            r = res.read(np.int32)
            assert r[0] == 130 and r[2] == 0, (grid, r)
            v = r[1:2].view(np.float32)[0]
            assert abs(v - ref[130]) <= 1e-6 * float(np.abs(ref).max())
            if i % 2 == 0:
                got = out.read(np.float32)
                assert rel_l2(got, ref) < 1e-6
                assert v == got[130] == got.max()
            else:
                assert (out.read(np.float32) == 9.0).all()
            assert counter.read(np.uint32)[0] == 0, grid
            out.free()
            res.free()
    finally:
        S.lib().emu_schedule(0, 0, 0)
    for d in (raw, tiles, xd, xq, am_val, am_idx, counter):
        d.free()
