"""l3g_matvec_q8_argmax_static: the matvec fused with an argmax over its rows,
reducing across CTAs in the library's static device scratch instead of any
allocation.  Checked against the existing entry point l3g_matvec_q8 (same
tiles, same accumulation) plus a host argmax, on consecutive calls (the
scratch's arrival counter must come back to zero after every launch).

The file name sorts last so that, in a full run, it executes after every
other GPU test; it passes alone as well.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


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


def test_static_argmax_rejects_more_ctas_than_slots(gpu_lib):
    import torch
    M = _matrix(gpu_lib, 64, 64, 9)
    _, d, q = _activation(64, 10)
    res = torch.zeros(4, dtype=torch.int32, device="cuda")
    with pytest.raises(gpu_lib.L3GError, match="static argmax scratch holds"):
        M.matvec_argmax_static(d.data_ptr(), q.data_ptr(), 0, res.data_ptr(),
                               max_ctas=gpu_lib.ARGMAX_STATIC_MAX_CTAS + 1)
    M.Close()


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
