"""Batched Q8_0 product on the tensor cores (l3g_gemm_*) against the
reference, through the C ABI.

- l3g_gemm_quantize writes the activation chunks bit-identically to the
  layout restated in test_gemm_layout.act_chunks (each row quantized by the
  oracle's QuantizeQ8_0Into);
- l3g_gemm_q8 matches the reference's own matvec_q8_c (simd.c:33-110) for
  every token within 1e-5 relative L2 (fp32 accumulation order only), and the
  single-token l3g_matvec_q8 on the same inputs;
- shapes cover ragged rows, columns that end inside a 128-column chunk, one
  token, every token tile (16 / 32 / 64 / 128) and several token tiles.
"""

import numpy as np
import pytest

from test_gemm_layout import _random_q8, act_chunks

pytestmark = pytest.mark.gpu

SHAPES = [(200, 288, 5), (4096, 4096, 1), (4096, 4096, 16), (1024, 4096, 17),
          (4096, 4096, 64), (2048, 8192, 100), (130, 512, 40), (256, 128, 300)]


def _case(rows, cols, n_tok):
    rng = np.random.default_rng(rows * 7919 + cols * 31 + n_tok)
    return _random_q8(rng, rows, cols), rng.normal(0, 1, (n_tok, cols)).astype(np.float32)


@pytest.mark.parametrize("n_tok,cols", [(5, 288), (17, 256), (40, 512), (130, 4096)])
def test_gemm_quantize_layout(gpu_lib, oracle_mod, n_tok, cols):
    import torch
    rng = np.random.default_rng(n_tok + cols)
    x = rng.normal(0, 1, (n_tok, cols)).astype(np.float32)
    x[0, :32] = 0.0  # an all-zero block (scale 1e-8)
    xd = torch.from_numpy(x).cuda()
    act = torch.full((gpu_lib.gemm_act_bytes(n_tok, cols),), 0x5A, dtype=torch.uint8, device="cuda")
    gpu_lib.gemm_quantize(xd.data_ptr(), n_tok, cols, act.data_ptr())
    torch.cuda.synchronize()
    want, _, _ = act_chunks(oracle_mod, x, cols)
    assert np.array_equal(act.cpu().numpy(), want)  # every byte written, padding zero


@pytest.mark.parametrize("rows,cols,n_tok", SHAPES)
def test_gemm_matches_reference(gpu_lib, oracle_mod, rows, cols, n_tok):
    import torch
    wq, x = _case(rows, cols, n_tok)
    w = gpu_lib.GemmMatrix(wq, rows, cols, device=0)
    xd = torch.from_numpy(x).cuda()
    act = torch.empty(gpu_lib.gemm_act_bytes(n_tok, cols), dtype=torch.uint8, device="cuda")
    out = torch.full((n_tok, rows), float("nan"), dtype=torch.float32, device="cuda")
    w.quantize(xd.data_ptr(), n_tok, act.data_ptr())
    w.gemm(act.data_ptr(), n_tok, out.data_ptr())
    assert w.status() == (0, 0)
    got = out.cpu().numpy()
    # the single-token matvec on the same quantized rows
    m = gpu_lib.Matrix(wq, rows, cols, device=0)
    for n in range(n_tok):
        d, qs = oracle_mod.quantize_q8_0(x[n])
        ref = oracle_mod.ref_matvec_q8(wq, d, qs, rows, cols)
        err = np.linalg.norm(got[n] - ref) / np.linalg.norm(ref)
        assert err < 1e-5, (n, err)
        if n in (0, n_tok - 1):
            dd, qd = torch.from_numpy(d).cuda(), torch.from_numpy(qs).cuda()
            mv = torch.empty(rows, dtype=torch.float32, device="cuda")
            m.matvec(dd.data_ptr(), qd.data_ptr(), mv.data_ptr())
            torch.cuda.synchronize()
            e2 = np.linalg.norm(got[n] - mv.cpu().numpy()) / np.linalg.norm(ref)
            assert e2 < 1e-5, (n, e2)
    m.Close()
    w.Close()


def test_gemm_rejects_bad_arguments(gpu_lib):
    import torch
    w = gpu_lib.GemmMatrix(np.zeros(4 * (128 // 32) * 34, np.uint8), 4, 128, device=0)
    buf = torch.empty(1 << 16, dtype=torch.uint8, device="cuda")
    with pytest.raises(gpu_lib.L3GError):
        w.gemm(buf.data_ptr(), 0, buf.data_ptr())
    with pytest.raises(gpu_lib.L3GError, match="16-byte aligned"):
        w.gemm(buf.data_ptr() + 4, 1, buf.data_ptr())
    w.Close()
