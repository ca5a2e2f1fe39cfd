"""CPU tests of the host side: GGUF container, synthetic models, the C ABI
library's exports and its host-only error paths (no GPU needed)."""
import ctypes
import os
import struct
import subprocess

import numpy as np
import pytest

from conftest import ROOT, synthetic_model


def test_gguf_round_trip(tmp_path):
    import gguf
    import synthetic
    cfg, T = synthetic_model("tiny")
    path = str(tmp_path / "t.gguf")
    synthetic.write_gguf(path, cfg, T)
    f = gguf.read_gguf(path)
    assert f.version == 3 and f.alignment == 32 and f.data_offset % 32 == 0
    assert f.get_u32("llama.embedding_length") == cfg.n_emb
    assert f.get_u32("llama.vocab_size") == cfg.vocab
    assert f.get_f32("llama.rope.freq_base") == 500000.0
    assert f.get_string("tokenizer.ggml.model") == "gpt2"
    assert {t.name for t in f.tensors} == set(T)
    for ti in f.tensors:
        assert ti.offset % 32 == 0
        assert np.array_equal(f.tensor_data(ti), T[ti.name][2].reshape(-1))
        assert list(ti.dims) == T[ti.name][0]


def test_gguf_typed_getters_follow_reference():
    """GetU32 takes UINT32 or a fitting UINT64 only; GetF32 FLOAT32 only
    (gguf.go:391-432)."""
    import gguf
    f = gguf.GGUFFile(version=3)
    f.kv = {"a": (gguf.T_UINT32, 7), "b": (gguf.T_UINT64, 9), "c": (gguf.T_UINT64, 1 << 40),
            "d": (gguf.T_INT32, 5), "e": (gguf.T_FLOAT32, 1.5), "g": (gguf.T_FLOAT64, 2.5)}
    assert f.get_u32("a") == 7 and f.get_u32("b") == 9
    assert f.get_u32("c") is None and f.get_u32("d") is None and f.get_u32("zz") is None
    assert f.get_f32("e") == 1.5 and f.get_f32("g") is None


def test_synthetic_q8_0_blocks():
    """Weights are N(0, 0.02): scales ~ maxabs/127 (never fp16-subnormal),
    q within [-127, 127], and the model is deterministic per seed."""
    import synthetic
    cfg, T = synthetic_model("tiny")
    b = T["blk.0.ffn_up.weight"][2].reshape(-1, 34)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)[:, 0]
    q = b[:, 2:].view(np.int8)
    assert (d > 6.1e-5).all() and (np.abs(q) <= 127).all()
    w = q.astype(np.float32) * d[:, None]
    assert abs(w.std() - 0.02) < 0.002
    T2 = synthetic.make_model(cfg, seed=0)
    assert all(np.array_equal(T[k][2], T2[k][2]) for k in T)


def test_workload_byte_counts():
    """Algorithmic bytes per token used for the roofline (Q8_0, 34 B / 32)."""
    import synthetic
    c8 = synthetic.CONFIGS["llama3.1-8b"]
    assert abs(c8.weight_bytes() / 1e9 - 7.9737) < 1e-3
    assert abs(synthetic.CONFIGS["llama3.2-1b"].weight_bytes() / 1e9 - 1.3130) < 1e-3
    assert abs(synthetic.CONFIGS["llama3.2-3b"].weight_bytes() / 1e9 - 3.4134) < 1e-3
    assert c8.kv_bytes(1) == 262144


def _lib():
    import build
    build.build(quiet=True)
    import l3g
    return l3g


def test_library_exports_every_declared_symbol():
    l3g = _lib()
    L = l3g.lib()
    declared = l3g.exported_symbols()
    assert len(declared) >= 25
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", l3g.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    assert all(f" {s}" in out for s in declared)
    assert L.l3g_version() == 1


def test_build_targets_sm100a_only():
    import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_gguf_loader_host_errors(tmp_path):
    """l3g_model_load_gguf rejects bad files before touching the GPU, with the
    reference's messages (gguf.go:73, model.go:210)."""
    l3g = _lib()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE" + b"\0" * 64)
    with pytest.raises(l3g.L3GError, match="not a gguf file") as e:
        l3g.LoadModel(str(bad))
    assert e.value.code == l3g.L3G_E_FORMAT
    import gguf
    w = gguf.GGUFWriter()
    w.add("llama.block_count", gguf.T_UINT32, 2)
    p = str(tmp_path / "nohp.gguf")
    w.write(p)
    with pytest.raises(l3g.L3GError, match="missing required llama"):
        l3g.LoadModel(p)
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(open(p, "rb").read()[:30])
    with pytest.raises(l3g.L3GError):
        l3g.LoadModel(str(trunc))
    with pytest.raises(l3g.L3GError, match="open"):
        l3g.LoadModel(str(tmp_path / "missing.gguf"))


def test_library_fails_loudly_without_a_gpu():
    """No silent CPU fallback: without a device every compute entry errors."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    l3g = _lib()
    n = ctypes.c_int32(-1)
    assert l3g.lib().l3g_device_count(ctypes.byref(n)) != 0
    with pytest.raises(l3g.L3GError):
        l3g.Matrix(np.zeros(34, np.uint8), 1, 32)


def test_c_abi_from_plain_c(tmp_path):
    """The header and the library as a cgo preamble sees them: tests/c_abi_check.c
    compiled as strict C99 (no C++), linked against libl3g.so and run without
    a GPU (host-only entries, error codes and messages, null handles)."""
    l3g = _lib()
    exe = str(tmp_path / "c_abi_check")
    libdir = os.path.dirname(l3g.LIB_PATH)
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic",
                    "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c_abi_check.c"),
                    "-L", libdir, "-ll3g", f"-Wl,-rpath,{libdir}", "-o", exe], check=True)
    out = subprocess.run([exe, str(tmp_path)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and out.stdout.strip() == "ok", out.stderr


def _split_args(text, open_at):
    """Top-level comma-separated arguments of the call whose '(' is at
    text[open_at]; returns (args, index after the closing ')')."""
    depth, cur, args, i = 0, "", [], open_at
    while True:
        ch = text[i]
        if ch in "([{":
            depth += 1
            if depth > 1:
                cur += ch
        elif ch in ")]}":
            depth -= 1
            if depth == 0:
                break
            cur += ch
        elif ch == "," and depth == 1:
            args.append(cur.strip())
            cur = ""
        else:
            cur += ch
        i += 1
    if cur.strip():
        args.append(cur.strip())
    return args, i + 1


def test_go_shim_calls_match_the_header():
    """Every C.l3g_* call of the Go shim (go/cuda.go, the cgo file a
    maintainer adds as internal/llama/cuda.go) names a function the header
    declares, with as many arguments as the
    declaration; every C.l3g_* type and C.L3G_* constant it uses exists."""
    import re
    hdr = open(os.path.join(ROOT, "include", "l3g.h")).read()
    nparams = {}
    for mt in re.finditer(r"\b(l3g_[a-z0-9_]+)\s*\(", hdr):
        args, _ = _split_args(hdr, mt.end() - 1)
        nparams[mt.group(1)] = 0 if args == ["void"] else len(args)
    go = open(os.path.join(ROOT, "go", "cuda.go")).read()
    assert "C.l3g_forward" in go
    calls = 0
    for mt in re.finditer(r"\bC\.(l3g_[a-z0-9_]+)\s*\(", go):
        name = mt.group(1)
        assert name in nparams, name
        args, _ = _split_args(go, mt.end() - 1)
        assert len(args) == nparams[name], (name, args, nparams[name])
        calls += 1
    assert calls >= 8
    for name in set(re.findall(r"\bC\.(l3g_[a-z0-9_]+)\b(?!\s*\()", go)):
        assert re.search(r"\b%s\s*;" % name, hdr), name  # a typedef name
    for name in set(re.findall(r"\bC\.(L3G_[A-Z0-9_]+)", go)):
        assert re.search(r"#define\s+%s\b" % name, hdr), name


def test_header_cites_reference_for_each_entry():
    hdr = open(os.path.join(ROOT, "include", "l3g.h")).read()
    for ref in ("simd.h:7-9", "workers.go", "infer.go:21-267", "infer.go:269-511",
                "model.go:55-156", "state.go:51-64", "workspace.go:35-69", "q8_0.go:22-79"):
        assert ref in hdr, ref


def test_philox_known_answers():
    """The test-side Philox4x32-10 reproduces the published known-answer
    values (counter, key) -> output of the algorithm."""
    from sampler_ref import philox4x32_10
    kat = [
        ([0, 0, 0, 0], [0, 0], [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]),
        ([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2, [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]),
        ([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0],
         [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]),
    ]
    for ctr, key, want in kat:
        assert philox4x32_10(ctr, key) == want


def test_sampler_restatement_is_a_distribution():
    """Over many draw indices the restated sampler picks each item with its
    softmax probability (chi-square-free check: every frequency within 4
    standard deviations)."""
    import math
    from sampler_ref import sample_topk
    ids = [10, 11, 12, 13]
    logits = [2.0, 1.0, 0.5, -1.0]
    T, n = 0.8, 20000
    counts = {i: 0 for i in ids}
    for c in range(n):
        counts[sample_topk(ids, logits, T, 1234, c)] += 1
    e = [math.exp((l - 2.0) / T) for l in logits]
    for i, p in zip(ids, [v / sum(e) for v in e]):
        assert abs(counts[i] - n * p) < 4 * math.sqrt(n * p * (1 - p)), (i, counts[i], n * p)
