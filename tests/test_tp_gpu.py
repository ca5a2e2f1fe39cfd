"""Tensor parallel on 2 GPUs: one process per GPU, the library's own NCCL
communicator (the unique id travels through a file), the shard split of
l3g_shard_plan.  Rank 0's logits must match the reference within the same
band as the single-GPU path, and both ranks must agree on every greedy id.
Skipped on a machine with fewer than two GPUs.
"""
import os
import time

import numpy as np
import pytest

from conftest import synthetic_model
from refspread import ReferenceRuns, rel_l2

pytestmark = pytest.mark.gpu

CONFIG, N_TOK, CTX = "mid", 12, 64


def _rank_main(rank, world, id_path, out_dir, path):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for sub in ("llama3.go_b200", "oracle", "tests"):
        sys.path.insert(0, os.path.join(root, sub))
    if path == "nccl":
        os.environ["L3G_TP_NCCL"] = "1"
    if path == "persistent":
        os.environ["L3G_PERSIST"] = "1"
    import l3g
    import synthetic
    from conftest import synthetic_model as sm
    cfg, T = sm(CONFIG)
    if rank == 0:
        nid = l3g.nccl_unique_id()
        with open(id_path + ".tmp", "wb") as f:
            f.write(nid)
        os.replace(id_path + ".tmp", id_path)
    else:
        t0 = time.time()
        while not os.path.exists(id_path):
            if time.time() - t0 > 120:
                raise TimeoutError("no NCCL id from rank 0")
            time.sleep(0.05)
        nid = open(id_path, "rb").read()
    opts = l3g.default_options(world, rank, rank, l3g.L3G_KV_F32, nid)
    m = l3g.LoadModelFromTensors(l3g.hparams_for(cfg), T, opts)
    s = m.NewState(CTX)
    ws = m.NewWorkspace(CTX, 40)
    if ws.tp_p2p() != (path != "nccl"):
        raise RuntimeError(f"workspace reduction path is not {path}")
    if ws.persistent() != (path == "persistent"):
        raise RuntimeError("persistent layer kernel not as requested")
    ids = synthetic.prompt_ids(cfg, N_TOK, seed=17)
    logits = np.empty(cfg.vocab, np.float32)
    out = []
    for t in ids:
        m.ForwardIntoWorkspace(s, int(t), logits, ws)
        out.append(logits.copy())
    # greedy continuation through the device argmax (allgathered per rank)
    tok, greedy = int(ids[-1]), []
    for _ in range(8):
        tok, _ = m.ForwardArgmax(s, tok, ws)
        greedy.append(tok)
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), logits=np.stack(out),
             greedy=np.array(greedy, np.int32))
    ws.Close()
    s.Close()
    m.Close()


def _threads_main(out_dir):
    """Both ranks as threads of this (spawned) process."""
    import sys
    import threading
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for sub in ("llama3.go_b200", "oracle", "tests"):
        sys.path.insert(0, os.path.join(root, sub))
    import l3g
    import synthetic
    from conftest import synthetic_model as sm
    cfg, T = sm(CONFIG)
    ids = synthetic.prompt_ids(cfg, N_TOK, seed=17)
    nid = l3g.nccl_unique_id()
    out, errors = {}, []

    def run(rank):
        try:
            opts = l3g.default_options(2, rank, rank, l3g.L3G_KV_F32, nid)
            m = l3g.LoadModelFromTensors(l3g.hparams_for(cfg), T, opts)
            s, ws = m.NewState(CTX), m.NewWorkspace(CTX, 40)
            p2p = ws.tp_p2p()
            logits = np.empty(cfg.vocab, np.float32)
            rows = []
            for t in ids:
                m.ForwardIntoWorkspace(s, int(t), logits, ws)
                rows.append(logits.copy())
            out[rank] = (p2p, np.stack(rows))
            ws.Close()
            s.Close()
            m.Close()
        except Exception as ex:
            errors.append(f"rank {rank}: {ex!r}")

    th = [threading.Thread(target=run, args=(r,), daemon=True) for r in range(2)]
    for x in th:
        x.start()
    for x in th:
        x.join(240)
    if any(x.is_alive() for x in th) or errors or len(out) != 2:
        with open(os.path.join(out_dir, "errors.txt"), "w") as f:
            f.write("\n".join(errors) or "a rank thread did not finish")
        os._exit(1)
    np.savez(os.path.join(out_dir, "threads.npz"), p2p=np.array([out[0][0], out[1][0]]),
             l0=out[0][1], l1=out[1][1])


def test_tp2_ranks_as_threads_of_one_process(gpu_lib, oracle_mod, tmp_path):
    """Two ranks driven by two threads of one process (the layout of a Go
    caller with one OS thread per GPU): the peer buffers are reached through
    unified addressing instead of IPC, and the results match the reference."""
    import torch
    import torch.multiprocessing as mp
    import synthetic
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    p = mp.get_context("spawn").Process(target=_threads_main, args=(str(tmp_path),))
    p.start()
    p.join(300)
    if p.is_alive():
        p.kill()
        p.join(10)
        pytest.fail("the two-thread run did not finish")
    err = tmp_path / "errors.txt"
    assert p.exitcode == 0, err.read_text() if err.exists() else p.exitcode
    z = np.load(tmp_path / "threads.npz")
    assert z["p2p"].all(), "same-process peers should use peer memory"
    assert np.array_equal(z["l0"], z["l1"])
    cfg, T = synthetic_model(CONFIG)
    ids = synthetic.prompt_ids(cfg, N_TOK, seed=17)
    R = ReferenceRuns(oracle_mod, cfg, T, ids, CTX, with_f64=False)
    errs = [rel_l2(z["l0"][i], R.cgo[i]) for i in range(N_TOK)]
    assert max(errs) < R.tol(), (errs, R.band())


@pytest.mark.parametrize("path", ["p2p", "nccl", "persistent"])
def test_tp2_matches_reference_and_single_gpu(gpu_lib, oracle_mod, tmp_path, path):
    """Both reductions: partial sums pushed over peer memory by the Wo / down
    matvecs and summed by the next kernel (p2p), and NCCL allreduces; and the
    persistent layer kernel, whose Wo / down phases push over peer memory
    and whose reduce phase sums the ranks' rows inside the same launch."""
    import torch
    import torch.multiprocessing as mp
    import synthetic
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    id_path = str(tmp_path / "nccl_id")
    procs = [ctx.Process(target=_rank_main, args=(r, 2, id_path, str(tmp_path), path)) for r in range(2)]
    for p in procs:
        p.start()
    deadline = time.time() + 600
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.time()))
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
        p.join(10)
    assert not alive, "a tensor-parallel rank did not finish"
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    r0 = np.load(tmp_path / "rank0.npz")
    r1 = np.load(tmp_path / "rank1.npz")
    assert np.array_equal(r0["greedy"], r1["greedy"])
    assert np.array_equal(r0["logits"], r1["logits"])  # allgathered: identical on every rank

    cfg, T = synthetic_model(CONFIG)
    ids = synthetic.prompt_ids(cfg, N_TOK, seed=17)
    R = ReferenceRuns(oracle_mod, cfg, T, ids, CTX, with_f64=False)
    errs = [rel_l2(r0["logits"][i], R.cgo[i]) for i in range(N_TOK)]
    assert max(errs) < R.tol(), (errs, R.band())
    # the single-GPU library on the same inputs
    m = gpu_lib.LoadModelFromTensors(gpu_lib.hparams_for(cfg), T, gpu_lib.default_options(device=0))
    s = m.NewState(CTX)
    ws = m.NewWorkspace(CTX, 40)
    logits = np.empty(cfg.vocab, np.float32)
    for i, t in enumerate(ids):
        m.ForwardIntoWorkspace(s, int(t), logits, ws)
        assert rel_l2(r0["logits"][i], logits) < R.tol()
