"""Tensor-parallel decomposition on CPU: two gloo ranks each take the shard
the library's l3g_shard_plan assigns them, run the decode step on their
shard in float64 numpy (heads for attention, rows for up/gate, the matching
columns for Wo / down, vocab rows for the logits), and exchange partial sums
with all_reduce / all_gather exactly where the GPU path calls NCCL.  The
result must equal the unsharded forward."""
import os

import numpy as np
import pytest

from conftest import ROOT, synthetic_model


def _tp_worker(rank, world, store_path, name, ntok, out_dir):
    import sys
    for sub in ("llama3.go_b200", "oracle", "tests"):
        sys.path.insert(0, os.path.join(ROOT, sub))
    import math

    import torch
    import torch.distributed as dist

    import l3g
    import npref
    import synthetic
    # file rendezvous: no TCP port to race for
    dist.init_process_group("gloo", init_method=f"file://{store_path}", rank=rank, world_size=world)
    cfg = synthetic.CONFIGS[name]
    T = synthetic.make_model(cfg, seed=0)
    sh = l3g.shard_plan(l3g.hparams_for(cfg), world, rank)
    full = npref.NpModel(cfg, T, 16)
    hd, e = cfg.head_dim, cfg.n_emb
    group = cfg.n_heads // cfg.n_heads_kv

    def rows(W, r0, n):
        return W[0][r0:r0 + n], W[1][r0:r0 + n]

    def cols(W, c0, n):
        return W[0][:, c0 // 32:(c0 + n) // 32], W[1][:, c0 // 32:(c0 + n) // 32]

    def mv(W, x):
        xs, xq = npref.quant_act(x)
        return npref.matvec(W[0], W[1], xs, xq)

    def allreduce(v):
        t = torch.from_numpy(v.copy())
        dist.all_reduce(t)
        return t.numpy()

    nq, nkv = sh.q_rows // hd, sh.kv_rows // hd
    K = np.zeros((cfg.n_layers, 16, nkv, hd))
    V = np.zeros_like(K)
    outs = []
    for pos, tok in enumerate(synthetic.prompt_ids(cfg, ntok, seed=3)):
        q8, d = full.emb[0][tok], full.emb[1][tok]
        x = (q8.astype(np.float64) * d[:, None]).reshape(-1)
        for l, L in enumerate(full.L):
            h = full._norm(x, L["an"])
            q = mv(rows(L["q"], sh.q_row0, sh.q_rows), h).reshape(nq, hd)
            k = mv(rows(L["k"], sh.kv_row0, sh.kv_rows), h).reshape(nkv, hd)
            v = mv(rows(L["v"], sh.kv_row0, sh.kv_rows), h).reshape(nkv, hd)
            full.pos = pos
            full._rope(q)
            full._rope(k)
            K[l, pos], V[l, pos] = k, v
            att = np.empty((nq, hd))
            for hh in range(nq):
                g = hh // group
                sc = K[l, :pos + 1, g, :] @ q[hh] / math.sqrt(hd)
                p = np.exp(sc - sc.max())
                att[hh] = (p / p.sum()) @ V[l, :pos + 1, g, :]
            x = x + allreduce(mv(cols(L["o"], sh.o_col0, sh.o_cols), att.reshape(-1)))
            h = full._norm(x, L["fn"])
            up = mv(rows(L["up"], sh.ff_row0, sh.ff_rows), h)
            gate = mv(rows(L["gate"], sh.ff_row0, sh.ff_rows), h)
            act = gate / (1 + np.exp(-gate)) * up
            x = x + allreduce(mv(cols(L["down"], sh.down_col0, sh.down_cols), act))
        h = full._norm(x, full.out_norm)
        local = np.full(sh.vocab_stride, -np.inf)
        local[:sh.vocab_rows] = mv(rows(full.out, sh.vocab_row0, sh.vocab_rows), h)
        parts = [torch.empty(sh.vocab_stride, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(local))
        outs.append(torch.cat(parts).numpy()[:cfg.vocab])
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.stack(outs))
    dist.destroy_process_group()


@pytest.mark.parametrize("name", ["tiny-gqa", "small"])
def test_tp2_decomposition_matches_single_rank(tmp_path, name):
    import torch.multiprocessing as mp

    import npref
    import synthetic
    cfg, T = synthetic_model(name)
    ntok = 4
    mp.start_processes(_tp_worker, args=(2, str(tmp_path / "store"), name, ntok, str(tmp_path)), nprocs=2,
                       join=True, start_method="spawn")
    ref_model = npref.NpModel(cfg, T, 16)
    ref = np.stack([ref_model.forward(int(t)) for t in synthetic.prompt_ids(cfg, ntok, seed=3)])
    for r in range(2):
        got = np.load(tmp_path / f"rank{r}.npy")
        assert np.allclose(got, ref, rtol=1e-9, atol=1e-9)


def test_shard_plan_covers_every_row_once():
    import l3g
    import synthetic
    for name, world in (("llama3.1-8b", 8), ("llama3.1-8b", 4), ("llama3.1-8b", 2), ("llama3.2-3b", 2),
                        ("llama3.2-3b", 4), ("llama3.2-3b", 8), ("llama3.2-1b", 8), ("tiny-gqa", 2)):
        cfg = synthetic.CONFIGS[name]
        hp = l3g.hparams_for(cfg)
        plans = [l3g.shard_plan(hp, world, r) for r in range(world)]
        for f0, fn, total in (("q_row0", "q_rows", cfg.n_emb), ("kv_row0", "kv_rows", cfg.n_heads_kv * cfg.head_dim),
                              ("o_col0", "o_cols", cfg.n_emb), ("ff_row0", "ff_rows", cfg.n_ff),
                              ("down_col0", "down_cols", cfg.n_ff), ("vocab_row0", "vocab_rows", cfg.vocab)):
            covered = []
            for p in plans:
                covered += list(range(getattr(p, f0), getattr(p, f0) + getattr(p, fn)))
            assert covered == list(range(total)), (name, world, f0)
        # Q8_0 blocks never straddle shards: column splits are multiples of 32
        assert all(p.o_col0 % 32 == 0 and p.down_col0 % 32 == 0 and p.down_cols % 32 == 0 for p in plans)
    with pytest.raises(l3g.L3GError, match="not divisible"):
        l3g.shard_plan(l3g.hparams_for(synthetic.CONFIGS["llama3.2-3b"]), 16, 0)
    with pytest.raises(l3g.L3GError, match="rank"):
        l3g.shard_plan(l3g.hparams_for(synthetic.CONFIGS["tiny-gqa"]), 2, 2)


def test_exchange_protocol_never_reads_overwritten_words():
    """Model of the tensor-parallel exchange under random interleavings of
    the ranks: rank r's program is push(1), reduce(1), push(2), reduce(2),
    ... (Wo / down push their partials for epoch e into slot r of parity
    e % 2 of every rank's buffer; the reduce kernel of epoch e waits until
    its buffer holds epoch e in every slot of that parity).  A rank's next
    kernel runs only after its previous one completed (stream order), so a
    push can never overwrite words a slower rank has not read yet: every
    reduce sees exactly its epoch, and no schedule deadlocks."""
    import random
    for world in (2, 3, 8):
        for trial in range(200):
            rng = random.Random(world * 1000 + trial)
            phases = 12
            buf = [[[0] * world for _ in range(2)] for _ in range(world)]  # [rank][parity][src]
            nxt = [0] * world  # index into the program: 2e = push(e+1), 2e+1 = reduce(e+1)
            done = 0
            while done < world:
                ready = []
                for r in range(world):
                    i = nxt[r]
                    if i >= 2 * phases:
                        continue
                    e = i // 2 + 1
                    if i % 2 == 0:
                        ready.append(r)  # a push depends only on the rank's own stream
                    elif all(buf[r][e % 2][s] == e for s in range(world)):
                        ready.append(r)  # a reduce waits for every rank's epoch e
                assert ready, "deadlock"
                r = rng.choice(ready)
                i = nxt[r]
                e = i // 2 + 1
                if i % 2 == 0:
                    for p in range(world):
                        # the words it replaces are from epoch e - 2, already read by p
                        assert buf[p][e % 2][r] in (0, e - 2)
                        assert buf[p][e % 2][r] == 0 or nxt[p] > 2 * (e - 2) - 1
                        buf[p][e % 2][r] = e
                else:
                    assert all(buf[r][e % 2][s] == e for s in range(world))
                nxt[r] += 1
                if nxt[r] == 2 * phases:
                    done += 1
