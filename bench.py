#!/usr/bin/env python
"""Decode benchmark of libl3g on B200.

Default workload: Llama-3.1-8B-shaped synthetic Q8_0 model (dim 4096, 32
layers, 32/8 heads, FFN 14336, vocab 128256, llama3 RoPE scaling), KV cache
prefilled with 4096 seeded tokens, then greedy decode at batch 1.  One
"step" is one decoded token.  With --gpus N (under torchrun) the model is
tensor-parallel over N GPUs.

Prints one JSON line:
  value  decode tok/s with the step loop resident on the device (each token
         fed from the previous step's on-device argmax), CUDA-event timed;
  e2e    the same tok/s through the public per-step call
         (l3g_forward_argmax: host token in, pinned H2D, graph, D2H result);
  roofline       the dominant kernel as the step runs it (the up/gate matvec
                 with its RMSNorm prologue and SwiGLU epilogue), its active
                 time on the step's device timeline against measured HBM
                 bandwidth (the standalone matvec, CUDA-event timed, beside it);
  decode_roofline  (weight + KV bytes per token) x tok/s / HBM bandwidth;
  cpu_baseline   the oracle (C restatement + the reference's own simd.c) on
                 the host cores, on a bounded sample of the same workload.

--impl reference times only the reference's CPU path (the oracle) on this
workload.  --workload matvec runs the Q8_0 matvec microbench instead;
--workload gemm the batched tensor-core product microbench, --workload
prefill batched prefill against token-by-token ingest, --workload batched the
64-session batched decode (tensor parallel under torchrun).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "llama3.go_b200"))

METRIC = "decode tok/s at 1/2/4/8 B200 (Llama-8B-shape Q8_0, bs1); % of HBM roofline"
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="l3g", choices=["l3g", "reference"])
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "matvec", "gemm", "prefill", "batched"])
    ap.add_argument("--config", default="llama3.1-8b")
    ap.add_argument("--prefill", type=int, default=4096)
    ap.add_argument("--kv", default="f32", choices=["f32", "f16"])
    ap.add_argument("--prefill-mode", default="batched", choices=["batched", "token"],
                    help="how the decode workload's prompt is ingested (not timed in value)")
    ap.add_argument("--persistent", action="store_true",
                    help="decode with the persistent layer kernel (every layer in one launch)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the matvec microbench and 1B-shape lines of the default run")
    ap.add_argument("--iters", type=int, default=1000, help="matvec microbench iterations")
    ap.add_argument("--tokens", default="16,64,128", help="gemm microbench token counts")
    ap.add_argument("--seqs", type=int, default=64, help="batched decode sessions")
    ap.add_argument("--ctx-min", type=int, default=512, help="batched decode shortest context")
    ap.add_argument("--ctx-max", type=int, default=8192, help="batched decode longest context")
    ap.add_argument("--shapes", default="4096x4096,1024x4096,14336x4096,4096x14336,128256x4096",
                    help="matvec microbench shapes, rows x cols")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(summary: str):
    """DRAM bytes (read + write) per launch that an ncu capture of the kernel
    measured, from the summary committed under profiles/ (None if absent)."""
    import re
    p = os.path.join(ROOT, "profiles", summary)
    if not os.path.exists(p):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*(\d+)", open(p).read())
    return int(m.group(1)) if m else None


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: str):
        """device: what nvidia-smi -i accepts (an index or a UUID)."""
        self.dev = device
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", device, f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "50"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def wait_first_sample(self, timeout_s: float = 5.0):
        """Blocks (bounded) until the sampler has written a row, so the timed
        region that follows is covered from its start."""
        if self.p is None:
            return
        t0 = time.time()
        while time.time() - t0 < timeout_s and self.p.poll() is None:
            try:
                with open(self.f.name) as g:
                    if any(len(r.split(",")) >= 9 for r in g.read().splitlines()):
                        return
            except OSError:
                pass
            time.sleep(0.02)

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        rows = [[c.strip() for c in r] for r in rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max((float(r[3]) for r in rows if r[3].replace(".", "").isdigit()), default=None)}


def physical_index(local: int) -> str:
    """The nvidia-smi identifier (index or UUID) of CUDA device `local`."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = [p.strip() for p in vis.split(",") if p.strip()]
        if local < len(parts):
            return parts[local]
    return str(local)


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class Dist:
    def __init__(self, world, rank, local):
        import torch
        self.world, self.rank, self.local = world, rank, local
        self.torch = torch
        self.pg = None
        if world > 1:
            import datetime
            import torch.distributed as dist
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
            self.dist = dist
            self.pg = True

    def barrier(self):
        if self.pg:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def bcast_bytes(self, b):
        if not self.pg:
            return b
        obj = [b]
        self.dist.broadcast_object_list(obj, src=0)
        return obj[0]

    def close(self):
        if self.pg:
            self.dist.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU path (the oracle): cpu_baseline and the reference arm
# ---------------------------------------------------------------------------
def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_decode_rate(cfg, T, prefill, seconds, max_steps, seed, warmup=1):
    """Greedy decode steps of the reference's chat path (ForwardTopK with
    topK 40 and its fastExp attention, argmax over the items) at position
    `prefill`, the KV cache of the earlier positions filled with seeded
    values (the step's cost does not depend on them).  It reads the same
    bytes per token as the full-logits greedy path timed on the GPU (every
    layer's weights, the whole KV prefix, the logits matrix); `warmup` steps
    run untimed first.  Returns (tok/s, steps, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle
    oracle.build()
    threads = host_cores()
    om = oracle.OracleModel(cfg, T, threads=threads)
    om.new_state(prefill + max_steps + 2)
    K, V = om.kv_arrays()
    rng = np.random.default_rng(seed)
    chunk = 1 << 24
    for arr in (K, V):
        for i in range(0, arr.size, chunk):
            n = min(chunk, arr.size - i)
            arr[i:i + n] = rng.random(n, dtype=np.float32) - 0.5
    om.pos = prefill - 1
    tok = int(rng.integers(0, cfg.vocab))
    for _ in range(max(0, warmup - 1)):
        ids, lg = om.forward_topk(tok, 40)
        tok = int(ids[int(np.argmax(lg))])
    t0 = time.perf_counter()
    ids, lg = om.forward_topk(tok, 40)
    first = time.perf_counter() - t0
    n = int(max(1, min(max_steps, round(seconds / max(first, 1e-6)))))
    tok = int(ids[int(np.argmax(lg))])
    t0 = time.perf_counter()
    for _ in range(n):
        ids, lg = om.forward_topk(tok, 40)
        tok = int(ids[int(np.argmax(lg))])
    el = time.perf_counter() - t0
    om.close()
    return n / el, n, om.threads


def make_host_model(cfg, seed, device):
    import synthetic
    return synthetic.make_model(cfg, seed=seed, device=device)


def run_reference(args):
    world, rank, local = dist_env()
    if rank != 0:
        return 0
    import synthetic
    import torch
    cfg = synthetic.CONFIGS[args.config]
    dev = f"cuda:{local}" if torch.cuda.is_available() else "cpu"
    T = make_host_model(cfg, args.seed, dev)
    # each step is one decoded token; at most ~90 s of timed CPU work so the
    # whole run ends within a few minutes
    rate, n, threads = cpu_decode_rate(cfg, T, args.prefill, 90.0, max(1, args.steps), args.seed + 1,
                                       warmup=max(1, args.warmup))
    sample = (f"{n} greedy decode steps of the {cfg.name} shape at position {args.prefill} "
              f"(KV of earlier positions seeded), after {max(1, args.warmup)} untimed steps; the "
              f"reference's ForwardTopKIntoWorkspace path (fastExp attention, topK 40), which reads "
              f"the same bytes per token as the greedy full-logits path the GPU arm times")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(rate, 4), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": n, "warmup": max(1, args.warmup),
        "ms_per_step": round(1000.0 / rate, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic",
        "config": {"workload": f"{cfg.name}-shape Q8_0 bs1 greedy decode after {args.prefill}-token prefill",
                   "model": cfg.name, "global_batch": 1, "seq_len": args.prefill, "parallelism": "cpu"},
        "cpu_baseline": {"value": round(rate, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sample,
                         "what": "C restatement of internal/llama/infer.go linked to the reference's own "
                                 "internal/llama/simd.c (AVX2, compiled from the reference tree)"},
        "e2e": {"value": round(rate, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# the GPU arm
# ---------------------------------------------------------------------------
def time_matvec_kernel(l3g, cfg, seed, hbm):
    """Live timing of the dominant kernel: the Q8_0 matvec on the FFN up/gate
    shape ([2*n_ff x n_emb], the largest per-layer matrix), rotating over
    copies that together exceed L2, CUDA events on the launching stream."""
    import numpy as np
    import synthetic
    import torch
    rows, cols = 2 * cfg.n_ff, cfg.n_emb
    ncopy = 3
    mats = []
    for i in range(ncopy):
        g = torch.Generator(device="cuda").manual_seed(seed * 31 + i)
        w = synthetic.quantize_q8_0_rows(torch.randn(rows, cols, generator=g, device="cuda") * 0.02, torch)
        mats.append(l3g.Matrix(w.cpu().numpy(), rows, cols))
        del w
    x = torch.randn(cols, device="cuda")
    nb = cols // 32
    d = torch.empty(nb, device="cuda")
    q = torch.empty(nb * 32, dtype=torch.int8, device="cuda")
    l3g.quantize_q8_0_device(x.data_ptr(), cols, d.data_ptr(), q.data_ptr())
    out = torch.empty(rows, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for i in range(6):
        mats[i % ncopy].matvec(d.data_ptr(), q.data_ptr(), out.data_ptr(), stream=stream)
    iters = 90
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for i in range(iters):
        mats[i % ncopy].matvec(d.data_ptr(), q.data_ptr(), out.data_ptr(), stream=stream)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    alg = rows * cols // 32 * 34 + cols + nb * 4 + rows * 4
    for mtx in mats:
        mtx.Close()
    return {"kernel": "k_matvec (Q8_0 matvec, FFN up/gate shape %dx%d)" % (rows, cols),
            "bytes_per_launch": alg, "ms_per_launch": ms, "achieved_gbs": alg / ms / 1e6}


def trace_summary(m, s, ws, tok, pos, reps=3):
    """Device timeline of one step replayed as its graph (kernels overlapping
    as in the timed loop): per kind, the time between consecutive kernel
    completions (sums to the step), the span from entry to exit, the active
    time from dependency release to the last exit, the time from dependency
    release to the end of the prologue, and the tail from the last CTA's end
    of tile loop to the last exit."""
    import numpy as np
    acc = {}
    step_us = []
    for _ in range(reps):
        s.Pos = pos
        recs = [(k, st) for k, st in m.TraceStep(s, tok, ws) if (st[:, 0] > 0).any()]
        first = min(st[:, 0][st[:, 0] > 0].min() for _, st in recs)
        prev_exit = first
        for kind, st in recs:
            live = st[:, 0] > 0
            ent = st[live, 0].min()
            ext = st[live, 4].max()
            released = st[live, 1].min()
            d = acc.setdefault(kind, {"critical": 0.0, "span": 0.0, "active": 0.0, "prologue": 0.0,
                                      "wake": 0.0, "tail": 0.0, "n": 0})
            d["critical"] += (ext - prev_exit) / 1e3
            d["span"] += (ext - ent) / 1e3
            d["active"] += (ext - released) / 1e3
            d["wake"] += max(0, released - prev_exit) / 1e3
            pro = st[live, 2]
            if (pro > 0).all():
                d["prologue"] += (pro.max() - released) / 1e3
            loop = st[live, 3]
            if (loop > 0).all():
                d["tail"] += max(0, ext - loop.max()) / 1e3
            d["n"] += 1
            prev_exit = max(prev_exit, ext)
        step_us.append((prev_exit - first) / 1e3)
    out = {k: {"critical_us": round(v["critical"] / reps, 1), "avg_span_us": round(v["span"] / v["n"], 2),
               "avg_active_us": round(v["active"] / v["n"], 3),
               "avg_wake_us": round(v["wake"] / v["n"], 2), "avg_prologue_us": round(v["prologue"] / v["n"], 2),
               "avg_tail_us": round(v["tail"] / v["n"], 2),
               "launches": v["n"] // reps}
           for k, v in sorted(acc.items(), key=lambda kv: -kv[1]["critical"])}
    out["traced_step_us"] = round(float(np.mean(step_us)), 1)
    return out


def persist_phases(bpl):
    """Names of a layer's phases, one per grid barrier, for the fusions in
    effect (7 barriers: none; 5: both; 6: the one whose variable is set)."""
    fuse_merge = bpl == 5 or (bpl == 6 and os.environ.get("L3G_PERSIST_FUSE_MERGE") == "1")
    fuse_quant = bpl == 5 or (bpl == 6 and not fuse_merge)
    names = ["qkv", "attention_merge" if fuse_merge else "attention"]
    if not fuse_merge:
        names.append("merge")
    names += ["wo", "upgate_act_quant" if fuse_quant else "upgate"]
    if not fuse_quant:
        names.append("act_quant")
    names.append("down")
    assert len(names) == bpl, (names, bpl)
    return tuple(names)


def persist_summary(m, s, ws, tok, pos, reps=3):
    """Barrier timeline of the persistent layer kernel (one traced step
    replayed as its graph): per phase, the mean time per layer from the
    last CTA's release at the previous barrier to the last CTA's arrival at
    this one (the phase's critical path), and the mean barrier latency (last
    arrival to last release)."""
    import numpy as np
    bpl = ws.persist_layout()["barriers_per_layer"]
    names = persist_phases(bpl)
    acc = {n: [] for n in names}
    lat = []
    for _ in range(reps):
        s.Pos = pos
        m.TraceStep(s, tok, ws)
        st = ws.persist_stamps()
        arr, rel = st[..., 0], st[..., 1]
        prev = None
        for b in range(st.shape[0]):
            if (arr[b] == 0).all():
                continue
            if prev is not None:
                acc[names[b % bpl]].append((arr[b].max() - prev) / 1e3)
            lat.append((rel[b].max() - arr[b].max()) / 1e3)
            prev = rel[b].max()
    out = {k: round(float(np.mean(v)), 2) for k, v in acc.items() if v}
    out["barrier_latency_us"] = round(float(np.mean(lat)), 2)
    return out


def progress(world, rank, msg):
    """Rank-tagged progress on stderr for multi-GPU runs (stdout keeps the
    single JSON line)."""
    if world > 1:
        print(f"[rank {rank} {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def run_l3g(args):
    world, rank, local = dist_env()
    if world != args.gpus:
        args.gpus = world
    import numpy as np
    import torch
    import build
    build.build(quiet=True)
    import l3g
    import synthetic
    D = Dist(world, rank, local)
    torch.cuda.set_device(local)
    hbm, hbm_kind = peaks()
    cfg = synthetic.CONFIGS[args.config]

    progress(world, rank, "generating the synthetic model")
    T = make_host_model(cfg, args.seed, f"cuda:{local}")
    torch.cuda.empty_cache()
    progress(world, rank, "loading the model")
    nid = D.bcast_bytes(l3g.nccl_unique_id() if (world > 1 and rank == 0) else None) if world > 1 else None
    kv = l3g.L3G_KV_F16 if args.kv == "f16" else l3g.L3G_KV_F32
    opts = l3g.default_options(world, rank, local, kv, nid)
    if args.persistent:
        os.environ["L3G_PERSIST"] = "1"
    m = l3g.LoadModelFromTensors(l3g.hparams_for(cfg), T, opts)
    os.environ.pop("L3G_PERSIST", None)
    ctx = args.prefill + args.warmup + args.steps + 2
    if ctx > cfg.ctx_len:
        raise SystemExit(f"prefill+warmup+steps exceeds the model context {cfg.ctx_len}")
    s = m.NewState(ctx)
    ws = m.NewWorkspace(ctx, 40)
    if args.persistent and not ws.persistent():
        raise SystemExit("--persistent: the workspace did not enable the persistent layer kernel")
    ps_layout = ws.persist_layout() if args.persistent else None
    prompt = synthetic.prompt_ids(cfg, args.prefill, seed=args.seed)
    progress(world, rank, "prefill")
    t0 = time.perf_counter()
    if args.prefill_mode == "batched":  # the tensor-core product, 512 tokens per pass
        m.PrefillBatched(s, prompt[:-1], ws)
    else:  # token by token, like the reference's ingest (main.go:276-286)
        m.Prefill(s, prompt[:-1], ws)
    prefill_s = time.perf_counter() - t0
    p0 = s.Pos

    # value: device-resident greedy loop
    progress(world, rank, "decode warm-up")
    warm, _ = m.DecodeGreedy(s, int(prompt[-1]), max(1, args.warmup), ws)
    clk = Clocks(physical_index(local))
    clk.wait_first_sample()
    # ranks enter the timed loop together (its steps wait on each other's
    # exchanges, so a late rank's start would count in an early rank's time)
    D.barrier()
    torch.cuda.nvtx.range_push("l3g_decode")
    toks, dev_ms = m.DecodeGreedy(s, int(warm[-1]), args.steps, ws)
    torch.cuda.nvtx.range_pop()
    D.barrier()
    clocks = clk.stop()
    dev_ms = D.max(dev_ms)
    value = args.steps / (dev_ms / 1000.0)
    kernels = ws.kernels_per_step()

    progress(world, rank, "e2e")
    # e2e: the public per-step call, host token in / host token out
    s.Pos = p0
    tok = int(prompt[-1])
    for _ in range(max(1, args.warmup)):
        tok, _ = m.ForwardArgmax(s, tok, ws)
    D.barrier()
    t0 = time.perf_counter()
    e2e_toks = []
    for _ in range(args.steps):
        tok, _ = m.ForwardArgmax(s, tok, ws)
        e2e_toks.append(tok)
    D.barrier()
    e2e_s = D.max(time.perf_counter() - t0)
    e2e = args.steps / e2e_s
    same = bool(np.array_equal(np.array(e2e_toks, np.int32), toks))

    progress(world, rank, "per-kernel profile")
    # per-kernel device time of one step at this context (eager, serialized)
    s.Pos = p0 + max(1, args.warmup)
    prof = {}
    for _ in range(3):
        for kind, us in m.ProfileStep(s, tok, ws):
            prof[kind] = prof.get(kind, 0.0) + us / 3
        s.Pos = p0 + max(1, args.warmup)
    prof = {k: round(v, 1) for k, v in sorted(prof.items(), key=lambda kv: -kv[1])}
    ws_grid = torch.cuda.get_device_properties(local).multi_processor_count
    progress(world, rank, "device timeline")
    timeline = trace_summary(m, s, ws, tok, p0 + max(1, args.warmup))
    phases = persist_summary(m, s, ws, tok, p0 + max(1, args.warmup)) if args.persistent else None
    progress(world, rank, "matvec timing and wrap-up")

    # roofline of the whole decode step (weights + KV read per token)
    es = 2 if args.kv == "f16" else 4
    first_pos = p0 + max(1, args.warmup)
    kv_bytes = sum(cfg.kv_bytes(first_pos + i + 1, es) for i in range(args.steps)) / args.steps
    step_bytes = cfg.weight_bytes() + kv_bytes
    decode_gbs = step_bytes * value / 1e9
    if args.persistent:
        # the dominant kernel is the persistent launch itself: every layer's
        # weights plus the KV cache at the profiled position, over its
        # CUDA-event time in the eager profile
        layer_bytes = cfg.weight_bytes() - cfg.vocab * cfg.n_emb // 32 * 34 - cfg.n_emb // 32 * 34
        alg = (layer_bytes + cfg.kv_bytes(first_pos + 1, es)) // world
        ms = prof["layers"] / 1e3
        mv = {"kernel": "k_layers (persistent: every layer of the step, %d CTAs)" % ws_grid,
              "bytes_per_launch": alg, "ms_per_launch": ms, "achieved_gbs": alg / ms / 1e6}
    else:
        # the dominant kernel as the step runs it: the up/gate matvec
        # (k_matvec<PRO_RMS, EPI_SWIGLU>: residual + RMSNorm + act-quant
        # prologue, the 2*n_ff x n_emb Q8_0 matrix, SwiGLU epilogue), its
        # active time on the step's device timeline (dependency release to
        # the last CTA's exit, averaged over the layers of the traced steps)
        ug = timeline.get("upgate_swiglu") if isinstance(timeline, dict) else None
        rows_ug = 2 * cfg.n_ff // world
        alg_ug = rows_ug * cfg.n_emb // 32 * 34 + 3 * cfg.n_emb * 4 + rows_ug // 2 * 4
        standalone = time_matvec_kernel(l3g, cfg, args.seed, hbm) if rank == 0 else None
        if ug and ug.get("avg_active_us", 0) > 0:
            ms = ug["avg_active_us"] / 1e3
            mv = {"kernel": "k_matvec<PRO_RMS, EPI_SWIGLU> in the decode step (FFN up/gate %dx%d)"
                            % (rows_ug, cfg.n_emb),
                  "bytes_per_launch": alg_ug, "ms_per_launch": ms, "achieved_gbs": alg_ug / ms / 1e6,
                  "timing": "device timeline of the step replayed as its graph: dependency release "
                            "to the last CTA's exit, mean over %d launches" % ug.get("launches", 0),
                  "standalone_events": None if standalone is None else {
                      "kernel": standalone["kernel"], "ms_per_launch": round(standalone["ms_per_launch"], 5),
                      "achieved_gbs": round(standalone["achieved_gbs"], 1),
                      "timing": "CUDA events over 90 launches of the pre-quantized matvec on rotating copies"}}
        else:
            mv = standalone

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, n, threads = cpu_decode_rate(cfg, T, args.prefill, args.cpu_seconds, 64, args.seed + 1)
        cpu = {"value": round(rate, 4), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"{n} greedy decode steps of the {cfg.name} shape at position {args.prefill} "
                         f"(KV of earlier positions seeded), the reference's ForwardTopKIntoWorkspace "
                         f"path (fastExp attention, topK 40: the same bytes per token as the greedy "
                         f"full-logits path timed on the GPU); C restatement of infer.go + the "
                         f"reference's own simd.c"}
    # workspace and state first: the workspace's step graphs hold NCCL calls
    # on the model's communicator
    ws.Close()
    s.Close()
    m.Close()
    D.close()
    extras = {}
    if rank == 0 and world == 1 and not args.no_extras:
        # the matvec microbench shapes and the 1B-shape decode, a few seconds
        progress(world, rank, "matvec microbench and the 1B-shape decode")
        del T
        torch.cuda.empty_cache()
        shapes = [tuple(int(v) for v in sh.split("x")) for sh in args.shapes.split(",") if sh]
        extras["matvec_microbench"] = matvec_sweep(l3g, shapes, 300, hbm, hbm_kind)
        extras["other_workloads"] = [small_config_decode(l3g, "llama3.2-1b", 16, 128, args.seed, hbm)]
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic",
        "config": {"workload": f"{cfg.name}-shape Q8_0 bs1 greedy decode after {args.prefill}-token prefill",
                   "model": cfg.name, "global_batch": 1, "seq_len": args.prefill,
                   "parallelism": f"tp{world}", "kv_dtype": args.kv,
                   "step_kernels": "persistent" if args.persistent else "per-kernel",
                   **({"persistent_layout": ps_layout} if ps_layout else {}),
                   "l2": "inputs larger than L2: every step streams %.2f GB of weights" % (cfg.weight_bytes() / 1e9),
                   "weights": "seeded N(0,0.02) quantized to Q8_0, norms 1.0; random-init synthetic"},
        "roofline": {"bound": "hbm", "achieved": round(mv["achieved_gbs"], 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(mv["achieved_gbs"] / hbm, 4),
                     "traffic": None if args.persistent else profiled_traffic(
                         "k_matvec_upgate_swiglu_in_step_28672x4096.md" if "timing" in mv
                         else "k_matvec_q8_upgate_28672x4096.md"),
                     "traffic_source": "not captured for the persistent kernel" if args.persistent else
                                       "ncu dram__bytes_read.sum + dram__bytes_write.sum per launch (%s)" % (
                                           "profiles/k_matvec_upgate_swiglu_in_step_28672x4096.md: the "
                                           "in-step kernel, mean of 3 launches" if "timing" in mv else
                                           "profiles/k_matvec_q8_upgate_28672x4096.md"),
                     "kernel": mv["kernel"], "bytes_per_launch": mv["bytes_per_launch"],
                     "ms_per_launch": round(mv["ms_per_launch"], 5), "peak_kind": hbm_kind,
                     **({"timing": mv["timing"]} if "timing" in mv else {}),
                     **({"standalone_events": mv["standalone_events"]} if mv.get("standalone_events") else {})},
        "decode_roofline": {"bytes_per_token": int(step_bytes), "weight_bytes": cfg.weight_bytes(),
                            "kv_bytes_avg": int(kv_bytes), "achieved_gbs": round(decode_gbs, 1),
                            "frac": round(decode_gbs / (hbm * world), 4), "peak_gbs_aggregate": hbm * world},
        "e2e": {"value": round(e2e, 3), "unit": "tok/s", "h2d_bytes_per_step": 16, "d2h_bytes_per_step": 16,
                "api": "l3g_forward_argmax per step (pinned H2D token+pos, graph, D2H result)",
                "tokens_match_device_loop": same},
        "gpu_launches": kernels * args.steps,
        "kernels_per_step": kernels,
        "step_profile_us": prof,
        "step_timeline_us": timeline,
        **({"persistent_phase_us": phases} if phases else {}),
        "clocks": clocks,
        "prefill_s": round(prefill_s, 3),
        "prefill_mode": args.prefill_mode,
        **extras,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    return 0


def matvec_sweep(l3g, shapes, iters, hbm, kind):
    """The Q8_0 matvec microbench over (rows, cols) shapes: each shape's
    weights rotated over copies that together exceed 4 x L2, CUDA events
    over `iters` launches; GB/s of weights + x + out against the HBM peak."""
    import torch
    import synthetic
    l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    rows_out = []
    for rows, cols in shapes:
        alg = rows * cols // 32 * 34 + cols + cols // 32 * 4 + rows * 4
        ncopy = max(1, -(-4 * l2 // alg))
        g = torch.Generator(device="cuda").manual_seed(rows + cols)
        w = synthetic.quantize_q8_0_rows(torch.randn(rows, cols, generator=g, device="cuda") * 0.02, torch)
        host = w.cpu().numpy()
        del w
        mats = [l3g.Matrix(host, rows, cols) for _ in range(ncopy)]
        x = torch.randn(cols, device="cuda")
        d = torch.empty(cols // 32, device="cuda")
        q = torch.empty(cols, dtype=torch.int8, device="cuda")
        l3g.quantize_q8_0_device(x.data_ptr(), cols, d.data_ptr(), q.data_ptr())
        out = torch.empty(rows, device="cuda")
        st = torch.cuda.current_stream().cuda_stream
        for i in range(5):
            mats[i % ncopy].matvec(d.data_ptr(), q.data_ptr(), out.data_ptr(), stream=st)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for i in range(iters):
            mats[i % ncopy].matvec(d.data_ptr(), q.data_ptr(), out.data_ptr(), stream=st)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        gbs = alg / ms / 1e6
        rows_out.append({"shape": [rows, cols], "iters": iters, "copies_rotated": ncopy,
                         "bytes_per_launch": alg, "us_per_launch": round(ms * 1e3, 3),
                         "achieved_gbs": round(gbs, 1), "peak_gbs": hbm, "frac": round(gbs / hbm, 4),
                         "peak_kind": kind})
        for mtx in mats:
            mtx.Close()
        torch.cuda.empty_cache()
    return rows_out


def run_matvec(args):
    """Q8_0 matvec microbench over the 8B shapes: GB/s of weights + x + out."""
    import build
    build.build(quiet=True)
    import l3g
    hbm, kind = peaks()
    shapes = [tuple(int(v) for v in s.split("x")) for s in args.shapes.split(",") if s]
    for r in matvec_sweep(l3g, shapes, args.iters, hbm, kind):
        print(json.dumps({"workload": "q8_0 matvec microbench", **r}), flush=True)
    return 0


def small_config_decode(l3g, name, prefill, steps, seed, hbm):
    """Greedy decode of another workload shape on this GPU (the 1B shape's
    16 prompt tokens + 128 greedy tokens by default): tok/s of the
    device-fed loop (CUDA events) and its decode roofline."""
    import torch
    import synthetic
    cfg = synthetic.CONFIGS[name]
    T = make_host_model(cfg, seed, "cuda")
    torch.cuda.empty_cache()
    m = l3g.LoadModelFromTensors(l3g.hparams_for(cfg), T, l3g.default_options(device=torch.cuda.current_device()))
    del T
    ctx = prefill + steps + 8
    s = m.NewState(ctx)
    ws = m.NewWorkspace(ctx, 40)
    prompt = synthetic.prompt_ids(cfg, prefill, seed=seed)
    m.Prefill(s, prompt[:-1], ws)
    p0 = s.Pos
    warm, _ = m.DecodeGreedy(s, int(prompt[-1]), 4, ws)
    s.Pos = p0
    toks, dev_ms = m.DecodeGreedy(s, int(prompt[-1]), steps, ws)
    value = steps / (dev_ms / 1000.0)
    kv = sum(cfg.kv_bytes(p0 + i + 1, 4) for i in range(steps)) / steps
    step_bytes = cfg.weight_bytes() + kv
    ws.Close()
    s.Close()
    m.Close()
    torch.cuda.empty_cache()
    return {"workload": f"{name}-shape Q8_0 bs1 greedy decode, {prefill} prompt + {steps} greedy tokens",
            "tok_s": round(value, 1), "ms_per_token": round(dev_ms / steps, 4),
            "bytes_per_token": int(step_bytes),
            "decode_roofline_frac": round(step_bytes * value / 1e9 / hbm, 4), "kv_dtype": "f32"}


def run_gemm(args):
    """Batched Q8_0 product (tcgen05 int8) microbench over the 8B shapes and
    token counts: GB/s of weights + activations + out, and int8 TOP/s."""
    import torch
    import build
    build.build(quiet=True)
    import l3g
    import synthetic
    hbm, kind = peaks()
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    shapes = [tuple(int(v) for v in s.split("x")) for s in args.shapes.split(",") if s]
    for rows, cols in shapes:
        g = torch.Generator(device="cuda").manual_seed(rows + cols)
        w = synthetic.quantize_q8_0_rows(torch.randn(rows, cols, generator=g, device="cuda") * 0.02, torch)
        host = w.cpu().numpy()
        del w
        wbytes = rows * cols // 32 * 34
        ncopy = max(1, -(-4 * l2 // wbytes))
        mats = [l3g.GemmMatrix(host, rows, cols, device=0) for _ in range(ncopy)]
        for n in [int(v) for v in args.tokens.split(",") if v]:
            x = torch.randn(n, cols, device="cuda")
            act = torch.empty(l3g.gemm_act_bytes(n, cols), dtype=torch.uint8, device="cuda")
            out = torch.empty(n, rows, device="cuda")
            st = torch.cuda.current_stream().cuda_stream
            l3g.gemm_quantize(x.data_ptr(), n, cols, act.data_ptr(), stream=st)
            for i in range(5):
                mats[i % ncopy].gemm(act.data_ptr(), n, out.data_ptr(), stream=st)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for i in range(args.iters):
                mats[i % ncopy].gemm(act.data_ptr(), n, out.data_ptr(), stream=st)
            e1.record()
            torch.cuda.synchronize()
            err = mats[0].status()
            ms = e0.elapsed_time(e1) / args.iters
            alg = wbytes + n * cols * 34 // 32 + n * rows * 4
            print(json.dumps({"workload": "q8_0 batched product (tcgen05 kind::i8) microbench",
                              "shape": [rows, cols], "tokens": n, "iters": args.iters,
                              "copies_rotated": ncopy, "bytes_per_launch": alg,
                              "us_per_launch": round(ms * 1e3, 3),
                              "achieved_gbs": round(alg / ms / 1e6, 1), "peak_gbs": hbm,
                              "frac": round(alg / ms / 1e6 / hbm, 4), "peak_kind": kind,
                              "int8_tops": round(2.0 * rows * cols * n / ms / 1e9, 2),
                              "device_status": list(err)}), flush=True)
        for mtx in mats:
            mtx.Close()
    return 0


def run_prefill(args):
    """Batched prefill of --prefill tokens against the token-by-token ingest
    (timed on a bounded sample), on one GPU."""
    import torch
    import build
    build.build(quiet=True)
    import l3g
    import synthetic
    cfg = synthetic.CONFIGS[args.config]
    T = make_host_model(cfg, args.seed, "cuda:0")
    torch.cuda.empty_cache()
    kv = l3g.L3G_KV_F16 if args.kv == "f16" else l3g.L3G_KV_F32
    m = l3g.LoadModelFromTensors(l3g.hparams_for(cfg), T, l3g.default_options(1, 0, 0, kv))
    ctx = args.prefill + 1
    s = m.NewState(ctx)
    ws = m.NewWorkspace(ctx, 40)
    prompt = synthetic.prompt_ids(cfg, args.prefill, seed=args.seed)
    m.PrefillBatched(s, prompt[:64], ws)  # first call builds the product's weight copies
    s.Pos = 0
    t0 = time.perf_counter()
    m.PrefillBatched(s, prompt, ws)
    batched_s = time.perf_counter() - t0
    sample = min(256, args.prefill)
    s.Pos = 0
    t0 = time.perf_counter()
    m.Prefill(s, prompt[:sample], ws)
    tbt_s = time.perf_counter() - t0
    ws.Close()
    s.Close()
    m.Close()
    print(json.dumps({"workload": f"{cfg.name}-shape batched prefill", "tokens": args.prefill,
                      "kv_dtype": args.kv, "seconds": round(batched_s, 4),
                      "tok_per_s": round(args.prefill / batched_s, 1),
                      "token_by_token_tok_per_s": round(sample / tbt_s, 1),
                      "token_by_token_sample": f"first {sample} positions"}), flush=True)
    return 0


def run_batched(args):
    """Batched decode: --seqs sessions with seeded context lengths uniform in
    [--ctx-min, --ctx-max], prefilled in batches, then --steps steps of top-k
    40 / temperature 0.8 sampling with a seed per session, tensor parallel
    over the ranks.  value: sampled tokens per second over all sessions,
    each step a host call (tokens in, samples out)."""
    world, rank, local = dist_env()
    import numpy as np
    import torch
    import build
    build.build(quiet=True)
    import l3g
    import synthetic
    D = Dist(world, rank, local)
    torch.cuda.set_device(local)
    hbm, hbm_kind = peaks()
    cfg = synthetic.CONFIGS[args.config]
    T = make_host_model(cfg, args.seed, f"cuda:{local}")
    torch.cuda.empty_cache()
    nid = D.bcast_bytes(l3g.nccl_unique_id() if (world > 1 and rank == 0) else None) if world > 1 else None
    kv = l3g.L3G_KV_F16 if args.kv == "f16" else l3g.L3G_KV_F32
    m = l3g.LoadModelFromTensors(l3g.hparams_for(cfg), T, l3g.default_options(world, rank, local, kv, nid))
    rng = np.random.default_rng(args.seed)
    lens = rng.integers(args.ctx_min, args.ctx_max + 1, args.seqs)
    seeds = rng.integers(1, 2**62, args.seqs).astype(np.uint64)
    ws = m.NewWorkspace(int(lens.max()) + args.warmup + args.steps + 1, 40)
    states = []
    # every session's KV pages come from one shared pool sized for the run
    # (pages of KV_PAGE positions per layer and local kv head)
    heads = cfg.n_layers * (cfg.n_heads_kv // world)
    need = [-(-(int(L) + args.warmup + args.steps + 1) // l3g.KV_PAGE) for L in lens]
    pool = m.NewKvPool(heads * sum(need))
    progress(world, rank, "batched prefill of the sessions")
    t0 = time.perf_counter()
    for i, L in enumerate(lens):
        s = m.NewStateInPool(pool, int(L) + args.warmup + args.steps + 1)
        m.PrefillBatched(s, synthetic.prompt_ids(cfg, int(L), seed=args.seed + 1 + i), ws)
        states.append(s)
    prefill_s = time.perf_counter() - t0
    batch = l3g.Batch(m, args.seqs)
    tokens = rng.integers(0, cfg.vocab, args.seqs)
    for _ in range(max(1, args.warmup)):
        tokens = batch.step(states, tokens, seeds)
    pos0 = np.array([s.Pos for s in states])
    clk = Clocks(physical_index(local))
    clk.wait_first_sample()
    D.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tokens = batch.step(states, tokens, seeds)
    D.barrier()
    clocks = clk.stop()
    wall = D.max(time.perf_counter() - t0)
    # one more step, untimed, inside an NVTX range: the launch list of a
    # single step for `ncu --nvtx --nvtx-include batched_step/`
    torch.cuda.nvtx.range_push("batched_step")
    tokens = batch.step(states, tokens, seeds)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    value = args.seqs * args.steps / wall
    es = 2 if args.kv == "f16" else 4
    kv_step = sum(cfg.kv_bytes(int(p) + i + 1, es) for p in pos0 for i in range(args.steps)) / args.steps
    step_bytes = cfg.weight_bytes() + kv_step
    gbs = step_bytes * args.steps / wall / 1e9
    kv_pool = {"pages": heads * sum(need), "page_bytes": m.KvPageBytes(),
               "pages_held": int(sum(s.Pages for s in states)), "page_positions": l3g.KV_PAGE}
    batch.Close()
    for s in states:
        s.Close()
    pool.Close()
    ws.Close()
    m.Close()
    D.close()
    if rank != 0:
        return 0
    print(json.dumps({"metric": "batched decode tok/s (all sessions)", "value": round(value, 1),
                      "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": round(wall * 1e3 / args.steps, 3), "higher_is_better": True,
                      "dtype": "int8", "data": "synthetic",
                      "config": {"workload": f"{cfg.name}-shape Q8_0 batched decode, {args.seqs} sessions, "
                                             f"contexts uniform in [{args.ctx_min}, {args.ctx_max}], "
                                             "top-k 40, temperature 0.8, a seed per session",
                                 "parallelism": f"tp{world}", "kv_dtype": args.kv},
                      "timing": "host wall clock per step call (tokens in, samples out), max over ranks",
                      "roofline": {"bound": "hbm", "bytes_per_step": int(step_bytes),
                                   "kv_bytes_per_step": int(kv_step), "achieved_gbs": round(gbs, 1),
                                   "peak_gbs_aggregate": hbm * world,
                                   "frac": round(gbs / (hbm * world), 4), "peak_kind": hbm_kind},
                      "kv_pool": kv_pool, "prefill_s": round(prefill_s, 2), "clocks": clocks}),
          flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "matvec":
        return run_matvec(args)
    if args.workload == "gemm":
        return run_gemm(args)
    if args.workload == "prefill":
        return run_prefill(args)
    if args.workload == "batched":
        return run_batched(args)
    return run_l3g(args)


if __name__ == "__main__":
    sys.exit(main())
