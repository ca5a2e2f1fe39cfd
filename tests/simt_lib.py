"""ctypes front end of the SIMT emulator build of the device kernels
(tests/simt/emu_l3g.cpp): builds it with g++ on first use and wraps its C
entry points.  Test infrastructure only (CPU tests)."""
import ctypes as C
import os
import subprocess
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(ROOT, "llama3.go_b200", "csrc")
SIMT = os.path.join(HERE, "simt")
_lib = None
_P = C.c_void_p


def _sources():
    files = [os.path.join(SIMT, f) for f in os.listdir(SIMT)]
    files += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return files


def build():
    """libemu.so in a per-user temp directory, rebuilt when a source changed."""
    out_dir = os.path.join(tempfile.gettempdir(), f"l3g_simt_{os.getuid()}")
    os.makedirs(out_dir, exist_ok=True)
    out = os.path.join(out_dir, "libemu.so")
    if os.path.exists(out) and all(os.path.getmtime(f) <= os.path.getmtime(out) for f in _sources()):
        return out
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    tmp = out + f".{os.getpid()}.tmp"
    subprocess.run(["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fPIC", "-shared",
                    "-I", cuda_inc, "-I", CSRC, "-I", SIMT,
                    os.path.join(SIMT, "emu_l3g.cpp"), "-o", tmp], check=True)
    os.replace(tmp, out)
    return out


class EmuLayers(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("grid", "n_layers", "n_emb", "n_ff", "hq", "hkv", "hd",
                                       "rope_half", "ctx", "kv_f16", "fuse_quant", "nsub",
                                       "max_stages", "max_splits", "launch_grid",
                                       "fuse_merge")] + [
        ("wait_ns", C.c_ulonglong), ("eps", C.c_float), ("w", C.POINTER(_P)), ("norm", C.POINTER(_P)),
        ("xa", _P), ("xb", _P), ("y", _P), ("attn", _P), ("act", _P), ("kv", _P),
        ("rope_cos", _P), ("rope_sin", _P), ("token", C.c_int), ("pos", C.c_int),
        ("step_count", C.c_int), ("err", C.c_int), ("where", C.c_int), ("splits", C.c_int), ("stages", C.c_int)]


def lib():
    global _lib
    if _lib is None:
        L = C.CDLL(build())
        L.emu_error.restype = C.c_char_p
        L.emu_malloc.restype = _P
        L.emu_malloc.argtypes = [C.c_ulonglong]
        L.emu_free.argtypes = [_P]
        L.emu_schedule.argtypes = [C.c_int, C.c_ulonglong, C.c_int]
        L.emu_tile_geometry.argtypes = [C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int)]
        L.emu_repack.argtypes = [C.POINTER(_P), C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_int,
                                 C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _P]
        L.emu_attf.argtypes = [_P, _P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _P,
                               _P, _P, _P, _P, _P, _P, _P]
        L.emu_layers.argtypes = [C.POINTER(EmuLayers)]
        L.emu_layers_tp.argtypes = [C.POINTER(EmuLayers), C.c_int]
        L.emu_gemm_quantize.argtypes = [_P, C.c_int, C.c_int, _P]
        L.emu_gemm_from_tiles.argtypes = [_P, C.c_int, C.c_int, C.c_int, _P]
        L.emu_prefill.argtypes = [C.c_void_p]
        L.emu_batch_step.argtypes = [C.c_void_p]
        L.emu_attention.argtypes = [_P, _P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _P, _P,
                                    _P, _P, C.c_int, C.c_int, C.POINTER(C.c_int)]
        L.emu_matvec.argtypes = [_P, C.c_int, C.c_int, C.c_int, _P, _P, _P, C.c_int, C.c_int,
                                 C.c_int]
        L.emu_matvec_epi.argtypes = [_P, C.c_int, C.c_int, C.c_int, _P, _P, _P, C.c_int, _P, _P,
                                     _P, _P, C.c_int]
        L.emu_bitonic.argtypes = [_P, C.c_int, C.c_int]
        L.emu_gemm.argtypes = [_P, C.c_int, C.c_int, _P, C.c_int, _P, C.c_int, _P, C.c_int,
                               C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int)]
        _lib = L
    return _lib


def check(rc):
    if rc != 0:
        raise RuntimeError(lib().emu_error().decode())


class Dev:
    """A device buffer of the emulator (guard page after its end)."""

    def __init__(self, nbytes_or_array):
        if isinstance(nbytes_or_array, np.ndarray):
            arr = np.ascontiguousarray(nbytes_or_array)
            self.nbytes = arr.nbytes
            self.ptr = lib().emu_malloc(max(1, self.nbytes))
            C.memmove(self.ptr, arr.ctypes.data, self.nbytes)
        else:
            self.nbytes = int(nbytes_or_array)
            self.ptr = lib().emu_malloc(max(1, self.nbytes))
        if not self.ptr:
            raise RuntimeError(lib().emu_error().decode())

    def read(self, dtype, count=None):
        dt = np.dtype(dtype)
        n = self.nbytes // dt.itemsize if count is None else count
        out = np.empty(n, dt)
        C.memmove(out.ctypes.data, self.ptr, n * dt.itemsize)
        return out

    def write(self, arr):
        arr = np.ascontiguousarray(arr)
        assert arr.nbytes <= self.nbytes
        C.memmove(self.ptr, arr.ctypes.data, arr.nbytes)

    def free(self):
        if self.ptr:
            lib().emu_free(self.ptr)
            self.ptr = None


def tile_geometry(rows, cols, rpw=4):
    out = (C.c_int * 5)()
    lib().emu_tile_geometry(rows, cols, rpw, out)
    return dict(zip(("wr", "ck", "nslices", "tile_bytes", "n_groups"), list(out)))


def repack(segments, cols_total, rows, blk0=0, cols=None, interleave2=False, rpw=4):
    """Tiles rows of GGUF Q8_0 matrices (segments: [(Dev of raw rows,
    first row, row count)]) with k_repack; returns the tiled Dev."""
    cols = cols_total if cols is None else cols
    g = tile_geometry(rows, cols, rpw)
    out = Dev(g["n_groups"] * g["nslices"] * g["tile_bytes"])
    src = (_P * 3)(*[s[0].ptr for s in segments] + [None] * (3 - len(segments)))
    r0 = (C.c_int * 3)(*[s[1] for s in segments] + [0] * (3 - len(segments)))
    nr = (C.c_int * 3)(*[s[2] for s in segments] + [0] * (3 - len(segments)))
    check(lib().emu_repack(src, r0, nr, len(segments), 1 if interleave2 else 0, cols_total // 32,
                           blk0, rows, cols, rpw, out.ptr))
    return out


KV_PAGE = 256  # positions per page of the library's KV cache (L3G_KV_PAGE)


def kv_len(ctx):
    """Positions per (layer, kv head) of a contiguous cache the kernels can
    reach through an identity page table: ctx rounded up to KV_PAGE."""
    return -(-ctx // KV_PAGE) * KV_PAGE


def rope_tables(cfg, ctx):
    """cos / sin [ctx][head_dim / 2] as the library builds them: inverse
    frequencies 1 / base^(2i / rope_dim) in f64 (rope.go:20-25), divided by
    the llama3 factors when the model has them, angles and cos / sin in f64,
    stored f32."""
    import synthetic
    half = cfg.head_dim // 2
    inv = np.array([1.0 / np.power(np.float64(cfg.rope_base), (2 * i) / cfg.head_dim)
                    for i in range(half)])
    if cfg.rope_scaling is not None:
        inv = inv / synthetic.llama3_freq_factors(cfg).astype(np.float64)
    ang = np.arange(ctx, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def embed_row(cfg, T, token):
    """k_embed: x[i] = f16(d) * q[i] of row `token` of token_embd."""
    raw = T["token_embd.weight"][2].reshape(cfg.vocab, cfg.n_emb // 32, 34)[token]
    d = raw[:, :2].copy().view(np.float16).astype(np.float32)[:, 0]
    q = raw[:, 2:].view(np.int8).astype(np.float32)
    return (d[:, None] * q).reshape(-1).astype(np.float32)


class PersistentModel:
    """A synthetic model's layers laid out as the library does for the
    persistent kernel (four rows per warp; QKV rows concatenated, up / gate
    interleaved), a KV cache [layer][kv head][ctx][K | V][hd] and the step's
    buffers, all in emulator device memory.  With world > 1 it holds rank
    `rank`'s shard as the library's shard plan (l3g_shard_plan) cuts it:
    heads of Q/K/V, head columns of Wo, rows of up/gate, columns of down.
    step() runs one token's layers through k_layers; step_tp() runs every
    rank's together."""

    def __init__(self, cfg, T, ctx, grid, kv_f16=False, world=1, rank=0):
        import synthetic
        self.cfg, self.T, self.ctx, self.grid, self.kv_f16 = cfg, T, ctx, grid, kv_f16
        self.world, self.rank = world, rank
        e, f, hd = cfg.n_emb, cfg.n_ff, cfg.head_dim
        if world > 1:
            import l3g
            sh = l3g.shard_plan(l3g.hparams_for(cfg), world, rank)
            q0, nq, k0, nk = sh.q_row0, sh.q_rows, sh.kv_row0, sh.kv_rows
            o0, no, f0, nf, d0, nd = sh.o_col0, sh.o_cols, sh.ff_row0, sh.ff_rows, sh.down_col0, sh.down_cols
        else:
            q0, nq, k0, nk = 0, e, 0, cfg.n_heads_kv * hd
            o0, no, f0, nf, d0, nd = 0, e, 0, f, 0, f
        self.hq, self.hkv, self.ff = nq // hd, nk // hd, nf
        self.kv_head0 = k0 // hd
        self._keep = []
        raw = {k: Dev(v[2]) for k, v in T.items() if v[1] == synthetic.GGML_Q8_0}
        self._keep += raw.values()
        w, norms = [], []
        for l in range(cfg.n_layers):
            p = f"blk.{l}."
            mats = [
                repack([(raw[p + "attn_q.weight"], q0, nq), (raw[p + "attn_k.weight"], k0, nk),
                        (raw[p + "attn_v.weight"], k0, nk)], e, nq + 2 * nk),
                repack([(raw[p + "attn_output.weight"], 0, e)], e, e, blk0=o0 // 32, cols=no),
                repack([(raw[p + "ffn_up.weight"], f0, nf), (raw[p + "ffn_gate.weight"], f0, nf)], e,
                       2 * nf, interleave2=True),
                repack([(raw[p + "ffn_down.weight"], 0, e)], f, e, blk0=d0 // 32, cols=nd),
            ]
            nv = [Dev(T[p + "attn_norm.weight"][2]), Dev(T[p + "ffn_norm.weight"][2])]
            w += [m.ptr for m in mats]
            norms += [n.ptr for n in nv]
            self._keep += mats + nv
        self.W = (_P * len(w))(*w)
        self.N = (_P * len(norms))(*norms)
        cos, sin = rope_tables(cfg, ctx)
        self.cos, self.sin = Dev(cos), Dev(sin)
        self.es = 2 if kv_f16 else 4
        self.kctx = kv_len(ctx)
        self.kv = Dev(cfg.n_layers * self.hkv * self.kctx * 2 * hd * self.es)
        self.xa, self.xb, self.y = Dev(e * 4), Dev(e * 4), Dev(e * 4)
        self.attn, self.act = Dev(self.hq * hd * 4), Dev(nf * 4)
        self._keep += [self.cos, self.sin, self.kv, self.xa, self.xb, self.y, self.attn, self.act]

    def load_kv(self, K, V, npos):
        """Positions [0, npos) of this rank's kv heads from the oracle's K, V
        ([layer][pos][kv head][hd], ctx positions)."""
        cfg = self.cfg
        hkv, hd, h0 = cfg.n_heads_kv, cfg.head_dim, self.kv_head0
        K = K.reshape(cfg.n_layers, self.ctx, hkv, hd)[:, :, h0:h0 + self.hkv]
        V = V.reshape(cfg.n_layers, self.ctx, hkv, hd)[:, :, h0:h0 + self.hkv]
        ours = np.zeros((cfg.n_layers, self.hkv, self.kctx, 2, hd), np.float32)
        ours[:, :, :npos, 0] = K[:, :npos].transpose(0, 2, 1, 3)
        ours[:, :, :npos, 1] = V[:, :npos].transpose(0, 2, 1, 3)
        self.kv.write(ours.astype(np.float16) if self.kv_f16 else ours)

    def read_kv(self):
        """[layer][local kv head][ctx][2][hd] as f32."""
        cfg = self.cfg
        a = self.kv.read(np.float16 if self.kv_f16 else np.float32).astype(np.float32)
        return a.reshape(cfg.n_layers, self.hkv, self.kctx, 2, cfg.head_dim)[:, :, :self.ctx]

    def record(self, token, pos, step_count=1, **kw):
        cfg = self.cfg
        self.xa.write(embed_row(cfg, self.T, int(token)))
        return EmuLayers(grid=self.grid, n_layers=cfg.n_layers, n_emb=cfg.n_emb, n_ff=self.ff,
                         hq=self.hq, hkv=self.hkv, hd=cfg.head_dim, rope_half=cfg.head_dim // 2,
                         ctx=self.kctx, kv_f16=1 if self.kv_f16 else 0, eps=cfg.rms_eps, w=self.W,
                         norm=self.N, xa=self.xa.ptr, xb=self.xb.ptr, y=self.y.ptr,
                         attn=self.attn.ptr, act=self.act.ptr, kv=self.kv.ptr,
                         rope_cos=self.cos.ptr, rope_sin=self.sin.ptr, token=int(token),
                         pos=int(pos), step_count=step_count, **kw)

    def hidden(self):
        # the residual add of the last down output is done by the logits kernel
        return (self.xa.read(np.float32) + self.y.read(np.float32)).astype(np.float32)

    def step(self, token, pos, **kw):
        """One token's layers; returns (hidden state after the last layer,
        the EmuLayers record).  kw: fuse_quant, fuse_merge, nsub, max_stages,
        max_splits, launch_grid, wait_ns."""
        a = self.record(token, pos, **kw)
        check(lib().emu_layers(C.byref(a)))
        return self.hidden(), a

    def close(self):
        for d in self._keep:
            d.free()
        self._keep = []


def step_tp(models, token, pos, step_count, **kw):
    """One token through every rank's shard at once (emulated GPUs pushing
    their Wo / down rows to each other); returns (hidden per rank, records)."""
    recs = (EmuLayers * len(models))(*[m.record(token, pos, step_count, **kw) for m in models])
    check(lib().emu_layers_tp(recs, len(models)))
    return [m.hidden() for m in models], list(recs)


class EmuPrefillLayer(C.Structure):
    _fields_ = [("g", _P * 4), ("attn_norm", _P), ("ffn_norm", _P)]


class EmuPrefill(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layers", "n_emb", "n_ff", "hq", "hkv", "hd", "rope_half",
                                       "ctx", "kv_f16", "vocab")] + [
        ("eps", C.c_float), ("layers", C.POINTER(EmuPrefillLayer)), ("emb", _P), ("kv", _P),
        ("rope_cos", _P), ("rope_sin", _P), ("ids", _P), ("P", C.c_int), ("pos0", C.c_int),
        ("nsm", C.c_int), ("err", C.c_int), ("where", C.c_int)]


def _gemm_chunks_bytes(rows, cols):
    return ((rows + 127) // 128) * ((cols + 127) // 128) * 17408


class PrefillModel:
    """A synthetic model laid out for batched prefill as the library builds it:
    decode tiles (k_repack, `rpw` rows per warp) turned into the batched
    product's weight chunks by k_gemm_from_tiles; a KV cache
    [layer][kv head][ctx][K | V][hd]; prefill() runs one pass."""

    def __init__(self, cfg, T, ctx, rpw=4, kv_f16=False):
        import synthetic
        self.cfg, self.ctx, self.kv_f16 = cfg, ctx, kv_f16
        e, f, hd, hkv = cfg.n_emb, cfg.n_ff, cfg.head_dim, cfg.n_heads_kv
        self._keep = []
        raw = {k: Dev(v[2]) for k, v in T.items() if v[1] == synthetic.GGML_Q8_0}
        self._keep += raw.values()
        layers = []
        for l in range(cfg.n_layers):
            p = f"blk.{l}."
            specs = [
                ([(raw[p + "attn_q.weight"], 0, e), (raw[p + "attn_k.weight"], 0, hkv * hd),
                  (raw[p + "attn_v.weight"], 0, hkv * hd)], e, e + 2 * hkv * hd, False),
                ([(raw[p + "attn_output.weight"], 0, e)], e, e, False),
                ([(raw[p + "ffn_up.weight"], 0, f), (raw[p + "ffn_gate.weight"], 0, f)], e, 2 * f, True),
                ([(raw[p + "ffn_down.weight"], 0, e)], f, e, False),
            ]
            chunks = []
            for segs, cols, rows, il in specs:
                tiles = repack(segs, cols, rows, interleave2=il, rpw=rpw)
                g = Dev(_gemm_chunks_bytes(rows, cols))
                check(lib().emu_gemm_from_tiles(tiles.ptr, rows, cols, rpw, g.ptr))
                tiles.free()
                chunks.append(g)
            nv = [Dev(T[p + "attn_norm.weight"][2]), Dev(T[p + "ffn_norm.weight"][2])]
            self._keep += chunks + nv
            L = EmuPrefillLayer()
            for i, g in enumerate(chunks):
                L.g[i] = g.ptr
            L.attn_norm, L.ffn_norm = nv[0].ptr, nv[1].ptr
            layers.append(L)
        self.layers = (EmuPrefillLayer * len(layers))(*layers)
        self.emb = Dev(T["token_embd.weight"][2])
        cos, sin = rope_tables(cfg, ctx)
        self.cos, self.sin = Dev(cos), Dev(sin)
        self.kctx = kv_len(ctx)
        self.kv = Dev(cfg.n_layers * hkv * self.kctx * 2 * hd * (2 if kv_f16 else 4))
        self._keep += [self.emb, self.cos, self.sin, self.kv]

    def prefill(self, ids, pos0, nsm=148):
        cfg = self.cfg
        d_ids = Dev(np.ascontiguousarray(ids, dtype=np.int32))
        a = EmuPrefill(n_layers=cfg.n_layers, n_emb=cfg.n_emb, n_ff=cfg.n_ff, hq=cfg.n_heads,
                       hkv=cfg.n_heads_kv, hd=cfg.head_dim, rope_half=cfg.head_dim // 2,
                       ctx=self.kctx, kv_f16=1 if self.kv_f16 else 0, vocab=cfg.vocab,
                       eps=cfg.rms_eps, layers=self.layers, emb=self.emb.ptr, kv=self.kv.ptr,
                       rope_cos=self.cos.ptr, rope_sin=self.sin.ptr, ids=d_ids.ptr, P=len(ids),
                       pos0=pos0, nsm=nsm)
        try:
            check(lib().emu_prefill(C.byref(a)))
        finally:
            d_ids.free()
        return a

    def read_kv(self):
        cfg = self.cfg
        a = self.kv.read(np.float16 if self.kv_f16 else np.float32).astype(np.float32)
        return a.reshape(cfg.n_layers, cfg.n_heads_kv, self.kctx, 2, cfg.head_dim)[:, :, :self.ctx]

    def close(self):
        for d in self._keep:
            d.free()
        self._keep = []


class SeqInfo(C.Structure):
    _fields_ = [("kv_pool", _P), ("kv_pages", _P), ("rope_cos", _P), ("rope_sin", _P),
                ("kv_pps", C.c_int), ("ctx", C.c_int), ("pos", C.c_int), ("token", C.c_int),
                ("seed", C.c_uint64), ("temperature", C.c_float), ("pad", C.c_int)]


class Result(C.Structure):
    _fields_ = [("token", C.c_int32), ("logit", C.c_float), ("err", C.c_int32), ("where", C.c_int32)]


class EmuBatch(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layers", "n_emb", "n_ff", "hq", "hkv", "hd", "rope_half",
                                       "kv_f16", "vocab")] + [
        ("eps", C.c_float), ("layers", C.POINTER(EmuPrefillLayer)), ("glogits", _P),
        ("out_norm", _P), ("emb", _P), ("seqs", _P), ("n", C.c_int), ("max_splits", C.c_int),
        ("top_k", C.c_int), ("nsm", C.c_int), ("logits", _P), ("out", _P), ("err", C.c_int),
        ("where", C.c_int)]


class BatchModel(PrefillModel):
    """PrefillModel plus the logits matrix as weight chunks (output.weight, or
    the tied token_embd) and the final norm; step() runs one batched decode
    step over sessions given as (KV cache Dev, position, token, seed)."""

    def __init__(self, cfg, T, ctx, rpw=4, kv_f16=False):
        super().__init__(cfg, T, ctx, rpw=rpw, kv_f16=kv_f16)
        name = "token_embd.weight" if cfg.tied else "output.weight"
        raw = Dev(T[name][2])
        tiles = repack([(raw, 0, cfg.vocab)], cfg.n_emb, cfg.vocab, rpw=rpw)
        self.glogits = Dev(_gemm_chunks_bytes(cfg.vocab, cfg.n_emb))
        check(lib().emu_gemm_from_tiles(tiles.ptr, cfg.vocab, cfg.n_emb, rpw, self.glogits.ptr))
        tiles.free()
        raw.free()
        self.out_norm = Dev(T["output_norm.weight"][2])
        # every session's cache is contiguous: one identity page table serves all
        self.pages = Dev(np.arange(cfg.n_layers * cfg.n_heads_kv * (self.kctx // KV_PAGE),
                                   dtype=np.int32))
        self._keep += [self.glogits, self.out_norm, self.pages]

    def new_cache(self):
        cfg = self.cfg
        d = Dev(cfg.n_layers * cfg.n_heads_kv * self.kctx * 2 * cfg.head_dim * (2 if self.kv_f16 else 4))
        self._keep.append(d)
        return d

    def step(self, caches, positions, tokens, seeds, top_k=40, temperature=0.8, nsm=148):
        cfg = self.cfg
        n = len(caches)
        seqs = (SeqInfo * n)(*[SeqInfo(kv_pool=c.ptr, kv_pages=self.pages.ptr,
                                       kv_pps=self.kctx // KV_PAGE, rope_cos=self.cos.ptr,
                                       rope_sin=self.sin.ptr, ctx=self.ctx, pos=int(p),
                                       token=int(t), seed=int(s), temperature=temperature)
                               for c, p, t, s in zip(caches, positions, tokens, seeds)])
        d_seqs = Dev(np.frombuffer(bytes(seqs), np.uint8))
        logits = Dev(n * cfg.vocab * 4)
        out = Dev(n * C.sizeof(Result))
        a = EmuBatch(n_layers=cfg.n_layers, n_emb=cfg.n_emb, n_ff=cfg.n_ff, hq=cfg.n_heads,
                     hkv=cfg.n_heads_kv, hd=cfg.head_dim, rope_half=cfg.head_dim // 2,
                     kv_f16=1 if self.kv_f16 else 0, vocab=cfg.vocab, eps=cfg.rms_eps,
                     layers=self.layers, glogits=self.glogits.ptr, out_norm=self.out_norm.ptr,
                     emb=self.emb.ptr, seqs=d_seqs.ptr, n=n, max_splits=(self.ctx + 255) // 256,
                     top_k=top_k, nsm=nsm, logits=logits.ptr, out=out.ptr)
        try:
            check(lib().emu_batch_step(C.byref(a)))
            lg = logits.read(np.float32).reshape(n, cfg.vocab)
            res = (Result * n).from_buffer_copy(out.read(np.uint8).tobytes())
            return lg, [r.token for r in res], a
        finally:
            for d in (d_seqs, logits, out):
                d.free()


def load_session_kv(dev, cfg, ctx, K, V, npos, f16=False):
    """Positions [0, npos) of a session's cache from the oracle's K, V."""
    hkv, hd = cfg.n_heads_kv, cfg.head_dim
    K = K.reshape(cfg.n_layers, ctx, hkv, hd)
    V = V.reshape(cfg.n_layers, ctx, hkv, hd)
    ours = np.zeros((cfg.n_layers, hkv, kv_len(ctx), 2, hd), np.float32)
    ours[:, :, :npos, 0] = K[:, :npos].transpose(0, 2, 1, 3)
    ours[:, :, :npos, 1] = V[:, :npos].transpose(0, 2, 1, 3)
    dev.write(ours.astype(np.float16) if f16 else ours)
