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
                                       "max_stages", "max_splits", "launch_grid")] + [
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
        self.kv = Dev(cfg.n_layers * self.hkv * ctx * 2 * hd * self.es)
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
        ours = np.zeros((cfg.n_layers, self.hkv, self.ctx, 2, hd), np.float32)
        ours[:, :, :npos, 0] = K[:, :npos].transpose(0, 2, 1, 3)
        ours[:, :, :npos, 1] = V[:, :npos].transpose(0, 2, 1, 3)
        self.kv.write(ours.astype(np.float16) if self.kv_f16 else ours)

    def read_kv(self):
        """[layer][local kv head][ctx][2][hd] as f32."""
        cfg = self.cfg
        a = self.kv.read(np.float16 if self.kv_f16 else np.float32).astype(np.float32)
        return a.reshape(cfg.n_layers, self.hkv, self.ctx, 2, cfg.head_dim)

    def record(self, token, pos, step_count=1, **kw):
        cfg = self.cfg
        self.xa.write(embed_row(cfg, self.T, int(token)))
        return EmuLayers(grid=self.grid, n_layers=cfg.n_layers, n_emb=cfg.n_emb, n_ff=self.ff,
                         hq=self.hq, hkv=self.hkv, hd=cfg.head_dim, rope_half=cfg.head_dim // 2,
                         ctx=self.ctx, kv_f16=1 if self.kv_f16 else 0, eps=cfg.rms_eps, w=self.W,
                         norm=self.N, xa=self.xa.ptr, xb=self.xb.ptr, y=self.y.ptr,
                         attn=self.attn.ptr, act=self.act.ptr, kv=self.kv.ptr,
                         rope_cos=self.cos.ptr, rope_sin=self.sin.ptr, token=int(token),
                         pos=int(pos), step_count=step_count, **kw)

    def hidden(self):
        # the residual add of the last down output is done by the logits kernel
        return (self.xa.read(np.float32) + self.y.read(np.float32)).astype(np.float32)

    def step(self, token, pos, **kw):
        """One token's layers; returns (hidden state after the last layer,
        the EmuLayers record).  kw: fuse_quant, nsub, max_stages, max_splits,
        launch_grid, wait_ns."""
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
