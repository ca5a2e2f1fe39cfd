"""ORACLE -- test infrastructure only (tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py).  Never imported by the product.

ctypes binding of oracle/liboracle.so, the C restatement of llama3.go's decode
loop, and of oracle/_ref/libref_simd.so, the reference's own simd.c.  See the
header of l3g_oracle.c for what is pinned to the reference and what is not.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_SIMD = os.path.join(HERE, "_ref", "libref_simd.so")


def build(quiet=True):
    """Compiles liboracle.so and, where the reference tree exists, _ref/."""
    subprocess.run(["make", "-s", "-C", HERE], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)


class Hparams(C.Structure):
    _fields_ = [("vocab_size", C.c_int), ("n_layers", C.c_int), ("n_emb", C.c_int),
                ("n_heads", C.c_int), ("n_heads_kv", C.c_int), ("n_ff", C.c_int),
                ("rope_dim", C.c_int), ("ctx_len", C.c_int), ("rms_eps", C.c_float),
                ("rope_base", C.c_float), ("rope_factor", C.c_float),
                ("rope_low_freq", C.c_float), ("rope_high_freq", C.c_float),
                ("rope_orig_ctx", C.c_int)]


class Layer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "wup", "wgate", "wdown",
                                          "attn_norm", "ffn_norm")]


_lib = None
_P = C.c_void_p
_FP = C.POINTER(C.c_float)


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB):
        build()
    L = C.CDLL(LIB)
    sig = {
        "orc_load_ref_simd": (C.c_int, [C.c_char_p]),
        "orc_have_ref_simd": (C.c_int, []),
        "orc_ref_matvec_q8": (C.c_int, [_P, _FP, _P, _FP, C.c_int, C.c_int, C.c_int]),
        "orc_ref_dot": (C.c_float, [_FP, _FP, C.c_int]),
        "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
        "orc_quantize_q8_0": (None, [_FP, C.c_int, _FP, _P]),
        "orc_dot_q8_0_row": (C.c_float, [_P, _FP, _P, C.c_int]),
        "orc_rmsnorm": (None, [_FP, _FP, _FP, C.c_int, C.c_float]),
        "orc_silu": (C.c_float, [C.c_float]),
        "orc_fast_exp": (C.c_float, [C.c_float]),
        "orc_rope_tables": (None, [C.POINTER(Hparams), C.c_int, _FP, _FP]),
        "orc_model_new": (_P, [C.POINTER(Hparams), _P, _P, _FP, C.POINTER(Layer), C.c_int]),
        "orc_model_free": (None, [_P]),
        "orc_model_threads": (C.c_int, [_P]),
        "orc_state_new": (_P, [_P, C.c_int]),
        "orc_state_free": (None, [_P]),
        "orc_state_pos": (C.c_int, [_P]),
        "orc_state_set_pos": (None, [_P, C.c_int]),
        "orc_state_ctx": (C.c_int, [_P]),
        "orc_state_k": (_FP, [_P]),
        "orc_state_v": (_FP, [_P]),
        "orc_state_hidden": (_FP, [_P]),
        "orc_state_q": (_FP, [_P]),
        "orc_state_attn": (_FP, [_P]),
        "orc_state_ffn_act": (_FP, [_P]),
        "orc_matvec_q8": (None, [_P, _P, _FP, _P, _FP, C.c_int, C.c_int, C.c_int]),
        "orc_forward": (C.c_int, [_P, _P, C.c_int32, _FP, C.c_int, C.c_char_p, C.c_int]),
        "orc_forward_topk": (C.c_int, [_P, _P, C.c_int32, C.c_int, C.POINTER(C.c_int32), _FP,
                                       C.c_int, C.c_char_p, C.c_int]),
        "orc_sample_topk": (C.c_int32, [C.POINTER(C.c_int32), _FP, C.c_int, C.c_float, C.c_double]),
        "orc_sample": (C.c_int32, [_FP, C.c_int, C.c_int, C.c_float, C.c_double]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    if os.path.exists(REF_SIMD):
        L.orc_load_ref_simd(REF_SIMD.encode())
    _lib = L
    return L


def have_ref_simd() -> bool:
    return bool(lib().orc_have_ref_simd())


def fp(a):
    return a.ctypes.data_as(_FP)


# ---- per-op helpers ---------------------------------------------------------
def quantize_q8_0(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    nb = (x.size + 31) // 32
    d = np.empty(nb, np.float32)
    qs = np.empty(nb * 32, np.int8)
    lib().orc_quantize_q8_0(fp(x), x.size, fp(d), qs.ctypes.data)
    return d, qs


def ref_matvec_q8(w: np.ndarray, d: np.ndarray, qs: np.ndarray, rows: int, cols: int,
                  start: int = 0, end: int | None = None) -> np.ndarray:
    """The reference's own matvec_q8_c (simd.c:33-110)."""
    end = rows if end is None else end
    out = np.zeros(rows, np.float32)
    if lib().orc_ref_matvec_q8(w.ctypes.data, fp(d), qs.ctypes.data, fp(out), start, end, cols):
        raise RuntimeError("reference simd.c library not loaded")
    return out


def dot_q8_0_row(row: np.ndarray, d: np.ndarray, qs: np.ndarray) -> float:
    return lib().orc_dot_q8_0_row(row.ctypes.data, fp(d), qs.ctypes.data, d.size)


def rmsnorm(x, w, eps):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib().orc_rmsnorm(fp(out), fp(x), fp(w), x.size, eps)
    return out


def f16_to_f32(bits: int) -> float:
    return lib().orc_f16_to_f32(bits)


def fast_exp(x: float) -> float:
    return lib().orc_fast_exp(x)


def silu(x: float) -> float:
    return lib().orc_silu(x)


def hparams_for(cfg) -> Hparams:
    hp = Hparams()
    hp.vocab_size, hp.n_layers, hp.n_emb = cfg.vocab, cfg.n_layers, cfg.n_emb
    hp.n_heads, hp.n_heads_kv, hp.n_ff = cfg.n_heads, cfg.n_heads_kv, cfg.n_ff
    hp.rope_dim, hp.ctx_len = cfg.head_dim, cfg.ctx_len
    hp.rms_eps, hp.rope_base = cfg.rms_eps, cfg.rope_base
    if cfg.rope_scaling is not None:
        hp.rope_factor, hp.rope_low_freq, hp.rope_high_freq, hp.rope_orig_ctx = cfg.rope_scaling
    return hp


class OracleModel:
    """Model + State of the restatement over in-memory tensors (name ->
    (dims, type, bytes)) as produced by synthetic.make_model."""

    def __init__(self, cfg, tensors: dict, threads: int = 0, rope_scaling: bool = True):
        self.cfg = cfg
        self.hp = hparams_for(cfg)
        if not rope_scaling:
            self.hp.rope_factor = 0.0
        self._keep = tensors

        def ptr(name):
            return tensors[name][2].ctypes.data

        layers = (Layer * cfg.n_layers)()
        for i in range(cfg.n_layers):
            p = f"blk.{i}."
            L = layers[i]
            L.wq, L.wk, L.wv = ptr(p + "attn_q.weight"), ptr(p + "attn_k.weight"), ptr(p + "attn_v.weight")
            L.wo = ptr(p + "attn_output.weight")
            L.wup, L.wgate, L.wdown = ptr(p + "ffn_up.weight"), ptr(p + "ffn_gate.weight"), ptr(p + "ffn_down.weight")
            L.attn_norm, L.ffn_norm = ptr(p + "attn_norm.weight"), ptr(p + "ffn_norm.weight")
        out = ptr("output.weight") if "output.weight" in tensors else None
        norm = tensors["output_norm.weight"][2].view(np.float32)
        self._norm = norm
        threads = threads or os.cpu_count() or 1
        self._h = lib().orc_model_new(C.byref(self.hp), ptr("token_embd.weight"), out, fp(norm),
                                      layers, threads)
        self.threads = lib().orc_model_threads(self._h)
        self.state = None

    def new_state(self, ctx: int):
        if self.state:
            lib().orc_state_free(self.state)
        self.state = lib().orc_state_new(self._h, ctx)
        self.ctx = lib().orc_state_ctx(self.state)
        return self.state

    @property
    def pos(self):
        return lib().orc_state_pos(self.state)

    @pos.setter
    def pos(self, p):
        lib().orc_state_set_pos(self.state, p)

    def forward(self, token: int, logits: bool = True, use_ref: bool = True):
        """ForwardIntoWorkspace (cgo build when use_ref)."""
        out = np.empty(self.cfg.vocab, np.float32) if logits else None
        err = C.create_string_buffer(256)
        rc = lib().orc_forward(self._h, self.state, int(token), fp(out) if logits else None,
                               1 if use_ref else 0, err, 256)
        if rc:
            raise RuntimeError(err.value.decode())
        return out

    def forward_topk(self, token: int, k: int = 40, use_ref: bool = True):
        """ForwardTopKIntoWorkspace: (ids, logits) unsorted, reference order."""
        ids = np.empty(k, np.int32)
        lg = np.empty(k, np.float32)
        err = C.create_string_buffer(256)
        n = lib().orc_forward_topk(self._h, self.state, int(token), k,
                                   ids.ctypes.data_as(C.POINTER(C.c_int32)), fp(lg),
                                   1 if use_ref else 0, err, 256)
        if n < 0:
            raise RuntimeError(err.value.decode())
        return ids[:n], lg[:n]

    def kv(self, layer: int, pos0: int, npos: int):
        """K, V of one layer for [pos0, pos0+npos): [npos][kv heads][hd]."""
        cfg = self.cfg
        hd, nkv = cfg.head_dim, cfg.n_heads_kv
        n = cfg.n_layers * self.ctx * nkv * hd
        K = np.ctypeslib.as_array(lib().orc_state_k(self.state), shape=(n,))
        V = np.ctypeslib.as_array(lib().orc_state_v(self.state), shape=(n,))
        K = K.reshape(cfg.n_layers, self.ctx, nkv, hd)
        V = V.reshape(cfg.n_layers, self.ctx, nkv, hd)
        return K[layer, pos0:pos0 + npos].copy(), V[layer, pos0:pos0 + npos].copy()

    def kv_arrays(self):
        cfg = self.cfg
        n = cfg.n_layers * self.ctx * cfg.n_heads_kv * cfg.head_dim
        K = np.ctypeslib.as_array(lib().orc_state_k(self.state), shape=(n,))
        V = np.ctypeslib.as_array(lib().orc_state_v(self.state), shape=(n,))
        return K, V

    def buffer(self, which: str) -> np.ndarray:
        cfg = self.cfg
        fn, n = {"hidden": (lib().orc_state_hidden, cfg.n_emb), "q": (lib().orc_state_q, cfg.n_emb),
                 "attn": (lib().orc_state_attn, cfg.n_emb),
                 "ffn_act": (lib().orc_state_ffn_act, cfg.n_ff)}[which]
        return np.ctypeslib.as_array(fn(self.state), shape=(n,)).copy()

    def matvec(self, w, d, qs, rows, cols, use_ref=True):
        out = np.empty(rows, np.float32)
        lib().orc_matvec_q8(self._h, w.ctypes.data, fp(d), qs.ctypes.data, fp(out), rows, cols,
                            1 if use_ref else 0)
        return out

    def close(self):
        if self.state:
            lib().orc_state_free(self.state)
            self.state = None
        if self._h:
            lib().orc_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def sample_topk(ids, logits, temperature, r01) -> int:
    ids = np.ascontiguousarray(ids, np.int32)
    lg = np.ascontiguousarray(logits, np.float32)
    return lib().orc_sample_topk(ids.ctypes.data_as(C.POINTER(C.c_int32)), fp(lg), ids.size,
                                 temperature, r01)
