"""Python host side of libl3g: a ctypes binding with the same shape as the
reference's Go API (internal/llama), so code and tests read like the
reference's own:

    m  = LoadModel(path)                        # model.go:55
    s  = m.NewState(ctx)                        # state.go:51
    ws = m.NewWorkspace(ctx, topK)              # workspace.go:35
    m.ForwardIntoWorkspace(s, tok, logits, ws)  # infer.go:21
    items = m.ForwardTopKIntoWorkspace(s, tok, topK, ws)   # infer.go:269
    smp = NewSampler(temp, topK, seed); smp.SampleTopK(items)  # sampling.go

Every call runs on the GPU through libl3g.so; there is no CPU fallback.  A
missing library or a failing call raises L3GError.
"""
from __future__ import annotations

import ctypes as C
import math
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libl3g.so")

L3G_OK, L3G_E_INVALID, L3G_E_CUDA, L3G_E_NCCL, L3G_E_CTX, L3G_E_TOKEN, \
    L3G_E_FORMAT, L3G_E_DEVICE = 0, -1, -2, -3, -4, -5, -6, -7
L3G_KV_F32, L3G_KV_F16 = 0, 1
BUF_HIDDEN, BUF_Q, BUF_ATTN, BUF_FFN_ACT, BUF_LOGITS = range(5)
ARGMAX_STATIC_MAX_CTAS = 1024  # L3G_ARGMAX_STATIC_MAX_CTAS


class L3GError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


class HyperParams(C.Structure):
    """HyperParams, model.go:10-21."""
    _fields_ = [("VocabSize", C.c_int32), ("NLayers", C.c_int32), ("NEmb", C.c_int32),
                ("NHeads", C.c_int32), ("NHeadsKV", C.c_int32), ("NFF", C.c_int32),
                ("RopeDim", C.c_int32), ("CtxLen", C.c_int32), ("RmsEps", C.c_float),
                ("RopeBase", C.c_float)]


class _Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("type", C.c_uint32), ("n_dims", C.c_uint32),
                ("dims", C.c_uint64 * 4), ("data", C.c_void_p), ("nbytes", C.c_uint64)]


class Options(C.Structure):
    _fields_ = [("world_size", C.c_int32), ("rank", C.c_int32), ("device", C.c_int32),
                ("kv_dtype", C.c_int32), ("nccl_id", C.c_uint8 * 128)]


class Shard(C.Structure):
    """l3g_shard: one tensor-parallel rank's row / column ranges."""
    _fields_ = [(n, C.c_int32) for n in (
        "q_row0", "q_rows", "kv_row0", "kv_rows", "o_col0", "o_cols", "ff_row0", "ff_rows",
        "down_col0", "down_cols", "vocab_row0", "vocab_rows", "vocab_stride")]


class TopKItem(C.Structure):
    """TopKItem, topk.go:5-8."""
    _fields_ = [("ID", C.c_int32), ("Logit", C.c_float)]

    def __repr__(self):
        return f"TopKItem(ID={self.ID}, Logit={self.Logit:.6g})"


_lib = None
_P = C.c_void_p


def lib():
    """Loads libl3g.so (built in-tree by build.py).  Raises when it is absent:
    the product path has no fallback."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise L3GError(L3G_E_INVALID, f"{LIB_PATH} is missing: run python llama3.go_b200/build.py")
    L = C.CDLL(LIB_PATH)
    sig = {
        "l3g_last_error": (C.c_char_p, []),
        "l3g_version": (C.c_int, []),
        "l3g_device_count": (C.c_int, [C.POINTER(C.c_int32)]),
        "l3g_nccl_unique_id": (C.c_int, [C.POINTER(C.c_uint8)]),
        "l3g_options_default": (None, [C.POINTER(Options)]),
        "l3g_shard_plan": (C.c_int, [C.POINTER(HyperParams), C.c_int32, C.c_int32, C.POINTER(Shard)]),
        "l3g_model_load": (C.c_int, [C.POINTER(HyperParams), C.POINTER(_Tensor), C.c_int32,
                                     C.POINTER(Options), C.POINTER(_P)]),
        "l3g_model_load_gguf": (C.c_int, [C.c_char_p, C.POINTER(Options), C.POINTER(_P)]),
        "l3g_model_hparams": (C.c_int, [_P, C.POINTER(HyperParams)]),
        "l3g_model_free": (None, [_P]),
        "l3g_state_new": (C.c_int, [_P, C.c_int32, C.POINTER(_P)]),
        "l3g_kvpool_page_bytes": (C.c_int, [_P, C.POINTER(C.c_uint64)]),
        "l3g_kvpool_new": (C.c_int, [_P, C.c_int32, C.POINTER(_P)]),
        "l3g_kvpool_free": (None, [_P]),
        "l3g_kvpool_free_pages": (C.c_int, [_P, C.POINTER(C.c_int32)]),
        "l3g_state_new_in_pool": (C.c_int, [_P, _P, C.c_int32, C.POINTER(_P)]),
        "l3g_state_pages": (C.c_int, [_P, C.POINTER(C.c_int32)]),
        "l3g_state_pos": (C.c_int, [_P, C.POINTER(C.c_int32)]),
        "l3g_state_ctx_len": (C.c_int, [_P, C.POINTER(C.c_int32)]),
        "l3g_state_set_pos": (C.c_int, [_P, C.c_int32]),
        "l3g_state_snapshot_bytes": (C.c_int, [_P, C.POINTER(C.c_uint64)]),
        "l3g_state_snapshot": (C.c_int, [_P, _P, C.c_uint64]),
        "l3g_state_restore": (C.c_int, [_P, _P, C.c_uint64]),
        "l3g_state_free": (None, [_P]),
        "l3g_workspace_new": (C.c_int, [_P, C.c_int32, C.c_int32, C.POINTER(_P)]),
        "l3g_workspace_free": (None, [_P]),
        "l3g_forward": (C.c_int, [_P, _P, _P, C.c_int32, C.POINTER(C.c_float)]),
        "l3g_forward_topk": (C.c_int, [_P, _P, _P, C.c_int32, C.c_int32, C.POINTER(TopKItem),
                                       C.POINTER(C.c_int32)]),
        "l3g_forward_argmax": (C.c_int, [_P, _P, _P, C.c_int32, C.POINTER(C.c_int32),
                                         C.POINTER(C.c_float)]),
        "l3g_prefill": (C.c_int, [_P, _P, _P, C.POINTER(C.c_int32), C.c_int32]),
        "l3g_prefill_batched": (C.c_int, [_P, _P, _P, C.POINTER(C.c_int32), C.c_int32]),
        "l3g_forward_sample": (C.c_int, [_P, _P, _P, C.c_int32, C.c_int32, C.c_float, C.c_uint64,
                                         C.POINTER(C.c_int32)]),
        "l3g_decode_sample": (C.c_int, [_P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_float,
                                        C.c_uint64, C.POINTER(C.c_int32), C.c_int32,
                                        C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                                        C.POINTER(C.c_float)]),
        "l3g_decode_greedy": (C.c_int, [_P, _P, _P, C.c_int32, C.c_int32, C.POINTER(C.c_int32),
                                        C.POINTER(C.c_float)]),
        "l3g_workspace_kernels_per_step": (C.c_int, [_P, C.POINTER(C.c_int32)]),
        "l3g_workspace_attention_layout": (C.c_int, [_P, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
        "l3g_workspace_tp_p2p": (C.c_int, [_P, C.POINTER(C.c_int32)]),
        "l3g_workspace_persistent": (C.c_int, [_P, C.POINTER(C.c_int32)]),
        "l3g_workspace_set_topk_fast_exp": (C.c_int, [_P, C.c_int32]),
        "l3g_persist_layout": (C.c_int, [_P] + [C.POINTER(C.c_int32)] * 6),
        "l3g_persist_stamps": (C.c_int, [_P, C.POINTER(C.c_uint64), C.c_int64, C.POINTER(C.c_int32),
                                         C.POINTER(C.c_int32)]),
        "l3g_profile_step": (C.c_int, [_P, _P, _P, C.c_int32, C.POINTER(C.c_int32), C.POINTER(C.c_float),
                                       C.POINTER(C.c_int32)]),
        "l3g_trace_step": (C.c_int, [_P, _P, _P, C.c_int32, C.POINTER(C.c_uint64), C.POINTER(C.c_int32),
                                     C.POINTER(C.c_int32)]),
        "l3g_matrix_upload": (C.c_int, [_P, C.c_int32, C.c_int32, C.c_int32, C.POINTER(_P)]),
        "l3g_matvec_q8": (C.c_int, [_P, _P, _P, _P, C.c_int32, C.c_int32, _P]),
        "l3g_matvec_q8_argmax_static": (C.c_int, [_P, _P, _P, _P, _P, C.c_int32, _P]),
        "l3g_matrix_free": (None, [_P]),
        "l3g_matrix_device_bytes": (C.c_int, [_P, C.POINTER(C.c_uint64)]),
        "l3g_quantize_q8_0": (C.c_int, [_P, C.c_int32, _P, _P, _P]),
        "l3g_batch_new": (C.c_int, [_P, C.c_int32, C.POINTER(_P)]),
        "l3g_batch_free": (None, [_P]),
        "l3g_batch_step": (C.c_int, [_P, C.POINTER(_P), C.c_int32, C.POINTER(C.c_int32), C.c_int32,
                                     C.c_float, C.POINTER(C.c_uint64), C.POINTER(C.c_int32),
                                     C.POINTER(C.c_float)]),
        "l3g_gemm_matrix_bytes": (C.c_int, [C.c_int32, C.c_int32, C.POINTER(C.c_uint64)]),
        "l3g_gemm_repack": (C.c_int, [_P, C.c_int32, C.c_int32, _P, C.c_uint64]),
        "l3g_gemm_matrix_upload": (C.c_int, [_P, C.c_int32, C.c_int32, C.c_int32, C.POINTER(_P)]),
        "l3g_gemm_matrix_free": (None, [_P]),
        "l3g_gemm_act_bytes": (C.c_int, [C.c_int32, C.c_int32, C.POINTER(C.c_uint64)]),
        "l3g_gemm_quantize": (C.c_int, [_P, C.c_int32, C.c_int32, _P, _P]),
        "l3g_gemm_q8": (C.c_int, [_P, _P, C.c_int32, _P, _P]),
        "l3g_gemm_status": (C.c_int, [_P, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
        "l3g_state_read_kv": (C.c_int, [_P, C.c_int32, C.c_int32, C.c_int32,
                                        C.POINTER(C.c_float), C.POINTER(C.c_float)]),
        "l3g_workspace_read": (C.c_int, [_P, C.c_int32, C.POINTER(C.c_float), C.c_int32]),
        "l3g_selftest_bounded_wait": (C.c_int, [C.c_int32, C.c_int32, C.POINTER(C.c_int32)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def exported_symbols():
    """Names the C header declares (checked against the library in tests)."""
    import re
    hdr = open(os.path.join(os.path.dirname(HERE), "include", "l3g.h")).read()
    return sorted(set(re.findall(r"\b(l3g_[a-z0-9_]+)\s*\(", hdr)))


def _check(rc):
    if rc != L3G_OK:
        raise L3GError(rc, lib().l3g_last_error().decode(errors="replace"))


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def default_options(world_size=1, rank=0, device=-1, kv_dtype=L3G_KV_F32, nccl_id=None):
    o = Options()
    lib().l3g_options_default(C.byref(o))
    o.world_size, o.rank, o.device, o.kv_dtype = world_size, rank, device, kv_dtype
    if nccl_id is not None:
        C.memmove(o.nccl_id, bytes(nccl_id), 128)
    return o


def shard_plan(hp: HyperParams, world_size: int, rank: int) -> Shard:
    """The library's tensor-parallel split for one rank (host-only)."""
    s = Shard()
    _check(lib().l3g_shard_plan(C.byref(hp), world_size, rank, C.byref(s)))
    return s


def nccl_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    _check(lib().l3g_nccl_unique_id(buf))
    return bytes(buf)


KV_PAGE = 256  # positions per KV page (L3G_KV_PAGE)


class Model:
    """Model (model.go:37-53): weights resident in HBM."""

    def __init__(self, handle):
        self._h = C.c_void_p(handle)
        hp = HyperParams()
        _check(lib().l3g_model_hparams(self._h, C.byref(hp)))
        self.HP = hp
        self._ws_cache = None

    # model.go:158-166
    def Close(self):
        if self._ws_cache is not None:
            self._ws_cache.Close()
            self._ws_cache = None
        if self._h:
            lib().l3g_model_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.Close()
        except Exception:
            pass

    def NewState(self, ctx_len: int = 0) -> "State":
        h = C.c_void_p()
        _check(lib().l3g_state_new(self._h, ctx_len, C.byref(h)))
        return State(self, h)

    def NewKvPool(self, n_pages: int) -> "KvPool":
        """A pool of n_pages KV pages (KV_PAGE positions of one layer and kv
        head each) that states made with NewState(pool=...) share."""
        h = C.c_void_p()
        _check(lib().l3g_kvpool_new(self._h, int(n_pages), C.byref(h)))
        return KvPool(self, h)

    def KvPageBytes(self) -> int:
        v = C.c_uint64()
        _check(lib().l3g_kvpool_page_bytes(self._h, C.byref(v)))
        return v.value

    def NewStateInPool(self, pool: "KvPool", ctx_len: int = 0) -> "State":
        """A state whose KV pages come from `pool` as its position grows."""
        h = C.c_void_p()
        _check(lib().l3g_state_new_in_pool(self._h, pool._h, ctx_len, C.byref(h)))
        return State(self, h)

    def NewWorkspace(self, ctx_len: int = 0, topK: int = 0) -> "Workspace":
        h = C.c_void_p()
        _check(lib().l3g_workspace_new(self._h, ctx_len, topK, C.byref(h)))
        ws = Workspace(self, h, topK)
        ws._ctx = ctx_len if 0 < ctx_len <= self.HP.CtxLen else self.HP.CtxLen
        return ws

    # infer.go:8-14
    def Forward(self, s: "State", token: int) -> np.ndarray:
        logits = np.empty(self.HP.VocabSize, dtype=np.float32)
        self.ForwardInto(s, token, logits)
        return logits

    # infer.go:16-19 (the reference builds a Workspace per call; the GPU keeps
    # one cached workspace with its captured graphs)
    def ForwardInto(self, s: "State", token: int, logitsOut) -> None:
        if self._ws_cache is None or self._ws_cache.CtxLen < s.CtxLen:
            if self._ws_cache is not None:
                self._ws_cache.Close()
            self._ws_cache = self.NewWorkspace(s.CtxLen, 0)
        self.ForwardIntoWorkspace(s, token, logitsOut, self._ws_cache)

    # infer.go:21-267
    def ForwardIntoWorkspace(self, s: "State", token: int, logitsOut, ws: "Workspace") -> None:
        if logitsOut is not None:
            if len(logitsOut) != self.HP.VocabSize:
                raise L3GError(L3G_E_INVALID, f"logitsOut len={len(logitsOut)}, want {self.HP.VocabSize}")
            buf = logitsOut if (isinstance(logitsOut, np.ndarray) and logitsOut.dtype == np.float32
                                and logitsOut.flags.c_contiguous) else np.empty(self.HP.VocabSize, np.float32)
            _check(lib().l3g_forward(self._h, s._h, _ws(ws), int(token), _fptr(buf)))
            if buf is not logitsOut:
                logitsOut[:] = buf
        else:
            _check(lib().l3g_forward(self._h, s._h, _ws(ws), int(token), None))

    # infer.go:269-511
    def ForwardTopKIntoWorkspace(self, s: "State", token: int, topK: int, ws: "Workspace"):
        k = topK if topK > 0 else 40
        items = (TopKItem * k)()
        n = C.c_int32()
        _check(lib().l3g_forward_topk(self._h, s._h, _ws(ws), int(token), k, items, C.byref(n)))
        return list(items[: n.value])

    def ForwardArgmax(self, s: "State", token: int, ws: "Workspace"):
        """Greedy step: (argmax id, its logit) of ForwardIntoWorkspace's logits."""
        nxt, lg = C.c_int32(), C.c_float()
        _check(lib().l3g_forward_argmax(self._h, s._h, _ws(ws), int(token), C.byref(nxt), C.byref(lg)))
        return nxt.value, lg.value

    def Prefill(self, s: "State", tokens, ws: "Workspace") -> None:
        """ingest, cmd/go-llama-chat/main.go:276-286."""
        arr = np.ascontiguousarray(tokens, dtype=np.int32)
        _check(lib().l3g_prefill(self._h, s._h, _ws(ws), arr.ctypes.data_as(C.POINTER(C.c_int32)),
                                 arr.size))

    def PrefillBatched(self, s: "State", tokens, ws: "Workspace") -> None:
        """The same ingest, up to 512 tokens per pass through the batched
        tensor-core product (l3g_prefill_batched)."""
        arr = np.ascontiguousarray(tokens, dtype=np.int32)
        _check(lib().l3g_prefill_batched(self._h, s._h, _ws(ws),
                                         arr.ctypes.data_as(C.POINTER(C.c_int32)), arr.size))

    KERNEL_KINDS = ("embed", "qkv_rope_kv", "attention", "wo", "upgate_swiglu", "down", "logits_argmax",
                    "other", "act_quant", "layers")

    def ProfileStep(self, s: "State", token: int, ws: "Workspace", cap: int = 4096):
        """One step run eagerly with every kernel timed alone: [(kind, us)]."""
        kinds = (C.c_int32 * cap)()
        us = (C.c_float * cap)()
        n = C.c_int32(cap)
        _check(lib().l3g_profile_step(self._h, s._h, _ws(ws), int(token), kinds, us, C.byref(n)))
        return [(self.KERNEL_KINDS[kinds[i]], float(us[i])) for i in range(n.value)]

    TRACE_CTAS = 256

    def TraceStep(self, s: "State", token: int, ws: "Workspace", cap: int = 256):
        """One greedy step replayed as its graph with the device timeline:
        [(kind, stamps[TRACE_CTAS][8] in ns)] per launch (zeros: untraced)."""
        per = self.TRACE_CTAS * 8
        stamps = np.zeros(cap * per, np.uint64)
        kinds = (C.c_int32 * cap)()
        n = C.c_int32(cap)
        _check(lib().l3g_trace_step(self._h, s._h, _ws(ws), int(token),
                                    stamps.ctypes.data_as(C.POINTER(C.c_uint64)), kinds, C.byref(n)))
        arr = stamps[: n.value * per].reshape(n.value, self.TRACE_CTAS, 8).astype(np.int64)
        return [(self.KERNEL_KINDS[kinds[i]], arr[i]) for i in range(n.value)]

    def DecodeGreedy(self, s: "State", first_token: int, n: int, ws: "Workspace"):
        """n greedy steps fed on the device; returns (tokens, device_ms)."""
        out = np.empty(n, np.int32)
        ms = C.c_float()
        _check(lib().l3g_decode_greedy(self._h, s._h, _ws(ws), int(first_token), n,
                                       out.ctypes.data_as(C.POINTER(C.c_int32)), C.byref(ms)))
        return out, ms.value

    def ForwardSample(self, s: "State", token: int, ws: "Workspace", top_k: int = 0,
                      temperature: float = 0.8, seed: int = 1) -> int:
        """ForwardTopKIntoWorkspace + SampleTopK on the device (Philox draw
        `seed`, counted per workspace); returns the sampled id."""
        nxt = C.c_int32()
        _check(lib().l3g_forward_sample(self._h, s._h, _ws(ws), int(token), int(top_k),
                                        float(temperature), int(seed) & (2**64 - 1), C.byref(nxt)))
        return nxt.value

    def DecodeSample(self, s: "State", first_token: int, n: int, ws: "Workspace", top_k: int = 0,
                     temperature: float = 0.8, seed: int = 1, stop_ids=()):
        """n sampled steps fed on the device; returns (tokens up to and
        including the first stop id, device_ms)."""
        out = np.empty(n, np.int32)
        stops = np.ascontiguousarray(np.asarray(stop_ids, np.int32))
        n_out = C.c_int32()
        ms = C.c_float()
        _check(lib().l3g_decode_sample(self._h, s._h, _ws(ws), int(first_token), n, int(top_k),
                                       float(temperature), int(seed) & (2**64 - 1),
                                       stops.ctypes.data_as(C.POINTER(C.c_int32)) if stops.size else None,
                                       stops.size, out.ctypes.data_as(C.POINTER(C.c_int32)),
                                       C.byref(n_out), C.byref(ms)))
        return out[:n_out.value], ms.value


def _ws(ws):
    return ws._h if ws is not None else None


class State:
    """State (state.go:45-49): position + HBM KV cache + RoPE tables."""

    def __init__(self, model: Model, h):
        self.model = model
        self._h = h

    @property
    def Pos(self) -> int:
        v = C.c_int32()
        _check(lib().l3g_state_pos(self._h, C.byref(v)))
        return v.value

    @Pos.setter
    def Pos(self, pos: int):
        _check(lib().l3g_state_set_pos(self._h, pos))

    @property
    def CtxLen(self) -> int:
        v = C.c_int32()
        _check(lib().l3g_state_ctx_len(self._h, C.byref(v)))
        return v.value

    def read_kv(self, layer: int, pos0: int, npos: int):
        """K, V of one layer, positions [pos0, pos0+npos): [npos][kv heads][hd]."""
        m = self.model.HP
        hd = m.NEmb // m.NHeads
        n = npos * self.local_kv_heads * hd
        k = np.empty(n, np.float32)
        v = np.empty(n, np.float32)
        _check(lib().l3g_state_read_kv(self._h, layer, pos0, npos, _fptr(k), _fptr(v)))
        shape = (npos, self.local_kv_heads, hd)
        return k.reshape(shape), v.reshape(shape)

    local_kv_heads = property(lambda self: self.model.HP.NHeadsKV // getattr(self.model, "world_size", 1))

    def Snapshot(self) -> np.ndarray:
        """The position and KV rows [0, Pos) of this rank, as host bytes."""
        n = C.c_uint64()
        _check(lib().l3g_state_snapshot_bytes(self._h, C.byref(n)))
        buf = np.empty(n.value, np.uint8)
        _check(lib().l3g_state_snapshot(self._h, buf.ctypes.data, n.value))
        return buf

    def Restore(self, snap: np.ndarray):
        """Loads a Snapshot of a state of the same model (any context length
        at least its position) and moves to its position."""
        snap = np.ascontiguousarray(snap, dtype=np.uint8)
        _check(lib().l3g_state_restore(self._h, snap.ctypes.data, snap.size))

    @property
    def Pages(self) -> int:
        """KV pages this state holds from a shared pool (0: a private pool)."""
        v = C.c_int32()
        _check(lib().l3g_state_pages(self._h, C.byref(v)))
        return v.value

    def Close(self):
        if self._h:
            lib().l3g_state_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.Close()
        except Exception:
            pass


class KvPool:
    """Pages of KV cache shared by the states of one model (l3g_kvpool)."""

    def __init__(self, model: Model, h):
        self.model = model
        self._h = h

    @property
    def FreePages(self) -> int:
        v = C.c_int32()
        _check(lib().l3g_kvpool_free_pages(self._h, C.byref(v)))
        return v.value

    def Close(self):
        if self._h:
            lib().l3g_kvpool_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.Close()
        except Exception:
            pass


class Workspace:
    """Workspace (workspace.go:3-33): device activations, scratch, graphs.
    NOT safe for concurrent use, like the reference's."""

    def __init__(self, model: Model, h, topK):
        self.model = model
        self._h = h
        self.TopK = topK if topK > 0 else 40

    @property
    def CtxLen(self):
        return self._ctx if hasattr(self, "_ctx") else self.model.HP.CtxLen

    def read(self, which: int, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        _check(lib().l3g_workspace_read(self._h, which, _fptr(out), n))
        return out

    def SetTopKFastExp(self, on: bool = True):
        """ForwardTopKIntoWorkspace's attention softmax as the reference
        computes it (fastExp of score - max over all positions,
        infer.go:376-423, 520-525) for this workspace's top-K and sampled
        calls; the full-logits, argmax and greedy calls keep the exact exp
        of ForwardIntoWorkspace.  Off by default."""
        _check(lib().l3g_workspace_set_topk_fast_exp(self._h, 1 if on else 0))

    def kernels_per_step(self) -> int:
        v = C.c_int32()
        _check(lib().l3g_workspace_kernels_per_step(self._h, C.byref(v)))
        return v.value

    def tp_p2p(self) -> bool:
        """True when the tensor-parallel reductions go over peer memory."""
        v = C.c_int32()
        _check(lib().l3g_workspace_tp_p2p(self._h, C.byref(v)))
        return bool(v.value)

    def persistent(self) -> bool:
        """True when this workspace's steps run every layer in one persistent
        launch (model loaded with L3G_PERSIST=1 in the environment)."""
        v = C.c_int32()
        _check(lib().l3g_workspace_persistent(self._h, C.byref(v)))
        return bool(v.value)

    def persist_layout(self) -> dict:
        """The persistent kernel's ring slots, slot bytes, attention splits,
        barrier counters, shared memory per CTA and grid barriers per layer."""
        v = [C.c_int32() for _ in range(6)]
        _check(lib().l3g_persist_layout(self._h, *[C.byref(x) for x in v]))
        return dict(zip(("stages", "slot_bytes", "splits", "barrier_counters", "smem_bytes",
                         "barriers_per_layer"), (x.value for x in v)))

    def persist_stamps(self) -> np.ndarray:
        """After Model.TraceStep on a persistent workspace: [barrier][cta][2]
        %globaltimer ns of each CTA's arrival at and release from each grid
        barrier (barriers_per_layer per layer; zeros where none ran)."""
        cap = 7 * self.model.HP.NLayers * 1024 * 2
        out = np.zeros(cap, np.uint64)
        nb, grid = C.c_int32(), C.c_int32()
        _check(lib().l3g_persist_stamps(self._h, out.ctypes.data_as(C.POINTER(C.c_uint64)), cap,
                                        C.byref(nb), C.byref(grid)))
        return out[: nb.value * grid.value * 2].reshape(nb.value, grid.value, 2).astype(np.int64)

    def attention_layout(self) -> tuple[int, int]:
        """(splits per kv head, cluster size or 0)."""
        sp, cl = C.c_int32(), C.c_int32()
        _check(lib().l3g_workspace_attention_layout(self._h, C.byref(sp), C.byref(cl)))
        return sp.value, cl.value

    def Close(self):
        if self._h:
            lib().l3g_workspace_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.Close()
        except Exception:
            pass


def _tensor_array(tensors: dict):
    arr = (_Tensor * len(tensors))()
    keep = []
    for i, (name, (dims, typ, data)) in enumerate(tensors.items()):
        data = np.ascontiguousarray(data)
        keep.append(data)
        nm = name.encode()
        keep.append(nm)
        arr[i].name = nm
        arr[i].type = typ
        arr[i].n_dims = len(dims)
        for j, d in enumerate(dims):
            arr[i].dims[j] = int(d)
        arr[i].data = data.ctypes.data
        arr[i].nbytes = data.nbytes
    return arr, keep


def hparams_for(cfg) -> HyperParams:
    hp = HyperParams()
    hp.VocabSize, hp.NLayers, hp.NEmb = cfg.vocab, cfg.n_layers, cfg.n_emb
    hp.NHeads, hp.NHeadsKV, hp.NFF = cfg.n_heads, cfg.n_heads_kv, cfg.n_ff
    hp.RopeDim, hp.CtxLen = cfg.head_dim, cfg.ctx_len
    hp.RmsEps, hp.RopeBase = cfg.rms_eps, cfg.rope_base
    return hp


def LoadModelFromTensors(hp: HyperParams, tensors: dict, options: Options | None = None) -> Model:
    """l3g_model_load: the path a Go shim takes with its mmapped tensors."""
    arr, keep = _tensor_array(tensors)
    h = C.c_void_p()
    _check(lib().l3g_model_load(C.byref(hp), arr, len(tensors),
                                C.byref(options) if options is not None else None, C.byref(h)))
    m = Model(h.value)
    m.world_size = options.world_size if options is not None else 1
    del keep
    return m


def LoadModel(path: str, threads: int = 0, options: Options | None = None) -> Model:
    """LoadModel, model.go:55-156 (threads is accepted for signature parity;
    the GPU grid replaces the goroutine pool)."""
    h = C.c_void_p()
    _check(lib().l3g_model_load_gguf(path.encode(), C.byref(options) if options is not None else None,
                                     C.byref(h)))
    m = Model(h.value)
    m.world_size = options.world_size if options is not None else 1
    return m


class Matrix:
    """A Q8_0 matrix resident on the device for the matvec_q8_c drop-in."""

    def __init__(self, q8_rows: np.ndarray, rows: int, cols: int, device: int = -1):
        q8_rows = np.ascontiguousarray(q8_rows, dtype=np.uint8)
        if q8_rows.size != rows * cols // 32 * 34:
            raise L3GError(L3G_E_INVALID, "matrix bytes do not match rows x cols")
        h = C.c_void_p()
        _check(lib().l3g_matrix_upload(q8_rows.ctypes.data, rows, cols, device, C.byref(h)))
        self._h = h
        self.rows, self.cols = rows, cols

    def device_bytes(self) -> int:
        v = C.c_uint64()
        _check(lib().l3g_matrix_device_bytes(self._h, C.byref(v)))
        return v.value

    def matvec(self, x_scales_ptr: int, x_qs_ptr: int, out_ptr: int, start: int = 0,
               end: int | None = None, stream: int = 0):
        """matvec_q8_c(w, x_scales, x_qs, out, start, end, cols) on device pointers."""
        end = self.rows if end is None else end
        _check(lib().l3g_matvec_q8(self._h, x_scales_ptr, x_qs_ptr, out_ptr, start, end, stream or None))

    def matvec_argmax_static(self, x_scales_ptr: int, x_qs_ptr: int, out_ptr: int,
                             result_ptr: int, max_ctas: int = 0, stream: int = 0):
        """The same matvec over all rows fused with the argmax of its output,
        using the library's static device scratch (no allocation).  out_ptr
        may be 0; result_ptr points at 16 device bytes that receive
        (int32 index, float32 value, int32 status, int32 detail)."""
        _check(lib().l3g_matvec_q8_argmax_static(self._h, x_scales_ptr, x_qs_ptr, out_ptr or None,
                                                 result_ptr, max_ctas, stream or None))

    def Close(self):
        if self._h:
            lib().l3g_matrix_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.Close()
        except Exception:
            pass


class Batch:
    """Batched decode over many sessions (l3g_state) of one model: one step
    ingests a token per session and samples its next token on the device."""

    def __init__(self, model: "Model", max_seqs: int):
        h = C.c_void_p()
        _check(lib().l3g_batch_new(model._h, max_seqs, C.byref(h)))
        self._h = h
        self.model = model
        self.max_seqs = max_seqs

    def step(self, states, tokens, seeds, top_k: int = 40, temperature: float = 0.8,
             want_logits: bool = False):
        """Returns next tokens [n] (and logits [n][vocab] when asked)."""
        n = len(states)
        arr = (C.c_void_p * n)(*[s._h.value if isinstance(s._h, C.c_void_p) else s._h
                                for s in states])
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        sd = np.ascontiguousarray(seeds, dtype=np.uint64)
        nxt = np.empty(n, np.int32)
        logits = np.empty((n, self.model.HP.VocabSize), np.float32) if want_logits else None
        _check(lib().l3g_batch_step(self._h, C.cast(arr, C.POINTER(C.c_void_p)), n,
                                    tok.ctypes.data_as(C.POINTER(C.c_int32)), top_k, temperature,
                                    sd.ctypes.data_as(C.POINTER(C.c_uint64)),
                                    nxt.ctypes.data_as(C.POINTER(C.c_int32)),
                                    _fptr(logits) if logits is not None else None))
        return (nxt, logits) if want_logits else nxt

    def Close(self):
        if self._h:
            lib().l3g_batch_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.Close()
        except Exception:
            pass


def gemm_matrix_bytes(rows: int, cols: int) -> int:
    v = C.c_uint64()
    _check(lib().l3g_gemm_matrix_bytes(rows, cols, C.byref(v)))
    return v.value


def gemm_repack(q8_rows: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Host-side repack of GGUF Q8_0 rows into the batched product's weight
    chunks (no device needed)."""
    q8_rows = np.ascontiguousarray(q8_rows, dtype=np.uint8)
    if q8_rows.size != rows * cols // 32 * 34:
        raise L3GError(L3G_E_INVALID, "matrix bytes do not match rows x cols")
    out = np.empty(gemm_matrix_bytes(rows, cols), np.uint8)
    _check(lib().l3g_gemm_repack(q8_rows.ctypes.data, rows, cols, out.ctypes.data, out.size))
    return out


def gemm_act_bytes(n_tok: int, cols: int) -> int:
    v = C.c_uint64()
    _check(lib().l3g_gemm_act_bytes(n_tok, cols, C.byref(v)))
    return v.value


def gemm_quantize(x_ptr: int, n_tok: int, cols: int, act_ptr: int, stream: int = 0):
    """QuantizeQ8_0Into of n_tok device rows of cols floats into the batched
    product's activation chunks (act: gemm_act_bytes(n_tok, cols) bytes)."""
    _check(lib().l3g_gemm_quantize(x_ptr, n_tok, cols, act_ptr, stream or None))


class GemmMatrix:
    """A Q8_0 matrix resident on the device for the batched product (n_tok
    matvec_q8_c products in one pass over the weights, on the tensor cores)."""

    def __init__(self, q8_rows: np.ndarray, rows: int, cols: int, device: int = -1):
        q8_rows = np.ascontiguousarray(q8_rows, dtype=np.uint8)
        if q8_rows.size != rows * cols // 32 * 34:
            raise L3GError(L3G_E_INVALID, "matrix bytes do not match rows x cols")
        h = C.c_void_p()
        _check(lib().l3g_gemm_matrix_upload(q8_rows.ctypes.data, rows, cols, device, C.byref(h)))
        self._h = h
        self.rows, self.cols = rows, cols

    def quantize(self, x_ptr: int, n_tok: int, act_ptr: int, stream: int = 0):
        """gemm_quantize with this matrix's column count."""
        gemm_quantize(x_ptr, n_tok, self.cols, act_ptr, stream)

    def gemm(self, act_ptr: int, n_tok: int, out_ptr: int, stream: int = 0):
        """out[n][r] for n < n_tok, r < rows (device pointers)."""
        _check(lib().l3g_gemm_q8(self._h, act_ptr, n_tok, out_ptr, stream or None))

    def status(self):
        """(err, where) of the kernel's bounded waits since the last call."""
        e, w = C.c_int32(), C.c_int32()
        _check(lib().l3g_gemm_status(self._h, C.byref(e), C.byref(w)))
        return e.value, w.value

    def Close(self):
        if self._h:
            lib().l3g_gemm_matrix_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.Close()
        except Exception:
            pass


def quantize_q8_0_device(x_ptr: int, n: int, d_ptr: int, qs_ptr: int, stream: int = 0):
    _check(lib().l3g_quantize_q8_0(x_ptr, n, d_ptr, qs_ptr, stream or None))


def selftest_bounded_wait(device: int = -1, timeout_us: int = 2000) -> int:
    st = C.c_int32()
    _check(lib().l3g_selftest_bounded_wait(device, timeout_us, C.byref(st)))
    return st.value


class Sampler:
    """Sampler (sampling.go:11-30): temperature softmax over the top-k, drawn
    from a seeded numpy Generator (Go's math/rand stream is not reproduced)."""

    def __init__(self, temp: float, topK: int, seed: int):
        if temp <= 0:
            temp = 0.8
        if topK <= 0:
            topK = 40
        if seed == 0:
            import time
            seed = time.time_ns()
        self.Temperature, self.TopK, self.Seed = float(np.float32(temp)), topK, seed
        self.rng = np.random.default_rng(seed)

    def _draw(self, ids, logits):
        # sampling.go:115-142: f64 softmax over items, cumulative pick
        mx = max(logits)
        invT = 1.0 / self.Temperature
        exps = [math.exp(float(np.float32(l - mx)) * invT) for l in logits]
        r = self.rng.random() * sum(exps)
        acc = 0.0
        for i, e in enumerate(exps):
            acc += e
            if r <= acc:
                return int(ids[i])
        return int(ids[-1])

    def SampleTopK(self, items) -> int:
        if not items:
            return 0
        return self._draw([it.ID for it in items], [np.float32(it.Logit) for it in items])

    def Sample(self, logits) -> int:
        k = min(self.TopK, len(logits))
        idx = np.argpartition(-np.asarray(logits), k - 1)[:k]
        return self._draw(list(idx), [np.float32(logits[i]) for i in idx])


def NewSampler(temp: float, topK: int, seed: int) -> Sampler:
    return Sampler(temp, topK, seed)
