"""Independent float64 numpy forward of the decode step, used only to
cross-check the oracle's restatement (the reference ships no golden vectors).
It follows the same algorithm -- Q8_0 weights, per-32-block activation
quantization, adjacent-pair RoPE, GQA softmax attention, SwiGLU -- but every
float operation runs in float64 with numpy's own ordering.
"""
import math

import numpy as np


def split_q8_0(b: np.ndarray, rows: int, cols: int):
    """GGUF Q8_0 bytes -> (q int8 [rows, nb, 32], d float64 [rows, nb])."""
    nb = cols // 32
    blk = b.reshape(rows, nb, 34)
    d = blk[:, :, :2].copy().view(np.float16)[..., 0].astype(np.float64)
    q = blk[:, :, 2:].view(np.int8)
    return q, d


def quant_act(x: np.ndarray):
    """The reference's activation scheme (q8_0.go:22-79) in float64 math."""
    n = x.size
    nb = (n + 31) // 32
    xp = np.zeros(nb * 32)
    xp[:n] = x
    blk = xp.reshape(nb, 32)
    scale = np.abs(blk).max(axis=1) / 127.0
    scale[scale == 0] = 1e-8
    f = blk / scale[:, None]
    q = np.where(f >= 0, np.trunc(f + 0.5), np.trunc(f - 0.5))
    return scale, np.clip(q, -128, 127)


def matvec(q, d, xs, xq):
    # sum_b d_w[r,b] * d_x[b] * sum_i q_w[r,b,i] q_x[b,i]
    isum = np.einsum("rbi,bi->rb", q.astype(np.float64), xq)
    return (isum * d * xs[None, :]).sum(axis=1)


class NpModel:
    def __init__(self, cfg, tensors, ctx, rope_factors=None):
        self.cfg = cfg
        e, f = cfg.n_emb, cfg.n_ff
        kv = cfg.n_heads_kv * cfg.head_dim

        def mat(name, rows, cols):
            return split_q8_0(tensors[name][2], rows, cols)

        def vec(name):
            return tensors[name][2].view(np.float32).astype(np.float64)

        self.emb = mat("token_embd.weight", cfg.vocab, e)
        self.out = mat("output.weight", cfg.vocab, e) if "output.weight" in tensors else self.emb
        self.out_norm = vec("output_norm.weight")
        self.L = []
        for i in range(cfg.n_layers):
            p = f"blk.{i}."
            self.L.append(dict(
                q=mat(p + "attn_q.weight", e, e), k=mat(p + "attn_k.weight", kv, e),
                v=mat(p + "attn_v.weight", kv, e), o=mat(p + "attn_output.weight", e, e),
                up=mat(p + "ffn_up.weight", f, e), gate=mat(p + "ffn_gate.weight", f, e),
                down=mat(p + "ffn_down.weight", e, f),
                an=vec(p + "attn_norm.weight"), fn=vec(p + "ffn_norm.weight")))
        hd = cfg.head_dim
        half = hd // 2
        inv = np.array([1.0 / math.pow(cfg.rope_base, 2 * i / hd) for i in range(half)])
        if rope_factors is not None:
            inv = inv / rope_factors
        ang = np.arange(ctx)[:, None] * inv[None, :]
        self.cos, self.sin = np.cos(ang), np.sin(ang)
        self.K = np.zeros((cfg.n_layers, ctx, cfg.n_heads_kv, hd))
        self.V = np.zeros_like(self.K)
        self.pos = 0

    def _norm(self, x, w):
        return x / math.sqrt((x * x).mean() + self.cfg.rms_eps) * w

    def _mv(self, W, x):
        xs, xq = quant_act(x)
        return matvec(W[0], W[1], xs, xq)

    def _rope(self, v):
        c, s = self.cos[self.pos], self.sin[self.pos]
        x0, x1 = v[..., 0::2].copy(), v[..., 1::2].copy()
        v[..., 0::2] = x0 * c - x1 * s
        v[..., 1::2] = x0 * s + x1 * c

    def forward(self, token):
        cfg = self.cfg
        hd, nh, nkv = cfg.head_dim, cfg.n_heads, cfg.n_heads_kv
        q8, d = self.emb[0][token], self.emb[1][token]
        x = (q8.astype(np.float64) * d[:, None]).reshape(-1)
        for l, L in enumerate(self.L):
            h = self._norm(x, L["an"])
            q = self._mv(L["q"], h).reshape(nh, hd)
            k = self._mv(L["k"], h).reshape(nkv, hd)
            v = self._mv(L["v"], h).reshape(nkv, hd)
            self._rope(q)
            self._rope(k)
            self.K[l, self.pos], self.V[l, self.pos] = k, v
            Kt, Vt = self.K[l, : self.pos + 1], self.V[l, : self.pos + 1]
            att = np.empty((nh, hd))
            for hh in range(nh):
                g = hh // (nh // nkv)
                sc = Kt[:, g, :] @ q[hh] / math.sqrt(hd)
                p = np.exp(sc - sc.max())
                att[hh] = (p / p.sum()) @ Vt[:, g, :]
            x = x + self._mv(L["o"], att.reshape(-1))
            h = self._norm(x, L["fn"])
            up, gate = self._mv(L["up"], h), self._mv(L["gate"], h)
            act = gate / (1 + np.exp(-gate)) * up
            x = x + self._mv(L["down"], act)
        self.pos += 1
        h = self._norm(x, self.out_norm)
        return self._mv(self.out, h)
