"""Seeded synthetic Llama-3-shaped Q8_0 models (no checkpoints, no network).

A model is a dict ``name -> (dims, ggml_type, uint8 bytes)`` with the tensor
names and ne0-first dims the reference loader expects
(internal/llama/model.go:83-138): weights drawn N(0, 0.02) and quantized to
Q8_0 (fp16 d = maxabs/127 per 32-element block, q = round(w/d)), norms 1.0.
It can be written as a GGUF file (with the tokenizer metadata LoadModel
requires, tokenizer_bpe.go:37-49, and UINT32 / FLOAT32 hyperparameters as
gguf.go:391-432 demands) or handed to ``l3g_model_load`` / the oracle as
in-memory tensors.

Generation runs on torch (CPU for small models, CUDA for the 8B shape where
it is much faster); a given (config, seed, device) always yields the same
bytes.
"""
from __future__ import annotations

import math
import zlib
from dataclasses import dataclass, field

import numpy as np

from gguf import (GGML_F32, GGML_Q8_0, T_ARRAY, T_FLOAT32, T_STRING, T_UINT32,
                  GGUFWriter)


@dataclass(frozen=True)
class Config:
    name: str
    n_emb: int
    n_layers: int
    n_heads: int
    n_heads_kv: int
    n_ff: int
    vocab: int
    tied: bool = True
    rope_base: float = 500000.0
    # llama3 frequency scaling (factor, low_freq, high_freq, original ctx)
    rope_scaling: tuple | None = None
    rms_eps: float = 1e-5
    ctx_len: int = 2048

    @property
    def head_dim(self):
        return self.n_emb // self.n_heads

    def weight_bytes(self) -> int:
        """Q8_0 bytes read per decoded token (all matvecs incl. logits, plus the
        embedding row): the algorithmic weight traffic of one step."""
        e, f, kv = self.n_emb, self.n_ff, self.n_heads_kv * self.head_dim
        per_layer = e * e + 2 * e * kv + e * e + 3 * e * f
        n = self.n_layers * per_layer + self.vocab * e
        return n // 32 * 34 + e // 32 * 34

    def kv_bytes(self, n_pos: int, elem_bytes: int = 4) -> int:
        """K and V bytes read by attention for one token attending n_pos."""
        return self.n_layers * 2 * self.n_heads_kv * self.head_dim * n_pos * elem_bytes


CONFIGS = {
    # the five shapes of the workload definitions
    "llama3.2-1b": Config("llama3.2-1b", 2048, 16, 32, 8, 8192, 128256, tied=True, ctx_len=2048),
    "llama3.2-3b": Config("llama3.2-3b", 3072, 28, 24, 8, 8192, 128256, tied=True, ctx_len=4096),
    "llama3.1-8b": Config("llama3.1-8b", 4096, 32, 32, 8, 14336, 128256, tied=False,
                          rope_scaling=(8.0, 1.0, 4.0, 8192), ctx_len=8320),
    # the 8B layer shapes with two layers (~1.1 GB): kernel-level profiling
    "llama3.1-8b-2l": Config("llama3.1-8b-2l", 4096, 2, 32, 8, 14336, 128256, tied=False,
                             rope_scaling=(8.0, 1.0, 4.0, 8192), ctx_len=8320),
    # small shapes for parity tests (same structure, seconds on the CPU oracle)
    "tiny": Config("tiny", 64, 2, 2, 1, 128, 97, tied=True, ctx_len=64),
    "tiny-gqa": Config("tiny-gqa", 128, 2, 4, 2, 256, 300, tied=False, ctx_len=128),
    "small": Config("small", 256, 2, 4, 2, 512, 1000, tied=True, ctx_len=512),
    "small-hd128": Config("small-hd128", 512, 2, 4, 1, 1024, 2048, tied=False,
                          rope_scaling=(8.0, 1.0, 4.0, 8192), ctx_len=4608),
    "mid": Config("mid", 1024, 4, 8, 2, 2816, 8000, tied=True, ctx_len=1024),
    # a GQA group of 3 (the 3B shape's 24 / 8), padded to 4 in attention
    "tiny-g3": Config("tiny-g3", 192, 2, 6, 2, 384, 500, tied=True, ctx_len=128),
    # the 1B layer shapes (head_dim 64, the full vocabulary) with two layers
    "llama3.2-1b-2l": Config("llama3.2-1b-2l", 2048, 2, 32, 8, 8192, 128256, tied=True, ctx_len=2048),
}


def llama3_freq_factors(cfg: Config) -> np.ndarray:
    """Divisors of the inverse RoPE frequencies by the published Llama-3.1
    scaling rule (an extension: the reference has no RoPE scaling)."""
    half = cfg.head_dim // 2
    factor, low, high, orig = cfg.rope_scaling
    low_wl, high_wl = orig / low, orig / high
    out = np.ones(half, dtype=np.float32)
    for i in range(half):
        freq = 1.0 / math.pow(cfg.rope_base, (2 * i) / cfg.head_dim)
        wl = 2 * math.pi / freq
        if wl < high_wl:
            out[i] = 1.0
        elif wl > low_wl:
            out[i] = factor
        else:
            smooth = (orig / wl - low) / (high - low)
            out[i] = 1.0 / ((1 - smooth) / factor + smooth)
    return out


def _seed_for(seed: int, name: str) -> int:
    return (seed * 1_000_003 + zlib.crc32(name.encode())) & 0x7FFF_FFFF_FFFF_FFFF


def quantize_q8_0_rows(w, torch):
    """[rows, cols] float tensor -> uint8 [rows, cols/32*34] GGUF Q8_0 bytes."""
    rows, cols = w.shape
    nb = cols // 32
    blk = w.reshape(rows, nb, 32)
    amax = blk.abs().amax(-1)
    d16 = (amax / 127.0).to(torch.float16)
    d = d16.float()
    inv = torch.where(d > 0, 1.0 / d, torch.zeros_like(d))
    q = torch.round(blk * inv[..., None]).clamp_(-127, 127).to(torch.int8)
    out = torch.empty(rows, nb, 34, dtype=torch.uint8, device=w.device)
    out[..., :2] = d16.view(torch.uint8).reshape(rows, nb, 2)
    out[..., 2:] = q.view(torch.uint8)
    # fp16 subnormal scales decode differently in simd.c:21-30; never emit one
    nz = d16[d16 != 0].float()
    if nz.numel() and float(nz.min()) < 6.104e-5:
        raise ValueError("Q8_0 scale would be an fp16 subnormal")
    return out.reshape(rows, nb * 34)


def _q8_tensor(name, rows, cols, seed, device, torch, std=0.02, chunk_elems=1 << 25):
    g = torch.Generator(device=device)
    g.manual_seed(_seed_for(seed, name))
    out = np.empty((rows, cols // 32 * 34), dtype=np.uint8)
    step = max(1, chunk_elems // cols)
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        w = torch.randn(r1 - r0, cols, generator=g, device=device, dtype=torch.float32) * std
        out[r0:r1] = quantize_q8_0_rows(w, torch).cpu().numpy()
    return out


def make_model(cfg: Config, seed: int = 0, device: str = "cpu") -> dict:
    """All tensors of a synthetic model, as host numpy byte arrays."""
    import torch
    e, f, kv = cfg.n_emb, cfg.n_ff, cfg.n_heads_kv * cfg.head_dim
    t = {}

    def q8(name, rows, cols):
        t[name] = ([cols, rows], GGML_Q8_0, _q8_tensor(name, rows, cols, seed, device, torch))

    def ones(name, n):
        t[name] = ([n], GGML_F32, np.ones(n, dtype=np.float32).view(np.uint8))

    q8("token_embd.weight", cfg.vocab, e)
    ones("output_norm.weight", e)
    if not cfg.tied:
        q8("output.weight", cfg.vocab, e)
    if cfg.rope_scaling is not None:
        ff = llama3_freq_factors(cfg)
        t["rope_freqs.weight"] = ([ff.size], GGML_F32, ff.view(np.uint8))
    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        ones(p + "attn_norm.weight", e)
        ones(p + "ffn_norm.weight", e)
        q8(p + "attn_q.weight", e, e)
        q8(p + "attn_k.weight", kv, e)
        q8(p + "attn_v.weight", kv, e)
        q8(p + "attn_output.weight", e, e)
        q8(p + "ffn_up.weight", f, e)
        q8(p + "ffn_gate.weight", f, e)
        q8(p + "ffn_down.weight", e, f)
    return t


def write_gguf(path: str, cfg: Config, tensors: dict):
    w = GGUFWriter()
    w.add("general.architecture", T_STRING, "llama")
    w.add("llama.vocab_size", T_UINT32, cfg.vocab)
    w.add("llama.block_count", T_UINT32, cfg.n_layers)
    w.add("llama.embedding_length", T_UINT32, cfg.n_emb)
    w.add("llama.feed_forward_length", T_UINT32, cfg.n_ff)
    w.add("llama.attention.head_count", T_UINT32, cfg.n_heads)
    w.add("llama.attention.head_count_kv", T_UINT32, cfg.n_heads_kv)
    w.add("llama.rope.dimension_count", T_UINT32, cfg.head_dim)
    w.add("llama.context_length", T_UINT32, cfg.ctx_len)
    w.add("llama.norm_rms_eps", T_FLOAT32, cfg.rms_eps)
    w.add("llama.rope.freq_base", T_FLOAT32, cfg.rope_base)
    # synthetic gpt2 tokenizer metadata (the tokenizer itself is out of scope)
    toks = [f"t{i}" for i in range(cfg.vocab)]
    specials = ["<|begin_of_text|>", "<|end_of_text|>", "<|eot_id|>"]
    for j, s in enumerate(specials):
        toks[cfg.vocab - len(specials) + j] = s
    w.add("tokenizer.ggml.model", T_STRING, "gpt2")
    w.add("tokenizer.ggml.tokens", T_ARRAY, toks, T_STRING)
    w.add("tokenizer.ggml.merges", T_ARRAY, ["t 0"], T_STRING)
    w.add("tokenizer.ggml.bos_token_id", T_UINT32, cfg.vocab - 3)
    w.add("tokenizer.ggml.eos_token_id", T_UINT32, cfg.vocab - 2)
    w.add("tokenizer.ggml.eot_token_id", T_UINT32, cfg.vocab - 1)
    for name, (dims, typ, data) in tensors.items():
        w.add_tensor(name, dims, typ, data)
    w.write(path)


def prompt_ids(cfg: Config, n: int, seed: int = 0) -> np.ndarray:
    """n seeded token ids uniform in [0, vocab)."""
    return np.random.default_rng(seed).integers(0, cfg.vocab, size=n, dtype=np.int64).astype(np.int32)
