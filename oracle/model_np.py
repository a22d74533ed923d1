"""Numpy restatement of the reference's LayerSkip-Llama math and packed ragged forward.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker, never the thing
measured or shipped.

Arithmetic follows the reference step by step, including where the reference rounds
to the model dtype.  ``bf16=True`` emulates PyTorch's bf16 tensor semantics: every
elementwise op computes in fp32 and rounds its result to bf16 (round to nearest even);
GEMMs take bf16-valued inputs, accumulate in fp32 and round the output.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

F32 = np.float32


def to_bf16(x) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even); returned as float32."""
    u = np.ascontiguousarray(x, dtype=F32).view(np.uint32)
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + r) & np.uint32(0xFFFF0000)).view(F32)


@dataclass
class OracleConfig:
    """Mirror of ``ModelConfig`` (common/model.py:39-108) restricted to what the math needs."""
    vocab_size: int
    dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    intermediate_size: int
    norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    tie_word_embeddings: bool = False
    rope_scaling: Optional[dict] = None


def _llama3_inv_freq(inv_freq: np.ndarray, s: dict) -> np.ndarray:
    """common/model.py:113-126 (llama3 frequency scaling)."""
    factor, low, high = s["factor"], s["low_freq_factor"], s["high_freq_factor"]
    old = s["original_max_position_embeddings"]
    low_w, high_w = old / low, old / high
    # ``scalar / tensor`` evaluates as reciprocal(tensor) * scalar in fp32
    wl = ((F32(1.0) / inv_freq).astype(F32) * F32(2 * math.pi)).astype(F32)
    out = np.where(wl > low_w, inv_freq / F32(factor), inv_freq).astype(F32)
    smooth = ((old / wl - low) / (high - low)).astype(F32)
    smoothed = ((1 - smooth) * out / F32(factor) + smooth * out).astype(F32)
    medium = ~(wl < high_w) & ~(wl > low_w)
    return np.where(medium, smoothed, out).astype(F32)


def rope_tables(cfg: OracleConfig, max_seq: int) -> tuple[np.ndarray, np.ndarray]:
    """common/model.py:129-140: fp32 table [max_seq, D] in the rotate-half layout cat(f, f)."""
    D = cfg.head_dim
    exps = (np.arange(0, D, 2, dtype=np.int64).astype(F32) / F32(D)).astype(F32)
    # ``theta ** t`` with a python-float base is evaluated in double and rounded to fp32
    inv_freq = (F32(1.0) / np.power(np.float64(cfg.rope_theta), exps.astype(np.float64)).astype(F32)).astype(F32)
    sc = cfg.rope_scaling or {}
    if sc.get("rope_type", sc.get("type")) == "llama3":
        inv_freq = _llama3_inv_freq(inv_freq, sc)
    t = np.arange(max_seq, dtype=F32)
    freqs = np.outer(t, inv_freq).astype(F32)
    emb = np.concatenate([freqs, freqs], axis=-1)
    return np.cos(emb).astype(F32), np.sin(emb).astype(F32)


class OracleModel:
    """Layer-range forward over packed ragged blocks, with a static per-row KV cache.

    Cache layout follows ``KVCache`` (common/model.py:171-183): per layer
    ``[max_batch, n_kv_heads, max_seq, head_dim]``."""

    def __init__(self, cfg: OracleConfig, weights: dict, bf16: bool, max_batch: int, max_seq: int):
        self.cfg, self.bf16 = cfg, bf16
        rnd = to_bf16 if bf16 else (lambda a: np.asarray(a, dtype=F32))
        self.r = rnd
        self.w = {k: rnd(v) for k, v in weights.items()}
        self.G = cfg.n_heads // cfg.n_kv_heads
        self.q_size = cfg.n_heads * cfg.head_dim
        self.kv_size = cfg.n_kv_heads * cfg.head_dim
        self.allocate(max_batch, max_seq)

    def allocate(self, max_batch: int, max_seq: int) -> None:
        c = self.cfg
        max_seq = (max_seq + 63) // 64 * 64                        # common/model.py:286
        shape = (c.n_layers, max_batch, c.n_kv_heads, max_seq, c.head_dim)
        self.kc = np.zeros(shape, dtype=F32)
        self.vc = np.zeros(shape, dtype=F32)
        cos, sin = rope_tables(c, max_seq)
        # cast to the model dtype before use (solutions/packed.py:106-107)
        self.cos, self.sin = self.r(cos), self.r(sin)
        self.max_seq = max_seq

    # ------------------------------------------------------------------ primitives
    def mm(self, a: np.ndarray, w: np.ndarray) -> np.ndarray:
        """F.linear: a @ w.T, fp32 accumulation, output rounded to the model dtype."""
        return self.r(np.asarray(a, dtype=F32) @ w.T)

    def rms_norm(self, x: np.ndarray, w: np.ndarray) -> np.ndarray:
        """common/model.py:153-156: fp32 normalise, cast to dtype, multiply by weight in dtype."""
        xf = np.asarray(x, dtype=F32)
        r = (F32(1.0) / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True, dtype=F32) + F32(self.cfg.norm_eps))).astype(F32)
        return self.r(w * self.r(xf * r))

    def rope(self, x: np.ndarray, pos: np.ndarray) -> np.ndarray:
        """common/model.py:143-150: x*cos + rotate_half(x)*sin, every product rounded to dtype.
        x [n, h, D]; cos/sin gathered by token position."""
        c = self.cos[pos][:, None, :]
        s = self.sin[pos][:, None, :]
        h = x.shape[-1] // 2
        rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
        return self.r(self.r(x * c) + self.r(rot * s))

    def embed(self, ids) -> np.ndarray:
        return self.w["embed"][np.asarray(ids, dtype=np.int64)].copy()

    def head(self, h: np.ndarray) -> np.ndarray:
        """common/model.py:328-330: final RMSNorm + LM head (shared by every exit)."""
        lm = self.w["embed"] if self.cfg.tie_word_embeddings else self.w["lm_head"]
        return self.mm(self.rms_norm(h, self.w["norm"]), lm)

    # ------------------------------------------------------------------ packed forward
    def _attend(self, i: int, q: np.ndarray, blocks, offsets) -> np.ndarray:
        """solutions/packed.py:142-166 without buckets: per block and KV head, the G query heads of
        every token read cache positions <= their own position (softmax in fp32)."""
        c = self.cfg
        D, G = c.head_dim, self.G
        out = np.zeros((q.shape[0], self.q_size), dtype=F32)
        scale = F32(1.0 / math.sqrt(D))
        for bi, (row, pos0, T) in enumerate(blocks):
            s0 = offsets[bi]
            L = pos0 + T
            qpos = np.arange(pos0, pos0 + T)
            keys = np.arange(L)
            masked = keys[None, :] > qpos[:, None]                          # [T, L]
            for h in range(c.n_kv_heads):
                K = self.kc[i, row, h, :L]
                V = self.vc[i, row, h, :L]
                for g in range(G):
                    hq = h * G + g
                    qq = q[s0:s0 + T, hq, :]                                 # [T, D]
                    sc = (qq @ K.T).astype(F32) * scale
                    sc = np.where(masked, -np.inf, sc)
                    m = sc.max(axis=-1, keepdims=True)
                    p = np.exp(sc - m).astype(F32)
                    p = p / p.sum(axis=-1, keepdims=True)
                    out[s0:s0 + T, hq * D:(hq + 1) * D] = p @ V
        return self.r(out)

    def packed_layer(self, i: int, x: np.ndarray, blocks, offsets, pos, rows) -> np.ndarray:
        """solutions/packed.py:169-185 (one decoder layer on packed tokens x [N, dim])."""
        c = self.cfg
        w = self.w
        N = x.shape[0]
        qkv = self.mm(self.rms_norm(x, w[f"l{i}.attn_norm"]), w[f"l{i}.wqkv"])
        q = qkv[:, :self.q_size].reshape(N, c.n_heads, c.head_dim)
        k = qkv[:, self.q_size:self.q_size + self.kv_size].reshape(N, c.n_kv_heads, c.head_dim)
        v = qkv[:, self.q_size + self.kv_size:].reshape(N, c.n_kv_heads, c.head_dim)
        q = self.rope(q, pos)
        k = self.rope(k, pos)
        self.kc[i, rows, :, pos] = k                                    # solutions/packed.py:180-181
        self.vc[i, rows, :, pos] = v
        x = self.r(x + self.mm(self._attend(i, q, blocks, offsets), w[f"l{i}.wo"]))
        gu = self.mm(self.rms_norm(x, w[f"l{i}.ffn_norm"]), w[f"l{i}.w13"])
        I = c.intermediate_size
        g, u = gu[:, :I], gu[:, I:]
        a = self.r(self.r(g / (F32(1.0) + np.exp(-g))) * u)             # F.silu(g) * u in dtype
        return self.r(x + self.mm(a, w[f"l{i}.w2"]))

    def packed_layers(self, x: np.ndarray, blocks, start: int, end: int, capture=()) -> tuple[np.ndarray, dict]:
        """solutions/packed.py:188-196.  ``blocks`` is a list of (row, pos0, T) in packed order;
        capture[k] = hidden state entering exit layer k for every k in ``capture``."""
        T = np.array([b[2] for b in blocks], dtype=np.int64)
        offsets = np.concatenate([[0], np.cumsum(T)]).astype(np.int64)
        pos = np.concatenate([np.arange(p0, p0 + t) for (_, p0, t) in blocks]).astype(np.int64)
        rows = np.concatenate([np.full(t, r) for (r, _, t) in blocks]).astype(np.int64)
        x = self.r(x)
        cap = {}
        for i in range(start, end):
            x = self.packed_layer(i, x, blocks, offsets, pos, rows)
            if (i + 1) in capture:
                cap[i + 1] = x.copy()
        return x, cap

    def prefill(self, tokens, slot: int, chunk: int = 512) -> np.ndarray:
        """Chunked causal prefill of one request into cache row ``slot`` through the packed
        rule (solutions/engine.py:217-234); returns the last position's logits."""
        h = None
        for s in range(0, len(tokens), chunk):
            c = min(chunk, len(tokens) - s)
            h, _ = self.packed_layers(self.embed(tokens[s:s + c]), [(slot, s, c)], 0, self.cfg.n_layers)
        return self.head(h[-1:])[0]


def argmax_first(logits: np.ndarray) -> np.ndarray:
    """torch.argmax semantics: the lowest index among equal maxima."""
    return np.argmax(logits, axis=-1)
