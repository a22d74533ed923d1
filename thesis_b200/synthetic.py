"""Seeded synthetic LayerSkip-Llama weights and ragged prompts.

The reference measures on real checkpoints and HF datasets (``common/data.py``), which
are not available here.  Seeded synthetic inputs with the benchmark's shapes stand in:

* weights: Normal(0, 0.02) for every matrix (HF ``initializer_range``), 1.0 for the norm
  weights unless ``norm_jitter`` asks for a perturbation (tests use it so the norm
  multiply is exercised);
* acceptance control: the residual-output projections (``wo`` and ``w2``) of layers
  ``>= residual_scale_from`` are multiplied by ``residual_scale``;
* prompts: token ids uniform in [0, vocab); lengths uniform or lognormal, clipped.

Layouts follow ``common/model.py:161-168`` / ``:259-276``: ``wqkv = [q; k; v]`` rows,
``w13 = [gate; up]`` rows, every matrix ``[out_features, in_features]``.

Two generators exist: ``synthetic_weights`` (numpy, bit-reproducible on any host, used
for everything the CPU oracle checks) and ``synthetic_weights_torch`` (a seeded torch
generator on the target device, for full-size benchmark models where a host-side
8B-parameter draw would dominate start-up).
"""

from __future__ import annotations

import zlib
from dataclasses import dataclass
from typing import Optional

import numpy as np

TENSORS = ("wqkv", "wo", "w13", "w2", "attn_norm", "ffn_norm")


@dataclass
class Prompt:
    """Same fields as the reference's ``common.data.Prompt`` (common/data.py:66-69)."""
    pid: str
    tokens: list
    reference: str = ""
    max_new: Optional[int] = None   # per-request output length (open-loop serving workloads)


def layer_shapes(cfg) -> dict:
    q = cfg.n_heads * cfg.head_dim
    kv = cfg.n_kv_heads * cfg.head_dim
    return {
        "wqkv": (q + 2 * kv, cfg.dim),
        "wo": (cfg.dim, q),
        "w13": (2 * cfg.intermediate_size, cfg.dim),
        "w2": (cfg.dim, cfg.intermediate_size),
        "attn_norm": (cfg.dim,),
        "ffn_norm": (cfg.dim,),
    }


def _rng(seed: int, name: str) -> np.random.Generator:
    return np.random.default_rng([seed, zlib.crc32(name.encode())])


def synthetic_weights(cfg, seed: int = 0, std: float = 0.02, residual_scale_from: Optional[int] = None,
                      residual_scale: float = 1.0, norm_jitter: float = 0.0) -> dict:
    """Float32 numpy weights keyed ``embed``, ``lm_head`` (untied only), ``norm`` and
    ``l{i}.{wqkv,wo,w13,w2,attn_norm,ffn_norm}``.  Each tensor has its own seeded stream,
    so any subset can be regenerated independently."""
    W = {}

    def mat(name, shape):
        return (_rng(seed, name).standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)

    def norm(name, n):
        w = np.ones(n, dtype=np.float32)
        if norm_jitter:
            w += _rng(seed, name).standard_normal(n, dtype=np.float32) * np.float32(norm_jitter)
        return w

    W["embed"] = mat("embed", (cfg.vocab_size, cfg.dim))
    if not cfg.tie_word_embeddings:
        W["lm_head"] = mat("lm_head", (cfg.vocab_size, cfg.dim))
    W["norm"] = norm("norm", cfg.dim)
    for i in range(cfg.n_layers):
        for t, shape in layer_shapes(cfg).items():
            name = f"l{i}.{t}"
            W[name] = norm(name, shape[0]) if len(shape) == 1 else mat(name, shape)
        if residual_scale_from is not None and i >= residual_scale_from:
            W[f"l{i}.wo"] *= np.float32(residual_scale)
            W[f"l{i}.w2"] *= np.float32(residual_scale)
    return W


def synthetic_weights_torch(cfg, seed: int, device, dtype, std: float = 0.02,
                            residual_scale_from: Optional[int] = None, residual_scale: float = 1.0) -> dict:
    """Same keys and distributions as ``synthetic_weights``, drawn on ``device`` with a seeded
    torch generator (not bit-identical to the numpy draw)."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    W = {}

    def mat(shape):
        t = torch.empty(shape, device=device, dtype=torch.float32)
        t.normal_(0.0, std, generator=g)
        return t.to(dtype)

    W["embed"] = mat((cfg.vocab_size, cfg.dim))
    if not cfg.tie_word_embeddings:
        W["lm_head"] = mat((cfg.vocab_size, cfg.dim))
    W["norm"] = torch.ones(cfg.dim, device=device, dtype=dtype)
    for i in range(cfg.n_layers):
        for t, shape in layer_shapes(cfg).items():
            W[f"l{i}.{t}"] = torch.ones(shape, device=device, dtype=dtype) if len(shape) == 1 else mat(shape)
        if residual_scale_from is not None and i >= residual_scale_from:
            W[f"l{i}.wo"].mul_(residual_scale)
            W[f"l{i}.w2"].mul_(residual_scale)
    return W


def synthetic_prompts(n: int, vocab: int, seed: int = 0, min_len: int = 32, max_len: int = 128,
                      lengths: str = "uniform", median: Optional[float] = None, sigma: float = 0.6,
                      pid_prefix: str = "p") -> list:
    """Ragged prompts: ids uniform in [0, vocab); lengths uniform in [min_len, max_len] or
    lognormal around ``median`` clipped to [min_len, max_len]."""
    rng = np.random.default_rng(seed)
    if lengths == "uniform":
        lens = rng.integers(min_len, max_len + 1, size=n)
    elif lengths == "lognormal":
        med = median if median is not None else (min_len + max_len) / 2
        lens = np.clip(np.round(rng.lognormal(np.log(med), sigma, size=n)), min_len, max_len).astype(np.int64)
    else:
        raise ValueError(lengths)
    return [Prompt(f"{pid_prefix}{i}", rng.integers(0, vocab, size=int(L)).tolist()) for i, L in enumerate(lens)]
