"""Model configuration (mirror of ``ModelConfig``, common/model.py:39-108) and named presets.

The presets are the synthetic LayerSkip-Llama shapes the benchmark configurations name
(Llama3.2-1B, Llama3-8B, Llama2-7B) plus small shapes used by the parity tests.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field, replace
from pathlib import Path
from typing import Optional


@dataclass
class ModelConfig:
    vocab_size: int
    dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    intermediate_size: int
    norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    max_position_embeddings: int = 4096
    tie_word_embeddings: bool = False
    rope_scaling: Optional[dict] = None
    bos_token_id: Optional[int] = None
    eos_token_ids: tuple = field(default_factory=tuple)

    @classmethod
    def from_hf_dir(cls, path) -> "ModelConfig":
        """HF ``config.json`` (+ ``generation_config.json`` EOS ids), old and new RoPE formats
        (common/model.py:56-91)."""
        path = Path(path)
        cfg = json.loads((path / "config.json").read_text())
        eos = cfg.get("eos_token_id")
        eos_ids = list(eos) if isinstance(eos, list) else ([eos] if eos is not None else [])
        gen = path / "generation_config.json"
        if gen.exists():
            g = json.loads(gen.read_text()).get("eos_token_id")
            eos_ids += g if isinstance(g, list) else ([g] if g is not None else [])
        rp = cfg.get("rope_parameters") or {}
        scaling = cfg.get("rope_scaling")
        if scaling is None and rp.get("rope_type", "default") != "default":
            scaling = rp
        n_heads = cfg["num_attention_heads"]
        return cls(
            vocab_size=cfg["vocab_size"], dim=cfg["hidden_size"], n_layers=cfg["num_hidden_layers"],
            n_heads=n_heads, n_kv_heads=cfg.get("num_key_value_heads", n_heads),
            head_dim=cfg.get("head_dim") or cfg["hidden_size"] // n_heads,
            intermediate_size=cfg["intermediate_size"], norm_eps=cfg.get("rms_norm_eps", 1e-5),
            rope_theta=cfg.get("rope_theta", rp.get("rope_theta", 10000.0)),
            max_position_embeddings=cfg.get("max_position_embeddings", 4096),
            tie_word_embeddings=cfg.get("tie_word_embeddings", False), rope_scaling=scaling,
            bos_token_id=cfg.get("bos_token_id"), eos_token_ids=tuple(dict.fromkeys(eos_ids)),
        )

    @property
    def group(self) -> int:
        return self.n_heads // self.n_kv_heads

    @property
    def layer_param_count(self) -> int:
        """common/model.py:98-102."""
        attn = self.dim * (self.n_heads + 2 * self.n_kv_heads) * self.head_dim + self.n_heads * self.head_dim * self.dim
        return attn + 3 * self.dim * self.intermediate_size + 2 * self.dim

    def kv_bytes_per_position_layer(self, elem_bytes: int) -> int:
        return 2 * self.n_kv_heads * self.head_dim * elem_bytes

    def head_params(self) -> int:
        return self.vocab_size * self.dim


PRESETS = {
    # Llama3.2-1B-shaped (BASELINE configs 1 and 2)
    "llama3-1b": ModelConfig(vocab_size=128256, dim=2048, n_layers=16, n_heads=32, n_kv_heads=8, head_dim=64,
                             intermediate_size=8192, rope_theta=500000.0, tie_word_embeddings=True),
    # Llama3-8B-shaped (configs 3 and 5)
    "llama3-8b": ModelConfig(vocab_size=128256, dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128,
                             intermediate_size=14336, rope_theta=500000.0),
    # Llama2-7B-shaped, MHA (config 4)
    "llama2-7b": ModelConfig(vocab_size=32000, dim=4096, n_layers=32, n_heads=32, n_kv_heads=32, head_dim=128,
                             intermediate_size=11008, rope_theta=10000.0),
    # small shapes for oracle parity (GQA groups 2 and 4, MHA, head_dim 64 and 128, tied head, llama3 RoPE)
    "tiny": ModelConfig(vocab_size=512, dim=256, n_layers=6, n_heads=4, n_kv_heads=2, head_dim=64,
                        intermediate_size=512, rope_theta=10000.0),
    "c1s": ModelConfig(vocab_size=2048, dim=512, n_layers=8, n_heads=8, n_kv_heads=2, head_dim=64,
                       intermediate_size=1024, rope_theta=500000.0, tie_word_embeddings=True),
    "d128": ModelConfig(vocab_size=1024, dim=512, n_layers=4, n_heads=4, n_kv_heads=1, head_dim=128,
                        intermediate_size=768, rope_theta=500000.0,
                        rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                      "high_freq_factor": 4.0, "original_max_position_embeddings": 64}),
    "mha": ModelConfig(vocab_size=512, dim=256, n_layers=4, n_heads=4, n_kv_heads=4, head_dim=64,
                       intermediate_size=384, rope_theta=10000.0),
}


def preset(name: str, **overrides) -> ModelConfig:
    return replace(PRESETS[name], **overrides)
