"""Loading helpers for the committed golden fixtures (``tests/golden/*.npz``)."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = ["tiny_fp32", "tiny_bf16", "c1s_fp32", "c1s_bf16", "d128_fp32", "mha_bf16"]
# benchmark-shaped cases with sparsely stored logits (every 16th column + each row's top 64)
FULL_CASES = ["c1_fp32", "c3s_bf16", "c3s_fp32", "c2s_bf16", "c4s_bf16"]

# Tolerances from the task statement: logits agree within 1e-4 relative in fp32 and 2e-2 in
# bf16.  "Relative" is max |a - b| / max |b| over the compared tensor.
TOL = {"fp32": 1e-4, "bf16": 2e-2}


class Golden:
    def __init__(self, name: str):
        z = np.load(GOLDEN / f"{name}.npz", allow_pickle=False)
        self.z = {k: z[k] for k in z.files}
        self.meta = json.loads(str(self.z["meta"]))
        self.name = name

    def __getitem__(self, k):
        return self.z[k]

    @property
    def dtype(self) -> str:
        return self.meta["dtype"]

    def config(self):
        from thesis_b200.config import ModelConfig

        return ModelConfig(**{k: (tuple(v) if k == "eos_token_ids" else v) for k, v in self.meta["config"].items()})

    def weights(self):
        from thesis_b200.synthetic import synthetic_weights

        return synthetic_weights(self.config(), seed=self.meta["seed"], **self.meta["weights"])

    def prompts(self) -> list:
        return [list(map(int, self["prompt_tokens"][i, :n])) for i, n in enumerate(self["prompt_lens"])]


def rel_err(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def sparse_rel_err(g: Golden, key: str, logits) -> float:
    """rel_err of full logits rows [n, V] against a sparsely stored golden ``key``: the stored
    columns (every stride-th one and each row's largest entries, which hold the row maximum)."""
    lg = np.asarray(logits, dtype=np.float64)
    stride = g.meta["sparse"]["stride"]
    a1, b1 = lg[:, ::stride], g[f"{key}_stride"].astype(np.float64)
    a2 = np.take_along_axis(lg, g[f"{key}_top_idx"], axis=1)
    b2 = g[f"{key}_top_val"].astype(np.float64)
    num = max(np.abs(a1 - b1).max(), np.abs(a2 - b2).max())
    return float(num / max(np.abs(b1).max(), np.abs(b2).max(), 1e-30))
