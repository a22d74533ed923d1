"""The numpy oracle against the reference's own outputs (golden fixtures), on CPU."""

import numpy as np
import pytest

from goldens import CASES, TOL, Golden, rel_err
from oracle.engine_np import ar_generate, spec_generate
from oracle.model_np import OracleConfig, OracleModel, argmax_first, rope_tables, to_bf16


def _oracle(g: Golden, max_batch: int = 4) -> OracleModel:
    c = g.config()
    oc = OracleConfig(vocab_size=c.vocab_size, dim=c.dim, n_layers=c.n_layers, n_heads=c.n_heads,
                      n_kv_heads=c.n_kv_heads, head_dim=c.head_dim, intermediate_size=c.intermediate_size,
                      norm_eps=c.norm_eps, rope_theta=c.rope_theta, tie_word_embeddings=c.tie_word_embeddings,
                      rope_scaling=c.rope_scaling)
    return OracleModel(oc, g.weights(), g.dtype == "bf16", max_batch, g.meta["max_seq"])


def test_bf16_rounding_is_round_to_nearest_even():
    import torch

    x = np.random.default_rng(0).standard_normal(100000).astype(np.float32) * 10
    x[:4] = [1.00390625, 1.01171875, -3.0e-39, 65504.0]      # ties (both parities), a denormal
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(to_bf16(x), ref)


@pytest.mark.parametrize("name", CASES)
def test_rope_table_matches_reference(name):
    g = Golden(name)
    c = g.config()
    oc = OracleConfig(c.vocab_size, c.dim, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.intermediate_size,
                      c.norm_eps, c.rope_theta, c.tie_word_embeddings, c.rope_scaling)
    cos, sin = rope_tables(oc, g.meta["max_seq"])
    assert np.abs(cos - g["rope_cos"]).max() < 2e-6
    assert np.abs(sin - g["rope_sin"]).max() < 2e-6


@pytest.mark.parametrize("name", CASES)
def test_prefill_and_packed_logits_match_reference(name):
    g = Golden(name)
    m = _oracle(g)
    tol = TOL[g.dtype]
    for i, p in enumerate(g.prompts()):
        got = m.prefill(p, slot=i)
        assert rel_err(got, g["prefill_logits"][i]) < tol, (i, rel_err(got, g["prefill_logits"][i]))
    blocks = [tuple(map(int, b)) for b in g["packed_blocks"]]
    E = g.meta["exit_layer"]
    h, cap = m.packed_layers(m.embed(g["packed_ids"]), blocks, 0, m.cfg.n_layers, capture=(E,))
    assert rel_err(m.head(cap[E]), g["packed_exit_logits"]) < tol
    assert rel_err(m.head(h), g["packed_final_logits"]) < tol


@pytest.mark.parametrize("name", [c for c in CASES if c.endswith("fp32")])
def test_greedy_tokens_match_reference_fp32(name):
    """fp32: identical token sequences (AR and speculative) to the reference's engines."""
    g = Golden(name)
    prompts = g.prompts()
    ar = ar_generate(_oracle(g), prompts, g.meta["max_new"])
    assert np.array_equal(np.array(ar), g["ar_tokens"])
    sp, st = spec_generate(_oracle(g), prompts, g.meta["max_new"], g.meta["exit_layer"], g.meta["gamma"])
    assert np.array_equal(np.array(sp), g["spec_tokens"])
    if "residual_scale_from" in g.meta["weights"]:      # acceptance is controllable only when scaled
        assert st["accepted"] > 0


def test_argmax_ties_take_the_lowest_index():
    assert int(argmax_first(np.array([1.0, 3.0, 3.0, 2.0]))) == 1


def test_oracle_at_benchmark_config1_matches_reference():
    """BASELINE configuration 1 at full size (Llama3.2-1B shape, fp32): the oracle's prefill, exit
    and final logits match the reference's within 1e-4 (stored columns of the 128256-entry rows)."""
    from goldens import sparse_rel_err

    g = Golden("c1_fp32")
    m = _oracle(g)
    rows = [m.prefill(p, slot=i) for i, p in enumerate(g.prompts())]
    assert sparse_rel_err(g, "prefill_logits", np.stack(rows)) < TOL["fp32"]
    blocks = [tuple(map(int, b)) for b in g["packed_blocks"]]
    E = g.meta["exit_layer"]
    h, cap = m.packed_layers(m.embed(g["packed_ids"]), blocks, 0, m.cfg.n_layers, capture=(E,))
    assert sparse_rel_err(g, "packed_exit_logits", m.head(cap[E])) < TOL["fp32"]
    assert sparse_rel_err(g, "packed_final_logits", m.head(h)) < TOL["fp32"]
