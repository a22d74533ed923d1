"""Generate the golden vectors that pin the CPU oracle to the reference.

Runs the UNMODIFIED reference (hsungo/thesis, pure PyTorch on CPU) on seeded synthetic
weights and prompts and stores its outputs as small ``.npz`` fixtures next to this
script.  The reference cannot travel to the GPU host, so the fixtures are committed;
rerun this script (in a checkout that has the reference) to regenerate them:

    python tests/golden/make_golden.py --reference /path/to/thesis      # or THESIS_REFERENCE=...

What is recorded per case (model preset x dtype):
* ``prefill_logits``   ``LayerSkipLlama.prefill`` last-position logits of every prompt
                       (common/model.py:392-403);
* ``packed_*``         one ragged ``build_packed`` + ``packed_layers`` call over decode (T=1)
                       and verify (T=gamma+1) blocks on top of the prefilled rows, with the
                       exit-layer and final logits (solutions/packed.py:81-196);
* ``ar_tokens``        greedy ``ARBatchEngine`` outputs (common/engine.py:302-331);
* ``spec_tokens``      ``SyncSpecEngine`` outputs (common/engine.py:336-421);
* ``eesd_tokens``      ``EESDEngine`` (fixed scheduler) outputs (solutions/engine.py);
* ``rope_cos/sin``     the reference's RoPE table (common/model.py:129-140).

Full-size cases (``FULL_CASES``) run the benchmark shapes: BASELINE configuration 1 verbatim
(Llama3.2-1B shape, fp32, batch 4, prompts 32..128, exit 4, draft length 4, 64 new tokens) and a
4-layer Llama3-8B-shaped bf16 model with prompts of 137..1027 tokens (several 64-key tiles, split-K
projections, the CTA-pair W13, the two-tile LM head, multi-chunk prefill on the B200 side), and the
same for the Llama3.2-1B shape (head_dim 64 attention, its split-K shapes, the tied head) and the
Llama2-7B shape (MHA, SwiGLU 11008, vocabulary 32000), and the 4-layer Llama3-8B case in fp32
(token identity at long contexts).  Their
weights are regenerated from the seed by ``thesis_b200.synthetic``; their logits rows (vocabulary
128256) are stored sparsely: every 16th column plus each row's 64 largest entries
(``<key>_stride``, ``<key>_top_idx``, ``<key>_top_val``).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from dataclasses import asdict
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from thesis_b200.config import preset  # noqa: E402
from thesis_b200.synthetic import synthetic_prompts, synthetic_weights  # noqa: E402

CASES = [
    # name, preset, dtype, exit layer, gamma, weight kwargs
    ("tiny_fp32", "tiny", "fp32", 2, 3, dict(norm_jitter=0.1)),
    ("tiny_bf16", "tiny", "bf16", 2, 3, dict(norm_jitter=0.1)),
    ("c1s_fp32", "c1s", "fp32", 4, 4, dict(residual_scale_from=4, residual_scale=0.05)),
    ("c1s_bf16", "c1s", "bf16", 4, 4, dict(residual_scale_from=4, residual_scale=0.05)),
    ("d128_fp32", "d128", "fp32", 2, 3, dict(norm_jitter=0.1)),
    ("mha_bf16", "mha", "bf16", 2, 2, dict(norm_jitter=0.1)),
]
N_PROMPTS = 4
MAX_NEW = 16
SEED = 0

FULL_CASES = [
    # BASELINE configuration 1 verbatim
    dict(name="c1_fp32", preset="llama3-1b", overrides={}, dtype="fp32", exit_layer=4, gamma=4,
         weights=dict(residual_scale_from=4, residual_scale=0.05), min_len=32, max_len=128, max_new=64,
         max_seq=256),
    # Llama3-8B shape cut to 4 layers; contexts up to ~1030 tokens
    dict(name="c3s_bf16", preset="llama3-8b", overrides=dict(n_layers=4), dtype="bf16", exit_layer=2, gamma=4,
         weights=dict(residual_scale_from=2, residual_scale=0.1), lens=(137, 449, 700, 1027), max_new=12,
         max_seq=1088),
    # Llama3.2-1B shape (BASELINE configuration 2's model: head_dim 64, tied head) cut to 4 layers,
    # bf16, draft length 6; contexts up to ~1030 tokens
    dict(name="c2s_bf16", preset="llama3-1b", overrides=dict(n_layers=4), dtype="bf16", exit_layer=2, gamma=6,
         weights=dict(residual_scale_from=2, residual_scale=0.1), lens=(64, 333, 702, 1024), max_new=12,
         max_seq=1088),
    # Llama3-8B shape cut to 4 layers in fp32: token identity at long contexts and head_dim 128
    dict(name="c3s_fp32", preset="llama3-8b", overrides=dict(n_layers=4), dtype="fp32", exit_layer=2, gamma=4,
         weights=dict(residual_scale_from=2, residual_scale=0.1), lens=(137, 449, 700, 1027), max_new=12,
         max_seq=1088),
    # Llama2-7B shape (BASELINE configuration 4's model: MHA, SwiGLU 11008, vocab 32000, RoPE theta
    # 10000) cut to 4 layers, bf16; contexts up to ~1030 tokens
    dict(name="c4s_bf16", preset="llama2-7b", overrides=dict(n_layers=4), dtype="bf16", exit_layer=2, gamma=4,
         weights=dict(residual_scale_from=2, residual_scale=0.1), lens=(40, 256, 640, 1020), max_new=12,
         max_seq=1088),
]
STRIDE, TOP = 16, 64


def sparse_logits(key: str, lg: np.ndarray) -> dict:
    """Every STRIDE-th column and the TOP largest entries (with their columns) of each row."""
    lg = np.asarray(lg, dtype=np.float32)
    top = np.argsort(-lg, axis=1, kind="stable")[:, :TOP]
    return {f"{key}_stride": lg[:, ::STRIDE].copy(), f"{key}_top_idx": top.astype(np.int64),
            f"{key}_top_val": np.take_along_axis(lg, top, axis=1)}


def build_reference_model(cfg, W, dtype, max_seq):
    import torch
    from common.model import LayerSkipLlama, LayerWeights, ModelConfig

    rc = ModelConfig(vocab_size=cfg.vocab_size, dim=cfg.dim, n_layers=cfg.n_layers, n_heads=cfg.n_heads,
                     n_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, intermediate_size=cfg.intermediate_size,
                     norm_eps=cfg.norm_eps, rope_theta=cfg.rope_theta, max_position_embeddings=max_seq,
                     tie_word_embeddings=cfg.tie_word_embeddings, rope_scaling=cfg.rope_scaling)

    def t(a):
        return torch.from_numpy(np.asarray(a)).to(dtype)

    layers = [LayerWeights(wqkv=t(W[f"l{i}.wqkv"]), wo=t(W[f"l{i}.wo"]), w13=t(W[f"l{i}.w13"]), w2=t(W[f"l{i}.w2"]),
                           attn_norm=t(W[f"l{i}.attn_norm"]), ffn_norm=t(W[f"l{i}.ffn_norm"]))
              for i in range(cfg.n_layers)]
    embed = t(W["embed"])
    lm = embed if cfg.tie_word_embeddings else t(W["lm_head"])
    return LayerSkipLlama(rc, embed, layers, t(W["norm"]), lm, "cpu", dtype, max_seq)


def tokens_by_pid(res, prompts):
    out = {}
    for c in res["completions"]:
        out.setdefault(c["pid"], c["tokens"])
    return np.array([out[p.pid] for p in prompts], dtype=np.int64)


def make_case(name, pname, dt, E, gamma, wkw):
    import torch
    from common.data import Prompt as RefPrompt
    from common.engine import ARBatchEngine, RunConfig, SyncSpecEngine
    from solutions.cost_model import synthetic_cost_model
    from solutions.engine import EESDEngine, EngineConfig
    from solutions.packed import Block, build_packed, packed_layers

    torch.manual_seed(0)
    dtype = {"fp32": torch.float32, "bf16": torch.bfloat16}[dt]
    cfg = preset(pname)
    W = synthetic_weights(cfg, seed=SEED, **wkw)
    prompts = synthetic_prompts(N_PROMPTS, cfg.vocab_size, seed=SEED + 1, min_len=5, max_len=40)
    max_seq = 256
    m = build_reference_model(cfg, W, dtype, max_seq)
    out = {}
    with torch.inference_mode():
        # --- prefill logits, one row per prompt
        m.allocate_cache(N_PROMPTS, max_seq)
        pre = []
        for i, p in enumerate(prompts):
            logits, _ = m.prefill(p.tokens, slot=i)
            pre.append(logits.float().numpy())
        out["prefill_logits"] = np.stack(pre)
        # --- one ragged packed call on top of the prefilled rows: decode and verify blocks
        lens = [len(p.tokens) for p in prompts]
        blocks = [Block(0, lens[0], 1), Block(1, lens[1], gamma + 1), Block(2, lens[2], 1),
                  Block(3, lens[3], gamma + 1)]
        pb = build_packed(m, blocks, "exact")
        order = np.array([[b.row, b.pos0, b.T] for b in pb.blocks], dtype=np.int64)
        rng = np.random.default_rng(SEED + 2)
        ids = rng.integers(0, cfg.vocab_size, size=pb.n_tokens)
        x = m.embed(torch.from_numpy(ids))
        cap = {}
        h = packed_layers(m, x, pb, 0, cfg.n_layers, cap, (E,))
        out["packed_blocks"] = order
        out["packed_ids"] = ids
        out["packed_exit_logits"] = m.head(cap[E]).float().numpy()
        out["packed_final_logits"] = m.head(h).float().numpy()
        out["rope_cos"] = m.rope_cos[:max_seq].numpy()
        out["rope_sin"] = m.rope_sin[:max_seq].numpy()
    # --- greedy engines (static mode, every prompt once)
    rp = [RefPrompt(p.pid, list(p.tokens)) for p in prompts]
    rc = RunConfig(mode="static", keep_outputs=True)
    ar = ARBatchEngine(m, 2, max(lens), MAX_NEW, (), ignore_eos=True)
    out["ar_tokens"] = tokens_by_pid(ar.run(rp, rc), prompts)
    sp = SyncSpecEngine(m, 3, max(lens), MAX_NEW, (), ignore_eos=True, exit_layer=E, gamma=gamma)
    out["spec_tokens"] = tokens_by_pid(sp.run(rp, rc), prompts)
    ee = EESDEngine(m, 3, max(lens), MAX_NEW, (), EngineConfig(mode="spec", sched="fixed", gamma=gamma, k=E, d_max=8),
                    synthetic_cost_model(m.cfg))
    res = ee.run(rp, "static", keep_outputs=True)
    out["eesd_tokens"] = tokens_by_pid(res, prompts)
    plen = np.array(lens, dtype=np.int64)
    ptok = np.zeros((N_PROMPTS, max(lens)), dtype=np.int64)
    for i, p in enumerate(prompts):
        ptok[i, :lens[i]] = p.tokens
    out["prompt_lens"], out["prompt_tokens"] = plen, ptok
    meta = dict(name=name, preset=pname, dtype=dt, exit_layer=E, gamma=gamma, weights=wkw, seed=SEED,
                max_new=MAX_NEW, max_seq=max_seq, config=asdict(cfg))
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / f"{name}.npz", **out)
    agree = (out["ar_tokens"] == out["spec_tokens"]).all(), (out["ar_tokens"] == out["eesd_tokens"]).all()
    print(f"{name}: wrote {HERE / (name + '.npz')}  spec==ar {agree[0]}  eesd==ar {agree[1]}")


def make_full_case(c: dict):
    """A benchmark-shaped case: prefill and packed logits (sparse), and the tokens of the
    reference's three greedy engines (batch = number of prompts)."""
    import torch
    from common.data import Prompt as RefPrompt
    from common.engine import ARBatchEngine, RunConfig, SyncSpecEngine
    from solutions.cost_model import synthetic_cost_model
    from solutions.engine import EESDEngine, EngineConfig
    from solutions.packed import Block, build_packed, packed_layers

    torch.manual_seed(0)
    dtype = {"fp32": torch.float32, "bf16": torch.bfloat16}[c["dtype"]]
    cfg = preset(c["preset"], **c["overrides"])
    E, gamma, max_seq, max_new = c["exit_layer"], c["gamma"], c["max_seq"], c["max_new"]
    W = synthetic_weights(cfg, seed=SEED, **c["weights"])
    if "lens" in c:
        rng = np.random.default_rng(SEED + 1)
        from thesis_b200.synthetic import Prompt
        prompts = [Prompt(f"p{i}", rng.integers(0, cfg.vocab_size, size=n).tolist()) for i, n in enumerate(c["lens"])]
    else:
        prompts = synthetic_prompts(N_PROMPTS, cfg.vocab_size, seed=SEED + 1, min_len=c["min_len"],
                                    max_len=c["max_len"])
    m = build_reference_model(cfg, W, dtype, max_seq)
    del W
    out = {}
    lens = [len(p.tokens) for p in prompts]
    with torch.inference_mode():
        m.allocate_cache(len(prompts), max_seq)
        pre = []
        for i, p in enumerate(prompts):
            logits, _ = m.prefill(p.tokens, slot=i)
            pre.append(logits.float().numpy())
        out.update(sparse_logits("prefill_logits", np.stack(pre)))
        blocks = [Block(i, lens[i], 1 if i % 2 == 0 else gamma + 1) for i in range(len(prompts))]
        pb = build_packed(m, blocks, "exact")
        order = np.array([[b.row, b.pos0, b.T] for b in pb.blocks], dtype=np.int64)
        rng = np.random.default_rng(SEED + 2)
        ids = rng.integers(0, cfg.vocab_size, size=pb.n_tokens)
        x = m.embed(torch.from_numpy(ids))
        cap = {}
        h = packed_layers(m, x, pb, 0, cfg.n_layers, cap, (E,))
        out["packed_blocks"] = order
        out["packed_ids"] = ids
        out.update(sparse_logits("packed_exit_logits", m.head(cap[E]).float().numpy()))
        out.update(sparse_logits("packed_final_logits", m.head(h).float().numpy()))
    rp = [RefPrompt(p.pid, list(p.tokens)) for p in prompts]
    rc = RunConfig(mode="static", keep_outputs=True)
    B = len(prompts)
    out["ar_tokens"] = tokens_by_pid(ARBatchEngine(m, B, max(lens), max_new, (), ignore_eos=True).run(rp, rc), prompts)
    sp = SyncSpecEngine(m, B, max(lens), max_new, (), ignore_eos=True, exit_layer=E, gamma=gamma)
    out["spec_tokens"] = tokens_by_pid(sp.run(rp, rc), prompts)
    ee = EESDEngine(m, B, max(lens), max_new, (), EngineConfig(mode="spec", sched="fixed", gamma=gamma, k=E, d_max=8),
                    synthetic_cost_model(m.cfg))
    out["eesd_tokens"] = tokens_by_pid(ee.run(rp, "static", keep_outputs=True), prompts)
    ptok = np.zeros((B, max(lens)), dtype=np.int64)
    for i, p in enumerate(prompts):
        ptok[i, :lens[i]] = p.tokens
    out["prompt_lens"], out["prompt_tokens"] = np.array(lens, dtype=np.int64), ptok
    meta = dict(name=c["name"], preset=c["preset"], dtype=c["dtype"], exit_layer=E, gamma=gamma, weights=c["weights"],
                seed=SEED, max_new=max_new, max_seq=max_seq, config=asdict(cfg), sparse=dict(stride=STRIDE, top=TOP))
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / f"{c['name']}.npz", **out)
    agree = (out["ar_tokens"] == out["spec_tokens"]).all(), (out["ar_tokens"] == out["eesd_tokens"]).all()
    print(f"{c['name']}: wrote {HERE / (c['name'] + '.npz')}  spec==ar {agree[0]}  eesd==ar {agree[1]}")


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("THESIS_REFERENCE"),
                    help="checkout of the reference repository (default: $THESIS_REFERENCE)")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference or set THESIS_REFERENCE to a checkout of the reference")
    sys.path.insert(0, str(Path(args.reference).resolve()))
    for name, pname, dt, E, g, wkw in CASES:
        if args.only and name != args.only:
            continue
        make_case(name, pname, dt, E, g, wkw)
    for c in FULL_CASES:
        if args.only and c["name"] != args.only:
            continue
        make_full_case(c)


if __name__ == "__main__":
    main()
