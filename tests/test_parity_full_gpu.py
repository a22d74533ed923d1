"""Parity at the benchmark shapes against the reference's own outputs (golden fixtures made by
the unmodified reference, ``tests/golden/make_golden.py``).

* ``c1_fp32``: BASELINE configuration 1 verbatim - Llama3.2-1B shape (16 layers, dim 2048, GQA 4,
  head_dim 64, vocab 128256, tied head), fp32, o_proj / down_proj of layers 4..15 x 0.05, batch 4,
  prompts of 32..128 tokens, exit layer 4, draft length 4, 64 new tokens.  Prefill, exit-layer and
  final logits within 1e-4; AR and speculative token sequences identical to the reference's
  ``ARBatchEngine``, ``SyncSpecEngine`` and ``EESDEngine`` (common/engine.py:302-436,
  solutions/engine.py:269-489), and so are the dynamic-exit engine's (both schedules) and the
  serving engine's with piggybacked prefill.
* ``c3s_bf16``: the Llama3-8B shape (dim 4096, GQA 4, head_dim 128, SwiGLU 14336, vocab 128256,
  untied head) cut to 4 layers, bf16, prompts of 137..1027 tokens (multi-chunk prefill, contexts over
  16 key tiles, split-K projections, CTA-pair W13, two-tile LM head).  Logits within 2e-2; the
  speculative output equals this engine's own AR output (lossless).
* ``c3s_fp32``: the same model in fp32: logits within 1e-4, and AR, speculative, dynamic-exit and
  piggyback tokens identical to the reference's at contexts up to ~1040 tokens and head_dim 128.
* ``c2s_bf16``: the same for the Llama3.2-1B shape (dim 2048, GQA 4, head_dim 64, SwiGLU 8192,
  tied head), 4 layers, bf16, draft length 6, prompts of 64..1024 tokens.
* ``c4s_bf16``: the same for the Llama2-7B shape (MHA: 32 KV heads of 128, SwiGLU 11008,
  vocabulary 32000, RoPE theta 10000), 4 layers, bf16, prompts of 40..1020 tokens.

Relative error = max |a - b| / max |b| over the stored logits columns.
"""

import numpy as np
import pytest
import torch

from goldens import FULL_CASES, TOL, Golden, sparse_rel_err
from thesis_b200.dynamic import B200DynamicSpecEngine
from thesis_b200.eesd import B200ARBatchEngine, B200SpecEngine
from thesis_b200.engine import RunConfig
from thesis_b200.model import DeviceModel, ModelWeights
from thesis_b200.serving import B200ServingEngine
from thesis_b200.synthetic import Prompt

pytestmark = pytest.mark.gpu

CHUNK = 512


@pytest.fixture(scope="module", params=FULL_CASES)
def case(request):
    g = Golden(request.param)
    dtype = torch.bfloat16 if g.dtype == "bf16" else torch.float32
    w = ModelWeights.from_numpy(g.config(), g.weights(), dtype, "cuda")
    yield g, w
    del w
    torch.cuda.empty_cache()


def _call(dm, blocks, ids):
    ph = dm.pack(blocks)
    b, (ids_d,) = dm.upload(ph, (np.asarray(ids, dtype=np.int32),))
    return b, dm.embed(ids_d)


def test_prefill_and_packed_logits_match_reference(cuda_dev, case):
    g, w = case
    dm = DeviceModel(w, max_batch=4, max_seq=g.meta["max_seq"], max_tokens=CHUNK)
    L, E, tol = dm.cfg.n_layers, g.meta["exit_layer"], TOL[g.dtype]
    rows = []
    for i, p in enumerate(g.prompts()):          # chunked prefill (the reference prefills in one pass)
        for s in range(0, len(p), CHUNK):
            c = min(CHUNK, len(p) - s)
            b, x = _call(dm, [(i, s, c)], p[s:s + c])
            dm.forward_layers(x, b, 0, L)
        _, lg = dm.head_argmax(x[-1:].contiguous(), logits=True)
        rows.append(lg[0].float().cpu().numpy())
    assert sparse_rel_err(g, "prefill_logits", np.stack(rows)) < tol
    blocks = [tuple(map(int, b)) for b in g["packed_blocks"]]
    b, x = _call(dm, blocks, g["packed_ids"])
    dm.forward_layers(x, b, 0, E)
    _, lg_exit = dm.head_argmax(x, logits=True)
    dm.forward_layers(x, b, E, L)
    ids, lg_final = dm.head_argmax(x, logits=True)
    dm.check()
    err_exit = sparse_rel_err(g, "packed_exit_logits", lg_exit.float().cpu().numpy())
    err_final = sparse_rel_err(g, "packed_final_logits", lg_final.float().cpu().numpy())
    assert err_exit < tol and err_final < tol, (err_exit, err_final)
    if g.dtype == "fp32":
        assert np.array_equal(ids.cpu().numpy(), g["packed_final_logits_top_idx"][:, 0])


def _tokens(res, prompts):
    out = {}
    for c in res["completions"]:
        out.setdefault(c["pid"], c["tokens"])
    return np.array([out[p.pid] for p in prompts])


def test_engine_tokens_match_reference(cuda_dev, case):
    g, w = case
    prompts = [Prompt(f"p{i}", p) for i, p in enumerate(g.prompts())]
    mp, B, n = max(len(p.tokens) for p in prompts), len(prompts), g.meta["max_new"]
    rc = RunConfig(mode="static", keep_outputs=True)
    ar = _tokens(B200ARBatchEngine(w, B, mp, n, (), ignore_eos=True).run(prompts, rc), prompts)
    sp_eng = B200SpecEngine(w, B, mp, n, (), ignore_eos=True, exit_layer=g.meta["exit_layer"], gamma=g.meta["gamma"])
    sp = _tokens(sp_eng.run(prompts, rc), prompts)
    sp_eng.dm.check()
    assert np.array_equal(sp, ar)                        # lossless
    if g.dtype == "fp32":
        assert np.array_equal(ar, g["ar_tokens"])
        assert np.array_equal(sp, g["spec_tokens"])
        assert np.array_equal(sp, g["eesd_tokens"])


@pytest.mark.parametrize("schedule", ["lockstep", "unified"])
def test_dynamic_engine_matches_reference_ar_tokens_fp32(cuda_dev, case, schedule):
    """Per-request exit layers {E/2, E, 3E/2 ...} and draft lengths 1..6 in fp32 at BASELINE
    configuration 1: the tokens equal the reference's ARBatchEngine tokens."""
    g, w = case
    if g.dtype != "fp32":
        pytest.skip("token identity with the reference is the fp32 contract")
    L, E = w.cfg.n_layers, g.meta["exit_layer"]
    exits = sorted({max(1, E // 2), E, min(L - 1, E + E // 2)})
    prompts = [Prompt(f"p{i}", p) for i, p in enumerate(g.prompts())]
    mp, B, n = max(len(p.tokens) for p in prompts), len(prompts), g.meta["max_new"]
    eng = B200DynamicSpecEngine(w, B, mp, n, (), ignore_eos=True, exit_layers=exits, gamma_range=(1, 6),
                                schedule=schedule)
    got = _tokens(eng.run(prompts, RunConfig(mode="static", keep_outputs=True)), prompts)
    eng.dm.check()
    assert np.array_equal(got, g["ar_tokens"])


@pytest.mark.parametrize("budget", [24, 1000])
def test_piggyback_engine_matches_reference_ar_tokens_fp32(cuda_dev, case, budget):
    """Two slots for four requests, so the later prompts are prefilled in chunks of at most
    `budget` tokens riding on the other requests' draft and verify steps (config 5's serving
    engine), fp32 at BASELINE configuration 1: the tokens equal the reference's ARBatchEngine
    tokens."""
    g, w = case
    if g.dtype != "fp32":
        pytest.skip("token identity with the reference is the fp32 contract")
    prompts = [Prompt(f"p{i}", p) for i, p in enumerate(g.prompts())]
    mp, n = max(len(p.tokens) for p in prompts), g.meta["max_new"]
    eng = B200ServingEngine(w, 2, mp, n, (), ignore_eos=True, exit_layer=g.meta["exit_layer"], gamma=g.meta["gamma"],
                            piggyback_budget=budget)
    got = _tokens(eng.run(prompts, RunConfig(mode="static", keep_outputs=True)), prompts)
    eng.dm.check()
    assert eng.stats["piggyback_tokens"] > 0
    assert np.array_equal(got, g["ar_tokens"])
