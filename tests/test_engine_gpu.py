"""Engine behaviour on the B200: losslessness (speculative == autoregressive, bit-exact),
EOS handling, the cyclic driver, and full-size shapes through size-independent properties."""

import numpy as np
import pytest
import torch

from thesis_b200.config import preset
from thesis_b200.dynamic import B200DynamicSpecEngine
from thesis_b200.eesd import B200ARBatchEngine, B200SpecEngine
from thesis_b200.engine import RunConfig
from thesis_b200.model import ModelWeights
from thesis_b200.serving import B200ServingEngine
from thesis_b200.synthetic import Prompt, synthetic_prompts, synthetic_weights

pytestmark = pytest.mark.gpu

MAX_NEW = 40


def _outputs(res):
    return {c["pid"]: c["tokens"] for c in res["completions"]}


@pytest.fixture(scope="module")
def c1s_bf16():
    cfg = preset("c1s")
    W = synthetic_weights(cfg, seed=5, residual_scale_from=4, residual_scale=0.05, norm_jitter=0.1)
    return ModelWeights.from_numpy(cfg, W, torch.bfloat16, "cuda")


@pytest.fixture(scope="module")
def ar_reference(c1s_bf16):
    prompts = synthetic_prompts(6, c1s_bf16.cfg.vocab_size, seed=11, min_len=5, max_len=60)
    eng = B200ARBatchEngine(c1s_bf16, 2, 60, MAX_NEW, (2,), ignore_eos=True)
    return prompts, _outputs(eng.run(prompts, RunConfig(mode="static", keep_outputs=True)))


@pytest.mark.parametrize("k,gamma,B", [(1, 3, 2), (3, 5, 3), (5, 2, 1), (2, 0, 2), (4, 8, 5)])
def test_spec_is_lossless_bf16(c1s_bf16, ar_reference, k, gamma, B):
    prompts, ref = ar_reference
    eng = B200SpecEngine(c1s_bf16, B, 60, MAX_NEW, (2,), ignore_eos=True, exit_layer=k, gamma=gamma)
    res = eng.run(prompts, RunConfig(mode="static", keep_outputs=True))
    assert _outputs(res) == ref
    if gamma and k >= 4:
        assert res["metrics"]["spec"]["accepted"] > 0


def test_eos_stops_generation(c1s_bf16, ar_reference):
    prompts, ref = ar_reference
    eos = ref["p0"][5]
    rc = RunConfig(mode="static", keep_outputs=True)
    ar = _outputs(B200ARBatchEngine(c1s_bf16, 2, 60, MAX_NEW, (eos,)).run(prompts, rc))
    sp = _outputs(B200SpecEngine(c1s_bf16, 2, 60, MAX_NEW, (eos,), exit_layer=3, gamma=4).run(prompts, rc))
    assert ar == sp
    assert ar["p0"][-1] == eos and len(ar["p0"]) <= 6


@pytest.mark.parametrize("kw", [{}, {"exit_layer": 3, "gamma": 4}])
def test_overlapped_steps_equal_synchronous_steps(c1s_bf16, ar_reference, kw):
    """Enqueueing step k+1 before reading step k back changes nothing: same tokens with EOS stops
    and slot refills (6 prompts through 2 slots), AR and speculative alike."""
    prompts, ref = ar_reference
    eos = ref["p1"][7]
    cls = B200SpecEngine if kw else B200ARBatchEngine
    rc = RunConfig(mode="static", keep_outputs=True)
    outs = [_outputs(cls(c1s_bf16, 2, 60, MAX_NEW, (eos,), overlap=o, **kw).run(prompts, rc)) for o in (True, False)]
    assert outs[0] == outs[1]
    assert len(outs[0]["p1"]) <= 8 and outs[0]["p1"][-1] == eos


def test_cyclic_run_converges_and_reports(c1s_bf16):
    prompts = synthetic_prompts(4, c1s_bf16.cfg.vocab_size, seed=2, min_len=5, max_len=20)
    eng = B200SpecEngine(c1s_bf16, 3, 20, 12, (2,), ignore_eos=True, exit_layer=4, gamma=3)
    res = eng.run(prompts, RunConfig(mode="cyclic", warmup_samples=2, max_eval_samples=6, converge=False))
    m = res["metrics"]
    assert m["stop_reason"] == "max_eval_samples"
    assert m["evaluated_completions"] == 6
    assert m["measured_tokens"] > 0 and m["throughput_tok_s"] > 0
    assert all(c["generated"] == 12 for c in res["completions"])
    assert "verify" in m["steps"] and m["steps"]["verify"]["p50_ms"] > 0


@pytest.mark.parametrize("name,E,gamma,B,lens", [("llama3-1b", 6, 6, 8, (64, 300)), ("llama3-8b", 8, 4, 4, (128, 256))])
def test_full_size_spec_equals_ar(cuda_dev, name, E, gamma, B, lens):
    """Full BASELINE shapes (bf16, residual outputs of the deep layers scaled by 0.1): the
    speculative tokens equal the AR tokens bit for bit."""
    cfg = preset(name)
    w = ModelWeights.synthetic(cfg, seed=0, dtype=torch.bfloat16, device="cuda", residual_scale_from=E,
                               residual_scale=0.1)
    prompts = synthetic_prompts(B, cfg.vocab_size, seed=1, min_len=lens[0], max_len=lens[1])
    rc = RunConfig(mode="static", keep_outputs=True)
    ar_e = B200ARBatchEngine(w, B, lens[1], 24, (), ignore_eos=True)
    ar = _outputs(ar_e.run(prompts, rc))
    ar_e.free()
    sp_e = B200SpecEngine(w, B, lens[1], 24, (), ignore_eos=True, exit_layer=E, gamma=gamma)
    res = sp_e.run(prompts, rc)
    sp_e.dm.check()
    assert _outputs(res) == ar
    assert res["metrics"]["spec"]["acceptance_rate"] > 0.2


@pytest.mark.parametrize("schedule", ["lockstep", "unified"])
@pytest.mark.parametrize("exits,grange,B,seed", [((1, 3, 5), (2, 8), 3, 0), ((2, 4), (0, 3), 4, 1), ((3,), (1, 1), 2, 2)])
def test_dynamic_exit_and_draft_length_is_lossless(c1s_bf16, ar_reference, exits, grange, B, seed, schedule):
    """Per-request exit layer and per-request, per-round draft length (coalesced ragged verify), in
    lock-step rounds or in the unified step (requests verify out of phase): the output equals the AR
    output bit for bit whatever the draws."""
    prompts, ref = ar_reference
    eng = B200DynamicSpecEngine(c1s_bf16, B, 60, MAX_NEW, (2,), ignore_eos=True, exit_layers=exits,
                                gamma_range=grange, policy_seed=seed, schedule=schedule)
    res = eng.run(prompts, RunConfig(mode="static", keep_outputs=True))
    eng.dm.check()
    assert _outputs(res) == ref
    spec = res["metrics"]["spec"]
    assert sum(spec["exit_hist"].values()) == spec["request_rounds"]
    if len(exits) > 1:
        assert sum(1 for v in spec["exit_hist"].values() if v) > 1     # several exits were in play
    if grange[1] > 0:
        assert spec["accepted"] > 0


def test_dynamic_full_size_llama2_7b_equals_ar(cuda_dev):
    """BASELINE config 4 shape (Llama2-7B, MHA, exits {4, 8, 12}, draft length 2..8 per request and
    round, lognormal prompt lengths): speculative tokens equal AR tokens bit for bit."""
    cfg = preset("llama2-7b")
    w = ModelWeights.synthetic(cfg, seed=0, dtype=torch.bfloat16, device="cuda", residual_scale_from=4,
                               residual_scale=0.1)
    prompts = synthetic_prompts(6, cfg.vocab_size, seed=3, min_len=32, max_len=1536, lengths="lognormal", median=256)
    rc = RunConfig(mode="static", keep_outputs=True)
    mp = max(len(p.tokens) for p in prompts)
    ar_e = B200ARBatchEngine(w, 6, mp, 20, (), ignore_eos=True)
    ar = _outputs(ar_e.run(prompts, rc))
    ar_e.free()
    sp_e = B200DynamicSpecEngine(w, 6, mp, 20, (), ignore_eos=True, exit_layers=(4, 8, 12), gamma_range=(2, 8))
    res = sp_e.run(prompts, rc)
    sp_e.dm.check()
    assert _outputs(res) == ar
    assert res["metrics"]["spec"]["acceptance_rate"] > 0.1


@pytest.mark.parametrize("B,budget,gamma", [(2, 7, 3), (3, 64, 4), (4, 1000, 2)])
def test_piggyback_prefill_is_lossless(c1s_bf16, ar_reference, B, budget, gamma):
    """New requests prefilled inside the draft/verify steps (chunks through [0, E) with the drafts,
    through [E, L) with the verify tokens; a flush through all layers when nothing decodes): the
    output equals the AR output bit for bit."""
    prompts, ref = ar_reference
    eng = B200ServingEngine(c1s_bf16, B, 60, MAX_NEW, (2,), ignore_eos=True, exit_layer=3, gamma=gamma,
                            piggyback_budget=budget)
    res = eng.run(prompts, RunConfig(mode="static", keep_outputs=True))
    eng.dm.check()
    assert _outputs(res) == ref
    assert eng.stats["piggyback_tokens"] > 0 and eng.stats["flush_steps"] > 0


def test_poisson_driver_with_per_request_lengths(c1s_bf16):
    """Open-loop Poisson arrivals, per-request output lengths, piggybacked prefill: every measured
    request completes with its own length and the AR tokens."""
    base = synthetic_prompts(8, c1s_bf16.cfg.vocab_size, seed=4, min_len=5, max_len=40)
    rng = np.random.default_rng(0)
    prompts = [Prompt(p.pid, p.tokens, max_new=int(rng.integers(4, 17))) for p in base]
    ar_e = B200ARBatchEngine(c1s_bf16, 4, 40, 16, (), ignore_eos=True)
    ar = _outputs(ar_e.run(base, RunConfig(mode="static", keep_outputs=True)))
    ar_e.free()
    eng = B200ServingEngine(c1s_bf16, 3, 40, 16, (), ignore_eos=True, exit_layer=3, gamma=3, piggyback_budget=16)
    res = eng.run_poisson(prompts, rate_per_s=200.0, n_requests=6, warm_requests=2, seed=0, keep_outputs=True)
    eng.dm.check()
    m = res["metrics"]
    # the run ends after n_requests + warm_requests completions; requests assigned before the warm-up
    # ended are not measured (solutions/engine.py:625-673)
    assert len(res["completions"]) >= 8
    assert 1 <= m["evaluated_completions"] <= 6 and m["ttft_ms_mean"] > 0 and m["wall_throughput_tok_s"] > 0
    by_pid = {p.pid: p for p in prompts}
    for c in res["completions"]:
        want = by_pid[c["pid"]].max_new
        assert c["generated"] == want and c["tokens"] == ar[c["pid"]][:want]
