"""Engine behaviour on the B200: losslessness (speculative == autoregressive, bit-exact),
EOS handling, the cyclic driver, and full-size shapes through size-independent properties."""

import numpy as np
import pytest
import torch

from thesis_b200.config import preset
from thesis_b200.eesd import B200ARBatchEngine, B200SpecEngine
from thesis_b200.engine import RunConfig
from thesis_b200.model import ModelWeights
from thesis_b200.synthetic import synthetic_prompts, synthetic_weights

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
