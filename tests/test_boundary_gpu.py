"""The drop-in boundary and the engine invariants of the reference's own tests, on the B200.

* The reference's harness builds ``b200_layerskip`` through its registry from its own
  ``LayerSkipLlama`` (evaluation/benchmark.py:86-92: ``spec.build(model, args, B, ...)`` then
  ``engine.run(prompts, run_cfg)``) and gets the reference ``SyncSpecEngine``'s tokens (fp32).
  Needs the reference (THESIS_REFERENCE or baseline/_ref, which travels with the repository).
* ``ModelWeights.from_pretrained`` on a tiny HF checkpoint written by transformers matches HF's
  own forward (tests/test_model.py:9-36 of the reference pins its model the same way).
* Rollback moves no KV: a step never rewrites cached positions below a request's committed
  position, and pos = prompt length + generated - 1 (tests/test_eesd.py:145-171).
* A prompt prefilled piggybacked on draft/verify steps leaves exactly the KV a normal prefill
  writes, and the same first token (tests/test_eesd.py:174-196).
* Device-to-host reads: one per round (the accepted counts and verified tokens), none in the draft
  steps (tests/test_eesd.py:199-223; here every round's read is a single pinned copy).
"""

import json
import sys

import numpy as np
import pytest
import torch

from goldens import Golden
from refpath import reference_dir
from thesis_b200.config import preset
from thesis_b200.eesd import B200SpecEngine
from thesis_b200.model import DeviceModel, ModelWeights
from thesis_b200.serving import B200ServingEngine
from thesis_b200.synthetic import Prompt, synthetic_prompts, synthetic_weights

pytestmark = pytest.mark.gpu


def _reference():
    ref = reference_dir()
    if ref is None:
        pytest.skip("the reference is not available (THESIS_REFERENCE or baseline/_ref)")
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    return ref


def test_reference_harness_builds_and_runs_b200_layerskip(cuda_dev):
    _reference()
    from common.data import Prompt as RefPrompt
    from common.engine import RunConfig as RefRunConfig
    from common.methods import METHODS, load_plugins
    from common.model import LayerSkipLlama, LayerWeights, ModelConfig as RefConfig
    from evaluation.benchmark import build_parser

    g = Golden("c1s_fp32")
    cfg, W = g.config(), g.weights()
    rc = RefConfig(vocab_size=cfg.vocab_size, dim=cfg.dim, n_layers=cfg.n_layers, n_heads=cfg.n_heads,
                   n_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, intermediate_size=cfg.intermediate_size,
                   norm_eps=cfg.norm_eps, rope_theta=cfg.rope_theta, max_position_embeddings=g.meta["max_seq"],
                   tie_word_embeddings=cfg.tie_word_embeddings, rope_scaling=cfg.rope_scaling)

    def t(a):
        return torch.from_numpy(np.asarray(a)).to(cuda_dev, torch.float32)

    layers = [LayerWeights(wqkv=t(W[f"l{i}.wqkv"]), wo=t(W[f"l{i}.wo"]), w13=t(W[f"l{i}.w13"]), w2=t(W[f"l{i}.w2"]),
                           attn_norm=t(W[f"l{i}.attn_norm"]), ffn_norm=t(W[f"l{i}.ffn_norm"]))
              for i in range(cfg.n_layers)]
    embed = t(W["embed"])
    model = LayerSkipLlama(rc, embed, layers, t(W["norm"]), embed, cuda_dev, torch.float32, g.meta["max_seq"])
    load_plugins(["thesis_b200.plugin"])
    args = build_parser().parse_args(["--method", "b200_layerskip", "--exit-layer", str(g.meta["exit_layer"]),
                                      "--gamma", str(g.meta["gamma"]), "--max-new-tokens", str(g.meta["max_new"])])
    prompts = [RefPrompt(f"p{i}", p) for i, p in enumerate(g.prompts())]
    engine = METHODS[args.method].build(model, args, 3, max(len(p.tokens) for p in prompts), ())
    res = engine.run(prompts, RefRunConfig(mode="static", keep_outputs=True))
    got = {c["pid"]: c["tokens"] for c in res["completions"]}
    assert np.array_equal(np.array([got[p.pid] for p in prompts]), g["spec_tokens"])
    m = res["metrics"]
    assert m["stop_reason"] == "pool_exhausted" and m["steps"]["verify"]["p50_ms"] > 0
    assert 0.0 <= m["spec"]["acceptance_rate"] <= 1.0
    json.dumps(m)                                       # the harness writes the metrics as JSON


def test_from_pretrained_matches_transformers(cuda_dev, tmp_path):
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    hf_cfg = LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=640, num_hidden_layers=3,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=64, rms_norm_eps=1e-5,
                         rope_theta=10000.0, max_position_embeddings=256, tie_word_embeddings=False)
    hf = LlamaForCausalLM(hf_cfg).float().eval()
    with torch.no_grad():                               # non-trivial norm weights
        for mod in hf.modules():
            if type(mod).__name__.endswith("RMSNorm"):
                mod.weight.add_(0.1 * torch.randn_like(mod.weight))
    hf.save_pretrained(tmp_path, safe_serialization=True)
    w = ModelWeights.from_pretrained(tmp_path, device=cuda_dev, dtype=torch.float32)
    assert (w.cfg.n_layers, w.cfg.dim, w.cfg.n_kv_heads, w.cfg.head_dim) == (3, 256, 2, 64)
    dm = DeviceModel(w, max_batch=2, max_seq=128, max_tokens=128)
    ids = list(np.random.default_rng(0).integers(0, 512, size=37))
    ph = dm.pack([(0, 0, len(ids))])
    b, (ids_d,) = dm.upload(ph, (np.asarray(ids, dtype=np.int32),))
    x = dm.embed(ids_d)
    dm.forward_layers(x, b, 0, 3)
    _, lg = dm.head_argmax(x, logits=True)
    with torch.no_grad():
        want = hf(torch.tensor([ids])).logits[0].float()
    got = lg.float().cpu()
    assert (got - want).abs().max().item() / want.abs().max().item() < 1e-4
    assert torch.equal(got.argmax(-1), want.argmax(-1))


def _c1s_bf16(seed=0):
    cfg = preset("c1s")
    return ModelWeights.from_numpy(cfg, synthetic_weights(cfg, seed=seed, residual_scale_from=4, residual_scale=0.05),
                                   torch.bfloat16, "cuda")


def test_rollback_moves_no_kv(cuda_dev):
    cfg = preset("c1s")                                 # unscaled residuals: drafts get rejected
    w = ModelWeights.from_numpy(cfg, synthetic_weights(cfg, seed=1, norm_jitter=0.1), torch.bfloat16, "cuda")
    prompts = synthetic_prompts(4, w.cfg.vocab_size, seed=3, min_len=20, max_len=60)
    eng = B200SpecEngine(w, 4, 64, 48, (), ignore_eos=True, exit_layer=4, gamma=4)
    eng.start(prompts)
    saw_reject = False
    for _ in range(12):
        live = [s for s in range(4) if not eng.slots[s].idle and eng.slots[s].finish_reason is None]
        if not live:
            break
        torch.cuda.synchronize()
        before = {s: eng.slots[s].pos for s in live}
        snap = {s: (eng.dm.k_cache[:, s, :, :before[s]].clone(), eng.dm.v_cache[:, s, :, :before[s]].clone())
                for s in live}
        eng.step()
        torch.cuda.synchronize()
        for s in live:
            assert torch.equal(eng.dm.k_cache[:, s, :, :before[s]], snap[s][0])
            assert torch.equal(eng.dm.v_cache[:, s, :, :before[s]], snap[s][1])
            st = eng.slots[s]
            if st.finish_reason is None:       # a finished request's output is cut at its budget
                assert st.pos == st.prompt_len + len(st.output) - 1
                if 0 < st.pos - before[s] < eng.gamma + 1:
                    saw_reject = True
    eng.dm.check()
    assert saw_reject, "the test needs a round with a rejected draft"


def test_piggyback_prefill_writes_the_same_kv_as_a_normal_prefill(cuda_dev):
    w = _c1s_bf16()
    ps = synthetic_prompts(2, w.cfg.vocab_size, seed=5, min_len=40, max_len=60)
    eng = B200ServingEngine(w, 3, 64, 32, (), ignore_eos=True, exit_layer=4, gamma=2, piggyback_budget=7)
    eng._assign_many([(0, 0, ps[0])])
    while 0 in eng.pf:                                  # nothing decodes yet: slot 0 is prefilled alone
        eng.step()
    eng._assign_many([(1, 1, ps[1])])
    steps = 0
    while 1 in eng.pf:
        eng.step()                                      # slot 1's prompt rides on slot 0's rounds
        steps += 1
        assert steps < 40
    assert steps > 1, "the prompt must take several piggybacked chunks"
    n = len(ps[1].tokens)
    first = eng.dm.prefill({2: list(ps[1].tokens)})[2]  # a normal prefill of the same prompt into row 2
    torch.cuda.synchronize()
    assert torch.equal(eng.dm.k_cache[:, 1, :, :n], eng.dm.k_cache[:, 2, :, :n])
    assert torch.equal(eng.dm.v_cache[:, 1, :, :n], eng.dm.v_cache[:, 2, :, :n])
    assert eng.slots[1].output[0] == first
    eng.dm.check()


def test_one_device_to_host_read_per_round(cuda_dev, monkeypatch):
    w = _c1s_bf16()
    prompts = synthetic_prompts(4, w.cfg.vocab_size, seed=7, min_len=20, max_len=60)
    eng = B200SpecEngine(w, 4, 64, 40, (), ignore_eos=True, exit_layer=4, gamma=4)
    eng.start(prompts)
    eng.step()
    calls = []
    orig = {name: getattr(torch.Tensor, name) for name in ("cpu", "item", "tolist", "numpy", "copy_")}

    def wrap(name):
        def f(self, *a, **k):
            if name == "copy_":
                src = a[0] if a else None
                if self.device.type == "cpu" and isinstance(src, torch.Tensor) and src.is_cuda:
                    calls.append("d2h")
            elif self.is_cuda:
                calls.append(name)
            return orig[name](self, *a, **k)
        return f

    for name in orig:
        monkeypatch.setattr(torch.Tensor, name, wrap(name))
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: calls.append("device_sync"))
    for _ in range(5):
        calls.clear()
        n_rec = len(eng.records)
        eng.step()
        kinds = [r.kind for r in eng.records[n_rec:]]
        assert kinds == ["draft"] * eng.gamma + ["verify"]
        assert calls == ["d2h"], calls                 # the round's one pinned read-back, nothing else
