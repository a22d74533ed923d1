"""Parity of the sm_100a path with the reference (golden vectors) and with the numpy oracle.

Tolerances (task statement): exit-layer and final logits within 1e-4 relative in fp32 and
2e-2 in bf16 (relative = max |a - b| / max |b|), identical token sequences in fp32.
"""

import numpy as np
import pytest
import torch

from goldens import CASES, TOL, Golden, rel_err
from thesis_b200.eesd import B200ARBatchEngine, B200SpecEngine
from thesis_b200.engine import RunConfig
from thesis_b200.model import DeviceModel, ModelWeights
from thesis_b200.synthetic import Prompt

pytestmark = pytest.mark.gpu


def _device_model(g: Golden, max_batch=4, max_tokens=512):
    dtype = torch.bfloat16 if g.dtype == "bf16" else torch.float32
    w = ModelWeights.from_numpy(g.config(), g.weights(), dtype, "cuda")
    return w, DeviceModel(w, max_batch=max_batch, max_seq=g.meta["max_seq"], max_tokens=max_tokens)


def _run_blocks(dm, blocks, ids):
    ph = dm.pack(blocks)
    b, (ids_d,) = dm.upload(ph, (np.asarray(ids, dtype=np.int32),))
    return ph, b, dm.embed(ids_d)


@pytest.mark.parametrize("name", CASES)
def test_prefill_and_packed_logits_match_reference(cuda_dev, name):
    g = Golden(name)
    _, dm = _device_model(g)
    tol = TOL[g.dtype]
    L = dm.cfg.n_layers
    for i, p in enumerate(g.prompts()):
        ph, b, x = _run_blocks(dm, [(i, 0, len(p))], p)
        dm.forward_layers(x, b, 0, L)
        _, lg = dm.head_argmax(x[-1:].contiguous(), logits=True)
        assert rel_err(lg[0].float().cpu().numpy(), g["prefill_logits"][i]) < tol
    blocks = [tuple(map(int, b)) for b in g["packed_blocks"]]
    E = g.meta["exit_layer"]
    ph, b, x = _run_blocks(dm, blocks, g["packed_ids"])
    dm.forward_layers(x, b, 0, E)
    _, lg_exit = dm.head_argmax(x, logits=True)
    dm.forward_layers(x, b, E, L)
    _, lg_final = dm.head_argmax(x, logits=True)
    dm.check()
    assert rel_err(lg_exit.float().cpu().numpy(), g["packed_exit_logits"]) < tol
    assert rel_err(lg_final.float().cpu().numpy(), g["packed_final_logits"]) < tol


@pytest.mark.parametrize("name", CASES)
def test_fused_head_argmax_equals_argmax_of_logits(cuda_dev, name):
    g = Golden(name)
    _, dm = _device_model(g)
    blocks = [tuple(map(int, b)) for b in g["packed_blocks"]]
    ph, b, x = _run_blocks(dm, blocks, g["packed_ids"])
    dm.forward_layers(x, b, 0, dm.cfg.n_layers)
    fused = dm.head_argmax(x)
    ids, lg = dm.head_argmax(x, logits=True)
    assert torch.equal(fused, ids)
    assert torch.equal(ids.long(), lg.float().argmax(-1))


def _tokens(res, prompts):
    out = {}
    for c in res["completions"]:
        out.setdefault(c["pid"], c["tokens"])
    return np.array([out[p.pid] for p in prompts])


@pytest.mark.parametrize("name", CASES)
def test_engine_tokens(cuda_dev, name):
    """fp32: AR and speculative tokens identical to the reference's engines.  Every dtype: the
    speculative output is bit-identical to this engine's own AR output (lossless)."""
    g = Golden(name)
    dtype = torch.bfloat16 if g.dtype == "bf16" else torch.float32
    w = ModelWeights.from_numpy(g.config(), g.weights(), dtype, "cuda")
    prompts = [Prompt(f"p{i}", p) for i, p in enumerate(g.prompts())]
    mp = max(len(p.tokens) for p in prompts)
    rc = RunConfig(mode="static", keep_outputs=True)
    ar = _tokens(B200ARBatchEngine(w, 2, mp, g.meta["max_new"], (), ignore_eos=True).run(prompts, rc), prompts)
    sp_eng = B200SpecEngine(w, 3, mp, g.meta["max_new"], (), ignore_eos=True, exit_layer=g.meta["exit_layer"],
                            gamma=g.meta["gamma"])
    sp = _tokens(sp_eng.run(prompts, rc), prompts)
    sp_eng.dm.check()
    assert np.array_equal(sp, ar)
    if g.dtype == "fp32":
        assert np.array_equal(ar, g["ar_tokens"])
        assert np.array_equal(sp, g["spec_tokens"])
