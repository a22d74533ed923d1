"""Cost-model calibration on the B200 engine (thesis_b200/calibrate.py): the fits and the step
prices on CPU, the file's compatibility with the reference's own cost model, and one quick
calibration on the GPU."""

import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from refpath import reference_dir
from thesis_b200.calibrate import StepCost, fit_linear, hinge_knee, model_dims
from thesis_b200.config import preset


def _synthetic_calibration(cfg):
    gpu = {"bw": 6.0e9, "flops": 1.5e12, "t_op": 0.004, "n_op_layer": 7.0, "n_op_bucket": 0.0, "n_op_head": 3.0,
           "n_op_segment": 1.0, "meta": {"source": "test"}, "flops_eff": 9.0e11, "knee_measured": 180.0}
    lin = {"a": 0.05, "b": 0.0004, "c": 2.0e-7, "head_a": 0.2, "head_b": 0.001, "n_layers": cfg.n_layers,
           "model_name": "llama3-8b", "seg_ms": 0.0}
    return {"model": "llama3-8b", "gpu": gpu, "model_dims": model_dims(cfg), "linear": lin}


def test_hinge_fit_recovers_the_knee():
    n = np.array([1, 2, 4, 8, 16, 32, 64, 96, 128, 160, 192, 256, 320, 384, 448, 512], dtype=float)
    t = 0.06 + 0.0005 * np.maximum(n - 128, 0)
    knee, (a, b) = hinge_knee(n, t)
    assert knee == 128 and abs(a - 0.06) < 1e-9 and abs(b - 0.0005) < 1e-9


def test_linear_fit_recovers_the_coefficients():
    rng = np.random.default_rng(0)
    rows = [{"n": int(n), "kv": int(kv), "ms": 0.05 + 0.0004 * n + 2e-7 * kv}
            for n, kv in zip(rng.integers(1, 600, 40), rng.integers(100, 200000, 40))]
    heads = [{"n": n, "ms": 0.2 + 0.001 * n} for n in (1, 4, 16, 64, 256)]
    fit = fit_linear(rows, heads)
    assert np.allclose([fit["a"], fit["b"], fit["c"], fit["head_a"], fit["head_b"]], [0.05, 0.0004, 2e-7, 0.2, 0.001])


def test_step_prices_follow_the_roofline_form():
    cfg = preset("llama3-8b")
    cal = _synthetic_calibration(cfg)
    d, g = cal["model_dims"], cal["gpu"]
    rf = StepCost(cal, "roofline")
    w = d["layer_params"] * 2
    layer = max(w / g["bw"], 2 * d["layer_params"] * 64 / g["flops_eff"]) + 5000 * d["kv_bytes_per_pos"] / g["bw"] \
        + 7 * 0.004
    head = max(d["head_params"] * 2 / g["bw"], 2 * d["head_params"] * 64 / g["flops_eff"]) + 3 * 0.004
    assert abs(rf.t_sh(64, 8, 5000) - (8 * layer + 0.004 + head)) < 1e-12
    lin = StepCost(cal, "linear")
    assert abs(lin.t_prefill(100, 300) - (32 * (0.05 + 0.04 + 6e-5) + 0.2 + 0.001)) < 1e-12


def test_calibration_file_loads_in_the_reference_cost_model(tmp_path):
    """The JSON layout is the one solutions/cost_model.py:load_cost_model reads, and the restated
    step prices equal the reference's own for the three model kinds.  Needs a checkout of the
    reference (THESIS_REFERENCE or baseline/_ref)."""
    ref = reference_dir()
    if ref is None:
        pytest.skip("the reference is not available (THESIS_REFERENCE or baseline/_ref)")
    cfg = preset("llama3-8b")
    cal = _synthetic_calibration(cfg)
    path = tmp_path / "cal.json"
    path.write_text(json.dumps(cal))
    queries = [("t_sh", (64, 8, 40000)), ("t_deep", (320, 8, 40000, 64)), ("t_prefill", (512, 600)),
               ("t_sh", (1, 8, 300)), ("t_deep", (17, 4, 3000, 1))]
    mine = {kind: [float(getattr(StepCost(cal, kind), q)(*a)) for q, a in queries]
            for kind in ("roofline", "roofline-peak", "linear")}
    code = f"""
import json, sys
sys.path[:0] = [{str(ref)!r}]
from common.model import ModelConfig
from solutions.cost_model import load_cost_model
cfg = ModelConfig(vocab_size=128256, dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128,
                  intermediate_size=14336, norm_eps=1e-5, rope_theta=500000.0, max_position_embeddings=8192)
queries = {queries!r}
out = {{}}
for kind in ("roofline", "roofline-peak", "linear"):
    cm = load_cost_model({str(path)!r}, cfg, kind)
    out[kind] = [float(getattr(cm, q)(*a)) for q, a in queries]
print(json.dumps(out))
"""
    r = subprocess.run([sys.executable, "-c", code], cwd=str(ref), capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    theirs = json.loads(r.stdout.strip().splitlines()[-1])
    for kind in mine:
        assert np.allclose(mine[kind], theirs[kind], rtol=1e-12, atol=0), (kind, mine[kind], theirs[kind])


@pytest.mark.gpu
def test_quick_calibration_on_the_gpu(cuda_dev, tmp_path):
    from thesis_b200.calibrate import main

    out = tmp_path / "c.json"
    main(["--preset", "c1s", "--quick", "--validate", "--k", "3", "--out", str(out)])
    res = json.loads(out.read_text())
    g = res["gpu"]
    assert g["bw"] > 0 and g["flops"] > 0 and g["flops_eff"] > 0 and g["t_op"] > 0
    assert g["n_op_layer"] >= 5 and g["n_op_head"] >= 1
    assert set(res["linear"]) >= {"a", "b", "c", "head_a", "head_b"}
    assert res["validation"]["roofline_all"]["n"] > 0
