"""Host-side logic on CPU: ragged packing, the method registry, and the DecodeEngine driver
(with a toy engine whose 'model' is a deterministic function, so no GPU is needed)."""

import argparse

import numpy as np
import pytest

from refpath import reference_dir

from thesis_b200.engine import DecodeEngine, RunConfig, StepRecord
from thesis_b200.packing import pack, qo_indptr
from thesis_b200.synthetic import Prompt, synthetic_prompts


def test_packing_metadata():
    blocks = [(2, 10, 3), (0, 5, 1), (1, 7, 40), (3, 9, 1)]
    ph = pack(blocks, item_tokens=16)
    assert ph.n_tokens == 45
    assert list(ph.offsets) == list(qo_indptr([3, 1, 40, 1]))
    for i, (r, p0, T) in enumerate(blocks):          # caller order kept, positions consecutive
        sl = ph.block_slice(i)
        assert list(ph.tok_pos[sl]) == list(range(p0, p0 + T))
        assert set(ph.tok_row[sl]) == {r}
        assert tuple(ph.blk[i]) == (ph.offsets[i], T, r, p0)
    # the 40-token block is tiled into items of 16 query tokens: 0, 16, 32
    assert sorted(tuple(x) for x in ph.items if x[0] == 2) == [(2, 0), (2, 16), (2, 32)]
    assert len(ph.items) == 6
    # items are ordered longest key range (pos0 + last query token + 1) first
    kv = [int(ph.blk[b][3]) + min(int(t0) + 16, int(ph.blk[b][1])) for b, t0 in ph.items]
    assert kv == sorted(kv, reverse=True) and kv[0] == 47
    assert ph.max_ctx == 47 and ph.kv_read == 13 + 6 + 47 + 10
    with pytest.raises(ValueError):
        pack([(0, 0, 0)], 16)


def test_registry_contract():
    from thesis_b200 import methods

    assert {"b200_autoregressive", "b200_layerskip", "b200_layerskip_dynamic",
            "b200_layerskip_piggyback"} <= set(methods.METHODS)
    with pytest.raises(ValueError):
        methods.register(methods.METHODS["b200_layerskip"])
    # the CLI groups coexist with a parser that already has --exit-layer / --gamma (the reference's)
    ap = argparse.ArgumentParser()
    ap.add_argument("--exit-layer", type=int)
    ap.add_argument("--gamma", type=int, default=4)
    for spec in methods.METHODS.values():
        spec.add_args(ap.add_argument_group(spec.name))
    a = ap.parse_args(["--exit-layer", "8", "--b200-prefill-chunk", "256"])
    assert a.exit_layer == 8 and a.b200_prefill_chunk == 256
    assert methods.METHODS["b200_layerskip"].tag(a) == "-k8-g4"
    assert methods.METHODS["b200_layerskip"].step_tokens(a) == 5
    a = ap.parse_args(["--b200-exit-layers", "4,8,12", "--b200-gamma-range", "2,8"])
    dyn = methods.METHODS["b200_layerskip_dynamic"]
    assert dyn.step_tokens(a) == 9 and dyn.tag(a) == "-e4_8_12-g2_8"
    assert dyn.params(a) == {"exit_layers": [4, 8, 12], "gamma_range": [2, 8], "policy_seed": 0}
    a = ap.parse_args(["--exit-layer", "8", "--b200-piggyback-budget", "128"])
    pb = methods.METHODS["b200_layerskip_piggyback"]
    assert pb.tag(a) == "-k8-g4-pb128" and pb.step_tokens(a) == 5


class ToyEngine(DecodeEngine):
    """next token = (7 * last + 3) % 97, one token per request per step."""

    def _prefill_slots(self, prompts):
        return {s: (sum(t) * 13) % 97 for s, t in prompts.items()}

    def _iteration(self, measured):
        committed = 0
        act = self._active()
        for s in act:
            st = self.slots[s]
            st.last_token = (7 * st.last_token + 3) % 97
            st.pos += 1
            committed += self._commit(s, [st.last_token])
        self.records.append(StepRecord("ar", 1.0, len(act), len(act), len(act), 0, measured))
        return committed


def _expected(p, n):
    t = (sum(p.tokens) * 13) % 97
    out = [t]
    while len(out) < n:
        t = (7 * t + 3) % 97
        out.append(t)
    return out


def test_static_run_generates_every_prompt_once():
    prompts = synthetic_prompts(5, 97, seed=0, min_len=3, max_len=9)
    eng = ToyEngine(None, 2, 9, 12, (), ignore_eos=True)
    res = eng.run(prompts, RunConfig(mode="static", keep_outputs=True))
    assert sorted(c["pid"] for c in res["completions"]) == sorted(p.pid for p in prompts)
    for c in res["completions"]:
        p = next(p for p in prompts if p.pid == c["pid"])
        assert c["tokens"] == _expected(p, 12) and c["finish_reason"] == "length"
    assert res["metrics"]["stop_reason"] == "pool_exhausted"
    assert res["metrics"]["steps"]["ar"]["p50_ms"] == 1.0


def test_cyclic_run_stops_at_max_eval_and_counts_tokens():
    prompts = synthetic_prompts(4, 97, seed=1, min_len=3, max_len=9)
    eng = ToyEngine(None, 3, 9, 5, (), ignore_eos=True)
    res = eng.run(prompts, RunConfig(mode="cyclic", warmup_samples=2, max_eval_samples=6, converge=False))
    m = res["metrics"]
    assert m["stop_reason"] == "max_eval_samples" and m["evaluated_completions"] == 6
    assert m["measured_tokens"] > 0 and m["throughput_tok_s"] > 0
    assert m["warmup_samples_effective"] == 3                # max(2, 1.0 * B)


def test_eos_and_stop_checker():
    prompts = [Prompt("a", [1, 2, 3])]
    first = _expected(prompts[0], 8)
    eng = ToyEngine(None, 1, 3, 8, (first[3],))
    res = eng.run(prompts, RunConfig(mode="static", keep_outputs=True))
    c = res["completions"][0]
    assert c["tokens"] == first[:4] and c["finish_reason"] == "eos"
    eng = ToyEngine(None, 1, 3, 8, ())
    eng.stop_checker = lambda out, n: 3 if len(out) >= 3 else None
    c = eng.run(prompts, RunConfig(mode="static", keep_outputs=True))["completions"][0]
    assert c["tokens"] == first[:3] and c["finish_reason"] == "stop"


def test_sampling_is_rejected():
    with pytest.raises(NotImplementedError):
        ToyEngine(None, 1, 3, 8, (), temperature=0.7)


def test_synthetic_inputs_are_seeded():
    from thesis_b200.config import preset
    from thesis_b200.synthetic import synthetic_weights

    a = synthetic_prompts(3, 1000, seed=4, min_len=10, max_len=20)
    b = synthetic_prompts(3, 1000, seed=4, min_len=10, max_len=20)
    assert [p.tokens for p in a] == [p.tokens for p in b]
    assert all(10 <= len(p.tokens) <= 20 for p in a)
    ln = synthetic_prompts(200, 1000, seed=4, min_len=32, max_len=1536, lengths="lognormal", median=256)
    assert 150 < np.median([len(p.tokens) for p in ln]) < 350
    cfg = preset("tiny")
    W = synthetic_weights(cfg, seed=0, residual_scale_from=3, residual_scale=0.1)
    W2 = synthetic_weights(cfg, seed=0)
    assert np.allclose(W["l3.wo"], 0.1 * W2["l3.wo"]) and np.array_equal(W["l2.wo"], W2["l2.wo"])
    assert W["l0.wqkv"].shape == (4 * 64 + 2 * 2 * 64, 256) and W["l0.w13"].shape == (2 * 512, 256)


def test_plugin_registers_into_the_reference_harness():
    """The drop-in boundary itself: the reference's registry takes the B200 methods through
    ``load_plugins`` and its benchmark parser accepts their flags next to the reference's own.
    Needs the reference (THESIS_REFERENCE or baseline/_ref); the CUDA library is not touched."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    ref = reference_dir()
    if ref is None:
        pytest.skip("the reference is not available (THESIS_REFERENCE or baseline/_ref)")
    repo = Path(__file__).resolve().parents[1]
    code = f"""
import sys
sys.path[:0] = [{str(ref)!r}, {str(repo)!r}]
from common.methods import METHODS, load_plugins
load_plugins(["thesis_b200.plugin"])
assert {{"b200_autoregressive", "b200_layerskip", "b200_layerskip_dynamic"}} <= set(METHODS), sorted(METHODS)
from evaluation.benchmark import build_parser
ap = build_parser()
a = ap.parse_args(["--method", "b200_layerskip", "--exit-layer", "8", "--gamma", "4"])
spec = METHODS[a.method]
assert spec.tag(a) == "-k8-g4" and spec.step_tokens(a) == 5 and spec.params(a) == {{"exit_layer": 8, "gamma": 4}}
a = ap.parse_args(["--method", "b200_layerskip_dynamic", "--b200-exit-layers", "4,8,12", "--b200-gamma-range", "2,8"])
assert METHODS[a.method].step_tokens(a) == 9
print("registered", sorted(m for m in METHODS if m.startswith("b200")))
"""
    r = subprocess.run([sys.executable, "-c", code], cwd=str(ref), capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    assert "b200_layerskip_dynamic" in r.stdout


def test_bench_kernel_floor():
    """The bench's per-kernel floor: at 64 tokens every projection is HBM-bound, so the floor is the
    bytes-only one; at 320 tokens the projections and the head are tensor-bound and it is higher."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench
    from thesis_b200.config import preset

    cfg = preset("llama3-8b")
    hbm, tf = 6549.4e9, 1400.3e12
    kv = bench.algorithmic("attn", 1, cfg, 576 * 64)[0]
    gemms = ("gemm_qkv", "gemm_o", "gemm_w13", "gemm_w2")
    bytes_64 = sum(bench.algorithmic(k, 64, cfg, 0.0)[0] for k in gemms) + kv
    f64 = bench.kernel_floor_ms(cfg, hbm, tf, kv, [(1, 64)], [])
    assert abs(f64 - 1000 * bytes_64 / hbm) < 1e-9
    f320 = bench.kernel_floor_ms(cfg, hbm, tf, kv, [(1, 320)], [])
    flops_320 = sum(bench.algorithmic(k, 320, cfg, 0.0)[1] for k in gemms)
    assert abs(f320 - 1000 * (flops_320 / tf + kv / hbm)) < 1e-9 and f320 > f64
    verify = bench.kernel_floor_ms(cfg, hbm, tf, kv, [(8, 64), (24, 320)], [320])
    assert 3.5 < verify < 4.5          # ms, against a bytes-only floor of ~2.8 ms
