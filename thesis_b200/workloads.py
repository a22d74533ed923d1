"""Measurement of the BASELINE configurations beyond the headline one (one JSON line each).

    python -m thesis_b200.workloads c2 [--requests 64] [--new 256]
    python -m thesis_b200.workloads c4 [--requests 32] [--new 256]
    python -m thesis_b200.workloads c5 [--requests 256] [--rate 40] [--budget 256]
    torchrun --nproc-per-node 8 -m thesis_b200.workloads c5        # config 5 as specified: 8 GPUs
    python -m thesis_b200.workloads strong [--rounds 20]
    python -m thesis_b200.workloads lossless [--new 512]
    python -m thesis_b200.workloads refgpu [--new 512]

c2  Llama3.2-1B shape (16 layers, dim 2048, 32 / 8 heads of 64, SwiGLU 8192, vocab 128256, tied
    embeddings, RoPE theta 500000), bf16, residual outputs of layers >= 6 scaled by 0.1; batch 64,
    prompt lengths uniform in 64..1024 (several 512-token prefill chunks), exit layer 6, gamma 6,
    256 new tokens greedy, through the public engine API (``B200SpecEngine.run``), next to the
    autoregressive engine on the same requests.  Reports decode throughput, the step p50s and the
    verify step's fraction of its weight + KV HBM floor.
c4  Llama2-7B shape (32 layers, dim 4096, 32 heads MHA of 128, SwiGLU 11008, vocab 32000, RoPE
    theta 10000), bf16, residual outputs of layers >= 4 scaled by 0.1; batch 32, prompt lengths
    lognormal (median 256, clipped to 32..1536), a per-request exit layer from {4, 8, 12} and a
    per-request draft length drawn from 2..8 every round (``B200DynamicSpecEngine``), 256 new
    tokens greedy.  Reports decode throughput next to the autoregressive engine's on the same
    requests, and whether the two outputs are identical.
c5  Llama3-8B shape, bf16, residual outputs of layers >= 8 scaled by 0.1; 256 slots, Poisson
    arrivals at ``--rate`` requests/s, prompt lengths lognormal (median 512, clipped to 64..2048),
    output lengths uniform in 128..1024, exit layer 8, gamma 4, new-request prefill piggybacked
    on the draft/verify steps (``B200ServingEngine.run_poisson``).  Reports throughput, TTFT and
    TPOT of the measured requests.  Under torchrun every rank serves its own request stream (the
    requests shard across the GPUs, seeds differ per rank); rank 0 reports the aggregate wall-clock
    throughput and every rank's latencies.

strong  Strong scaling of config 3 (Llama3-8B shape, E=8, gamma=4, 64 requests in total, prompts
    U[128,512]) over 1, 2, 4 and 8 GPUs, measured shard by shard on one GPU: ranks share nothing
    but the final output gather, so an N-GPU run is N independent engines of 64 / N requests
    (`bench.py --strong --gpus N` runs them concurrently).  For each N every shard runs 3 warm-up
    and ``--rounds`` timed draft/verify rounds (CUDA events); the aggregate is all shards' tokens
    over the slowest shard's time, as in the bench.

lossless  Config 3 in full (Llama3-8B shape, bf16, 64 requests, prompts U[128,512], E=8, gamma=4,
    ``--new`` tokens): the speculative engine's output against the autoregressive engine's, token
    for token, for every request (the bench line checks a subset only).

refgpu  Config 3 through the reference's OWN packed engine (``solutions/engine.py`` EESDEngine,
    fixed schedule, gamma 4, exit layer 8: PyTorch eager with cuBLAS and SDPA) on this GPU, on
    the same synthetic weights (shared, not copied) and prompts, next to this library's engine.
    The reference is imported from ``baseline/_ref`` (``baseline/install_reference.sh``).

Weights and prompts are seeded synthetic stand-ins for the checkpoints and datasets the
reference would use; no dataset item is reproduced.
"""

from __future__ import annotations

import argparse
import json
import time

import numpy as np
import torch

from .config import preset
from .engine import RunConfig
from .model import ModelWeights
from .synthetic import Prompt, synthetic_prompts


def run_c4(args) -> dict:
    from .dynamic import B200DynamicSpecEngine
    from .eesd import B200ARBatchEngine

    cfg = preset("llama2-7b")
    w = ModelWeights.synthetic(cfg, seed=0, dtype=torch.bfloat16, device="cuda", residual_scale_from=4,
                               residual_scale=0.1)
    prompts = synthetic_prompts(args.requests, cfg.vocab_size, seed=7, min_len=32, max_len=1536, lengths="lognormal",
                                median=256)
    mp = max(len(p.tokens) for p in prompts)
    rc = RunConfig(mode="static", keep_outputs=True)
    out = {}
    def dyn(schedule):
        return lambda: B200DynamicSpecEngine(w, args.requests, mp, args.new, (), ignore_eos=True,
                                             exit_layers=(4, 8, 12), gamma_range=(2, 8), schedule=schedule)

    for name, make in (("dynamic", dyn("lockstep")), ("dynamic_unified", dyn("unified")),
                       ("ar", lambda: B200ARBatchEngine(w, args.requests, mp, args.new, (), ignore_eos=True))):
        eng = make()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        res = eng.run(prompts, rc)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        m = res["metrics"]
        toks = {c["pid"]: c["tokens"] for c in res["completions"]}
        out[name] = {"throughput_tok_s": m["throughput_tok_s"], "e2e_tok_s": sum(len(t) for t in toks.values()) / wall,
                     "steps": m["steps"], "spec": m.get("spec"), "tokens": toks}
        eng.free()
        del eng
        torch.cuda.empty_cache()
    ar_tokens = out["ar"].pop("tokens")
    same = out["dynamic"].pop("tokens") == ar_tokens
    same_unified = out["dynamic_unified"].pop("tokens") == ar_tokens
    return {"workload": "c4", "metric": "generated tokens/s (decode device time), 1 GPU", "unit": "tokens/s",
            "value": out["dynamic"]["throughput_tok_s"], "unified_value": out["dynamic_unified"]["throughput_tok_s"],
            "ar_value": out["ar"]["throughput_tok_s"],
            "speedup_vs_ar": out["dynamic"]["throughput_tok_s"] / out["ar"]["throughput_tok_s"],
            "unified_speedup_vs_ar": out["dynamic_unified"]["throughput_tok_s"] / out["ar"]["throughput_tok_s"],
            "identical_to_ar": same, "unified_identical_to_ar": same_unified, "requests": args.requests,
            "new_tokens": args.new, "detail": out}


def run_c2(args) -> dict:
    from .eesd import B200ARBatchEngine, B200SpecEngine

    cfg = preset("llama3-1b")
    E, gamma = 6, 6
    w = ModelWeights.synthetic(cfg, seed=0, dtype=torch.bfloat16, device="cuda", residual_scale_from=E,
                               residual_scale=0.1)
    prompts = synthetic_prompts(args.requests, cfg.vocab_size, seed=11, min_len=64, max_len=1024)
    mp = max(len(p.tokens) for p in prompts)
    rc = RunConfig(mode="static", keep_outputs=True)
    out = {}
    for name, make in (("spec", lambda: B200SpecEngine(w, args.requests, mp, args.new, (), ignore_eos=True,
                                                       exit_layer=E, gamma=gamma)),
                       ("ar", lambda: B200ARBatchEngine(w, args.requests, mp, args.new, (), ignore_eos=True))):
        eng = make()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        res = eng.run(prompts, rc)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        m = res["metrics"]
        toks = {c["pid"]: c["tokens"] for c in res["completions"]}
        out[name] = {"throughput_tok_s": m["throughput_tok_s"], "e2e_tok_s": sum(len(t) for t in toks.values()) / wall,
                     "steps": m["steps"], "spec": m.get("spec"), "tokens": toks}
        eng.free()
        del eng
        torch.cuda.empty_cache()
    same = out["spec"].pop("tokens") == out["ar"].pop("tokens")
    # verify step floor: every layer's weights (the last draft through [0, E), the deep tokens through
    # [E, L)), the LM head, and the batch's KV at the mean context in all layers, at the measured HBM peak
    peaks_file = __import__("pathlib").Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    hbm = json.loads(peaks_file.read_text())["hbm_gbs"] if peaks_file.exists() else 6650.0
    lens = np.array([len(p.tokens) for p in prompts])
    ctx = float(lens.mean() + args.new / 2)
    w_bytes = cfg.n_layers * cfg.layer_param_count * 2 + cfg.vocab_size * cfg.dim * 2
    kv_bytes = cfg.n_layers * args.requests * ctx * cfg.kv_bytes_per_position_layer(2)
    floor_ms = 1000 * (w_bytes + kv_bytes) / (hbm * 1e9)
    v50 = out["spec"]["steps"]["verify"]["p50_ms"]
    return {"workload": "c2", "metric": "generated tokens/s (decode device time), 1 GPU", "unit": "tokens/s",
            "value": out["spec"]["throughput_tok_s"], "ar_value": out["ar"]["throughput_tok_s"],
            "speedup_vs_ar": out["spec"]["throughput_tok_s"] / out["ar"]["throughput_tok_s"],
            "identical_to_ar": same, "requests": args.requests, "new_tokens": args.new,
            "verify_step": {"p50_ms": v50, "bytes": w_bytes + kv_bytes, "floor_ms": floor_ms, "frac": floor_ms / v50,
                            "mean_context": ctx, "peak_gbs": hbm},
            "detail": out}


def run_c5(args) -> dict:
    from .serving import B200ServingEngine

    cfg = preset("llama3-8b")
    w = ModelWeights.synthetic(cfg, seed=0, dtype=torch.bfloat16, device="cuda", residual_scale_from=8,
                               residual_scale=0.1)
    n_pool = args.requests + args.warm
    rank = int(__import__("os").environ.get("RANK", "0"))
    base = synthetic_prompts(n_pool, cfg.vocab_size, seed=9 + 1000 * rank, min_len=64, max_len=2048,
                             lengths="lognormal", median=512, pid_prefix=f"r{rank}p")
    rng = np.random.default_rng(9 + 1000 * rank)
    prompts = [Prompt(p.pid, p.tokens, max_new=int(rng.integers(128, 1025))) for p in base]
    eng = B200ServingEngine(w, args.slots, 2048, 1024, (), ignore_eos=True, exit_layer=8, gamma=4,
                            piggyback_budget=args.budget)
    res = eng.run_poisson(prompts, rate_per_s=args.rate, n_requests=args.requests, warm_requests=args.warm,
                          seed=rank)
    eng.dm.check()
    m = res["metrics"]
    return {"workload": "c5", "metric": "generated tokens/s (wall clock, open loop), 1 GPU", "unit": "tokens/s",
            "value": m["wall_throughput_tok_s"], "slots": args.slots, "rate_per_s": args.rate,
            "requests_measured": m["evaluated_completions"], "metrics": m}


def run_strong(args) -> dict:
    from .eesd import B200SpecEngine
    from .shard import shard_requests

    cfg = preset("llama3-8b")
    w = ModelWeights.synthetic(cfg, seed=0, dtype=torch.bfloat16, device="cuda", residual_scale_from=8,
                               residual_scale=0.1)
    allp = synthetic_prompts(64, cfg.vocab_size, seed=1000, min_len=128, max_len=512)
    rows = []
    for n in (1, 2, 4, 8):
        shard_ms, tokens = [], 0
        for r in range(n):
            prompts = [allp[i] for i in shard_requests(64, r, n)]
            eng = B200SpecEngine(w, len(prompts), 512, 512, (), ignore_eos=True, exit_layer=8, gamma=4)
            eng.start(prompts)
            for _ in range(3):
                eng.step(measured=False)
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            got = sum(eng.step(measured=True) for _ in range(args.rounds))
            b.record()
            torch.cuda.synchronize()
            shard_ms.append(a.elapsed_time(b))
            tokens += got
            eng.free()
            del eng
            torch.cuda.empty_cache()
        agg = tokens / (max(shard_ms) / 1000.0)
        rows.append({"gpus": n, "requests_per_gpu": 64 // n, "ms_per_round_max": max(shard_ms) / args.rounds,
                     "ms_per_round_min": min(shard_ms) / args.rounds, "aggregate_tok_s": agg})
    for r in rows:
        r["speedup"] = r["aggregate_tok_s"] / rows[0]["aggregate_tok_s"]
        r["efficiency"] = r["speedup"] / r["gpus"]
    return {"workload": "strong", "metric": "generated tokens/s, 64 requests in total (strong scaling)",
            "unit": "tokens/s", "rounds": args.rounds, "rows": rows}


def run_lossless(args) -> dict:
    from .eesd import B200ARBatchEngine, B200SpecEngine

    cfg = preset("llama3-8b")
    w = ModelWeights.synthetic(cfg, seed=0, dtype=torch.bfloat16, device="cuda", residual_scale_from=8,
                               residual_scale=0.1)
    prompts = synthetic_prompts(64, cfg.vocab_size, seed=1000, min_len=128, max_len=512)
    rc = RunConfig(mode="static", keep_outputs=True)
    out = {}
    for name, make in (("ar", lambda: B200ARBatchEngine(w, 64, 512, args.new, (), ignore_eos=True)),
                       ("spec", lambda: B200SpecEngine(w, 64, 512, args.new, (), ignore_eos=True, exit_layer=8,
                                                       gamma=4))):
        eng = make()
        res = eng.run(prompts, rc)
        eng.dm.check()
        out[name] = {c["pid"]: list(c["tokens"]) for c in res["completions"]}
        out[name + "_metrics"] = res["metrics"]
        eng.free()
        del eng
        torch.cuda.empty_cache()
    same = [out["ar"][p.pid] == out["spec"][p.pid] for p in prompts]
    first_diff = None
    for p in prompts:
        a, b = out["ar"][p.pid], out["spec"][p.pid]
        if a != b:
            first_diff = {"pid": p.pid, "index": next(i for i in range(min(len(a), len(b)) + 1)
                                                      if i >= min(len(a), len(b)) or a[i] != b[i])}
            break
    sm = out["spec_metrics"]
    return {"workload": "lossless", "config": "C3: Llama3-8B shape, bf16, 64 requests, prompts U[128,512], E=8, "
                                              f"gamma=4, {args.new} new tokens",
            "requests": len(prompts), "tokens_per_request": args.new,
            "identical_requests": int(sum(same)), "spec_equals_ar": all(same), "first_difference": first_diff,
            "acceptance_rate": sm.get("spec", {}).get("acceptance_rate"),
            "spec_throughput_tok_s": sm.get("throughput_tok_s"), "ar_throughput_tok_s": out["ar_metrics"].get("throughput_tok_s")}


def run_refgpu(args) -> dict:
    import statistics
    import sys
    from pathlib import Path

    from .eesd import B200SpecEngine

    ref = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
    if not (ref / "solutions" / "engine.py").exists():
        return {"workload": "refgpu", "unavailable": "the reference is not installed under baseline/_ref"}
    sys.path.insert(0, str(ref))
    from common.data import Prompt as RefPrompt
    from common.model import LayerSkipLlama, LayerWeights, ModelConfig as RefConfig
    from solutions.cost_model import synthetic_cost_model
    from solutions.engine import EESDEngine, EngineConfig

    cfg = preset("llama3-8b")
    w = ModelWeights.synthetic(cfg, seed=0, dtype=torch.bfloat16, device="cuda", residual_scale_from=8,
                               residual_scale=0.1)
    prompts = synthetic_prompts(64, cfg.vocab_size, seed=1000, min_len=128, max_len=512)
    t = w.t
    rc = RefConfig(vocab_size=cfg.vocab_size, dim=cfg.dim, n_layers=cfg.n_layers, n_heads=cfg.n_heads,
                   n_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, intermediate_size=cfg.intermediate_size,
                   norm_eps=cfg.norm_eps, rope_theta=cfg.rope_theta, max_position_embeddings=2048,
                   tie_word_embeddings=cfg.tie_word_embeddings, rope_scaling=cfg.rope_scaling)
    layers = [LayerWeights(wqkv=t[f"l{i}.wqkv"], wo=t[f"l{i}.wo"], w13=t[f"l{i}.w13"], w2=t[f"l{i}.w2"],
                           attn_norm=t[f"l{i}.attn_norm"], ffn_norm=t[f"l{i}.ffn_norm"]) for i in range(cfg.n_layers)]
    model = LayerSkipLlama(rc, t["embed"], layers, t["norm"], t["lm_head"], w.device, torch.bfloat16, 2048)
    rp = [RefPrompt(p.pid, list(p.tokens)) for p in prompts]
    eng = EESDEngine(model, 64, 512, args.new, (), EngineConfig(mode="spec", sched="fixed", gamma=4, k=8),
                     synthetic_cost_model(model.cfg))
    res = eng.run(rp, "static", keep_outputs=True)
    m = res["metrics"]
    deep = [r.ms for r in eng.records if r.kind == "deep" and r.measured]
    shallow = [r.ms for r in eng.records if r.kind == "shallow" and r.measured]
    ref_tok = {c["pid"]: list(c["tokens"]) for c in res["completions"]}
    del eng, model
    torch.cuda.empty_cache()
    ours = B200SpecEngine(w, 64, 512, args.new, (), ignore_eos=True, exit_layer=8, gamma=4)
    r2 = ours.run(prompts, RunConfig(mode="static", keep_outputs=True))
    ours.dm.check()
    om = r2["metrics"]
    same = sum(ref_tok.get(c["pid"]) == list(c["tokens"]) for c in r2["completions"])

    def common_prefix(a, b):
        n = 0
        while n < min(len(a), len(b)) and a[n] == b[n]:
            n += 1
        return n
    prefix = [common_prefix(ref_tok.get(c["pid"], []), list(c["tokens"])) for c in r2["completions"]]
    return {"workload": "refgpu", "config": f"C3: Llama3-8B shape, bf16, 64 requests, prompts U[128,512], E=8, "
                                            f"gamma=4, {args.new} new tokens, static mode, one B200",
            "reference": {"engine": "solutions/engine.py EESDEngine (fixed, gamma 4, k 8)",
                          "throughput_tok_s": m["throughput_tok_s"], "wall_throughput_tok_s": m["wall_throughput_tok_s"],
                          "verify_step_p50_ms": statistics.median(deep) if deep else None,
                          "draft_step_p50_ms": statistics.median(shallow) if shallow else None,
                          "acceptance_rate": m["acceptance_rate"]},
            "ours": {"engine": "thesis_b200 B200SpecEngine", "throughput_tok_s": om["throughput_tok_s"],
                     "wall_throughput_tok_s": om.get("wall_throughput_tok_s"),
                     "verify_step_p50_ms": om["steps"]["verify"]["p50_ms"],
                     "draft_step_p50_ms": om["steps"]["draft"]["p50_ms"],
                     "acceptance_rate": om["spec"]["acceptance_rate"]},
            "speedup_decode": om["throughput_tok_s"] / m["throughput_tok_s"] if m["throughput_tok_s"] else None,
            "speedup_wall": (om["wall_throughput_tok_s"] / m["wall_throughput_tok_s"]
                             if om.get("wall_throughput_tok_s") and m["wall_throughput_tok_s"] else None),
            "requests_with_identical_tokens": int(same),
            "common_prefix_tokens": {"mean": float(np.mean(prefix)), "min": int(min(prefix)), "max": int(max(prefix))},
            "note": "both in bf16 with different kernels; bf16 outputs may differ after a near-tie, so identical "
                    "tokens are counted, not required"}


def _multi_rank_c5(args) -> None:
    """Config 5 over the ranks of a torchrun launch: one request stream per GPU, no collective on the
    data path; the per-rank results are gathered once at the end."""
    import datetime
    import os

    import torch.distributed as dist

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    try:
        res = run_c5(args)
        m = res["metrics"]
        mine = {"rank": rank, "wall_tok_s": m["wall_throughput_tok_s"], "measured_tokens": m["measured_tokens"],
                "wall_s": m["wall_s"], "decode_tok_s": m["throughput_tok_s"], "ttft_ms_mean": m["ttft_ms_mean"],
                "ttft_ms_p99": m["ttft_ms_p99"], "tpot_ms_mean": m["tpot_ms_mean"], "tpot_ms_p99": m["tpot_ms_p99"],
                "acceptance_rate": m["acceptance_rate"], "queue_left": m["queue_left"],
                "requests_measured": m["evaluated_completions"]}
        allr = [None] * world
        dist.all_gather_object(allr, mine)
        if rank == 0:
            wall = max(r["wall_s"] for r in allr)
            tokens = sum(r["measured_tokens"] for r in allr)
            print(json.dumps({"workload": "c5", "metric": "generated tokens/s (wall clock, open loop), all GPUs",
                              "unit": "tokens/s", "value": tokens / wall, "n_gpus": world, "slots_per_gpu": args.slots,
                              "rate_per_s_per_gpu": args.rate, "requests_per_gpu": args.requests, "ranks": allr}),
                  flush=True)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("workload", choices=["c2", "c4", "c5", "strong", "lossless", "refgpu"])
    ap.add_argument("--rounds", type=int, default=20)
    ap.add_argument("--requests", type=int, default=None)
    ap.add_argument("--new", type=int, default=None, help="new tokens per request (lossless: 512, else 256)")
    ap.add_argument("--rate", type=float, default=40.0)
    ap.add_argument("--slots", type=int, default=256)
    ap.add_argument("--warm", type=int, default=16)
    ap.add_argument("--budget", type=int, default=256)
    args = ap.parse_args(argv)
    if args.requests is None:
        args.requests = {"c2": 64, "c4": 32}.get(args.workload, 256)
    if args.new is None:
        args.new = 512 if args.workload in ("lossless", "refgpu") else 256
    if args.workload == "c5" and int(__import__("os").environ.get("WORLD_SIZE", "1")) > 1:
        _multi_rank_c5(args)
        return
    res = {"c2": run_c2, "c4": run_c4, "c5": run_c5, "strong": run_strong, "lossless": run_lossless,
           "refgpu": run_refgpu}[args.workload](args)
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
