"""Benchmark of the packed LayerSkip draft/verify step on B200 (driver contract: one JSON line).

Workload (the headline metric's configuration): synthetic LayerSkip-Llama3-8B
shape, bf16, random init (seed 0) with the residual outputs of layers >= 8 scaled by 0.1,
B=64 requests per GPU with prompt lengths uniform in [128, 512] (token ids uniform), exit layer 8,
draft length gamma=4, greedy, 512 new tokens.  The reference's datasets and checkpoints are not
available; seeded synthetic inputs with these shapes stand in for them.

A "step" is one draft/verify round over the GPU's batch: gamma shallow steps (layers [0, 8) + head)
and one verify step (the last draft through [0, 8), then 5 tokens per request through [8, 32) +
head + greedy acceptance).  Multi-GPU runs shard requests (each rank owns its own 64 requests and
a full weight replica; weak scaling); the only collective is the final gather of the generated
tokens (NCCL all_gather) inside the timed region.  ``--strong`` shards the 64 requests of the
1-GPU run over the GPUs instead (strong scaling, 64 / N requests per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--strong]

``--impl reference`` times the reference's own CPU implementation of the path - its
``common/model.py`` + ``solutions/packed.py``, installed unmodified under ``baseline/_ref`` (see
``baseline/install_reference.sh``), fp32 as the reference runs on CPU (common/cli.py:22-24) - on a
bounded sample of the same workload; without that install it falls back to the numpy port of the
same algorithm under ``oracle/`` and says so (``kind``).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

B_PER_GPU, EXIT, GAMMA, MAX_NEW = 64, 8, 4, 512
PROMPT_LEN = (128, 512)
# Tokens committed per draft/verify round by the B200 engine on this workload (64 requests, default
# --warmup 3 --steps 20), as measured by this script's own arm.  The reference arm composes a round
# from timed pieces and divides these tokens by it: the reference decodes the same prompts with
# the same greedy draft/verify rule, so a round of it commits the same tokens (its fp32 arithmetic
# can move an acceptance by a near-tie; the arm states the value it used).
TOKENS_PER_ROUND = 157.6
REF_DIR = ROOT / "baseline" / "_ref"
METRIC = "generated tokens/s/GPU, LayerSkip-8B bf16 B=64 E=8 k=4; verify-step p50 ms"
WORKLOAD = ("C3: LayerSkip-Llama3-8B-shaped bf16 (32 layers, dim 4096, 32q/8kv heads of 128, SwiGLU 14336, "
            "vocab 128256, untied), random init seed 0, residual outputs of layers >= 8 scaled by 0.1; "
            "B=64 requests per GPU, prompts U[128,512], exit layer 8, gamma 4, greedy, 512 new tokens")


def recorded_traffic(key: str):
    """dram read+write bytes per launch of a kernel group, recorded from one ncu capture in
    profiles/ncu_traffic.txt (None when that kernel group was not captured)."""
    p = ROOT / "profiles" / "ncu_traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        f = line.split()
        if len(f) == 2 and not line.startswith("#") and f[0] == key:
            return int(f[1])
    return None


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
            # nvidia-smi takes a moment to start: wait (at most 5 s) for its first sample, so that a
            # short timed region still falls inside the sampled window
            t_end = time.time() + 5.0
            while time.time() < t_end and self.proc.poll() is None:
                if Path(self.path).stat().st_size > 0:
                    break
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if self.proc is None or not self.path:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in Path(self.path).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------------- CPU baseline
def cpu_baseline(tokens_per_round: float, n_samples: int = 1) -> dict:
    """Reference algorithm on the host cores: the numpy port of common/model.py + packed.py (fp32)
    at the C3 shapes.  Bounded sample: one shallow layer (64 tokens), one deep layer (64 blocks of
    5 tokens) at the workload's mean context, and the head on 64 and 320 rows are timed; a round
    is composed from them (gamma+1 shallow passes of 8 layers, 24 deep layers, gamma+1 heads) and
    tokens/s uses the tokens per round the GPU engine measured on the same workload."""
    import numpy as np

    from oracle.model_np import OracleConfig, OracleModel
    from thesis_b200.config import preset

    try:
        from threadpoolctl import threadpool_info
        cores = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        cores = os.cpu_count() or 1
    c = preset("llama3-8b")
    oc = OracleConfig(c.vocab_size, c.dim, 1, c.n_heads, c.n_kv_heads, c.head_dim, c.intermediate_size, c.norm_eps,
                      c.rope_theta)
    from thesis_b200.synthetic import layer_shapes

    W = {f"l0.{k}": np.full(s, 0.01, dtype=np.float32) for k, s in layer_shapes(c).items()}
    W["l0.attn_norm"][:] = 1.0
    W["l0.ffn_norm"][:] = 1.0
    # the head GEMM is linear in the vocabulary: time 1/8 of it and scale (keeps host memory small)
    vshare = 8
    W["embed"] = np.full((c.vocab_size // vshare, c.dim), 0.01, dtype=np.float32)
    W["lm_head"] = W["embed"]
    W["norm"] = np.ones(c.dim, dtype=np.float32)
    B = B_PER_GPU
    ctx = (PROMPT_LEN[0] + PROMPT_LEN[1]) // 2 + MAX_NEW // 2          # mean context over a run
    m = OracleModel(oc, W, False, B, ctx + GAMMA + 64)
    rng = np.random.default_rng(0)
    m.kc[:] = rng.standard_normal(m.kc.shape[1:], dtype=np.float32)[None] * 0.1
    m.vc[:] = m.kc
    x_sh = rng.standard_normal((B, c.dim), dtype=np.float32)
    x_dp = rng.standard_normal((B * (GAMMA + 1), c.dim), dtype=np.float32)
    sh_blocks = [(r, ctx, 1) for r in range(B)]
    dp_blocks = [(r, ctx - GAMMA, GAMMA + 1) for r in range(B)]

    def layer(x, blocks):
        T = np.array([b[2] for b in blocks])
        off = np.concatenate([[0], np.cumsum(T)])
        pos = np.concatenate([np.arange(p0, p0 + t) for (_, p0, t) in blocks])
        rows = np.concatenate([np.full(t, r) for (r, _, t) in blocks])
        t0 = time.perf_counter()
        m.packed_layer(0, x, blocks, off, pos, rows)
        return time.perf_counter() - t0

    def head(x):
        t0 = time.perf_counter()
        m.head(x)
        return (time.perf_counter() - t0) * vshare

    samples = []
    for _ in range(n_samples):
        t_sh, t_dp, h_sh, h_dp = layer(x_sh, sh_blocks), layer(x_dp, dp_blocks), head(x_sh), head(x_dp)
        rnd = (GAMMA + 1) * EXIT * t_sh + GAMMA * h_sh + (c.n_layers - EXIT) * t_dp + h_dp
        samples.append(tokens_per_round / rnd)
    return {"value": float(statistics.median(samples)), "unit": "tokens/s", "cores": int(cores), "kind": "port",
            "sample": (f"numpy fp32 port of the reference path at C3 shapes: 1 shallow layer (64 tok), 1 deep layer "
                       f"(64x5 tok), head on 64 and 320 rows (1/{vshare} of the vocab, x{vshare}) at context {ctx}, composed into a round "
                       f"(5x8 shallow + 24 deep layers + 5 heads), {tokens_per_round:.1f} tokens/round, "
                       f"{n_samples} sample(s)")}


def reference_installed() -> bool:
    return (REF_DIR / "common" / "model.py").exists() and (REF_DIR / "solutions" / "packed.py").exists()


def cpu_reference_sample(tokens_per_round: float, n_samples: int = 1, warmup: int = 1) -> dict:
    """The reference's own path on the host cores: ``common/model.py`` + ``solutions/packed.py``
    from the unmodified install under baseline/_ref, fp32, torch with every host thread.  Bounded
    sample at the C3 shapes: ``build_packed`` + ``packed_layer`` on one shallow layer (64 blocks of
    1 token) and one deep layer (64 blocks of 5 tokens) at the workload's mean context, and the
    shared head on 64 and 320 rows (1/8 of the vocabulary, scaled x8: the head GEMM is linear in
    it); a round = gamma + 1 shallow packings and passes of 8 layers, gamma draft heads, one deep
    packing and 24 deep layers, one verify head."""
    import torch

    from thesis_b200.config import preset

    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    from common.model import LayerSkipLlama, LayerWeights, ModelConfig
    from solutions.packed import Block, build_packed, packed_layer

    torch.set_num_threads(len(os.sched_getaffinity(0)))
    c = preset("llama3-8b")
    vshare = 8
    B = B_PER_GPU
    ctx = (PROMPT_LEN[0] + PROMPT_LEN[1]) // 2 + MAX_NEW // 2          # mean context over a run
    max_seq = ctx + GAMMA + 64
    rc = ModelConfig(vocab_size=c.vocab_size // vshare, dim=c.dim, n_layers=1, n_heads=c.n_heads,
                     n_kv_heads=c.n_kv_heads, head_dim=c.head_dim, intermediate_size=c.intermediate_size,
                     norm_eps=c.norm_eps, rope_theta=c.rope_theta, max_position_embeddings=max_seq,
                     tie_word_embeddings=False)
    g = torch.Generator().manual_seed(0)

    def mat(r, k):
        return torch.randn(r, k, generator=g) * 0.02

    qkv_rows = (c.n_heads + 2 * c.n_kv_heads) * c.head_dim
    lw = LayerWeights(wqkv=mat(qkv_rows, c.dim), wo=mat(c.dim, c.n_heads * c.head_dim),
                      w13=mat(2 * c.intermediate_size, c.dim), w2=mat(c.dim, c.intermediate_size),
                      attn_norm=torch.ones(c.dim), ffn_norm=torch.ones(c.dim))
    m = LayerSkipLlama(rc, mat(rc.vocab_size, c.dim), [lw], torch.ones(c.dim), mat(rc.vocab_size, c.dim), "cpu",
                       torch.float32, max_seq)
    m.allocate_cache(B, max_seq)
    m.cache.k[0].normal_(0.0, 0.1, generator=g)
    m.cache.v[0].normal_(0.0, 0.1, generator=g)
    x_sh = torch.randn(B, c.dim, generator=g)
    x_dp = torch.randn(B * (GAMMA + 1), c.dim, generator=g)
    sh_blocks = [Block(r, ctx, 1) for r in range(B)]
    dp_blocks = [Block(r, ctx - GAMMA, GAMMA + 1) for r in range(B)]

    def step(x, blocks):
        t0 = time.perf_counter()
        pb = build_packed(m, blocks, "exact")
        t1 = time.perf_counter()
        packed_layer(m, 0, x, pb)
        t2 = time.perf_counter()
        m.head(x)
        t3 = time.perf_counter()
        return t1 - t0, t2 - t1, (t3 - t2) * vshare

    samples = []
    with torch.inference_mode():
        for i in range(warmup + n_samples):
            p_sh, l_sh, h_sh = step(x_sh, sh_blocks)
            p_dp, l_dp, h_dp = step(x_dp, dp_blocks)
            rnd = (GAMMA + 1) * (p_sh + EXIT * l_sh) + GAMMA * h_sh + p_dp + (c.n_layers - EXIT) * l_dp + h_dp
            if i >= warmup:
                samples.append(tokens_per_round / rnd)
    return {"value": float(statistics.median(samples)), "unit": "tokens/s", "cores": int(torch.get_num_threads()),
            "kind": "reference",
            "sample": (f"the reference's common/model.py + solutions/packed.py (baseline/_ref, unmodified), fp32 on "
                       f"{torch.get_num_threads()} torch threads, C3 shapes: build_packed + packed_layer for 1 shallow "
                       f"layer (64x1 tok) and 1 deep layer (64x5 tok) at context {ctx}, head on 64 and 320 rows "
                       f"(1/{vshare} of the vocab, x{vshare}), composed into a round (5 x (pack + 8 shallow layers) + "
                       f"4 heads + pack + 24 deep layers + head); {tokens_per_round:.1f} tokens/round; median of "
                       f"{n_samples} sample(s) after {warmup} warm-up")}


def cpu_sample(tokens_per_round: float, n_samples: int, warmup: int) -> dict:
    """The reference's own CPU path when it is installed, else the numpy port of it."""
    if reference_installed():
        return cpu_reference_sample(tokens_per_round, n_samples, warmup)
    for _ in range(warmup):
        cpu_baseline(tokens_per_round, 1)
    cb = cpu_baseline(tokens_per_round, n_samples)
    cb["sample"] += " (baseline/_ref absent: numpy port)"
    return cb


def _all_host_threads():
    """Let the CPU sample's BLAS / OpenMP pools use every core this process may run on (a
    launcher such as torchrun sets OMP_NUM_THREADS=1 for each rank)."""
    import contextlib

    try:
        import numpy  # noqa: F401 - its BLAS must be loaded for the limit to reach it
        from threadpoolctl import threadpool_limits

        return threadpool_limits(limits=len(os.sched_getaffinity(0)))
    except Exception:
        return contextlib.nullcontext()


def run_reference(args) -> None:
    if int(os.environ.get("RANK", "0")) != 0:
        return
    tpr = args.tokens_per_round
    with _all_host_threads():
        t0 = time.perf_counter()
        cb = cpu_sample(tpr, max(args.steps, 1), args.warmup)
        wall = time.perf_counter() - t0
    line = {"metric": METRIC, "value": cb["value"], "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * wall / max(args.steps, 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD + " (CPU sample)", "global_batch": B_PER_GPU, "seq_len": MAX_NEW,
                       "parallelism": "host cores"},
            "impl": "reference", "cpu_baseline": cb, "tokens_per_round": tpr,
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------- our engine
def algorithmic(kind: str, n_tok: int, cfg, ctx: float, eb: int = 2) -> tuple[float, float]:
    """(bytes, flops) of one launch of a runtime kernel kind on n_tok packed tokens."""
    D, H, Hkv, dim, I = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.dim, cfg.intermediate_size
    shapes = {"gemm_qkv": ((H + 2 * Hkv) * D, dim), "gemm_o": (dim, H * D), "gemm_w13": (2 * I, dim),
              "gemm_w2": (dim, I), "head": (cfg.vocab_size, dim)}
    if kind in shapes:
        n, k = shapes[kind]
        out = I if kind == "gemm_w13" else n
        return float(n * k * eb + n_tok * k * eb + n_tok * out * eb), float(2 * n * k * n_tok)
    if kind == "attn":
        # KV bytes read per launch: every block reads its context once per KV head
        return float(ctx * 2 * Hkv * D * eb), float(4 * H * D * ctx * n_tok / max(n_tok, 1))
    return float(2 * n_tok * dim * eb), 0.0


def kernel_floor_ms(cfg, hbm: float, tflops: float, kv_layer: float, layers_by_tokens, head_tokens) -> float:
    """Floor of a step (ms): the sum over its kernels of max(algorithmic bytes / HBM peak, FLOPs /
    sustained bf16 peak).  layers_by_tokens: (layers, packed tokens) segments; kv_layer: one layer's
    KV bytes for the batch; head_tokens: the token count of each LM-head call.  At 320 tokens the
    projections and the head are tensor-bound, so this floor is above the bytes-only one."""
    t = 0.0
    for n_layers, n_tok in layers_by_tokens:
        for kind in ("gemm_qkv", "gemm_o", "gemm_w13", "gemm_w2"):
            by, fl = algorithmic(kind, n_tok, cfg, 0.0)
            t += n_layers * max(by / hbm, fl / tflops)
        t += n_layers * kv_layer / hbm
    for n_tok in head_tokens:
        by, fl = algorithmic("head", n_tok, cfg, 0.0)
        t += max(by / hbm, fl / tflops)
    return 1000 * t


def run_ours(args) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist

    from thesis_b200.config import preset
    from thesis_b200.eesd import B200ARBatchEngine, B200SpecEngine
    from thesis_b200.engine import RunConfig
    from thesis_b200.shard import gather_outputs, shard_requests
    from thesis_b200.model import ModelWeights
    from thesis_b200.synthetic import synthetic_prompts
    from thesis_b200 import lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg = preset("llama3-8b")
    w = ModelWeights.synthetic(cfg, seed=0, dtype=torch.bfloat16, device=dev, residual_scale_from=EXIT,
                               residual_scale=0.1)
    if args.strong:
        # strong scaling: the 64 requests of the 1-GPU run, sharded over the ranks
        allp = synthetic_prompts(B_PER_GPU, cfg.vocab_size, seed=1000, min_len=PROMPT_LEN[0], max_len=PROMPT_LEN[1])
        ids = shard_requests(B_PER_GPU, rank, world)
        prompts = [allp[i] for i in ids]
        n_total = B_PER_GPU
    else:
        # weak scaling: 64 requests per GPU
        prompts = synthetic_prompts(B_PER_GPU, cfg.vocab_size, seed=1000 + rank, min_len=PROMPT_LEN[0],
                                    max_len=PROMPT_LEN[1])
        ids = [rank + world * i for i in range(B_PER_GPU)]
        n_total = B_PER_GPU * world
    nb = len(prompts)
    eng = B200SpecEngine(w, nb, PROMPT_LEN[1], MAX_NEW, (), ignore_eos=True, exit_layer=EXIT, gamma=GAMMA)
    eng.start(prompts)
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        eng.step(measured=False)
    launches0 = eng.dm.launch_count() + lib.direct_launches
    n_rec0 = len(eng.records)
    if world > 1:
        # the output gather's first NCCL all_gather sets up its channels (~30 ms, once per process);
        # it is warmed here like the steps, and runs again inside the timed region
        gather_outputs({ids[i]: eng.slots[i].output for i in range(nb)}, n_total, world, device=dev)
    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    committed = 0
    with ClockSampler(local) as clk:
        # the sampler is running before the ranks line up, so its start-up is outside the timed region
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed")          # lets a profiler select exactly the timed rounds
        ev0.record(stream)
        for _ in range(args.steps):
            committed += eng.step(measured=True)
        if world > 1:          # final output gather (the only collective): tokens generated so far
            outs = {ids[i]: eng.slots[i].output for i in range(nb)}
            gather_outputs(outs, n_total, world, device=dev)
        ev1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = ev0.elapsed_time(ev1)
    launches = eng.dm.launch_count() + lib.direct_launches - launches0
    eng.dm.check()
    # per-kernel CUDA events on a few rounds right after the timed region (events between launches
    # would serialise the programmatic-dependent-launch overlap, so the timed rounds carry none)
    eng.dm.profile(True)
    for _ in range(args.profile_rounds):
        eng.step(measured=False)
    torch.cuda.synchronize()
    recs = eng.dm.profile_records()
    eng.dm.profile(False)
    acc_rate = eng.extra_metrics()["spec"]["acceptance_rate"]
    verify = [r.forward_ms for r in eng.records[n_rec0:] if r.kind == "verify"]
    draft = [r.forward_ms for r in eng.records[n_rec0:] if r.kind == "draft"]
    t = torch.tensor([ms, float(committed)], dtype=torch.float64, device=dev)
    if world > 1:
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tot = t.clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        ms_max, tokens_all = float(mx[0]), float(tot[1])
        per = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(per, t)
        rank_ms = [round(float(x[0]) / args.steps, 3) for x in per]
    else:
        ms_max, tokens_all = ms, float(committed)
        rank_ms = [round(ms / args.steps, 3)]
    value = tokens_all / (ms_max / 1000.0)

    # ---- dominant kernel group (kind, token count) and its roofline from the live launch timings
    groups = {}
    for kind, n_tok, t_ms in recs:
        g = groups.setdefault((kind, n_tok), [0, 0.0])
        g[0] += 1
        g[1] += t_ms
    if not groups:                                   # --profile-rounds 0
        groups[("none", 0)] = [1, 1.0]
    (dk, dn), (dcount, dms) = max(groups.items(), key=lambda kv: kv[1][1])
    pk = peaks()
    ctx_mean = float(np.mean([s.pos for s in eng.slots]))
    by, fl = algorithmic(dk, dn, cfg, ctx_mean * nb)
    avg_s = dms / dcount / 1000.0
    tensor_bound = fl / max(by, 1.0) > pk["bf16_tflops_sustained"] * 1e12 / (pk["hbm_gbs"] * 1e9)
    if tensor_bound:
        achieved, peak, unit = fl / avg_s / 1e12, pk["bf16_tflops_sustained"], "TFLOP/s"
    else:
        achieved, peak, unit = by / avg_s / 1e9, pk["hbm_gbs"], "GB/s"
    total_ms = sum(g[1] for g in groups.values())
    # ---- whole-step rooflines: weight + KV bytes each step must read, over the measured HBM peak
    # (the north star's "fraction of the weight-plus-KV-bytes HBM roofline")
    L = cfg.n_layers
    w_layer = sum(algorithmic(k, 0, cfg, 0.0)[0] for k in ("gemm_qkv", "gemm_o", "gemm_w13", "gemm_w2"))
    w_head = algorithmic("head", 0, cfg, 0.0)[0]
    kv_layer = algorithmic("attn", 1, cfg, ctx_mean * nb)[0]      # one layer's KV of the batch
    draft_bytes = EXIT * (w_layer + kv_layer) + w_head
    verify_bytes = L * (w_layer + kv_layer) + w_head                    # last draft [0, E) + deep [E, L)
    hbm = pk["hbm_gbs"] * 1e9

    tflops = pk["bf16_tflops_sustained"] * 1e12

    def step_roof(nbytes, ms, kfloor):
        return {"bytes": nbytes, "floor_ms": 1000 * nbytes / hbm, "measured_ms": ms,
                "frac": (1000 * nbytes / hbm) / ms if ms else None,
                "kernel_floor_ms": kfloor, "frac_of_kernel_floor": kfloor / ms if ms else None}
    kf_draft = kernel_floor_ms(cfg, hbm, tflops, kv_layer, [(EXIT, nb)], [nb])
    kf_verify = kernel_floor_ms(cfg, hbm, tflops, kv_layer, [(EXIT, nb), (L - EXIT, nb * (GAMMA + 1))],
                                [nb * (GAMMA + 1)])
    share = {f"{k}@{n}": round(v[1] / total_ms, 4) for (k, n), v in sorted(groups.items(), key=lambda kv: -kv[1][1])}

    # ---- losslessness on the headline workload: the speculative output of a fixed subset of the
    # requests equals the same engine's autoregressive output, token for token
    lossless = None
    if args.lossless_requests > 0:
        sub = prompts[:args.lossless_requests]
        rc_ll = RunConfig(mode="static", keep_outputs=True)
        toks = []
        for make in (lambda: B200ARBatchEngine(w, len(sub), PROMPT_LEN[1], args.lossless_new, (), ignore_eos=True),
                     lambda: B200SpecEngine(w, len(sub), PROMPT_LEN[1], args.lossless_new, (), ignore_eos=True,
                                            exit_layer=EXIT, gamma=GAMMA)):
            e = make()
            res = e.run(sub, rc_ll)
            by = {c["pid"]: c["tokens"] for c in res["completions"]}
            toks.append([by[p.pid] for p in sub])
            e.free()
        lossless = {"spec_equals_ar": toks[0] == toks[1], "requests": len(sub), "new_tokens": args.lossless_new,
                    "check": "B200SpecEngine vs B200ARBatchEngine token lists on the first requests of this rank"}
    eng.free()
    del eng
    torch.cuda.empty_cache()

    # ---- strong scaling next to weak scaling (multi-GPU runs): the 64 requests of the 1-GPU run
    # sharded over the ranks, run concurrently, timed like the weak case
    strong = None
    if world > 1 and not args.strong and not args.no_strong_sub:
        allp = synthetic_prompts(B_PER_GPU, cfg.vocab_size, seed=1000, min_len=PROMPT_LEN[0], max_len=PROMPT_LEN[1])
        sids = shard_requests(B_PER_GPU, rank, world)
        sp_prompts = [allp[i] for i in sids]
        s_eng = B200SpecEngine(w, len(sp_prompts), PROMPT_LEN[1], MAX_NEW, (), ignore_eos=True, exit_layer=EXIT,
                               gamma=GAMMA)
        s_eng.start(sp_prompts)
        for _ in range(args.warmup):
            s_eng.step(measured=False)
        gather_outputs({sids[i]: s_eng.slots[i].output for i in range(len(sids))}, B_PER_GPU, world, device=dev)
        n0 = len(s_eng.records)
        dist.barrier()
        torch.cuda.synchronize()
        s_committed = 0
        ev0.record(stream)
        for _ in range(args.steps):
            s_committed += s_eng.step(measured=True)
        gather_outputs({sids[i]: s_eng.slots[i].output for i in range(len(sids))}, B_PER_GPU, world, device=dev)
        ev1.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        st = torch.tensor([ev0.elapsed_time(ev1), float(s_committed)], dtype=torch.float64, device=dev)
        per = [torch.zeros_like(st) for _ in range(world)]
        dist.all_gather(per, st)
        s_ms = max(float(x[0]) for x in per)
        s_tok = sum(float(x[1]) for x in per)
        sv = [r.forward_ms for r in s_eng.records[n0:] if r.kind == "verify"]
        sd = [r.forward_ms for r in s_eng.records[n0:] if r.kind == "draft"]
        strong = {"value": s_tok / (s_ms / 1000.0), "unit": "tokens/s", "requests_total": B_PER_GPU,
                  "requests_per_gpu": len(sids), "ms_per_step": s_ms / args.steps,
                  "rank_ms_per_step": [round(float(x[0]) / args.steps, 3) for x in per],
                  "verify_step_p50_ms": statistics.median(sv) if sv else None,
                  "draft_step_p50_ms": statistics.median(sd) if sd else None,
                  "limiter": (f"every rank streams the full 16 GB of weights per round for {len(sids)} requests "
                              "(weight-bound steps), plus the final NCCL all_gather of the outputs")}
        s_eng.free()
        del s_eng
        torch.cuda.empty_cache()

    # ---- end to end through the public engine API (host prompts in, token lists out)
    e2e = None
    if not args.no_e2e:
        e2e_eng = B200SpecEngine(w, nb, PROMPT_LEN[1], args.e2e_new, (), ignore_eos=True, exit_layer=EXIT,
                                 gamma=GAMMA)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        res = e2e_eng.run(prompts, RunConfig(mode="static", keep_outputs=True))
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        toks = sum(c["generated"] for c in res["completions"])
        tt = torch.tensor([wall, float(toks)], dtype=torch.float64, device=dev)
        if world > 1:
            mx = tt.clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
            tot = tt.clone()
            dist.all_reduce(tot, op=dist.ReduceOp.SUM)
            wall, toks = float(mx[0]), float(tot[1])
        n_steps = max(len(e2e_eng.records), 1)
        e2e = {"value": toks / wall, "unit": "tokens/s", "h2d_bytes_per_step": int(e2e_eng.h2d_bytes / n_steps),
               "d2h_bytes_per_step": int(e2e_eng.d2h_bytes / n_steps), "new_tokens_per_request": args.e2e_new,
               "includes": "prefill of all prompts, every draft/verify step, host bookkeeping"}
        e2e_eng.free()

    if rank == 0:
        acc_tokens_per_round = committed / max(args.steps, 1)
        cb = None
        if not args.no_cpu and world == 1:         # the CPU baseline is taken on 1 GPU runs only
            with _all_host_threads():               # same sample count and warm-up as the reference arm
                cb = cpu_sample(acc_tokens_per_round, args.steps, args.warmup)
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "rank_ms_per_step": rank_ms,
            "higher_is_better": True, "scaling": "strong" if args.strong else "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD if not args.strong else WORKLOAD.replace(
                           "B=64 requests per GPU", f"B=64 requests in total, {nb} per GPU"),
                       "global_batch": n_total, "seq_len": MAX_NEW,
                       "parallelism": f"request-sharded x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2: each round streams the 16 GB of weights",
                       "value_is": "aggregate over all GPUs"},
            "tokens_per_gpu_per_s": value / world,
            "verify_step_p50_ms": statistics.median(verify) if verify else None,
            "draft_step_p50_ms": statistics.median(draft) if draft else None,
            "tokens_per_round_per_gpu": acc_tokens_per_round,
            "acceptance_rate": acc_rate,
            "clocks": clk.summary(),
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor" if tensor_bound else "hbm", "achieved": achieved, "peak": peak,
                         "unit": unit, "frac": achieved / peak, "traffic": recorded_traffic(f"{dk}@{dn}"),
                         "traffic_source": "dram read+write bytes per launch from the ncu capture recorded in "
                                           "profiles/ncu_traffic.txt (an earlier run of the same kernel, not this one)",
                         "kernel": f"{dk}@{dn} tokens",
                         "launches": dcount, "avg_ms": avg_s * 1000, "peak_source": pk["source"],
                         "timing": f"per-launch CUDA events over {args.profile_rounds} profiled rounds after the timed region"},
            "kernel_time_share": share,
            "step_roofline": {
                "peak_gbs": pk["hbm_gbs"], "peak_source": pk["source"],
                "verify": step_roof(verify_bytes, statistics.median(verify) if verify else None, kf_verify),
                "draft": step_roof(draft_bytes, statistics.median(draft) if draft else None, kf_draft),
                "round": step_roof(GAMMA * draft_bytes + verify_bytes, ms_max / args.steps,
                                   GAMMA * kf_draft + kf_verify),
                "bytes_are": "bf16 weights of the layers each step runs + LM head + the batch's KV cache at the mean "
                             "context; activations excluded",
                "kernel_floor_is": "sum over the step's kernels of max(bytes / HBM peak, FLOPs / sustained bf16 peak); "
                                   "frac (bytes only) is the north star's measure"},
            "e2e": e2e,
            "cpu_baseline": cb,
            "lossless": lossless,
            "strong": strong,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-new", type=int, default=MAX_NEW, help="new tokens per request in the end-to-end run")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--strong", action="store_true",
                    help="strong scaling: the 64 requests of the 1-GPU run sharded over the GPUs (default: 64 per GPU)")
    ap.add_argument("--profile-rounds", type=int, default=3, help="profiled rounds after the timed region")
    ap.add_argument("--lossless-requests", type=int, default=8,
                    help="requests of the speculative == autoregressive check after the timed region (0 = skip)")
    ap.add_argument("--lossless-new", type=int, default=64, help="new tokens per request of that check")
    ap.add_argument("--no-strong-sub", action="store_true",
                    help="multi-GPU runs: skip the strong-scaling measurement reported next to weak scaling")
    ap.add_argument("--tokens-per-round", type=float, default=TOKENS_PER_ROUND,
                    help="reference arm: tokens committed per round (default: the B200 engine's measured value "
                         "on this workload)")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
