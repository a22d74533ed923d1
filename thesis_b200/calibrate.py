"""Calibration of the reference's step-cost model on the B200 engine.

    python -m thesis_b200.calibrate [--preset llama3-8b] [--out FILE] [--validate] [--quick]

The reference's adaptive schedulers (the M1 knee rule, ASPIRE, the FSM) price shallow, deep and
prefill steps with the portable cost model of solutions/cost_model.py:1-31, calibrated once per
GPU by solutions/calibrate.py:1-20.  This module measures the same quantities through this
package's kernels and writes a JSON in the layout solutions/cost_model.py:202-216
(``load_cost_model``) reads - "gpu" (the GPUParams fields), "model_dims" and "linear" - so the
reference's schedulers run on B200 step costs unchanged.

Measured through the C ABI with CUDA events (medians):

  bw        bytes/ms of a 1-token GEMM through a 28672 x 8192 bf16 weight
  flops     flop/ms of an 8192 x 8192 x 8192 bf16 GEMM
  F_eff     highest flop/ms of the layer's GEMMs (QKV, O, W13 + SwiGLU, W2) over 1..512 tokens
  knee      hinge fit t = a + b max(n - knee, 0) of one packed layer, n requests x 1 token
  t_op      ms per launch of a one-CTA kernel issued back to back
  n_op      launches of one packed layer and of one head call; a packed segment's metadata is one
            host-to-device copy (there are no attention buckets: n_op_bucket = 0)
  linear    least squares a + b n + c KV of one packed layer over a (requests, tokens per request,
            context) grid, and head_a + head_b n

``--validate`` times real shallow steps, deep steps and prefill chunks of the engine's packed path
(full depth) and reports the MAPE of the roofline, roofline-peak and linear predictions, as
solutions/calibrate.py:169-225 does.  Weights and the KV cache hold seeded random values: step
times do not depend on them.
"""

from __future__ import annotations

import argparse
import json
from dataclasses import replace
from pathlib import Path

import numpy as np
import torch

from . import lib
from .config import ModelConfig, preset
from .model import DeviceModel, ModelWeights

N_GRID = (1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256, 320, 384, 448, 512)


def _t(fn, reps: int = 20, warm: int = 5) -> float:
    """Median device time of fn() in ms: `warm` untimed calls, then `reps` calls each bracketed by
    its own pair of CUDA events."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    pairs = []
    for _ in range(reps):
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record()
        fn()
        ev[1].record()
        pairs.append(ev)
    torch.cuda.synchronize()
    return float(np.median([a.elapsed_time(b) for a, b in pairs]))


# ---------------------------------------------------------------------------------- fits
def _lsq(X: np.ndarray, y: np.ndarray) -> np.ndarray:
    """Least-squares coefficients through a QR factorisation of the design matrix."""
    q, r = np.linalg.qr(X)
    return np.linalg.solve(r, q.T @ y)


def hinge_knee(ns, ms, grid=None) -> tuple:
    """Knee of the hinge t(n) = a + b max(n - knee, 0), b >= 0, that minimises the squared relative
    error.  For a fixed knee the model is linear in (a, b) and solved directly; the knee is searched
    over the measured token counts (or `grid`), then refined inside the two neighbouring intervals
    of the best one by golden-section search (the error is smooth between measured points).
    Returns (knee, (a, b))."""
    n = np.asarray(ns, dtype=np.float64)
    y = np.asarray(ms, dtype=np.float64)
    w = 1.0 / y

    def fit(kn: float):
        X = np.stack([np.ones_like(n), np.maximum(n - kn, 0.0)], axis=1) * w[:, None]
        coef = _lsq(X, y * w)
        if coef[1] < 0:
            return np.inf, coef
        return float(np.sum((X @ coef - y * w) ** 2)), coef

    pts = np.unique(n)
    cand = np.asarray(grid, dtype=np.float64) if grid is not None else pts[:-1]
    errs = [fit(k)[0] for k in cand]
    i = int(np.argmin(errs))
    if not np.isfinite(errs[i]):
        raise ValueError("no knee with a non-negative slope")
    best_k, best_e = float(cand[i]), errs[i]
    if grid is None and best_e > 0:
        lo = pts[max(i - 1, 0)]
        hi = pts[min(i + 1, len(pts) - 1)]
        g = (np.sqrt(5.0) - 1) / 2
        a, b = lo, hi
        for _ in range(40):
            c, d = b - g * (b - a), a + g * (b - a)
            if fit(c)[0] < fit(d)[0]:
                b = d
            else:
                a = c
        k = 0.5 * (a + b)
        if fit(k)[0] < best_e * (1 - 1e-9):
            best_k, best_e = float(k), fit(k)[0]
    coef = fit(best_k)[1]
    return best_k, (float(coef[0]), float(coef[1]))


def fit_linear(layer_rows, head_rows) -> dict:
    """Plain least squares of t_layer = a + b n + c KV (n packed tokens, KV positions read) and
    t_head = head_a + head_b n."""
    a, b, c = _lsq(np.array([[1.0, r["n"], r["kv"]] for r in layer_rows]), np.array([r["ms"] for r in layer_rows]))
    ha, hb = _lsq(np.array([[1.0, h["n"]] for h in head_rows]), np.array([h["ms"] for h in head_rows]))
    return {"a": float(a), "b": float(b), "c": float(c), "head_a": float(ha), "head_b": float(hb)}


def model_dims(cfg: ModelConfig, dtype_bytes: int = 2) -> dict:
    """The ModelDims fields of solutions/cost_model.py:44-70 for this configuration."""
    return {"n_layers": cfg.n_layers, "dim": cfg.dim, "vocab": cfg.vocab_size,
            "layer_params": cfg.layer_param_count, "head_params": cfg.vocab_size * cfg.dim + cfg.dim,
            "kv_bytes_per_pos": cfg.kv_bytes_per_position_layer(dtype_bytes), "dtype_bytes": dtype_bytes}


# ---------------------------------------------------------------------------------- predictions
class StepCost:
    """Step prices of the calibrated model, as solutions/cost_model.py:91-198 defines them.

    kind "roofline": a layer costs max(W / bw, 2 P n / F) + KV C / bw + n_op_layer t_op with F =
    F_eff; "roofline-peak": the same with the 8192^3 peak F; "linear": a + b n + c C.  A segment of
    m layers adds its metadata ops, a head call costs the head's roofline (or head_a + head_b n)."""

    def __init__(self, cal: dict, kind: str):
        self.kind, self.g, self.d = kind, cal["gpu"], cal["model_dims"]
        self.lin = cal.get("linear")
        self.F = self.g["flops_eff"] if kind == "roofline" and self.g.get("flops_eff") else self.g["flops"]

    def _layer(self, n, C):
        d, g = self.d, self.g
        if self.kind == "linear":
            return self.lin["a"] + self.lin["b"] * n + self.lin["c"] * C
        w = d["layer_params"] * d["dtype_bytes"]
        return (max(w / g["bw"], 2.0 * d["layer_params"] * n / self.F) + C * d["kv_bytes_per_pos"] / g["bw"]
                + g["n_op_layer"] * g["t_op"])

    def head(self, n):
        if n <= 0:
            return 0.0
        if self.kind == "linear":
            return self.lin["head_a"] + self.lin["head_b"] * n
        d, g = self.d, self.g
        return (max(d["head_params"] * d["dtype_bytes"] / g["bw"], 2.0 * d["head_params"] * n / self.F)
                + g["n_op_head"] * g["t_op"])

    def segment(self, m, n, C):
        if m == 0 or n <= 0:
            return 0.0
        seg = self.lin.get("seg_ms", 0.0) if self.kind == "linear" else self.g["n_op_segment"] * self.g["t_op"]
        return m * self._layer(n, C) + seg

    def t_sh(self, B, k, C):
        return self.segment(k, B, C) + self.head(B)

    def t_deep(self, n, k, C, n_req):
        return self.segment(k, n_req, C) + self.segment(self.d["n_layers"] - k, n, C) + self.head(n)

    def t_prefill(self, n, C):
        return self.segment(self.d["n_layers"], n, C) + self.head(1)


# ---------------------------------------------------------------------------------- measurements
class _Gemm:
    """eesd_gemm with its output and workspace kept per shape."""

    def __init__(self, dev):
        self.dev, self.bufs = dev, {}

    def __call__(self, x, w, epi=lib.EPI_STORE, n_out=None, up=0, residual=None):
        n, k = x.shape
        n_out = n_out or w.shape[0]
        key = (n, n_out, k, epi)
        if key not in self.bufs:
            ws_b = int(lib.load().eesd_gemm_workspace_bytes(n, n_out, k, epi))
            self.bufs[key] = (torch.empty(n, n_out, dtype=torch.bfloat16, device=self.dev),
                              torch.empty(max(ws_b, 16), dtype=torch.uint8, device=self.dev), ws_b)
        y, ws, ws_b = self.bufs[key]
        lib.call("eesd_gemm", lib.BF16, epi, x.data_ptr(), w.data_ptr(), lib.ptr(residual), y.data_ptr(), n, n_out,
                 k, up, ws.data_ptr(), ws_b, lib.stream_ptr())
        return y


def micro(dev, quick: bool = False) -> dict:
    """bw, flops and t_op (solutions/calibrate.py:59-76 measures the same three with eager torch)."""
    g = _Gemm(dev)
    rows, k = (8192, 4096) if quick else (28672, 8192)
    w = (torch.randn(rows, k, device=dev) * 0.02).bfloat16()
    x = torch.randn(1, k, device=dev).bfloat16()
    bw = w.numel() * 2 / _t(lambda: g(x, w))
    del w
    s = 4096 if quick else 8192
    a = torch.randn(s, s, device=dev).bfloat16()
    bm = (torch.randn(s, s, device=dev) * 0.02).bfloat16()
    flops = 2.0 * s ** 3 / _t(lambda: g(a, bm), reps=10)
    del a, bm
    ids = torch.zeros(1, dtype=torch.int32, device=dev)
    table = torch.zeros(1, dtype=torch.int32, device=dev)

    def loop():
        for _ in range(1000):
            lib.call("eesd_scatter_ids", ids.data_ptr(), ids.data_ptr(), table.data_ptr(), 1, lib.stream_ptr())
    t_op = _t(loop, reps=5, warm=1) / 1000
    torch.cuda.empty_cache()
    return {"bw": bw, "flops": flops, "t_op": t_op}


def measure_flops_eff(cfg: ModelConfig, dev, ns=N_GRID) -> dict:
    """F_eff: the highest flop rate of one layer's four GEMMs with their fused epilogues over ns."""
    g = _Gemm(dev)
    q = cfg.n_heads * cfg.head_dim
    qkv = (cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim
    inter = cfg.intermediate_size

    def wt(r, c):
        return (torch.randn(r, c, device=dev) * 0.02).bfloat16()
    wqkv, wo, w13, w2 = wt(qkv, cfg.dim), wt(cfg.dim, q), wt(2 * inter, cfg.dim), wt(cfg.dim, inter)
    params = qkv * cfg.dim + cfg.dim * q + 2 * inter * cfg.dim + cfg.dim * inter
    rows = []
    for n in ns:
        xd = torch.randn(n, cfg.dim, device=dev).bfloat16()
        xq = torch.randn(n, q, device=dev).bfloat16()
        xi = torch.randn(n, inter, device=dev).bfloat16()
        res = torch.randn(n, cfg.dim, device=dev).bfloat16()

        def layer():
            g(xd, wqkv)
            g(xq, wo, lib.EPI_RESIDUAL, residual=res)
            g(xd, w13, lib.EPI_SWIGLU, n_out=inter, up=inter)
            g(xi, w2, lib.EPI_RESIDUAL, residual=res)
        ms = _t(layer)
        rows.append({"n": n, "ms": ms, "flop_per_ms": 2.0 * params * n / ms})
    best = max(rows, key=lambda r: r["flop_per_ms"])
    del wqkv, wo, w13, w2
    torch.cuda.empty_cache()
    return {"flops_eff": best["flop_per_ms"], "flops_eff_at_n": best["n"], "gemm_grid": rows}


def _layer_model(cfg: ModelConfig, dev, max_batch: int, max_seq: int, max_tokens: int) -> DeviceModel:
    """Two layers of the configuration (layer 1 is the one timed), KV cache filled with noise."""
    w = ModelWeights.synthetic(replace(cfg, n_layers=2), seed=0, dtype=torch.bfloat16, device=dev)
    dm = DeviceModel(w, max_batch=max_batch, max_seq=max_seq, max_tokens=max_tokens)
    dm.k_cache.normal_(0, 0.5)
    dm.v_cache.normal_(0, 0.5)
    return dm


def _x(dm: DeviceModel, n: int) -> torch.Tensor:
    return (torch.randn(n, dm.cfg.dim, device=dm.device) * 0.5).to(dm.dtype)


def measure_knee(dm: DeviceModel, ns=N_GRID, ctx: int = 128) -> dict:
    """One packed layer on n requests x 1 token at a short context, hinge-fitted
    (solutions/calibrate.py:140-152)."""
    rows = []
    for n in ns:
        b, _ = dm.upload(dm.pack([(r, ctx, 1) for r in range(n)]))
        x = _x(dm, n)
        rows.append({"n": n, "ms": _t(lambda: dm.forward_layers(x, b, 1, 2))})
    knee, (a, slope) = hinge_knee([r["n"] for r in rows], [r["ms"] for r in rows])
    return {"knee_measured": knee, "knee_fit": {"a": a, "b": slope}, "layer_grid": rows}


def trace_ops(dm: DeviceModel) -> dict:
    """Launches of one packed layer and of one head call, counted by the library."""
    b, _ = dm.upload(dm.pack([(0, 100, 1), (1, 100, 3)]))
    x = _x(dm, 4)
    dm.forward_layers(x, b, 1, 2)
    torch.cuda.synchronize()
    c0 = dm.launch_count()
    dm.forward_layers(x, b, 1, 2)
    c1 = dm.launch_count()
    dm.head_argmax(x)
    c2 = dm.launch_count()
    return {"n_op_layer": float(c1 - c0), "n_op_bucket": 0.0, "n_op_head": float(c2 - c1), "n_op_segment": 1.0}


def layer_grid(dm: DeviceModel, Bs=(1, 8, 32, 64, 128), Ts=(1, 2, 5, 9), ctxs=(128, 640, 1536)) -> tuple:
    """One packed layer over B requests x T tokens at context C, the quantities of
    solutions/calibrate.py:93-113.  The grid follows the engines here: draft (T = 1), verify
    (T = gamma + 1 = 5) and per-request draft lengths up to 8 (T = 9), batches up to the
    serving configuration's, contexts of the benchmark configurations."""
    rows, heads = [], []
    for C in ctxs:
        for B in Bs:
            for T in Ts:
                ph = dm.pack([(r, C - T, T) for r in range(B)])
                b, _ = dm.upload(ph)
                x = _x(dm, B * T)
                ms = _t(lambda: dm.forward_layers(x, b, 1, 2), reps=10, warm=3)
                rows.append({"n": B * T, "kv": ph.kv_read, "ms": ms, "B": B, "T": T, "ctx": C})
                if C == ctxs[0]:
                    heads.append({"n": B * T, "ms": _t(lambda: dm.head_argmax(x), reps=10, warm=3)})
    return rows, heads


def validate(cfg: ModelConfig, dev, cal: dict, k: int, quick: bool = False) -> tuple:
    """Real shallow steps, deep steps and prefill chunks of the full-depth packed path against the
    three predictions (solutions/calibrate.py:169-225); returns (rows, MAPE summary)."""
    L = cfg.n_layers
    ctxs, Bs, Ts, pre = ((256,), (1, 4), (2, 4), (64,)) if quick else \
        ((256, 1024, 2048), (1, 4, 8, 16, 32), (2, 4, 6, 9, 17), (64, 256, 1024))
    w = ModelWeights.synthetic(cfg, seed=0, dtype=torch.bfloat16, device=dev)
    dm = DeviceModel(w, max_batch=max(Bs), max_seq=max(ctxs) + max(pre) + max(Ts) + 64,
                     max_tokens=max(max(pre), max(Bs) * max(Ts)))
    dm.k_cache.normal_(0, 0.5)
    dm.v_cache.normal_(0, 0.5)
    models = {kind: StepCost(cal, kind) for kind in ("roofline", "roofline-peak", "linear") if
              kind != "linear" or cal.get("linear")}
    rows = []
    for C in ctxs:
        for B in Bs:
            ph = dm.pack([(r, C, 1) for r in range(B)])
            b, _ = dm.upload(ph)
            x = _x(dm, B)

            def shallow():
                dm.forward_layers(x, b, 0, k)
                dm.head_argmax(x)
            rows.append({"kind": "shallow", "B": B, "ctx": C, "T": 1, "n": B,
                         **{m: c.t_sh(B, k, ph.kv_read) for m, c in models.items()},
                         "ms": _t(shallow, reps=10, warm=3)})
            for T in Ts:
                phs = dm.pack([(r, C + T - 1, 1) for r in range(B)])
                phd = dm.pack([(r, C, T) for r in range(B)])
                bs, _ = dm.upload(phs)
                bd, _ = dm.upload(phd)
                xd = _x(dm, B * T)

                def deep():
                    dm.forward_layers(x, bs, 0, k)
                    dm.forward_layers(xd, bd, k, L)
                    dm.head_argmax(xd)
                rows.append({"kind": "deep", "B": B, "ctx": C, "T": T, "n": B * T,
                             **{m: c.t_deep(B * T, k, phd.kv_read, B) for m, c in models.items()},
                             "ms": _t(deep, reps=10, warm=3)})
            if B == 1:
                for n_tok in pre:
                    php = dm.pack([(0, C, n_tok)])
                    bp, _ = dm.upload(php)
                    xp = _x(dm, n_tok)
                    last = torch.tensor([n_tok - 1], dtype=torch.int32, device=dev)

                    def prefill():
                        dm.forward_layers(xp, bp, 0, L)
                        dm.head_argmax(xp, last)
                    rows.append({"kind": "prefill", "B": 1, "ctx": C, "T": n_tok, "n": n_tok,
                                 **{m: c.t_prefill(n_tok, php.kv_read) for m, c in models.items()},
                                 "ms": _t(prefill, reps=5, warm=2)})
    dm.check()
    summary = {}
    for m in models:
        for kind in ("shallow", "deep", "prefill", "all", "n64_256"):
            if kind == "n64_256":
                rr = [r for r in rows if 64 <= r["n"] <= 256]
            else:
                rr = [r for r in rows if kind == "all" or r["kind"] == kind]
            if rr:
                ape = np.array([abs(r[m] - r["ms"]) / r["ms"] for r in rr])
                summary[f"{m}_{kind}"] = {"n": len(rr), "mape": float(ape.mean()), "max_ape": float(ape.max())}
    return rows, summary


def calibrate(cfg: ModelConfig, name: str, dev, quick: bool = False, linear: bool = True) -> dict:
    ns = (1, 8, 32, 64, 128) if quick else N_GRID
    mic = micro(dev, quick)
    fe = measure_flops_eff(cfg, dev, ns)
    grid = ((1, 4), (1, 4), (256, 512)) if quick else ((1, 4, 16, 32, 64), (1, 4, 8, 17), (256, 1024, 2048))
    dm = _layer_model(cfg, dev, max_batch=max(max(ns), max(grid[0])), max_seq=max(grid[2]) + 64,
                      max_tokens=max(max(ns), max(grid[0]) * max(grid[1])))
    ops = trace_ops(dm)
    kn = measure_knee(dm, ns)
    gpu = {**mic, **ops, "flops_eff": fe["flops_eff"], "knee_measured": kn["knee_measured"],
           "meta": {"source": "thesis_b200 kernels (C ABI), CUDA events", "device": torch.cuda.get_device_name(dev),
                    "flops_eff_at_n": fe["flops_eff_at_n"], "knee_fit": kn["knee_fit"],
                    "knee_analytic_peak": mic["flops"] / mic["bw"],   # F W / (2 P bw) with W = 2 P bytes
                    "gemm_grid": fe["gemm_grid"], "knee_layer_grid": kn["layer_grid"]}}
    res = {"model": name, "gpu": gpu, "model_dims": model_dims(cfg)}
    if linear:
        rows, heads = layer_grid(dm, *grid)
        res["linear"] = {**fit_linear(rows, heads), "n_layers": cfg.n_layers, "model_name": name, "seg_ms": 0.0}
        res["linear_grid"] = rows
    dm.close()
    del dm
    torch.cuda.empty_cache()
    return res


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--preset", default="llama3-8b")
    ap.add_argument("--k", type=int, default=8, help="exit layer of the validation steps")
    ap.add_argument("--validate", action="store_true")
    ap.add_argument("--quick", action="store_true", help="small grids (tests)")
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("calibration needs a CUDA GPU")
    dev = torch.device("cuda")
    cfg = preset(args.preset)
    res = calibrate(cfg, args.preset, dev, quick=args.quick)
    g = res["gpu"]
    print(f"[calibrate] bw {g['bw'] / 1e6:.0f} GB/s, F {g['flops'] / 1e9:.0f} TFLOP/s, F_eff "
          f"{g['flops_eff'] / 1e9:.0f} TFLOP/s (n={g['meta']['flops_eff_at_n']}), knee {g['knee_measured']:.0f} "
          f"tokens, t_op {1000 * g['t_op']:.2f} us, ops/layer {g['n_op_layer']:.0f}", flush=True)
    if args.validate:
        rows, summ = validate(cfg, dev, res, min(args.k, cfg.n_layers - 1), args.quick)
        res["validation"], res["validation_rows"] = summ, rows
        for key, v in summ.items():
            print(f"[calibrate] {key:28s} n={v['n']:3d}  MAPE {100 * v['mape']:5.1f}%  max {100 * v['max_ape']:5.1f}%")
    out = Path(args.out) if args.out else Path(f"b200_calibration_{args.preset}.json")
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(res, indent=2))
    print(f"[calibrate] wrote {out}", flush=True)


if __name__ == "__main__":
    main()
