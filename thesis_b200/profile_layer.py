"""Small, self-contained profiling workload for single-kernel captures (ncu) of the hot path.

    python -m thesis_b200.profile_layer [--iters N] [--layers 2] [--ctx 300 700] [--prefill] [--mma-split N]

Builds a LayerSkip-Llama3-8B-shaped model with only ``--layers`` layers (random bf16 weights,
about 2 GB on the device with the KV cache), fills the KV cache with random values, and runs a
verify-shaped packed call (64 blocks of 5 tokens), a draft-shaped call (64 blocks of 1 token) and
the exit head on both, ``--iters`` times, then the same again under per-launch CUDA events and
prints the average time of every (kernel kind, token count).  Inputs are larger than L2 (436 MB
of weights per layer, ~130 MB of KV per attention launch).  ``--prefill`` adds a prefill-shaped
call (4 requests x 512 prompt tokens from position 0), which runs the separate RoPE/KV-append
kernel.  ``--mma-split N`` sets the N of the first of the two MMAs a k-step issues for token tiles
above 256 (``EESD_OPT_MMA_SPLIT``; 0 = two equal halves).
"""

from __future__ import annotations

import argparse
from dataclasses import replace

import numpy as np
import torch

from .config import preset
from .model import DeviceModel, ModelWeights


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--iters", type=int, default=1)
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--ctx", type=int, nargs=2, default=(300, 700))
    ap.add_argument("--prefill", action="store_true")
    ap.add_argument("--mma-split", type=int, default=None)
    args = ap.parse_args(argv)
    if args.mma_split is not None:
        from . import lib

        lib.call("eesd_set_option", lib.OPT_MMA_SPLIT, args.mma_split)
    cfg = replace(preset("llama3-8b"), n_layers=args.layers)
    w = ModelWeights.synthetic(cfg, seed=0, dtype=torch.bfloat16, device="cuda")
    dm = DeviceModel(w, max_batch=64, max_seq=max(args.ctx[1], 512) + 64, max_tokens=2048 if args.prefill else 512)
    dm.k_cache.normal_(0, 0.5)
    dm.v_cache.normal_(0, 0.5)
    rng = np.random.default_rng(0)
    ctx = rng.integers(args.ctx[0], args.ctx[1], size=64)
    deep = dm.upload(dm.pack([(r, int(ctx[r]), 5) for r in range(64)]))
    shal = dm.upload(dm.pack([(r, int(ctx[r]), 1) for r in range(64)]))
    g = torch.Generator(device="cuda").manual_seed(0)
    xd = torch.randn(320, cfg.dim, device="cuda", generator=g).bfloat16()
    xs = torch.randn(64, cfg.dim, device="cuda", generator=g).bfloat16()

    if args.prefill:
        pre = dm.upload(dm.pack([(r, 0, 512) for r in range(60, 64)]))
        xp = torch.randn(2048, cfg.dim, device="cuda", generator=g).bfloat16()

    def once():
        dm.forward_layers(xd.clone(), deep, 0, cfg.n_layers)
        dm.forward_layers(xs.clone(), shal, 0, cfg.n_layers)
        dm.head_argmax(xs)
        dm.head_argmax(xd)
        if args.prefill:
            dm.forward_layers(xp.clone(), pre, 0, cfg.n_layers)

    for _ in range(args.iters):
        once()
    torch.cuda.synchronize()
    dm.check()
    dm.profile(True)
    for _ in range(max(args.iters, 3)):
        once()
    torch.cuda.synchronize()
    agg = {}
    for kind, n, t in dm.profile_records():
        a = agg.setdefault((kind, n), [0, 0.0])
        a[0] += 1
        a[1] += t
    dm.profile(False)
    for (kind, n), (c, t) in sorted(agg.items()):
        print(f"{kind:10s} N={n:4d} launches={c:3d} avg_us={1000 * t / c:9.2f}")


if __name__ == "__main__":
    main()
