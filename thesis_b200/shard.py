"""Request sharding across GPUs (one process per GPU, full weight replica each).

Requests are independent, so rank r owns requests r, r + W, r + 2W, ... and runs them with no
per-step communication.  The only collective is the final gather of the generated tokens
(``gather_outputs``): every rank contributes a padded int32 ``[n_local, max_len]`` block plus
lengths through ``all_gather`` (NCCL over NVLink on B200; gloo in the CPU tests).
"""

from __future__ import annotations

import numpy as np
import torch


def shard_requests(n: int, rank: int, world: int) -> list:
    if not 0 <= rank < world:
        raise ValueError("rank outside [0, world)")
    return list(range(rank, n, world))


def gather_outputs(outputs: dict, n_total: int, world: int, device=None, group=None) -> dict:
    """outputs: {request index: token list} of this rank -> {request index: tokens} of all ranks."""
    import torch.distributed as dist

    dev = device if device is not None else torch.device("cpu")
    keys = sorted(outputs)
    max_len = max((len(outputs[k]) for k in keys), default=0)
    n_local = torch.tensor([len(keys), max_len], dtype=torch.int64, device=dev)
    sizes = [torch.zeros(2, dtype=torch.int64, device=dev) for _ in range(world)]
    dist.all_gather(sizes, n_local, group=group)
    rows = max(int(s[0]) for s in sizes)
    width = max(int(s[1]) for s in sizes)
    block = torch.full((max(rows, 1), width + 2), -1, dtype=torch.int32)
    for i, k in enumerate(keys):
        t = outputs[k]
        block[i, 0] = k
        block[i, 1] = len(t)
        block[i, 2:2 + len(t)] = torch.tensor(t, dtype=torch.int32)
    block = block.to(dev)
    parts = [torch.empty_like(block) for _ in range(world)]
    dist.all_gather(parts, block, group=group)
    out = {}
    for p in parts:
        p = p.cpu().numpy()
        for row in p:
            if row[0] >= 0:
                out[int(row[0])] = row[2:2 + int(row[1])].tolist()
    if len(out) != n_total:
        raise RuntimeError(f"gathered {len(out)} of {n_total} requests")
    return out
