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
    """outputs: {request index: token list} of this rank -> {request index: tokens} of all ranks.

    Two ``all_gather`` calls (the [rows, width] of every rank, then the padded blocks) and one
    read-back of each; the blocks are filled and split with numpy."""
    import torch.distributed as dist

    dev = device if device is not None else torch.device("cpu")
    keys = sorted(outputs)
    lens = np.array([len(outputs[k]) for k in keys], dtype=np.int64)
    n_local = torch.tensor([len(keys), int(lens.max(initial=0))], dtype=torch.int64, device=dev)
    sizes = [torch.zeros(2, dtype=torch.int64, device=dev) for _ in range(world)]
    dist.all_gather(sizes, n_local, group=group)
    sz = torch.stack(sizes).cpu().numpy()
    rows, width = max(int(sz[:, 0].max()), 1), int(sz[:, 1].max())
    block = np.full((rows, width + 2), -1, dtype=np.int32)
    if keys:
        block[:len(keys), 0] = keys
        block[:len(keys), 1] = lens
        if width:
            filled = np.arange(width) < lens[:, None]
            block[:len(keys), 2:][filled] = np.concatenate([np.asarray(outputs[k], dtype=np.int32) for k in keys])
    blk = torch.from_numpy(block).to(dev)
    parts = [torch.empty_like(blk) for _ in range(world)]
    dist.all_gather(parts, blk, group=group)
    allb = torch.cat(parts).cpu().numpy()
    out = {int(row[0]): row[2:2 + int(row[1])].tolist() for row in allb if row[0] >= 0}
    if len(out) != n_total:
        raise RuntimeError(f"gathered {len(out)} of {n_total} requests")
    return out
