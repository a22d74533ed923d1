"""Ragged token packing for one call of the layer-range forward.

Counterpart of ``build_packed`` / ``qo_indptr`` (solutions/packed.py:81-139, 199-201).  Blocks
keep the caller's order (no bucketing: the attention kernel handles every block length in one
launch and derives causality from positions, so there is no mask to build and no KV gather).
The host builds four small int32 arrays and ships them in ONE pinned host-to-device copy:

    tok_pos [N]        absolute position of every packed token
    tok_row [N]        KV-cache row of every packed token
    blk     [nb, 4]    (start, T, row, pos0) per block; start = qo_indptr[b]
    items   [ni, 2]    attention work items (block, first token) tiling each block by
                       ``item_tokens`` query tokens
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


def qo_indptr(lengths) -> np.ndarray:
    """cumsum of per-block token counts with a leading 0 (solutions/packed.py:199-201)."""
    return np.concatenate([[0], np.cumsum(np.asarray(lengths, dtype=np.int64))]).astype(np.int64)


@dataclass
class PackedHost:
    blocks: list               # [(row, pos0, T)] in packed order
    offsets: np.ndarray        # qo_indptr [nb + 1]
    tok_pos: np.ndarray
    tok_row: np.ndarray
    blk: np.ndarray
    items: np.ndarray
    max_ctx: int

    @property
    def n_tokens(self) -> int:
        return int(self.offsets[-1])

    @property
    def n_blocks(self) -> int:
        return len(self.blocks)

    def block_slice(self, i: int) -> slice:
        return slice(int(self.offsets[i]), int(self.offsets[i + 1]))

    @property
    def kv_read(self) -> int:
        """KV positions attention reads per layer (sum over blocks of pos0 + T, no padding)."""
        return int(sum(p0 + T for (_, p0, T) in self.blocks))


def pack(blocks, item_tokens: int) -> PackedHost:
    """blocks: iterable of (row, pos0, T) with T >= 1."""
    blocks = [(int(r), int(p), int(t)) for (r, p, t) in blocks]
    if any(t < 1 or p < 0 or r < 0 for (r, p, t) in blocks):
        raise ValueError("blocks need row >= 0, pos0 >= 0 and T >= 1")
    Ts = np.array([t for (_, _, t) in blocks], dtype=np.int64)
    offsets = qo_indptr(Ts)
    N = int(offsets[-1])
    tok_pos = np.empty(N, dtype=np.int32)
    tok_row = np.empty(N, dtype=np.int32)
    blk = np.empty((len(blocks), 4), dtype=np.int32)
    items = []
    for i, (r, p0, T) in enumerate(blocks):
        s = int(offsets[i])
        tok_pos[s:s + T] = np.arange(p0, p0 + T)
        tok_row[s:s + T] = r
        blk[i] = (s, T, r, p0)
        items.extend((i, t0) for t0 in range(0, T, item_tokens))
    # longest key range first: the attention grid then finishes its long items before the short
    # ones fill the last wave (an item's result does not depend on its place in the grid)
    items.sort(key=lambda it_: -(blocks[it_[0]][1] + min(it_[1] + item_tokens, blocks[it_[0]][2])))
    it = np.array(items, dtype=np.int32).reshape(-1, 2)
    max_ctx = max((p0 + T for (_, p0, T) in blocks), default=0)
    return PackedHost(blocks, offsets, tok_pos, tok_row, blk, it, int(max_ctx))


class MetaUploader:
    """Pinned staging ring + device buffer for the packed metadata of one model.

    Each upload copies the four arrays with one ``cudaMemcpyAsync`` from a pinned slot; a slot is
    reused only after the event recorded behind its previous copy has completed."""

    def __init__(self, max_tokens: int, max_blocks: int, max_items: int, device, slots: int = 4,
                 max_extra: int = 0):
        import torch

        self.cap = 2 * max_tokens + 4 * max_blocks + 2 * max_items + max_extra
        self.max_extra = max_extra
        self.max_tokens, self.max_blocks, self.max_items = max_tokens, max_blocks, max_items
        self.host = [torch.empty(self.cap, dtype=torch.int32, pin_memory=True) for _ in range(slots)]
        self.dev = [torch.empty(self.cap, dtype=torch.int32, device=device) for _ in range(slots)]
        self.events = [None] * slots
        self.i = 0
        self.bytes_uploaded = 0

    def upload(self, ph: PackedHost, extra=(), stream=None):
        """Returns (lib.Batch struct, [device views of the ``extra`` int32 arrays]) for ``ph``; the
        extra arrays (step indices) travel in the same copy."""
        import torch

        from . import lib

        N, nb, ni = ph.n_tokens, ph.n_blocks, len(ph.items)
        n_extra = sum(int(np.asarray(e).size) for e in extra)
        if N > self.max_tokens or nb > self.max_blocks or ni > self.max_items or n_extra > self.max_extra:
            raise ValueError(f"packed call too large: tokens {N}/{self.max_tokens}, blocks {nb}/{self.max_blocks}, "
                             f"items {ni}/{self.max_items}")
        k = self.i
        self.i = (self.i + 1) % len(self.host)
        if self.events[k] is not None:
            self.events[k].synchronize()
        h = self.host[k].numpy()
        o = 0
        parts = []
        for arr in (ph.tok_pos, ph.tok_row, ph.blk.reshape(-1), ph.items.reshape(-1), *extra):
            arr = np.asarray(arr, dtype=np.int32).reshape(-1)
            h[o:o + arr.size] = arr
            parts.append((o, arr.size))
            o += arr.size
        d = self.dev[k]
        s = stream if stream is not None else torch.cuda.current_stream()
        with torch.cuda.stream(s):
            d[:o].copy_(self.host[k][:o], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(s)
        self.events[k] = ev
        self.bytes_uploaded += 4 * o
        base = d.data_ptr()
        b = lib.Batch(N, nb, ni, ph.max_ctx, *(base + 4 * parts[i][0] for i in range(4)))
        return b, [d[o:o + n] for (o, n) in parts[4:]]
