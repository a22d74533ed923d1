"""Greedy decoding drivers over ``OracleModel`` (small cases only).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

* ``ar_generate``    one token per request per step through all layers
                     (common/engine.py:302-331, solutions/engine.py:244-267);
* ``spec_generate``  synchronous draft/verify rounds: ``gamma`` drafts through layers
                     [0, E) + head, then the last draft through [0, E) and all gamma+1
                     tokens (cached exit hidden states) through [E, L) + head, greedy
                     acceptance = first mismatch (common/engine.py:356-421).

Every request lives in its own cache row and all requests of a call are packed into
one ragged batch (solutions/packed.py semantics).
"""

from __future__ import annotations

import numpy as np

from .model_np import OracleModel, argmax_first


def _prefill_all(m: OracleModel, prompts) -> list:
    return [int(argmax_first(m.prefill(list(p), slot=i))) for i, p in enumerate(prompts)]


def ar_generate(m: OracleModel, prompts, max_new: int) -> list:
    L = m.cfg.n_layers
    first = _prefill_all(m, prompts)
    out = [[t] for t in first]
    pos = [len(p) for p in prompts]
    while True:
        live = [i for i in range(len(prompts)) if len(out[i]) < max_new]
        if not live:
            return out
        blocks = [(i, pos[i], 1) for i in live]
        h, _ = m.packed_layers(m.embed([out[i][-1] for i in live]), blocks, 0, L)
        y = argmax_first(m.head(h))
        for j, i in enumerate(live):
            out[i].append(int(y[j]))
            pos[i] += 1


def spec_generate(m: OracleModel, prompts, max_new: int, exit_layer: int, gamma: int) -> tuple[list, dict]:
    L, E = m.cfg.n_layers, exit_layer
    first = _prefill_all(m, prompts)
    out = [[t] for t in first]
    pos = [len(p) for p in prompts]
    stats = {"rounds": 0, "accepted": 0, "drafted": 0}
    while True:
        live = [i for i in range(len(prompts)) if len(out[i]) < max_new]
        if not live:
            return out, stats
        inp = [out[i][-1] for i in live]
        exit_h = [[] for _ in live]
        drafts = [[] for _ in live]
        for j in range(gamma + 1):                       # gamma drafts + the last draft's shallow pass
            blocks = [(i, pos[i] + j, 1) for i in live]
            h, _ = m.packed_layers(m.embed(inp), blocks, 0, E)
            for r in range(len(live)):
                exit_h[r].append(h[r])
            if j < gamma:
                inp = [int(t) for t in argmax_first(m.head(h))]
                for r in range(len(live)):
                    drafts[r].append(inp[r])
        x = np.stack([e for r in range(len(live)) for e in exit_h[r]])
        blocks = [(i, pos[i], gamma + 1) for i in live]
        hd, _ = m.packed_layers(x, blocks, E, L)
        Y = argmax_first(m.head(hd)).reshape(len(live), gamma + 1)
        stats["rounds"] += 1
        for r, i in enumerate(live):
            acc = 0
            while acc < gamma and Y[r, acc] == drafts[r][acc]:
                acc += 1
            new = [int(t) for t in Y[r, :acc + 1]]
            stats["accepted"] += acc
            stats["drafted"] += gamma
            room = max_new - len(out[i])
            out[i].extend(new[:room])
            pos[i] += acc + 1
