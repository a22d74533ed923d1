"""Engine contract of the reference's benchmark harness, restated for the B200 engines.

Mirrors ``common/engine.py``: ``StepRecord`` (:36-44), ``SlotState`` (:47-58), ``RunConfig``
(:61-77), the cyclic-replay / static driver ``DecodeEngine.run`` (:178-297) and the commit rule
``_commit`` (:144-164), with the same argument meanings, result keys and errors, so an engine
built here can be returned from a ``MethodSpec.build`` and driven by ``evaluation/benchmark.py``.

Subclasses implement ``_prefill_slots`` (fill a set of slots, return their first tokens) and
``_iteration`` (one scheduling iteration over the occupied slots).  Differences from the
reference are confined to the device work; the host protocol is the same:
* throughput counts decode forward time only (CUDA-event intervals of the decode steps);
* the warm-up completions are dropped, cyclic mode stops when the cumulative decode throughput
  is stable within ``converge_threshold`` for ``converge_window`` completions, or after
  ``max_eval_samples`` / ``max_steps``;
* static mode generates every prompt once.
"""

from __future__ import annotations

import math
import time
from dataclasses import asdict, dataclass, field
from typing import Optional

import numpy as np
import torch


@dataclass
class StepRecord:
    kind: str               # "ar" | "draft" | "verify"
    forward_ms: float
    batch: int
    shallow_tokens: int
    deep_tokens: int
    kv_read: int
    measured: bool


@dataclass
class SlotState:
    prompt_idx: int = -1
    pid: str = ""
    prompt_len: int = 0
    pos: int = 0            # position of `last_token` (its KV is not written yet)
    last_token: int = 0
    output: list = field(default_factory=list)
    finish_reason: Optional[str] = None
    idle: bool = True
    t_assigned: float = 0.0
    decode_ms: float = 0.0
    max_new: Optional[int] = None   # per-request output budget (None: the engine's max_new_tokens)


@dataclass
class RunConfig:
    mode: str = "cyclic"             # cyclic | static
    warmup_samples: int = 8
    max_eval_samples: int = 256
    converge: bool = True
    converge_threshold: float = 0.01
    converge_window: int = 4
    converge_min_samples: int = 16
    max_steps: Optional[int] = None
    keep_outputs: bool = False
    warmup_per_slot: float = 1.0
    min_eval_per_slot: float = 2.0


class Interval:
    """CUDA-event interval on the current stream (common/timing.py:16-47)."""

    def __init__(self, device: torch.device):
        self.cuda = device.type == "cuda"
        if self.cuda:
            self._a = torch.cuda.Event(enable_timing=True)
            self._b = torch.cuda.Event(enable_timing=True)
        self._t0 = self._t1 = 0.0

    def start(self) -> "Interval":
        if self.cuda:
            self._a.record()
        else:
            self._t0 = time.perf_counter()
        return self

    def stop(self) -> "Interval":
        if self.cuda:
            self._b.record()
        else:
            self._t1 = time.perf_counter()
        return self

    @property
    def ms(self) -> float:
        if self.cuda:
            self._b.synchronize()
            return float(self._a.elapsed_time(self._b))
        return (self._t1 - self._t0) * 1000.0


class DecodeEngine:
    name = "base"

    def __init__(self, model, batch_size: int, max_prompt_len: int, max_new_tokens: int, eos_ids, *,
                 ignore_eos: bool = False, spec_slack: int = 32, temperature: float = 0.0, top_k: int = 50,
                 top_p: float = 0.9, seed: int = 0):
        if temperature > 0:
            raise NotImplementedError(f"{type(self).__name__} implements greedy decoding only (temperature 0)")
        self.B = int(batch_size)
        self.max_new = int(max_new_tokens)
        self.eos = set(int(e) for e in eos_ids)
        self.ignore_eos = ignore_eos
        self.temperature, self.top_k, self.top_p, self.seed = temperature, top_k, top_p, seed
        self.max_seq = max_prompt_len + max_new_tokens + spec_slack + 2     # common/engine.py:118
        self.slots = [SlotState() for _ in range(self.B)]
        self.records: list[StepRecord] = []
        self.probe = None
        self.stop_checker = None

    # ---------------------------------------------------------------- slot helpers
    def _commit(self, slot: int, tokens) -> int:
        """Append tokens, stopping at EOS / max_new / a stop string; returns the useful count."""
        s = self.slots[slot]
        n = 0
        for t in tokens:
            if s.finish_reason is not None:
                break
            t = int(t)
            s.output.append(t)
            n += 1
            if not self.ignore_eos and t in self.eos:
                s.finish_reason = "eos"
            elif len(s.output) >= (s.max_new or self.max_new):
                s.finish_reason = "length"
        if n and self.stop_checker and not self.ignore_eos:
            cut = self.stop_checker(s.output, n)
            if cut is not None:
                n -= len(s.output) - cut
                del s.output[cut:]
                s.finish_reason = "stop"
        return n

    def _active(self) -> list:
        return [i for i, s in enumerate(self.slots) if not s.idle]

    def _assign_many(self, items) -> None:
        """items: [(slot, prompt_idx, prompt)]; prefill them together, then commit first tokens."""
        if not items:
            return
        for slot, _, prompt in items:
            if len(prompt.tokens) + self.max_new + 2 > self.max_seq_alloc():
                raise ValueError(f"prompt of {len(prompt.tokens)} tokens does not fit max_seq={self.max_seq_alloc()}")
        first = self._prefill_slots({slot: list(prompt.tokens) for slot, _, prompt in items})
        now = time.perf_counter()
        for slot, idx, prompt in items:
            s = self.slots[slot]
            s.prompt_idx, s.pid, s.prompt_len = idx, prompt.pid, len(prompt.tokens)
            s.pos, s.last_token = len(prompt.tokens), int(first[slot])
            s.output, s.finish_reason, s.idle = [], None, False
            s.t_assigned, s.decode_ms = now, 0.0
            s.max_new = min(int(prompt.max_new), self.max_new) if getattr(prompt, "max_new", None) else None
            self._on_assigned(slot)
            self._commit(slot, [first[slot]])

    # ---------------------------------------------------------------- subclass hooks
    def max_seq_alloc(self) -> int:
        return self.max_seq

    def _prefill_slots(self, prompts: dict) -> dict:
        raise NotImplementedError

    def _on_assigned(self, slot: int) -> None:
        pass

    def _iteration(self, measured: bool) -> int:
        raise NotImplementedError

    def extra_metrics(self) -> dict:
        return {}

    # ---------------------------------------------------------------- driver
    @torch.inference_mode()
    def run(self, prompts: list, cfg: RunConfig) -> dict:
        self.records = []
        n_pool = len(prompts)
        B = self.B
        warmup_n = max(cfg.warmup_samples, math.ceil(cfg.warmup_per_slot * B)) if cfg.warmup_samples else 0
        min_eval_n = max(cfg.converge_min_samples, math.ceil(cfg.min_eval_per_slot * B))
        max_eval_n = max(cfg.max_eval_samples, min_eval_n) if cfg.converge else cfg.max_eval_samples
        warm = cfg.mode == "static" or warmup_n == 0
        state = {"cursor": 0}
        completions = []
        total_completed = evaluated = stable = steps = 0
        anchor = None
        stop_reason = None
        measured_tokens, measured_ms = 0, 0.0
        wall_t0 = time.perf_counter() if warm else None
        wall_measured = 0.0

        def take(slot):
            c = state["cursor"]
            state["cursor"] += 1
            return (slot, c % n_pool, prompts[c % n_pool])

        fill = []
        for slot in range(B):
            if cfg.mode == "static" and state["cursor"] >= n_pool:
                break
            fill.append(take(slot))
        self._assign_many(fill)

        while True:
            if not self._active():
                stop_reason = "pool_exhausted"
                break
            n_before = len(self.records)
            committed = self._iteration(measured=warm)
            new = self.records[n_before:]
            step_ms = sum(r.forward_ms for r in new)
            steps += len(new)
            for i in self._active():
                self.slots[i].decode_ms += step_ms
            if warm:
                measured_tokens += committed
                measured_ms += step_ms
            was_warm = warm
            refill = []
            for slot, s in enumerate(self.slots):
                if s.idle or s.finish_reason is None:
                    continue
                if stop_reason is not None:
                    break
                comp = {"pid": s.pid, "prompt_idx": s.prompt_idx, "prompt_len": s.prompt_len,
                        "generated": len(s.output), "finish_reason": s.finish_reason, "decode_ms": s.decode_ms,
                        "measured": was_warm}
                if cfg.keep_outputs:
                    comp["tokens"] = list(s.output)
                completions.append(comp)
                total_completed += 1
                s.idle = True
                if not was_warm:
                    if not warm and total_completed >= warmup_n:
                        warm = True
                        wall_t0 = time.perf_counter()
                elif cfg.mode == "cyclic":
                    evaluated += 1
                    if cfg.converge and evaluated >= min_eval_n and measured_ms > 0:
                        thr = measured_tokens / (measured_ms / 1000)
                        if anchor is None:
                            anchor = thr
                        elif abs(thr - anchor) / anchor < cfg.converge_threshold:
                            stable += 1
                        else:
                            stable, anchor = 0, thr
                        if stable >= cfg.converge_window:
                            stop_reason = "converged"
                    if stop_reason is None and evaluated >= max_eval_n:
                        stop_reason = "max_eval_samples"
                if cfg.mode == "cyclic" or state["cursor"] < n_pool:
                    refill.append(take(slot))
            if stop_reason is not None:
                break
            self._assign_many(refill)
            if cfg.max_steps is not None and steps >= cfg.max_steps:
                stop_reason = "max_steps"
                break
        if wall_t0 is not None:
            wall_measured = time.perf_counter() - wall_t0

        rec = [r for r in self.records if r.measured]
        per_kind = {}
        for kind in sorted({r.kind for r in rec}):
            ms = [r.forward_ms for r in rec if r.kind == kind]
            per_kind[kind] = {"steps": len(ms), "mean_ms": float(np.mean(ms)), "p50_ms": float(np.median(ms))}
        meas = [c for c in completions if c["measured"]]
        tpot = [c["decode_ms"] / max(c["generated"] - 1, 1) for c in meas]
        metrics = {
            "stop_reason": stop_reason,
            "warmup_samples_effective": warmup_n,
            "min_eval_samples_effective": min_eval_n,
            "total_completions": total_completed,
            "evaluated_completions": evaluated if cfg.mode == "cyclic" else total_completed,
            "measured_tokens": measured_tokens,
            "measured_forward_s": measured_ms / 1000,
            "measured_wall_s": wall_measured,
            "throughput_tok_s": measured_tokens / (measured_ms / 1000) if measured_ms else None,
            "wall_throughput_tok_s": measured_tokens / wall_measured if wall_measured else None,
            "mean_tpot_ms": float(np.mean(tpot)) if tpot else None,
            "steps": per_kind,
            **self.extra_metrics(),
        }
        return {"metrics": metrics, "completions": completions, "steps": [asdict(r) for r in self.records]}
