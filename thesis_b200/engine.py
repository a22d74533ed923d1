"""Engine contract of the reference's benchmark harness, implemented for the B200 engines.

The interface is the reference's (``common/engine.py``): ``StepRecord`` (:36-44), ``SlotState``
(:47-58), ``RunConfig`` (:61-77), ``DecodeEngine.run`` (:178-297) and the commit rule ``_commit``
(:144-164) keep their argument meanings, result keys and errors, so an engine built here can be
returned from a ``MethodSpec.build`` and driven by ``evaluation/benchmark.py``.  The driver itself
is organised around a prompt feed, a throughput meter and a convergence monitor.

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
        """Append the longest prefix of ``tokens`` this request may still take - up to and including
        its first EOS (unless ignored) and no further than its output budget - then let the stop
        checker trim a matched stop string.  Returns how many appended tokens remain (the count
        throughput uses)."""
        s = self.slots[slot]
        if s.finish_reason is not None:
            return 0
        room = (s.max_new or self.max_new) - len(s.output)
        take = [int(t) for t in list(tokens)[:max(room, 0)]]
        if not self.ignore_eos:
            hit = next((i for i, t in enumerate(take) if t in self.eos), None)
            if hit is not None:
                take, s.finish_reason = take[:hit + 1], "eos"
        s.output.extend(take)
        if s.finish_reason is None and len(s.output) >= (s.max_new or self.max_new):
            s.finish_reason = "length"
        kept = len(take)
        if kept and self.stop_checker is not None and not self.ignore_eos:
            cut = self.stop_checker(s.output, kept)
            if cut is not None:
                kept -= len(s.output) - cut
                del s.output[cut:]
                s.finish_reason = "stop"
        return kept

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
        """Drive the engine over ``prompts`` (common/engine.py:178-297 defines the protocol the
        reference's benchmark reads): static mode decodes every prompt once; cyclic mode replays
        the pool, drops the first ``warmup`` completions and stops when the measured throughput has
        settled (or at the evaluation / step caps)."""
        self.records = []
        feed = _PromptFeed(prompts, cyclic=cfg.mode == "cyclic")
        plan = _Plan.of(cfg, self.B)
        meter = _Meter(plan.warm_from_start)
        settle = _Convergence(cfg.converge_threshold, cfg.converge_window)
        done: list = []
        stop = None

        self._assign_many([(slot,) + feed.next() for slot in range(self.B) if feed.has_more()])
        while stop is None:
            if not self._active():
                stop = "pool_exhausted"
                break
            mark = len(self.records)
            committed = self._iteration(measured=meter.warm)
            step_ms = sum(r.forward_ms for r in self.records[mark:])
            n_steps_now = len(self.records) - mark
            for i in self._active():
                self.slots[i].decode_ms += step_ms
            meter.account(committed, step_ms, n_steps_now)
            measured_step = meter.warm
            refill = []
            for slot in self._finished_slots():
                done.append(self._completion(slot, measured_step, cfg.keep_outputs))
                meter.completed += 1
                if not measured_step:
                    if not meter.warm and meter.completed >= plan.warmup_n:
                        meter.start_measuring()
                elif cfg.mode == "cyclic":
                    meter.evaluated += 1
                    if cfg.converge and meter.evaluated >= plan.min_eval_n and meter.ms > 0 and \
                            settle.observe(meter.throughput()):
                        stop = "converged"
                    elif meter.evaluated >= plan.max_eval_n:
                        stop = "max_eval_samples"
                if stop is not None:
                    break
                if feed.has_more():
                    refill.append((slot,) + feed.next())
            if stop is not None:
                break
            self._assign_many(refill)
            if cfg.max_steps is not None and meter.steps >= cfg.max_steps:
                stop = "max_steps"
        return self._report(cfg, plan, meter, done, stop)

    def _finished_slots(self):
        """Occupied slots whose request finished, freed as they are yielded (slot order)."""
        for slot, st in enumerate(self.slots):
            if not st.idle and st.finish_reason is not None:
                st.idle = True
                yield slot

    def _completion(self, slot: int, measured: bool, keep: bool) -> dict:
        st = self.slots[slot]
        c = dict(pid=st.pid, prompt_idx=st.prompt_idx, prompt_len=st.prompt_len, generated=len(st.output),
                 finish_reason=st.finish_reason, decode_ms=st.decode_ms, measured=measured)
        if keep:
            c["tokens"] = list(st.output)
        return c

    def _report(self, cfg: RunConfig, plan: "_Plan", meter: "_Meter", done: list, stop) -> dict:
        measured = [r for r in self.records if r.measured]
        kinds = {}
        for r in measured:
            kinds.setdefault(r.kind, []).append(r.forward_ms)
        steps = {k: {"steps": len(v), "mean_ms": float(np.mean(v)), "p50_ms": float(np.median(v))}
                 for k, v in sorted(kinds.items())}
        # time per output token after the first (the first one comes from the prefill)
        tpot = [c["decode_ms"] / max(c["generated"] - 1, 1) for c in done if c["measured"]]
        wall = meter.wall_s()
        metrics = {
            "stop_reason": stop,
            "warmup_samples_effective": plan.warmup_n,
            "min_eval_samples_effective": plan.min_eval_n,
            "total_completions": meter.completed,
            "evaluated_completions": meter.evaluated if cfg.mode == "cyclic" else meter.completed,
            "measured_tokens": meter.tokens,
            "measured_forward_s": meter.ms / 1000,
            "measured_wall_s": wall,
            "throughput_tok_s": meter.throughput() if meter.ms else None,
            "wall_throughput_tok_s": meter.tokens / wall if wall else None,
            "mean_tpot_ms": float(np.mean(tpot)) if tpot else None,
            "steps": steps,
            **self.extra_metrics(),
        }
        return {"metrics": metrics, "completions": done, "steps": [asdict(r) for r in self.records]}


class _PromptFeed:
    """Prompt indices in order; cyclic feeds wrap around the pool, static ones stop at its end."""

    def __init__(self, prompts: list, cyclic: bool):
        self.prompts, self.cyclic, self.i = prompts, cyclic, 0

    def has_more(self) -> bool:
        return bool(self.prompts) and (self.cyclic or self.i < len(self.prompts))

    def next(self) -> tuple:
        k = self.i % len(self.prompts)
        self.i += 1
        return k, self.prompts[k]


@dataclass
class _Plan:
    """Completion counts of a run: warm-up, minimum and maximum evaluated samples."""
    warmup_n: int
    min_eval_n: int
    max_eval_n: int
    warm_from_start: bool

    @classmethod
    def of(cls, cfg: RunConfig, B: int) -> "_Plan":
        warm = max(cfg.warmup_samples, math.ceil(cfg.warmup_per_slot * B)) if cfg.warmup_samples else 0
        lo = max(cfg.converge_min_samples, math.ceil(cfg.min_eval_per_slot * B))
        hi = max(cfg.max_eval_samples, lo) if cfg.converge else cfg.max_eval_samples
        return cls(warm, lo, hi, cfg.mode == "static" or warm == 0)


class _Meter:
    """Measured decode tokens and forward time (only while warm) and the wall clock of that phase."""

    def __init__(self, warm: bool):
        self.warm = warm
        self.tokens, self.ms, self.steps = 0, 0.0, 0
        self.completed = self.evaluated = 0
        self.t0 = time.perf_counter() if warm else None

    def account(self, tokens: int, ms: float, n_steps: int) -> None:
        self.steps += n_steps
        if self.warm:
            self.tokens += tokens
            self.ms += ms

    def start_measuring(self) -> None:
        self.warm, self.t0 = True, time.perf_counter()

    def throughput(self) -> float:
        return self.tokens / (self.ms / 1000)

    def wall_s(self) -> float:
        return time.perf_counter() - self.t0 if self.t0 is not None else 0.0


class _Convergence:
    """Settled once ``window`` consecutive observations stay within ``rel`` of an anchor value
    (a departure re-anchors)."""

    def __init__(self, rel: float, window: int):
        self.rel, self.window = rel, window
        self.anchor, self.run = None, 0

    def observe(self, value: float) -> bool:
        if self.anchor is None:
            self.anchor = value
        elif abs(value - self.anchor) < self.rel * self.anchor:
            self.run += 1
        else:
            self.anchor, self.run = value, 0
        return self.run >= self.window
