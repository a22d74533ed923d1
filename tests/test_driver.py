"""The engine driver (``DecodeEngine.run`` and ``_commit``) against the reference's own driver
(common/engine.py:178-297, :144-164) on the CPU: the same host-only fake engine is driven by both,
and every completion, step record and metric must agree, except the wall-clock fields.  Needs the
reference (THESIS_REFERENCE or baseline/_ref); no GPU."""

import sys

import pytest

from refpath import reference_dir
from thesis_b200.engine import DecodeEngine, RunConfig, SlotState, StepRecord
from thesis_b200.synthetic import Prompt

WALL_KEYS = {"measured_wall_s", "wall_throughput_tok_s"}
EOS = 7


def _first_token(prompt):
    return (sum(prompt.tokens) * 7 + 3) % 40


def _step(engine, records_cls, slot_state, measured):
    """One fake iteration: every occupied slot gets 1-3 deterministic tokens (EOS among them)."""
    engine.t += 1
    committed = 0
    for i, s in enumerate(engine.slots):
        if s.idle:
            continue
        n = 1 + (engine.t * 31 + i * 7) % 3
        toks = [((s.prompt_idx * 13 + len(s.output) + j) * 11 + engine.t) % 40 for j in range(n)]
        committed += engine._commit(i, toks)
    engine.records.append(records_cls("verify", 1.0 + (engine.t % 5) * 0.25, engine.B, engine.B, engine.B, 0,
                                      measured))
    return committed


class OurFake(DecodeEngine):
    def __init__(self, B, max_new, ignore_eos):
        super().__init__(None, B, 64, max_new, (EOS,), ignore_eos=ignore_eos)
        self.t = 0

    def _prefill_slots(self, prompts):
        return {slot: _first_token(Prompt("", toks)) for slot, toks in prompts.items()}

    def _iteration(self, measured):
        return _step(self, StepRecord, SlotState, measured)


def _reference_fake(ref_engine):
    class RefFake(ref_engine.DecodeEngine):
        def __init__(self, B, max_new, ignore_eos):      # no model: only the driver state
            self.B, self.max_new, self.eos, self.ignore_eos = B, max_new, {EOS}, ignore_eos
            self.slots = [ref_engine.SlotState() for _ in range(B)]
            self.records, self.probe, self.stop_checker, self.t = [], None, None, 0

        def _assign(self, slot, prompt_idx, prompt):
            s = self.slots[slot]
            s.prompt_idx, s.pid, s.prompt_len = prompt_idx, prompt.pid, len(prompt.tokens)
            s.pos, s.last_token = len(prompt.tokens), _first_token(prompt)
            s.output, s.finish_reason, s.idle, s.decode_ms = [], None, False, 0.0
            self._commit(slot, [s.last_token])

        def _iteration(self, measured):
            return _step(self, ref_engine.StepRecord, ref_engine.SlotState, measured)

    return RefFake


def _strip(res):
    m = {k: v for k, v in res["metrics"].items() if k not in WALL_KEYS}
    return m, res["completions"], res["steps"]


@pytest.mark.parametrize("mode,kw,B,max_new,ignore_eos", [
    ("cyclic", dict(warmup_samples=3, converge_min_samples=4, converge_window=2, converge_threshold=0.2), 4, 12, False),
    ("cyclic", dict(warmup_samples=2, max_eval_samples=9, converge=False), 3, 9, False),
    ("cyclic", dict(warmup_samples=0, max_steps=17), 5, 30, True),
    ("static", {}, 4, 10, False),
    ("static", {}, 8, 6, True),
])
def test_driver_matches_the_reference_driver(mode, kw, B, max_new, ignore_eos):
    ref = reference_dir()
    if ref is None:
        pytest.skip("the reference is not available (THESIS_REFERENCE or baseline/_ref)")
    sys.path.insert(0, str(ref))
    try:
        import common.engine as ref_engine
    finally:
        sys.path.remove(str(ref))
    prompts = [Prompt(f"p{i}", list(range(i, i + 3 + i % 4))) for i in range(6)]
    ours = OurFake(B, max_new, ignore_eos).run(prompts, RunConfig(mode=mode, keep_outputs=True, **kw))
    theirs = _reference_fake(ref_engine)(B, max_new, ignore_eos).run(
        prompts, ref_engine.RunConfig(mode=mode, keep_outputs=True, **kw))
    mo, co, so = _strip(ours)
    mt, ct, st = _strip(theirs)
    assert co == ct
    assert so == st
    assert mo == mt
    assert len(co) > 0
