"""Decoding-method registry (mirror of ``common/methods.py``) with the B200 engines registered.

Same contract as the reference: ``MethodSpec`` fields (:27-37), ``register`` raising
``ValueError`` on a duplicate name (:43-47), ``METHODS`` (:40) and ``load_plugins`` (:50-60).
``SPECS`` lists the methods this package contributes; ``thesis_b200.plugin`` registers the same
specs into the reference's own registry so ``evaluation/benchmark.py`` can select them.
"""

from __future__ import annotations

import importlib
from dataclasses import dataclass, field
from typing import Callable, Optional


@dataclass
class MethodSpec:
    name: str
    description: str
    add_args: Callable
    build: Callable
    tag: Callable = field(default=lambda args: "")
    supports_sampling: bool = False
    spec_slack: int = 0
    step_tokens: Callable = field(default=lambda args: 1)
    params: Callable = field(default=lambda args: {})


METHODS: dict = {}


def register(spec: MethodSpec) -> MethodSpec:
    if spec.name in METHODS:
        raise ValueError(f"method {spec.name!r} already registered")
    METHODS[spec.name] = spec
    return spec


def load_plugins(modules: Optional[list] = None) -> list:
    """Import extra modules so they can register methods (the B200 methods are built in)."""
    loaded = []
    for name in list(modules or []):
        try:
            importlib.import_module(name)
            loaded.append(name)
        except ModuleNotFoundError as e:
            if e.name != name:
                raise
    return loaded


def _has(group, flag: str) -> bool:
    return flag in getattr(group, "_option_string_actions", {})


def _b200_ar_args(g) -> None:
    if not _has(g, "--b200-prefill-chunk"):
        g.add_argument("--b200-prefill-chunk", type=int, default=512, help="[b200_*] prefill chunk (tokens)")


def _b200_spec_args(g) -> None:
    # the reference registers --exit-layer / --gamma for sync_layerskip; reuse them when present
    if not _has(g, "--exit-layer"):
        g.add_argument("--exit-layer", type=int, default=None, help="[b200_layerskip] exit layer E")
    if not _has(g, "--gamma"):
        g.add_argument("--gamma", type=int, default=4, help="[b200_layerskip] draft length")
    _b200_ar_args(g)


def _kw(args) -> dict:
    return dict(ignore_eos=getattr(args, "ignore_eos", False), temperature=getattr(args, "temperature", 0.0),
                prefill_chunk=getattr(args, "b200_prefill_chunk", 512))


def _b200_ar_build(model, args, batch_size, max_prompt_len, eos):
    from .eesd import B200ARBatchEngine

    return B200ARBatchEngine(model, batch_size, max_prompt_len, args.max_new_tokens, eos, **_kw(args))


def _b200_spec_build(model, args, batch_size, max_prompt_len, eos):
    from .eesd import B200SpecEngine

    if args.exit_layer is None:
        raise SystemExit("--exit-layer is required for b200_layerskip")
    return B200SpecEngine(model, batch_size, max_prompt_len, args.max_new_tokens, eos, exit_layer=args.exit_layer,
                          gamma=args.gamma, **_kw(args))


def _b200_dyn_args(g) -> None:
    g.add_argument("--b200-exit-layers", type=str, default="4,8,12",
                   help="[b200_layerskip_dynamic] exit layers a request may draw (comma-separated)")
    g.add_argument("--b200-gamma-range", type=str, default="2,8",
                   help="[b200_layerskip_dynamic] draft length range lo,hi drawn per request and round")
    g.add_argument("--b200-policy-seed", type=int, default=0, help="[b200_layerskip_dynamic] draw seed")
    g.add_argument("--b200-schedule", choices=("lockstep", "unified"), default="lockstep",
                   help="[b200_layerskip_dynamic] lockstep rounds, or the unified step (each request verifies "
                        "when its own draft length is reached)")
    _b200_ar_args(g)


def _ints(text: str) -> list:
    return [int(v) for v in str(text).split(",") if v.strip()]


def _b200_dyn_build(model, args, batch_size, max_prompt_len, eos):
    from .dynamic import B200DynamicSpecEngine

    g = _ints(args.b200_gamma_range)
    if len(g) != 2:
        raise SystemExit("--b200-gamma-range takes lo,hi")
    return B200DynamicSpecEngine(model, batch_size, max_prompt_len, args.max_new_tokens, eos,
                                 exit_layers=_ints(args.b200_exit_layers), gamma_range=(g[0], g[1]),
                                 schedule=getattr(args, "b200_schedule", "lockstep"),
                                 policy_seed=args.b200_policy_seed, **_kw(args))


def _b200_piggy_args(g) -> None:
    _b200_spec_args(g)
    if not _has(g, "--b200-piggyback-budget"):
        g.add_argument("--b200-piggyback-budget", type=int, default=256,
                       help="[b200_layerskip_piggyback] prompt tokens carried by each shallow step")


def _b200_piggy_build(model, args, batch_size, max_prompt_len, eos):
    from .serving import B200ServingEngine

    if args.exit_layer is None:
        raise SystemExit("--exit-layer is required for b200_layerskip_piggyback")
    return B200ServingEngine(model, batch_size, max_prompt_len, args.max_new_tokens, eos, exit_layer=args.exit_layer,
                             gamma=args.gamma, piggyback_budget=args.b200_piggyback_budget, **_kw(args))


SPECS = [
    MethodSpec("b200_autoregressive", "all N layers per token on the sm_100a packed path (lossless reference)",
               _b200_ar_args, _b200_ar_build),
    MethodSpec("b200_layerskip", "synchronous batched LayerSkip on the sm_100a packed path (fixed E, gamma)",
               _b200_spec_args, _b200_spec_build, tag=lambda a: f"-k{a.exit_layer}-g{a.gamma}", spec_slack=64,
               step_tokens=lambda a: a.gamma + 1, params=lambda a: {"exit_layer": a.exit_layer, "gamma": a.gamma}),
    MethodSpec("b200_layerskip_piggyback",
               "LayerSkip (fixed E, gamma) with new-request prefill piggybacked on the draft / verify steps",
               _b200_piggy_args, _b200_piggy_build, tag=lambda a: f"-k{a.exit_layer}-g{a.gamma}-pb{a.b200_piggyback_budget}",
               spec_slack=64, step_tokens=lambda a: a.gamma + 1,
               params=lambda a: {"exit_layer": a.exit_layer, "gamma": a.gamma,
                                 "piggyback_budget": a.b200_piggyback_budget}),
    MethodSpec("b200_layerskip_dynamic",
               "LayerSkip with a per-request exit layer and per-request draft length, coalesced ragged verify",
               _b200_dyn_args, _b200_dyn_build,
               tag=lambda a: f"-e{a.b200_exit_layers.replace(',', '_')}-g{a.b200_gamma_range.replace(',', '_')}",
               spec_slack=64, step_tokens=lambda a: _ints(a.b200_gamma_range)[-1] + 1,
               params=lambda a: {"exit_layers": _ints(a.b200_exit_layers), "gamma_range": _ints(a.b200_gamma_range),
                                 "policy_seed": a.b200_policy_seed}),
]

for _s in SPECS:
    register(_s)
