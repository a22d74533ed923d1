"""Plugin for the reference harness: registers the B200 methods in ``common.methods``.

Importing this module inside a checkout of the reference (``common`` importable) adds
``b200_autoregressive``, ``b200_layerskip``, ``b200_layerskip_dynamic`` and
``b200_layerskip_piggyback`` to ``common.methods.METHODS``; after that
``evaluation/benchmark.py --method b200_layerskip --exit-layer 8 --gamma 4`` builds a
``B200SpecEngine`` from the ``LayerSkipLlama`` the harness loaded (weights are shared, not
copied).  Load it with ``common.methods.load_plugins(["thesis_b200.plugin"])`` or by importing
it from ``solutions/__init__.py`` (common/methods.py:50-60).
"""

from __future__ import annotations

from dataclasses import asdict

from common.methods import METHODS, MethodSpec, register  # noqa: the reference's registry

from .methods import SPECS

for _s in SPECS:
    if _s.name not in METHODS:
        register(MethodSpec(**{k: v for k, v in asdict(_s).items()}))
