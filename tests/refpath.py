"""Where the CPU tests find the unmodified reference (hsungo/thesis): ``$THESIS_REFERENCE`` if it
points to a checkout, else the offline install under ``baseline/_ref``
(``baseline/install_reference.sh``).  Tests that need it skip when neither exists."""

from __future__ import annotations

import os
from pathlib import Path
from typing import Optional

ROOT = Path(__file__).resolve().parents[1]


def reference_dir() -> Optional[Path]:
    for cand in (os.environ.get("THESIS_REFERENCE"), ROOT / "baseline" / "_ref"):
        if cand and (Path(cand) / "common" / "engine.py").exists():
            return Path(cand).resolve()
    return None
