"""Where the reference package (turfur44/MuZO-Clip's ``muzo_clip``) is imported from — TEST
INFRASTRUCTURE.

``MUZO_REFERENCE_PATH`` names a directory that holds the ``muzo_clip`` package (a source checkout,
or a ``pip install --target`` directory). Without it, the offline install under ``baseline/_ref``
at the repository root is used when present (``pip install --no-index --no-deps --target
baseline/_ref <reference checkout>``; it is not committed, and travels with the working tree).
Tests that need the reference skip when neither exists.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]


def reference_path() -> Path | None:
    env = os.environ.get("MUZO_REFERENCE_PATH")
    candidates = [Path(env)] if env else [ROOT / "baseline" / "_ref"]
    for c in candidates:
        if (c / "muzo_clip" / "__init__.py").exists():
            return c
    return None


def import_reference():
    """The reference's ``muzo_clip`` module (its directory put first on sys.path), or None."""
    p = reference_path()
    if p is None:
        return None
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))
    import muzo_clip

    return muzo_clip
