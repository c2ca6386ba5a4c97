"""Locates the host framework: the reference MIRA compiler package `mira`.

The cuda target is a plug-in for MIRA, so the `mira` package must be importable.  It is taken
from sys.path when installed, else from the directory named by $MIRA_PATH, else from the
`baseline/_ref` install next to this package.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def import_mira():
    try:
        import mira  # noqa: F401
        return sys.modules["mira"]
    except ImportError:
        pass
    for cand in (os.environ.get("MIRA_PATH"), str(REPO / "baseline" / "_ref")):
        if cand and (Path(cand) / "mira" / "__init__.py").exists():
            if cand not in sys.path:
                sys.path.insert(0, cand)
            import mira  # noqa: F401
            return sys.modules["mira"]
    raise ImportError("the MIRA host framework (package `mira`) is not importable: install it, or set MIRA_PATH "
                      "to the directory that contains it")
