"""Locating the reference package (MaskAhead's src/maskahead) for the drop-in tests.

It is imported from MASKAHEAD_REF_SRC (a folder holding maskahead/) when that is set,
else from baseline/_ref, where baseline/install_reference.sh installs it. None when
neither holds it: the drop-in tests skip.
"""

from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def reference_package():
    """The imported reference package, or None."""
    if "maskahead" in sys.modules:
        return sys.modules["maskahead"]
    where = os.environ.get("MASKAHEAD_REF_SRC") or str(ROOT / "baseline" / "_ref")
    if not (Path(where) / "maskahead" / "runtime" / "session.py").is_file():
        return None
    sys.path.insert(0, where)
    try:
        pkg = importlib.import_module("maskahead")
        importlib.import_module("maskahead.runtime.session")
    except Exception:
        sys.path.remove(where)
        return None
    return pkg
