"""Locate and import the B200 package from a model.py that the harness loaded by path."""
from __future__ import annotations

import importlib
import sys
from pathlib import Path


def load_b200_package():
    pkg_dir = Path(__file__).resolve().parents[2]  # .../lumen-sosp26-ae_b200
    root = str(pkg_dir.parent)
    if root not in sys.path:
        sys.path.insert(0, root)
    pkg = importlib.import_module(pkg_dir.name)
    pkg._cabi.load()  # raises if liblumen_b200.so is absent: no fallback
    return pkg
