"""The reference package installed beside this repository, for drop-in checks.

``baseline/_ref`` holds the reference (kvsnap) as its own installer built it
(``pip install --target baseline/_ref``, with its CUDA pool). It is not part
of the product and is not in version control; tests that need it skip when it
is absent. Its modules import under their own package name, ``kvsnap``.
"""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

import pytest

INSTALL = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def reference(module: str):
    """Import ``kvsnap.<module>`` from the installed reference, or skip the calling test."""
    if not (INSTALL / "kvsnap" / "__init__.py").is_file():
        pytest.skip("the reference is not installed under baseline/_ref")
    if str(INSTALL) not in sys.path:
        sys.path.append(str(INSTALL))
    return importlib.import_module(f"kvsnap.{module}")
