"""Where the tests find the reference ``thetascan`` package.

``$THETASCAN_REFERENCE_PATH`` names a directory that holds the package (for
instance the reference project's ``src``); without it the tests use the
offline install under ``baseline/_ref`` at the repository root, which travels
with the repository to a GPU host.  ``import_reference()`` puts that directory
on ``sys.path`` and imports the package, or skips the calling test when it is
not there.
"""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def reference_dir():
    env = os.environ.get("THETASCAN_REFERENCE_PATH")
    if env:
        return env
    path = os.path.join(ROOT, "baseline", "_ref")
    return path if os.path.isdir(os.path.join(path, "thetascan")) else None


def import_reference():
    path = reference_dir()
    if path and path not in sys.path:
        sys.path.insert(0, path)
    return pytest.importorskip("thetascan")
