"""The C-ABI library loads without a GPU and exports every declared symbol."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "thetascan_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ts_b200_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "ts_b200_scan_fwd" in names and "ts_b200_scan_bwd" in names
    assert len(names) >= 8


def test_library_exports_every_declared_symbol():
    from thetascan_b200 import _lib, build
    build.build()
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_binding_table_covers_the_header():
    from thetascan_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_version_and_error_reporting_without_a_gpu():
    from thetascan_b200 import _lib
    lib = _lib.load()
    assert b"sm_100a" in lib.ts_b200_version()
    # A null argument struct is rejected on the host with TS_ERR_VALUE.
    assert lib.ts_b200_scan_fwd(None, None) == _lib.TS_ERR_VALUE
    code, message = _lib.last_error()
    assert code == _lib.TS_ERR_VALUE and "null" in message
    with pytest.raises(ValueError):
        _lib.check(code)
