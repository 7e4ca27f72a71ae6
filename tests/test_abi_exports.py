"""The C-ABI library loads without a GPU and exports every function include/rfsn_b200.h declares.

No compute calls are made here (no GPU is needed); the ctypes signature table
in apple_b200/_lib.py is also checked against the header so the Python
binding and the ABI cannot drift apart.
"""
import ctypes
import re

import pytest

from tests.conftest import ROOT

HEADER = ROOT / "include" / "rfsn_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(rfsn_[a-z_0-9]+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("rfsn_encode", "rfsn_decode_codes", "rfsn_decode_attention", "rfsn_attention_workspace_size",
                     "rfsn_cold_prefetch", "rfsn_version", "rfsn_status_string"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from apple_b200 import _lib
    if not _lib.LIB_PATH.exists():
        pytest.fail(f"{_lib.LIB_PATH} is not built (python apple_b200/csrc/build.py)")
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_table_matches_header():
    from apple_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_status_strings_without_gpu():
    from apple_b200 import _lib
    lib = _lib.lib()
    assert lib.rfsn_version() // 1000 == 1
    assert lib.rfsn_status_string(0) == b"ok"
    assert b"timed out" in lib.rfsn_status_string(-5)
