"""The C-ABI library loads without a GPU and exports every function that
include/sarbon_sparse.h declares; calls that need no device behave."""
import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "sarbon_sparse.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^SB_API\s+[\w\s\*]+?\b(sb_\w+)\s*\(", text, re.M)))


def test_header_declares_the_api():
    names = declared()
    for must in ("sb_create", "sb_step", "sb_reset", "sb_upload_weights", "sb_set_extra", "sb_cache_ptr",
                 "sb_debug_lists", "sb_stats", "sb_destroy"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from sarbon_b200 import _lib
    lib = _lib.lib()  # raises if the .so is missing or lacks a prototype symbol
    for name in declared():
        assert hasattr(lib, name), name
    assert set(declared()) == set(_lib.PROTOTYPES), "ctypes prototypes out of sync with the header"


def test_host_only_calls():
    from sarbon_b200 import _lib
    lib = _lib.lib()
    assert b"sm_100a" in lib.sb_version()
    assert lib.sb_destroy(None) == _lib.SB_OK
    # argument validation happens before any device call
    out = C.c_void_p()
    rc = lib.sb_create(None, 0, 1, 64, 64, 32, 0, 0.0, 0, 4, C.byref(out))
    assert rc == _lib.SB_EINVAL
    assert b"null" in lib.sb_last_error()
    descs = (_lib.LayerDesc * 1)(_lib.LayerDesc(0, -1, 3, 32, 2, 2, 1, 1))
    assert lib.sb_create(descs, 1, 1, 100, 64, 32, 0, 0.0, 0, 4, C.byref(out)) == _lib.SB_EINVAL
    assert b"divisible" in lib.sb_last_error()


def test_engine_fails_loudly_without_library(monkeypatch, tmp_path):
    from sarbon_b200 import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "missing.so")
    with pytest.raises(_lib.SarbonLibraryError):
        _lib.lib()
