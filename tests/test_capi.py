"""libocb.so loads and exports every entry point that include/ocb.h declares
(no device calls: this runs without a GPU)."""
import ctypes
import re
from pathlib import Path

import pytest

from opencuda import _lib

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    text = "\n".join(p.read_text() for p in sorted((ROOT / "include").glob("*.h")))
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ocb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "ocb_create" in names and "ocb_lex_batch" in names
    assert len(names) >= 8


def test_library_exports_every_declared_symbol():
    if not _lib.LIB_PATH.is_file():
        pytest.fail("libocb.so not built: python -m opencuda.build")
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_signatures_cover_header():
    bound = {n for n, _, _ in _lib.SIGNATURES}
    assert set(declared_functions()) <= bound


def test_version_string():
    lib = _lib.load()
    assert b"sm_100a" in lib.ocb_version()
