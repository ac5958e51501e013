"""The C-ABI library loads on a machine without a GPU and exports every entry point include/fp4x.h declares
(no compute calls here)."""
import ctypes
import os
import re

import fp4x_native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "fp4x.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(fp4x_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(N.LIB_PATH)
    decl = declared_functions()
    assert len(decl) >= 10
    for name in decl:
        assert hasattr(lib, name), name


def test_binding_covers_header():
    assert sorted(N.exported_symbols()) == declared_functions()


def test_version_and_error_message_without_gpu():
    L = N.lib()
    assert L.fp4x_version() >= 100
    assert isinstance(L.fp4x_last_error_message(), bytes)
