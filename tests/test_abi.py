"""The C-ABI library loads and exports every entry point include/*.h declares
(no GPU needed: symbols only, no compute calls)."""
import ctypes
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "scratchtape_b200", "libst_b200.so")


def _declared():
    names = set()
    for hdr in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(hdr).read()
        names.update(re.findall(r"^ST_API\s+[\w\s\*]+?\b(st_\w+)\s*\(", src, flags=re.M))
    return sorted(names)


def test_header_declares_entry_points():
    names = _declared()
    assert "st_gemm" in names and "st_create" in names
    assert len(names) >= 10


def test_library_exports_every_declared_symbol():
    assert os.path.exists(LIB), "build the library first (__graft_entry__.build())"
    lib = ctypes.CDLL(LIB)
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    import scratchtape_b200._native as N
    assert set(N.SIGNATURES) == set(_declared())


def test_null_handle_is_an_error_not_a_crash():
    lib = ctypes.CDLL(LIB)
    lib.st_gemm.restype = ctypes.c_int
    assert lib.st_gemm(None, None, None, None, 1, 1, 1, 1, None, 0) == 1  # ST_INVALID_ARG
    lib.st_last_error.restype = ctypes.c_char_p
    assert lib.st_last_error(None) == b"null handle"
