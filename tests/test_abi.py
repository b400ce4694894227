"""The C-ABI library loads, exports every symbol include/flashgmm.h declares,
and rejects bad arguments before touching any device (no GPU needed)."""

import ctypes
import os
import re

import pytest

import _fgmm_lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = []
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            names += re.findall(r"FGMM_API\s+[\w\s\*]+?\b(fgmm_\w+)\s*\(", src)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(L.LIB_PATH):
        import build_lib
        build_lib.build()
    return L.load()


def test_header_declares_entry_points():
    names = declared_symbols()
    for n in ("fgmm_estep_iso", "fgmm_estep_diag", "fgmm_estep_full",
              "fgmm_workspace_bytes", "fgmm_last_error", "fgmm_version"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(L.LIB_PATH)
    for n in declared_symbols():
        assert hasattr(raw, n), f"{n} declared in include/ but not exported"


def test_version_and_workspace(lib):
    assert lib.fgmm_version() >= 100
    for v in (0, 1, 2):
        assert L.workspace_bytes(v, 1000, 64, 32) > 0
    assert L.workspace_bytes(0, 0, 1, 1) >= 0
    assert lib.fgmm_workspace_bytes(7, 10, 1, 1) == 0   # unknown variant


def test_bad_arguments_are_reported_without_a_device(lib):
    # negative N: rejected during validation, before any CUDA call
    code = lib.fgmm_estep_iso(None, 1, 1, None, 1, 1, None, None, -1, 4, 4,
                              None, None, None, None, None, 0, 0, None)
    assert code == 1
    assert b"invalid shape" in lib.fgmm_last_error()
    code = lib.fgmm_estep_full(None, 1, 1, None, 1, 1, None, None, 10, 4, 4,
                               None, None, None, None, None, 0, 0, None)
    assert code == 1 and b"null pointer" in lib.fgmm_last_error()


def test_estep_x_rejects_unknown_types_without_a_device(lib):
    f = ctypes.CDLL(L.LIB_PATH).fgmm_estep_x
    f.restype = ctypes.c_int
    args = [None, 1, 1, None, 1, 1, None, None, ctypes.c_int64(10), 4, 4,
            None, None, None, None, None, ctypes.c_size_t(0), ctypes.c_uint(0), None]
    assert f(0, 7, *args) == 1
    assert b"unknown x_type" in lib.fgmm_last_error()
    assert f(5, 0, *args) == 1
    assert b"unknown variant" in lib.fgmm_last_error()
