"""The C-ABI library builds, loads and exports what include/bfknn.h declares
(no compute calls: this runs without a GPU)."""
import ctypes
import os
import re

import pytest

from gpu_algo_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "bfknn.h")).read()
    return sorted(set(re.findall(r"BFK_API\s+[\w\s\*]*?\b(bfk_\w+)\s*\(", src)))


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(_lib.EXPORTS)


def test_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
    out = os.popen(f"nm -D --defined-only {_lib.LIB_PATH}").read()
    exported = set(re.findall(r"\bT (bfk_\w+)", out))
    assert exported == set(declared_symbols())


def test_version_and_status_strings(lib):
    assert _lib.version() == (0, 1)
    for code in range(7):
        assert _lib.status_string(code) not in ("", "unknown status")
    assert _lib.status_string(99) == "unknown status"


def test_argument_validation_without_gpu(lib):
    nb = ctypes.c_uint64()
    o = _lib.make_opts()
    assert lib.bfk_workspace_size(-1, 10, 8, 1, ctypes.byref(o), ctypes.byref(nb)) == 1
    assert lib.bfk_workspace_size(10, 10, 8, 0, ctypes.byref(o), ctypes.byref(nb)) == 1
    assert lib.bfk_workspace_size(10, 10, 8, 5000, ctypes.byref(o), ctypes.byref(nb)) == 2
    o.reserved[2] = 1
    assert lib.bfk_workspace_size(10, 10, 8, 1, ctypes.byref(o), ctypes.byref(nb)) == 1
    o = _lib.make_opts()
    o.shards = -1
    assert lib.bfk_workspace_size(10, 10, 8, 1, ctypes.byref(o), ctypes.byref(nb)) == 1
    o = _lib.make_opts("direct")
    assert lib.bfk_workspace_size(1024, 65536, 128, 10, ctypes.byref(o), ctypes.byref(nb)) == 0
    assert nb.value % 256 == 0 and nb.value >= 256
    # invalid arguments are rejected before any device work
    assert lib.bfk_search(None, 4, None, 4, 8, 1, 0, None, None, None, 0, None, None) == 1
    assert lib.bfk_merge(None, None, 4, 0, 1, None, None, None) == 1


def test_workspace_has_room_for_partials(lib):
    o = _lib.make_opts("direct", slices=8)
    nb = ctypes.c_uint64()
    assert lib.bfk_workspace_size(100, 10_000, 16, 10, ctypes.byref(o), ctypes.byref(nb)) == 0
    assert nb.value >= 8 * 100 * 10 * 8
