"""The C-ABI library loads without a GPU and exports every symbol include/ckl_b200.h declares."""
from __future__ import annotations

import ctypes as C
import re

import pytest

from conftest import ROOT
from ckl import _native

HEADER = (ROOT / "include" / "ckl_b200.h").read_text()


def declared_functions():
    body = re.sub(r"/\*.*?\*/", "", HEADER, flags=re.S)
    names = set(re.findall(r"\b(ckl_[a-z0-9_]+)\s*\(", body))
    return sorted(names - {"ckl_entry_fn"})


def test_library_loads_and_exports_every_declared_symbol():
    lib = _native.load()
    missing = [name for name in declared_functions() if not hasattr(lib, name)]
    assert not missing, missing
    assert set(_native.EXPORTED) >= set(declared_functions())


def test_no_device_reports_unavailable_not_crash():
    lib = _native.load()
    count = C.c_int(-1)
    assert lib.ckl_device_count(C.byref(count)) == 0
    if count.value == 0:
        assert lib.ckl_cuda_available() == 0
        handle = C.c_void_p()
        assert lib.ckl_device_create(0, C.byref(handle)) != 0
        assert _native.message()


def test_runtime_symbols_are_the_eight_callbacks():
    lib = _native.load()
    table = (_native.RuntimeSymbol * 8)()
    assert lib.ckl_runtime_symbols(table) == 0
    names = [entry.name.decode() for entry in table]
    assert names == ["ckl_begin", "ckl_heap", "ckl_resource", "ckl_kernel",
                     "ckl_argument_resource", "ckl_argument_value", "ckl_dependency", "ckl_commit"]
    for entry in table:
        assert entry.address == C.cast(getattr(lib, entry.name.decode()), C.c_void_p).value


def test_library_catalogue_and_geometry():
    from ckl.compile import library_geometry
    from ckl.library import pack
    lib = _native.load()
    names = {lib.ckl_library_name(i).decode() for i in range(lib.ckl_library_count())}
    assert {"ckl.pointwise.add_scalar", "ckl.fused.attention", "ckl.decoder.greedy"} <= names
    grid, block, shared = library_geometry("ckl.decoder.linear", pack(512, 1024, 4096, 4, 1, 0, 0, 0, 0, 0, 512))
    assert grid[0] >= 1 and block[0] in (128, 256) and shared == 0
    with pytest.raises(Exception):
        library_geometry("ckl.decoder.linear", pack(1, 2, 3))          # wrong spec size
    with pytest.raises(Exception):
        library_geometry("no.such.kernel", b"")


def test_bind_rejects_before_device_work():
    lib = _native.load()
    handle = C.c_void_p()
    assert lib.ckl_program_create_from_plan(b"not a plan", None, C.byref(handle)) == _native.INVALID_ARGUMENT
    assert "unknown plan record" in _native.message() or "header" in _native.message()
