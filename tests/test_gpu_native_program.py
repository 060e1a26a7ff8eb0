"""The eight plan-building callbacks driven by hand with a CUBIN, through the C ABI.

Restates tests/Runtime/NvidiaProgramValidation.cpp:23-108: a hand-written packed entry stands
in for generated host code; scalars of four types are packed; two `join` nodes with one
dependency run in ordinary, graph and capture modes with batch 2; a mismatched scalar type is
rejected; a failing callback latches its error and binding reports it.
"""
from __future__ import annotations

import ctypes as C
import struct

import numpy as np
import pytest

from conftest import ROOT
from ckl import _native

pytestmark = pytest.mark.gpu
CUBIN = (ROOT / "tests" / "native" / "runtime_kernels.cubin").read_bytes()


def callbacks():
    lib = _native.load()
    table = (_native.RuntimeSymbol * 8)()
    assert lib.ckl_runtime_symbols(table) == 0
    proto = {
        "ckl_begin": C.CFUNCTYPE(None, C.c_void_p, C.c_char_p, C.c_uint64),
        "ckl_heap": C.CFUNCTYPE(None, C.c_void_p, C.c_uint64, C.c_uint64),
        "ckl_resource": C.CFUNCTYPE(None, C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_void_p),
        "ckl_kernel": C.CFUNCTYPE(None, C.c_void_p, C.c_char_p, *([C.c_uint64] * 7)),
        "ckl_argument_resource": C.CFUNCTYPE(None, C.c_void_p, C.c_uint64, C.c_uint64),
        "ckl_argument_value": C.CFUNCTYPE(None, C.c_void_p, C.c_void_p, C.c_uint64),
        "ckl_dependency": C.CFUNCTYPE(None, C.c_void_p, C.c_uint64),
        "ckl_commit": C.CFUNCTYPE(None, C.c_void_p, C.c_uint64),
    }
    return {e.name.decode(): proto[e.name.decode()](e.address) for e in table}


CB = callbacks()


@_native.ENTRY
def entry(packed):
    frame = C.cast(packed[0], C.POINTER(C.c_void_p))[0]
    args = C.cast(C.cast(packed[1], C.POINTER(C.c_void_p))[0], C.POINTER(C.c_void_p))
    assert C.cast(args[4], C.POINTER(C.c_float))[0] == 1.25
    assert C.cast(args[5], C.POINTER(C.c_double))[0] == -2.5
    assert C.cast(args[6], C.POINTER(C.c_int64))[0] == -1234567890123
    CB["ckl_begin"](frame, CUBIN, len(CUBIN))
    CB["ckl_heap"](frame, 0, 128)
    for i in range(3):
        CB["ckl_resource"](frame, i, 0, 0, args[i])
    CB["ckl_resource"](frame, 3, 0, 0, None)
    for node in (2, 5):
        CB["ckl_kernel"](frame, b"join", 1, 1, 1, 32, 1, 1, 0)
        CB["ckl_argument_resource"](frame, 0 if node == 2 else 3, 0)
        CB["ckl_argument_resource"](frame, 1, 0)
        CB["ckl_argument_resource"](frame, 3 if node == 2 else 2, 0)
        CB["ckl_argument_value"](frame, args[3], 4)
        if node == 5:
            CB["ckl_dependency"](frame, 2)
        CB["ckl_commit"](frame, node)


@_native.ENTRY
def failing_entry(packed):
    frame = C.cast(packed[0], C.POINTER(C.c_void_p))[0]
    CB["ckl_argument_resource"](frame, 999, 0)   # records an error instead of unwinding
    CB["ckl_argument_resource"](frame, 0, 0)     # later callbacks are no-ops


def program(lib, function):
    sizes = (C.c_uint64 * 7)(128, 128, 128, 0, 0, 0, 0)
    types = (C.c_char_p * 7)(b"", b"", b"", b"i32", b"f32", b"f64", b"i64")
    handle = C.c_void_p()
    _native.check(lib.ckl_program_create(function, 7, sizes, types, None, C.byref(handle)))
    return handle


def arguments(buffers, scalar3=("i32", 32)):
    args = (_native.Argument * 7)()
    for i, b in enumerate(buffers):
        args[i].kind, args[i].buffer = _native.ARG_BUFFER, b
    kinds = {"i32": (_native.ARG_I32, "<i"), "f32": (_native.ARG_F32, "<f")}
    kind, code = kinds[scalar3[0]]
    args[3].kind, args[3].bits = kind, int.from_bytes(struct.pack(code, scalar3[1]).ljust(8, b"\0"), "little")
    args[4].kind, args[4].bits = _native.ARG_F32, int.from_bytes(struct.pack("<f", 1.25).ljust(8, b"\0"), "little")
    args[5].kind, args[5].bits = _native.ARG_F64, int.from_bytes(struct.pack("<d", -2.5), "little")
    args[6].kind, args[6].bits = _native.ARG_I64, int.from_bytes(struct.pack("<q", -1234567890123), "little")
    return args


def test_callback_protocol_modes_and_errors():
    lib = _native.load()
    device = C.c_void_p()
    _native.check(lib.ckl_device_create(0, C.byref(device)))
    buffers = []
    for values in (np.ones(32, np.float32), np.full(32, 3, np.float32), np.zeros(32, np.float32)):
        handle = C.c_void_p()
        _native.check(lib.ckl_buffer_allocate(device, 128, C.byref(handle)))
        _native.check(lib.ckl_buffer_copy_from_host(handle, values.ctypes.data, 128))
        buffers.append(handle.value)
    prog = program(lib, entry)
    inv = C.c_void_p()
    _native.check(lib.ckl_bind(prog, device, 7, arguments(buffers), C.byref(inv)))
    count = C.c_uint64()
    _native.check(lib.ckl_node_count(inv, C.byref(count)))
    assert count.value == 2
    result = np.zeros(32, np.float32)
    timing = (C.c_double * 3)()
    for mode in (0, 1, 2):
        _native.check(lib.ckl_run(inv, mode, 2))
        _native.check(lib.ckl_buffer_copy_to_host(buffers[2], result.ctypes.data, 128))
        assert np.all(result == np.float32(2.21875))
        _native.check(lib.ckl_benchmark(inv, mode, 2, 2, timing))
        assert all(v >= 0 for v in timing)
    wrong = C.c_void_p()
    assert lib.ckl_bind(prog, device, 7, arguments(buffers, ("f32", 32.0)), C.byref(wrong)) == _native.INVALID_ARGUMENT
    failing = program(lib, failing_entry)
    assert lib.ckl_bind(failing, device, 7, arguments(buffers), C.byref(wrong)) == _native.RUNTIME_ERROR
    again = C.c_void_p()
    _native.check(lib.ckl_bind(prog, device, 7, arguments(buffers), C.byref(again)))
    _native.check(lib.ckl_run(again, 1, 1))
    assert lib.ckl_run(again, 1, 1000001) == _native.INVALID_ARGUMENT
    for h in (inv, again):
        lib.ckl_invocation_release(h)
    for h in (prog, failing):
        lib.ckl_program_release(h)
    for b in buffers:
        lib.ckl_buffer_release(b)
    lib.ckl_device_release(device)
