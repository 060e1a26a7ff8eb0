"""ctypes binding of libckl_b200.so (declared in include/ckl_b200.h).

The library is built in-tree (``composable-kernel-language_b200/build.py``); ``CKL_NATIVE_LIBRARY``
may point at another build.  There is no pure-Python fallback: a missing library raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_LIBRARY = None

OK, INVALID_ARGUMENT, RUNTIME_ERROR, OUT_OF_RANGE = 0, 1, 2, 3
ARG_BUFFER, ARG_I32, ARG_I64, ARG_F32, ARG_F64 = 0, 1, 2, 3, 4


class Argument(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("reserved", C.c_uint32), ("buffer", C.c_void_p),
                ("bits", C.c_uint64)]


class GraphNode(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("unknown", C.c_uint32), ("first_access", C.c_uint32),
                ("access_count", C.c_uint32)]


class GraphAccess(C.Structure):
    _fields_ = [("resource", C.c_uint32), ("bits", C.c_uint32), ("offset", C.c_int64),
                ("length", C.c_int64)]


class GraphResource(C.Structure):
    _fields_ = [("temporary", C.c_uint32), ("device", C.c_int32), ("bytes", C.c_uint64),
                ("alignment", C.c_uint64)]


class RuntimeSymbol(C.Structure):
    _fields_ = [("name", C.c_char_p), ("address", C.c_size_t)]


ENTRY = C.CFUNCTYPE(None, C.POINTER(C.c_void_p))

_PROTOTYPES = {
    "ckl_last_error": (C.c_char_p, []),
    "ckl_cuda_available": (C.c_int, []),
    "ckl_device_count": (C.c_int, [C.POINTER(C.c_int)]),
    "ckl_device_create": (C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    "ckl_device_release": (None, [C.c_void_p]),
    "ckl_device_name": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t]),
    "ckl_device_ordinal": (C.c_int, [C.c_void_p]),
    "ckl_buffer_allocate": (C.c_int, [C.c_void_p, C.c_uint64, C.POINTER(C.c_void_p)]),
    "ckl_buffer_import": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint64, C.POINTER(C.c_void_p)]),
    "ckl_buffer_slice": (C.c_int, [C.c_void_p, C.c_uint64, C.c_uint64, C.POINTER(C.c_void_p)]),
    "ckl_buffer_release": (None, [C.c_void_p]),
    "ckl_buffer_address": (C.c_uint64, [C.c_void_p]),
    "ckl_buffer_size": (C.c_uint64, [C.c_void_p]),
    "ckl_buffer_copy_from_host": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64]),
    "ckl_buffer_copy_to_host": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64]),
    "ckl_buffer_fill_zero": (C.c_int, [C.c_void_p]),
    "ckl_host_alloc": (C.c_int, [C.c_uint64, C.POINTER(C.c_void_p)]),
    "ckl_host_free": (None, [C.c_void_p]),
    "ckl_program_create": (C.c_int, [ENTRY, C.c_uint32, C.POINTER(C.c_uint64),
                                     C.POINTER(C.c_char_p), C.c_void_p, C.POINTER(C.c_void_p)]),
    "ckl_program_create_from_plan": (C.c_int, [C.c_char_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    "ckl_program_release": (None, [C.c_void_p]),
    "ckl_bind": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.POINTER(Argument),
                           C.POINTER(C.c_void_p)]),
    "ckl_invocation_release": (None, [C.c_void_p]),
    "ckl_run": (C.c_int, [C.c_void_p, C.c_int, C.c_uint64]),
    "ckl_benchmark": (C.c_int, [C.c_void_p, C.c_int, C.c_uint64, C.c_uint64,
                                C.POINTER(C.c_double)]),
    "ckl_node_count": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint64)]),
    "ckl_node_name": (C.c_int, [C.c_void_p, C.c_uint64, C.c_char_p, C.c_size_t]),
    "ckl_node_argument_sizes": (C.c_int, [C.c_void_p, C.c_uint64, C.POINTER(C.c_uint64),
                                          C.c_uint32, C.POINTER(C.c_uint32)]),
    "ckl_update_kernel": (C.c_int, [C.c_void_p, C.c_int, C.c_uint64, C.c_uint64, C.c_uint32,
                                    C.POINTER(C.c_void_p), C.POINTER(C.c_uint64),
                                    C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.c_int64]),
    "ckl_launch": (C.c_int, [C.c_void_p, C.c_int, C.c_uint64]),
    "ckl_synchronize": (C.c_int, [C.c_void_p]),
    "ckl_copy_in_async": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64]),
    "ckl_copy_out_async": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64]),
    "ckl_record": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "ckl_wait_for": (C.c_int, [C.c_void_p, C.c_void_p]),
    "ckl_completion_query": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "ckl_completion_wait": (C.c_int, [C.c_void_p, C.c_uint64, C.POINTER(C.c_int)]),
    "ckl_completion_release": (None, [C.c_void_p]),
    "ckl_time_launches": (C.c_int, [C.c_void_p, C.c_int, C.c_uint64, C.c_uint64,
                                    C.POINTER(C.c_double)]),
    "ckl_profile_nodes": (C.c_int, [C.c_void_p, C.c_uint64, C.POINTER(C.c_double), C.c_uint64]),
    "ckl_greedy_head_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float,
                                          C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_void_p,
                                          C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "ckl_profiler_start": (C.c_int, []),
    "ckl_profiler_stop": (C.c_int, []),
    "ckl_runtime_symbols": (C.c_int, [C.POINTER(RuntimeSymbol)]),
    "ckl_library_geometry": (C.c_int, [C.c_char_p, C.c_void_p, C.c_uint64,
                                       C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                       C.POINTER(C.c_uint32)]),
    "ckl_library_signature": (C.c_int, [C.c_char_p, C.c_char_p, C.c_size_t]),
    "ckl_library_faults": (C.c_int, [C.POINTER(C.c_uint32), C.c_int]),
    "ckl_set_wait_limit": (C.c_int, [C.c_int, C.c_uint64]),
    "ckl_inject_unsignalled_wait": (C.c_int, [C.c_int, C.c_int]),
    "ckl_library_count": (C.c_uint32, []),
    "ckl_library_name": (C.c_char_p, [C.c_uint32]),
    "ckl_cuda_compile": (C.c_int, [C.c_char_p, C.c_char_p, C.POINTER(C.c_void_p),
                                   C.POINTER(C.c_uint64)]),
    "ckl_binary_free": (None, [C.c_void_p]),
    "ckl_graph_plan_create": (C.c_int, [C.c_uint32, C.POINTER(GraphNode), C.c_uint32,
                                        C.POINTER(GraphAccess), C.c_uint32,
                                        C.POINTER(GraphResource), C.c_uint32,
                                        C.POINTER(C.c_void_p)]),
    "ckl_graph_plan_release": (None, [C.c_void_p]),
    "ckl_graph_plan_edge_count": (C.c_uint64, [C.c_void_p]),
    "ckl_graph_plan_edges": (None, [C.c_void_p, C.POINTER(C.c_uint32)]),
    "ckl_graph_plan_dependency_count": (C.c_uint64, [C.c_void_p, C.c_uint32]),
    "ckl_graph_plan_dependencies": (None, [C.c_void_p, C.c_uint32, C.POINTER(C.c_uint32)]),
    "ckl_graph_plan_resource_count": (C.c_uint64, [C.c_void_p]),
    "ckl_graph_plan_resources": (None, [C.c_void_p, C.POINTER(C.c_uint32)]),
    "ckl_graph_plan_memory": (None, [C.c_void_p, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                     C.POINTER(C.c_uint32)]),
    "ckl_graph_plan_heaps": (None, [C.c_void_p, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "ckl_graph_plan_assignment": (C.c_int, [C.c_void_p, C.c_uint32, C.POINTER(C.c_uint64),
                                            C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "ckl_memory_plan": (C.c_int, [C.c_uint32, C.c_uint32, C.POINTER(C.c_uint32), C.c_uint32,
                                  C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                  C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                  C.POINTER(C.c_uint32), C.c_int, C.POINTER(C.c_uint64),
                                  C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                  C.POINTER(C.c_uint64)]),
    "ckl_repeat_dependencies": (C.c_int, [C.c_uint32, C.POINTER(C.c_uint32),
                                          C.POINTER(C.c_uint32), C.c_uint32,
                                          C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                          C.c_uint64]),
}

#: Every function the C header declares (checked by the CPU tests against the header).
EXPORTED = tuple(_PROTOTYPES) + ("ckl_begin", "ckl_heap", "ckl_resource", "ckl_kernel",
                                 "ckl_argument_resource", "ckl_argument_value",
                                 "ckl_dependency", "ckl_commit")


def library_path() -> Path:
    configured = os.environ.get("CKL_NATIVE_LIBRARY")
    return Path(configured) if configured else Path(__file__).with_name("libckl_b200.so")


def load():
    """Load (once) and return the native library with prototypes applied."""
    global _LIBRARY
    if _LIBRARY is not None:
        return _LIBRARY
    path = library_path()
    if not path.is_file():
        raise RuntimeError(f"CKL native library is not built ({path}); run "
                           "composable-kernel-language_b200/build.py")
    lib = C.CDLL(str(path))
    for name, (restype, argtypes) in _PROTOTYPES.items():
        function = getattr(lib, name)
        function.restype = restype
        function.argtypes = argtypes
    _LIBRARY = lib
    return lib


def compile_cuda(source: str, name: str = "ckl_generated.cu") -> bytes:
    """sm_100a CUBIN of CUDA C++ source (NVRTC through the native library)."""
    lib = load()
    binary, size = C.c_void_p(), C.c_uint64()
    check(lib.ckl_cuda_compile(source.encode(), name.encode(), C.byref(binary), C.byref(size)),
          "ckl_cuda_compile")
    try:
        return C.string_at(binary, size.value)
    finally:
        lib.ckl_binary_free(binary)


def library_faults(reset: bool = False) -> int:
    """The kernel library's fault word on the current device (``ckl_library_faults``)."""
    value = C.c_uint32()
    check(load().ckl_library_faults(C.byref(value), int(reset)), "ckl_library_faults")
    return value.value


def message() -> str:
    return (load().ckl_last_error() or b"").decode(errors="replace")


def check(status: int, what: str = "") -> None:
    """Map a C ABI status to the reference's Python exception classes."""
    if status == OK:
        return
    text = message()
    if what:
        text = f"{what}: {text}"
    if status in (INVALID_ARGUMENT, OUT_OF_RANGE):
        raise ValueError(text)
    raise RuntimeError(text)
