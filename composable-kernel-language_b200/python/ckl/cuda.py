"""Devices, buffers, compiled programs and bound invocations on the B200 runtime.

Same public surface and argument validation as the reference (``python/ckl/cuda.py:65-300``):
``Device``, ``DeviceBuffer``, ``CompiledProgram.bind/run`` and ``Invocation.run/benchmark/
node_count``, context-manager scopes with idempotent ``close()``, ``TypeError``/``ValueError``
for bad arguments before native code runs, ``RuntimeError`` for runtime failures.  Additions
for the B200 build: ``Device(ordinal)`` for multi-GPU jobs, asynchronous submission and
host copies on the invocation's stream, and node inspection.
"""
from __future__ import annotations

import ctypes as C
import math
import struct
import weakref
from contextlib import AbstractContextManager
from pathlib import Path

from . import _native as _abi
from .compiler import NVIDIATarget, SUPPORTED_CHIPS
from .types import BufferSpec, f32, f64, i32, i64

_SCALARS = {f32: ("f", 4), f64: ("d", 8), i32: ("i", 4), i64: ("q", 8)}
_ARG_KIND = {f32: _abi.ARG_F32, f64: _abi.ARG_F64, i32: _abi.ARG_I32, i64: _abi.ARG_I64}
_MODES = {"ordinary": 0, "graph": 1, "capture": 2}


def _byte_count(spec) -> int:
    if not isinstance(spec, BufferSpec) or spec.dtype not in _SCALARS:
        raise TypeError("device storage requires a numeric BufferSpec")
    size = math.prod(spec.shape) * _SCALARS[spec.dtype][1]
    if not 0 < size < (1 << 64):
        raise ValueError("device storage byte count must fit a positive 64-bit size")
    return size


class _Handle:
    """Owns one native handle; released when the last Python reference goes away."""

    __slots__ = ("value", "__weakref__")

    def __init__(self, value: int, release):
        self.value = value
        weakref.finalize(self, release, value)


def _host_pointer(obj, writable: bool):
    """(pointer, nbytes, keepalive) of a contiguous Python buffer."""
    view = memoryview(obj)
    if not view.contiguous:
        raise ValueError("host buffers must be contiguous")
    view = view.cast("B")
    if writable and view.readonly:
        raise ValueError("destination must be writable and match device storage byte count")
    if view.nbytes == 0:
        return 0, 0, view
    import numpy as np  # pointer extraction only

    array = np.frombuffer(view, dtype=np.uint8)
    return array.ctypes.data, view.nbytes, (view, array)


class _ContextManager(AbstractContextManager):
    _resource = None

    @property
    def _native_resource(self):
        if self._resource is None:
            raise RuntimeError(f"{type(self).__name__} is closed")
        return self._resource

    @property
    def closed(self):
        return self._resource is None

    def close(self):
        self._resource = None

    def __enter__(self):
        _ = self._native_resource
        return self

    def __exit__(self, exc_type, exc_value, traceback):
        self.close()
        return False


class Device(_ContextManager):
    """One CUDA device (default ordinal 0).  Construction initializes CUDA on it."""

    def __init__(self, ordinal: int = 0):
        if type(ordinal) is not int or ordinal < 0:
            raise ValueError("device ordinal must be a nonnegative int")
        self._lib = _abi.load()
        if not self._lib.ckl_cuda_available():
            raise RuntimeError("no CUDA device is available to the CKL runtime")
        handle = C.c_void_p()
        _abi.check(self._lib.ckl_device_create(ordinal, C.byref(handle)), "device")
        self._resource = _Handle(handle.value, self._lib.ckl_device_release)
        self.ordinal = ordinal

    @property
    def native_library(self) -> Path:
        return _abi.library_path().resolve()

    @property
    def name(self) -> str:
        buffer = C.create_string_buffer(256)
        _abi.check(self._lib.ckl_device_name(self._native_resource.value, buffer, 256))
        return buffer.value.decode()

    def empty(self, spec: BufferSpec) -> "DeviceBuffer":
        size = _byte_count(spec)
        handle = C.c_void_p()
        _abi.check(self._lib.ckl_buffer_allocate(self._native_resource.value, size,
                                                    C.byref(handle)), "allocate")
        return DeviceBuffer(self, _Handle(handle.value, self._lib.ckl_buffer_release), spec)

    def import_buffer(self, address: int, spec: BufferSpec, *, owner) -> "DeviceBuffer":
        """Borrow device storage, retaining its Python owner for the buffer's lifetime."""
        size = _byte_count(spec)
        if type(address) is not int or not 0 < address < (1 << 64) or owner is None:
            raise ValueError("imported storage requires a valid address and a live owner")
        handle = C.c_void_p()
        _abi.check(self._lib.ckl_buffer_import(self._native_resource.value, address, size,
                                                  C.byref(handle)), "import")
        return DeviceBuffer(self, _Handle(handle.value, self._lib.ckl_buffer_release), spec, owner)


class DeviceBuffer(_ContextManager):
    def __init__(self, device, resource, spec, owner=None):
        self.device, self.spec, self._owner = device, spec, owner
        self._lib = device._lib
        self._resource = resource
        # Borrowed storage keeps its owner's native allocation alive as well.
        self._owner_resource = owner._resource if isinstance(owner, DeviceBuffer) else None

    def close(self):
        super().close()
        self.device = self._owner = None

    @property
    def address(self) -> int:
        return int(self._lib.ckl_buffer_address(self._native_resource.value))

    @property
    def nbytes(self) -> int:
        return int(self._lib.ckl_buffer_size(self._native_resource.value))

    def subview(self, *, offset: int, shape: tuple) -> "DeviceBuffer":
        """A bounded contiguous view; ``offset`` is in elements of this buffer."""
        spec = BufferSpec(shape, self.spec.dtype)
        size = _byte_count(spec)
        if type(offset) is not int or offset < 0:
            raise ValueError("subview requires a nonnegative element offset")
        byte_offset = offset * _SCALARS[self.spec.dtype][1]
        if byte_offset > self.nbytes or size > self.nbytes - byte_offset:
            raise ValueError("subview exceeds its source buffer")
        handle = C.c_void_p()
        _abi.check(self._lib.ckl_buffer_slice(self._native_resource.value, byte_offset, size,
                                                 C.byref(handle)), "subview")
        return DeviceBuffer(self.device, _Handle(handle.value, self._lib.ckl_buffer_release),
                            spec, self)

    def copy_from_host(self, source):
        pointer, nbytes, keep = _host_pointer(source, writable=False)
        if nbytes != self.nbytes:
            raise ValueError("host buffer byte count does not match device storage")
        _abi.check(self._lib.ckl_buffer_copy_from_host(self._native_resource.value, pointer,
                                                          nbytes), "copy_from_host")

    def fill_zero(self):
        _abi.check(self._lib.ckl_buffer_fill_zero(self._native_resource.value), "fill_zero")

    def copy_to_host(self, destination):
        pointer, nbytes, keep = _host_pointer(destination, writable=True)
        if nbytes != self.nbytes:
            raise ValueError("destination must be writable and match device storage byte count")
        _abi.check(self._lib.ckl_buffer_copy_to_host(self._native_resource.value, pointer,
                                                        nbytes), "copy_to_host")


class _NativeProgram:
    """A native program built from an executable plan (optionally with a fallback)."""

    def __init__(self, lib, plans):
        self._lib = lib
        fallback = None
        if plans.fallback is not None:
            handle = C.c_void_p()
            _abi.check(lib.ckl_program_create_from_plan(plans.fallback.text.encode(), None,
                                                           C.byref(handle)), "program")
            fallback = _Handle(handle.value, lib.ckl_program_release)
        handle = C.c_void_p()
        _abi.check(lib.ckl_program_create_from_plan(
            plans.primary.text.encode(), fallback.value if fallback else None, C.byref(handle)),
            "program")
        self.fallback = fallback
        self.handle = _Handle(handle.value, lib.ckl_program_release)


class CompiledProgram(_ContextManager):
    """A program resolved onto the sm_100a kernel library (and kernels generated from the bodies
    the library does not implement) with its planned graph and storage."""

    def __init__(self, program, target: NVIDIATarget, *, fuse_pointwise=True, reuse_storage=True,
                 fuse_library=True, tensor_cores=True, library=True, whole_step=True):
        if type(fuse_pointwise) is not bool:
            raise TypeError("fuse_pointwise must be bool")
        if type(reuse_storage) is not bool:
            raise TypeError("reuse_storage must be bool")
        if any(type(v) is not bool for v in (fuse_library, tensor_cores, library, whole_step)):
            raise TypeError("fuse_library, tensor_cores, library and whole_step must be bool")
        if not isinstance(target, NVIDIATarget) or target.binary_format != "bin":
            raise ValueError("CKL CUDA compilation requires a binary target")
        if target.chip not in SUPPORTED_CHIPS:
            raise ValueError(f"this build generates sm_100a code only; got chip {target.chip!r}")
        from .compile import plan_program

        self.signature, self.target = program.signature, target
        self.lowered = program
        self._lib = _abi.load()
        self.plans = plan_program(program, fuse_pointwise=fuse_pointwise,
                                  fuse_library=fuse_library, reuse_storage=reuse_storage,
                                  tensor_cores=tensor_cores, library=library,
                                  whole_step=whole_step)
        self._resource = _NativeProgram(self._lib, self.plans)

    @classmethod
    def from_plans(cls, signature, plans, target: NVIDIATarget | None = None) -> "CompiledProgram":
        """A program from plans built directly on library kernels (e.g. the batched prefill),
        bound and run like a compiled DSL program."""
        self = cls.__new__(cls)
        self.signature, self.target = signature, target or NVIDIATarget("sm_100a")
        self.lowered = None
        self._lib = _abi.load()
        self.plans = plans
        self._resource = _NativeProgram(self._lib, plans)
        return self

    def to_json(self) -> str:
        """Signature, native plans (with any generated device code) and ``ckl_exec`` text as
        JSON; :func:`ckl.load_program` / :func:`ckl.plan_io.from_json` rebuild the program."""
        from .plan_io import to_json
        return to_json(self)

    def save(self, path) -> None:
        from .plan_io import save
        save(self, path)

    @property
    def plan_stats(self) -> dict:
        """The reference harness's statistics (nodes, edges, topology, temporaries, heap
        bytes) of the primary plan."""
        from .plan_io import plan_stats
        return plan_stats(self.executable_ir)

    @property
    def prepared_ir(self) -> str:
        return self.plans.prepared_ir

    @property
    def executable_ir(self) -> str:
        return self.plans.primary.executable_ir

    @property
    def fallback_ir(self) -> str:
        return self.plans.fallback.executable_ir if self.plans.fallback else ""

    @property
    def device_ir(self) -> str:
        return self.plans.device_ir

    @property
    def host_ir(self) -> str:
        return self.plans.host_ir

    @property
    def host_mlir(self) -> str:
        return self.plans.host_ir

    def bind(self, *arguments, device: Device | None = None) -> "Invocation":
        parameters = self.signature.runtime
        if len(arguments) != len(parameters):
            raise TypeError(f"expected {len(parameters)} runtime arguments, got {len(arguments)}")
        buffers = [a for a in arguments if isinstance(a, DeviceBuffer)]
        device = device or (buffers[0].device if buffers else None)
        if device is None:
            raise ValueError("pass a Device for programs without buffer arguments")
        packed = (_abi.Argument * max(len(arguments), 1))()
        for index, (parameter, value) in enumerate(zip(parameters, arguments)):
            if isinstance(parameter.dtype, BufferSpec):
                if not isinstance(value, DeviceBuffer) or value.spec != parameter.dtype:
                    raise TypeError(f"{parameter.name} requires {parameter.dtype}")
                if value.device is not device:
                    raise ValueError("all buffers must belong to the selected Device")
                packed[index].kind = _abi.ARG_BUFFER
                packed[index].buffer = value._native_resource.value
                continue
            code, width = _SCALARS[parameter.dtype]
            if parameter.dtype in (i32, i64):
                bits = width * 8
                if type(value) is not int or not -(1 << (bits - 1)) <= value < (1 << (bits - 1)):
                    raise TypeError(f"{parameter.name} requires a {bits}-bit integer")
            elif type(value) not in (int, float) or not math.isfinite(float(value)):
                raise TypeError(f"{parameter.name} requires a finite numeric value")
            if parameter.dtype in (f32, f64):
                try:
                    rounded = struct.unpack(code, struct.pack(code, value))[0]
                except (OverflowError, struct.error):
                    raise ValueError(f"{parameter.name} overflows {parameter.dtype.name}") from None
                if not math.isfinite(rounded):
                    raise ValueError(f"{parameter.name} overflows {parameter.dtype.name}")
            raw = struct.pack("<" + code, value)
            packed[index].kind = _ARG_KIND[parameter.dtype]
            packed[index].bits = int.from_bytes(raw.ljust(8, b"\0"), "little")
        handle = C.c_void_p()
        _abi.check(self._lib.ckl_bind(self._native_resource.handle.value,
                                         device._native_resource.value, len(arguments), packed,
                                         C.byref(handle)), "bind")
        return Invocation(self, device, arguments, _Handle(handle.value,
                                                           self._lib.ckl_invocation_release))

    def run(self, *arguments, graph=False, device=None) -> "Invocation":
        return self.bind(*arguments, device=device).run(graph=graph)


class Invocation(_ContextManager):
    """A bound program owning its temporaries, stream and lazily built CUDA graphs."""

    def __init__(self, program, device, arguments, resource):
        self.program, self.device, self.arguments = program, device, arguments
        self._lib = program._lib
        # The native invocation retains its program, device and buffers; keep the Python
        # owners of imported storage alive as well.
        self._keep = (program._resource, [getattr(a, "_owner", None) for a in arguments],
                      [getattr(a, "_owner_resource", None) for a in arguments],
                      [getattr(a, "_resource", None) for a in arguments])
        self._resource = resource

    def close(self):
        super().close()
        self.program = self.device = self.arguments = None

    @staticmethod
    def _execution(graph, mode, batch_size) -> int:
        if type(batch_size) is not int or not 0 < batch_size < (1 << 64):
            raise ValueError("batch_size must be a positive 64-bit count")
        if mode is not None and graph:
            raise ValueError("specify either graph or mode")
        if mode is not None and mode not in _MODES:
            raise ValueError("mode must be ordinary, graph, or capture")
        return _MODES[mode] if mode is not None else int(bool(graph))

    def run(self, *, graph=False, mode=None, batch_size=1) -> "Invocation":
        execution = self._execution(graph, mode, batch_size)
        _abi.check(self._lib.ckl_run(self._native_resource.value, execution, batch_size), "run")
        return self

    @property
    def node_count(self) -> int:
        """Kernel nodes of one program execution (after fusion or the overlap fallback)."""
        out = C.c_uint64()
        _abi.check(self._lib.ckl_node_count(self._native_resource.value, C.byref(out)))
        return int(out.value)

    @property
    def node_names(self) -> list:
        names = []
        for i in range(self.node_count):
            buffer = C.create_string_buffer(128)
            _abi.check(self._lib.ckl_node_name(self._native_resource.value, i, buffer, 128))
            names.append(buffer.value.decode())
        return names

    def node_argument_sizes(self, node: int) -> list:
        """Byte sizes of plan node `node`'s argument slots (what :meth:`update_kernel` takes)."""
        sizes, count = (C.c_uint64 * 64)(), C.c_uint32()
        _abi.check(self._lib.ckl_node_argument_sizes(self._native_resource.value, node, sizes, 64,
                                                     C.byref(count)), "node arguments")
        if count.value > 64:
            sizes = (C.c_uint64 * count.value)()
            _abi.check(self._lib.ckl_node_argument_sizes(self._native_resource.value, node, sizes,
                                                         count.value, C.byref(count)),
                       "node arguments")
        return [int(sizes[i]) for i in range(count.value)]

    def update_kernel(self, node: int, arguments, *, mode="graph", batch_size=1, grid=None,
                      block=None, shared_memory=None) -> None:
        """Replace one kernel node's launch parameters in this invocation's explicit graph for
        `batch_size` repetitions, without re-instantiating it (the reference's
        ``NvidiaGraphExecutable::updateKernel``, ``NvidiaRuntime.cpp:466-496``).

        `arguments` has one entry per argument slot of the node (:meth:`node_argument_sizes`):
        ``None`` keeps the slot, a :class:`DeviceBuffer` of this device gives its address, and
        ``bytes`` or a numpy scalar give the slot's new bytes.  Graph node ``r * node_count + i``
        is repetition r's node i.  Only ``mode="graph"`` has updatable nodes (a captured graph
        is rejected, as in the reference); the update applies to that graph only."""
        import numpy as np

        if type(node) is not int or node < 0:
            raise ValueError("node must be a nonnegative int")
        if mode not in _MODES:
            raise ValueError("mode must be ordinary, graph, or capture")
        arguments = list(arguments)
        pointers = (C.c_void_p * max(1, len(arguments)))()
        sizes = (C.c_uint64 * max(1, len(arguments)))()
        keep = []
        for i, value in enumerate(arguments):
            if value is None:
                continue
            if isinstance(value, DeviceBuffer):
                if value.device is not self.device and \
                        getattr(value.device, "ordinal", None) != getattr(self.device, "ordinal", None):
                    raise ValueError("updated buffer belongs to another device")
                keep.append(value)
                value = C.c_uint64(value.address)
                raw = bytes(value)
            elif isinstance(value, (bytes, bytearray)):
                raw = bytes(value)
            elif isinstance(value, np.generic):
                raw = value.tobytes()
            else:
                raise TypeError("kernel arguments are None, a DeviceBuffer, bytes or a numpy scalar")
            holder = C.create_string_buffer(raw, len(raw))
            keep.append(holder)
            pointers[i] = C.cast(holder, C.c_void_p)
            sizes[i] = len(raw)
        shape = lambda v: None if v is None else (C.c_uint32 * 3)(*(list(v) + [1, 1])[:3])
        shared = -1 if shared_memory is None else int(shared_memory)
        _abi.check(self._lib.ckl_update_kernel(self._native_resource.value, _MODES[mode],
                                               batch_size, node, len(arguments), pointers, sizes,
                                               shape(grid), shape(block), shared), "update_kernel")
        # Buffers now referenced by the graph stay alive with the invocation.
        self._updated = getattr(self, "_updated", []) + [k for k in keep
                                                         if isinstance(k, DeviceBuffer)]

    def benchmark(self, *, iterations=200, graph=False, mode=None, batch_size=1) -> dict:
        """Time ``iterations`` submissions of ``batch_size`` programs; report per program."""
        if type(iterations) is not int or not 0 < iterations < (1 << 64):
            raise ValueError("iterations must be a positive 64-bit count")
        execution = self._execution(graph, mode, batch_size)
        out = (C.c_double * 3)()
        _abi.check(self._lib.ckl_benchmark(self._native_resource.value, execution, iterations,
                                              batch_size, out), "benchmark")
        return {"stream_us": out[0], "wall_us": out[1], "graph_setup_ms": out[2]}

    # ---- asynchronous interface (B200 build) ------------------------------------------
    def launch(self, *, graph=False, mode=None, batch_size=1) -> None:
        """Submit without waiting; pair with :meth:`synchronize`."""
        execution = self._execution(graph, mode, batch_size)
        _abi.check(self._lib.ckl_launch(self._native_resource.value, execution, batch_size),
                      "launch")

    def synchronize(self) -> None:
        _abi.check(self._lib.ckl_synchronize(self._native_resource.value), "synchronize")

    def copy_in_async(self, buffer: DeviceBuffer, source_pointer: int, nbytes: int) -> None:
        """Enqueue a host-to-device copy from page-locked memory on the invocation stream."""
        _abi.check(self._lib.ckl_copy_in_async(self._native_resource.value,
                                                  buffer._native_resource.value, source_pointer,
                                                  nbytes), "copy_in_async")

    def copy_out_async(self, buffer: DeviceBuffer, destination_pointer: int, nbytes: int) -> None:
        _abi.check(self._lib.ckl_copy_out_async(self._native_resource.value,
                                                   buffer._native_resource.value,
                                                   destination_pointer, nbytes), "copy_out_async")

    def record(self) -> "Completion":
        """A completion at the current end of this invocation's stream."""
        handle = C.c_void_p()
        _abi.check(self._lib.ckl_record(self._native_resource.value, C.byref(handle)), "record")
        return Completion(self, _Handle(handle.value, self._lib.ckl_completion_release))

    def wait_for(self, completion: "Completion") -> None:
        """Make this invocation's later work wait (on the device) for `completion`."""
        if not isinstance(completion, Completion):
            raise TypeError("wait_for requires a Completion")
        _abi.check(self._lib.ckl_wait_for(self._native_resource.value,
                                          completion._native_resource.value), "wait_for")

    def submit(self, *, graph=False, mode=None, batch_size=1, after=(),
               observe=()) -> "Completion":
        """Enqueue one execution of ``batch_size`` programs and return its completion without
        waiting.  ``after``: completions (of this or other invocations, on any device) the
        execution waits for on the device.  ``observe``: ``(buffer, host)`` pairs copied to
        page-locked host memory (:class:`PinnedHostBuffer` or a numpy view of one) after the
        execution, in stream order; :meth:`Completion.wait` makes them readable.  Submissions
        on one invocation run in order; the completion keeps the invocation, its buffers and
        the observed host memory alive."""
        execution = self._execution(graph, mode, batch_size)
        observed = []
        for buffer, host in observe:
            if not isinstance(buffer, DeviceBuffer):
                raise TypeError("observe takes (DeviceBuffer, host memory) pairs")
            pointer, nbytes, keep = _pinned_pointer(host)
            if nbytes < buffer.nbytes:
                raise ValueError("observed host memory is smaller than the buffer")
            observed.append((buffer, pointer, keep))
        for completion in after:
            self.wait_for(completion)
        _abi.check(self._lib.ckl_launch(self._native_resource.value, execution, batch_size),
                   "submit")
        for buffer, pointer, _ in observed:
            self.copy_out_async(buffer, pointer, buffer.nbytes)
        completion = self.record()
        completion._keep = (tuple(after), tuple(observed))
        return completion

    def profile_nodes(self, iterations: int = 1) -> list:
        """Per-node device milliseconds over ``iterations`` ordinary executions (state advances)."""
        count = self.node_count
        out = (C.c_double * count)()
        _abi.check(self._lib.ckl_profile_nodes(self._native_resource.value, iterations, out,
                                                  count), "profile")
        return list(out)

    def time_launches(self, steps: int, *, mode="graph", batch_size=1) -> float:
        """Device milliseconds of ``steps`` back-to-back submissions (CUDA events)."""
        out = C.c_double()
        _abi.check(self._lib.ckl_time_launches(self._native_resource.value, _MODES[mode],
                                                  batch_size, steps, C.byref(out)), "timing")
        return out.value


class Completion(_ContextManager):
    """A point on an invocation's stream (asynchronous invocation/completion interface).

    Holding it keeps the invocation's stream, temporaries and bound buffers alive; ``done``
    polls, ``wait`` blocks (optionally up to ``timeout`` seconds) and returns whether the work
    before it has finished."""

    def __init__(self, invocation, resource):
        self.invocation = invocation
        self._lib = invocation._lib
        self._resource = resource
        self._keep = ()

    def done(self) -> bool:
        flag = C.c_int()
        _abi.check(self._lib.ckl_completion_query(self._native_resource.value, C.byref(flag)),
                   "completion query")
        return bool(flag.value)

    def wait(self, timeout: float | None = None) -> bool:
        if timeout is not None and (not math.isfinite(timeout) or timeout < 0):
            raise ValueError("timeout must be a finite nonnegative number of seconds")
        micros = (1 << 64) - 1 if timeout is None else int(timeout * 1e6)
        flag = C.c_int()
        _abi.check(self._lib.ckl_completion_wait(self._native_resource.value, micros,
                                                 C.byref(flag)), "completion wait")
        return bool(flag.value)


def _pinned_pointer(host):
    """(pointer, nbytes, keepalive) of page-locked host memory: a PinnedHostBuffer or a
    contiguous writable array viewing one."""
    if isinstance(host, PinnedHostBuffer):
        return host.pointer, host.nbytes, host
    pointer, nbytes, keep = _host_pointer(host, writable=True)
    return pointer, nbytes, (host, keep)


class PinnedHostBuffer:
    """Page-locked host memory for asynchronous copies."""

    def __init__(self, nbytes: int):
        self._lib = _abi.load()
        pointer = C.c_void_p()
        _abi.check(self._lib.ckl_host_alloc(nbytes, C.byref(pointer)), "pinned allocation")
        self.pointer, self.nbytes = pointer.value, nbytes
        self._handle = _Handle(pointer.value, self._lib.ckl_host_free)

    def view(self):
        return (C.c_char * self.nbytes).from_address(self.pointer)

    def array(self, dtype, shape):
        """A numpy array over this memory (the buffer must outlive it)."""
        import numpy as np
        count = int(np.prod(shape))
        if count * np.dtype(dtype).itemsize > self.nbytes:
            raise ValueError("array exceeds the pinned buffer")
        return np.frombuffer(self.view(), dtype=dtype, count=count).reshape(shape)


def cuda_available() -> bool:
    return bool(_abi.load().ckl_cuda_available())


class _NativeModule:
    """The subset of the reference's ``_ckl_native`` module that harness code calls."""

    def __init__(self):
        self._lib = _abi.load()
        self.__file__ = str(_abi.library_path())
        self.has_cuda_runtime = True

    def cuda_available(self) -> bool:
        return bool(self._lib.ckl_cuda_available())

    def profiler_start(self) -> None:
        _abi.check(self._lib.ckl_profiler_start(), "profiler_start")

    def profiler_stop(self) -> None:
        _abi.check(self._lib.ckl_profiler_stop(), "profiler_stop")


_MODULE = None


def _native_module():
    global _MODULE
    if _MODULE is None:
        _MODULE = _NativeModule()
    return _MODULE


def _native():
    """The reference exposes its native module as ``ckl.cuda._native()`` (cuda.py:31-62)."""
    return _native_module()
