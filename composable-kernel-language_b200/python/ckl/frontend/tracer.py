"""Trace a ``@ckl.program`` into an ordered list of allocations, dispatches and frees.

This replaces the reference's MLIR emitter (``python/ckl/frontend/emitter.py:162-749``)
for programs.  The semantics it keeps:

* program loops unroll (compile-time ``range`` bounds, at most 1024 iterations) and
  program ``if`` statements need compile-time predicates (``emitter.py:490-502``);
* ``ckl.empty`` / ``ckl.empty_like`` create temporaries, freed in reverse order at the end
  of the program (``emitter.py:176-177, 406-427``);
* ``ckl.subview`` creates a static contiguous view of a buffer (``emitter.py:428-439``);
* each ``ckl.launch`` binds the kernel's signature from its actual arguments and
  specializes it by content identity (``emitter.py:578-646``): constexpr parameters take
  compile-time values, scalar parameters take a constant or a forwarded program scalar;
* program-level arithmetic exists only on compile-time values.

The result is a :class:`LoweredProgram` whose ``trace`` feeds the B200 compiler
(:mod:`ckl.compile`).  Its ``mlir`` attribute holds a readable rendering of the trace.
"""
from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass, field

from ..types import BufferSpec, ConstexprType, ScalarType, i32, i64, index
from .checker import BoundSignature, bind, constant, parameter_type
from .source import Definition, describe
from .walker import BodyWalker


def identity(definition: Definition, signature: BoundSignature) -> str:
    """Specialization identity: definition content plus every bound parameter."""
    lines = [f"specialization of {definition.identity}"]
    for p in signature.parameters:
        if isinstance(p.dtype, ScalarType):
            kind = describe(p.dtype)
        else:
            kind = f"{p.dtype.dtype.name} buffer {tuple(p.dtype.shape)} {p.dtype.layout}"
        bound = f"constant {p.value!r}" if p.is_constant else "runtime"
        lines.append(f"{p.name}: {kind} {bound}")
    return hashlib.sha256("\n".join(lines).encode()).hexdigest()


@dataclass(frozen=True)
class Specialization:
    symbol: str
    identity: str
    signature: BoundSignature
    definition: Definition = field(compare=False, repr=False, default=None)


@dataclass
class Resource:
    """A program buffer: a runtime argument, a temporary, or a static view of either."""

    id: int
    kind: str               # "argument" | "temporary" | "view"
    spec: BufferSpec
    argument: int = -1      # runtime parameter position (arguments)
    base: int = -1          # base resource id (views)
    byte_offset: int = 0    # offset from the base resource (views)
    name: str = ""

    @property
    def root(self) -> int:
        return self.base if self.kind == "view" else self.id


@dataclass(frozen=True)
class Operand:
    """A dispatch argument: a resource, a forwarded program scalar, or a constant."""

    kind: str               # "resource" | "scalar" | "constant"
    dtype: object           # BufferSpec | ScalarType
    resource: int = -1
    argument: int = -1
    value: object = None


@dataclass
class Dispatch:
    specialization: Specialization
    operands: list
    grid: tuple
    block: tuple
    shared_memory: int
    location: str


@dataclass
class Event:
    kind: str               # "alloc" | "dispatch" | "free"
    resource: int = -1
    dispatch: Dispatch = None


@dataclass
class ProgramTrace:
    name: str
    signature: BoundSignature
    resources: list
    events: list

    @property
    def dispatches(self):
        return [e.dispatch for e in self.events if e.kind == "dispatch"]


@dataclass(frozen=True)
class LoweredProgram:
    mlir: str
    signature: BoundSignature
    specializations: tuple
    cache_key: str
    diagnostics: tuple = ()
    trace: ProgramTrace = field(default=None, compare=False, repr=False)

    def analyze(self, *passes, ckl_opt=None):
        """Structural analysis of the traced program: the inferred reference plan as text."""
        from ..compile import reference_plan_text

        return reference_plan_text(self)

    def verify(self, *, ckl_opt=None) -> "LoweredProgram":
        from ..compile import plan_program

        plan_program(self, fuse_pointwise=False, fuse_library=False, reuse_storage=True)
        return self

    def compile(self, *, target, fuse_pointwise=True, reuse_storage=True, fuse_library=True,
                tensor_cores=True, library=True, whole_step=True):
        """Select sm_100a kernels, infer the dependency graph and plan temporary storage.

        Kernel bodies the library does not implement are generated (CUDA C++, compiled by
        NVRTC for sm_100a).  ``tensor_cores=False`` keeps batched fused projections on FFMA
        instead of tcgen05; ``library=False`` generates every kernel from its body;
        ``whole_step=False`` keeps a small decode step as per-layer nodes instead of one
        whole-step kernel.
        """
        from ..cuda import CompiledProgram

        return CompiledProgram(self, target, fuse_pointwise=fuse_pointwise,
                               reuse_storage=reuse_storage, fuse_library=fuse_library,
                               tensor_cores=tensor_cores, library=library,
                               whole_step=whole_step)


@dataclass(frozen=True)
class _Runtime:
    """A runtime program parameter (buffer or scalar) seen inside the program body."""

    position: int
    dtype: object


@dataclass(frozen=True)
class _BufferValue:
    resource: int
    spec: BufferSpec


_RUNTIME_SCALAR = ("computed runtime host scalars are unsupported; forward the parameter "
                   "unchanged")


class ProgramTracer(BodyWalker):
    """Walks a program body at compile time: loops unroll, branches must be static, buffers
    are program resources, and every launch becomes a dispatch of a kernel specialization."""

    def __init__(self, definition: Definition, signature: BoundSignature):
        super().__init__(definition, signature.dimensions)
        self.signature = signature
        self.resources: list[Resource] = []
        self.events: list[Event] = []
        self.temporaries: list[int] = []
        self.specializations: dict[str, Specialization] = {}
        for position, parameter in enumerate(signature.runtime):
            if isinstance(parameter.dtype, BufferSpec):
                resource = self._resource("argument", parameter.dtype, argument=position,
                                          name=f"arg{position}")
                self.env[parameter.name] = _BufferValue(resource, parameter.dtype)
            else:
                self.env[parameter.name] = _Runtime(position, parameter.dtype)
        self.env.update((p.name, p.value) for p in signature.parameters if p.is_constant)

    def _resource(self, kind, spec, **fields) -> int:
        rid = len(self.resources)
        self.resources.append(Resource(rid, kind, spec, **fields))
        return rid

    # ---- walker hooks ----------------------------------------------------------------------
    def is_dynamic(self, value) -> bool:
        return isinstance(value, _Runtime)

    def buffer_spec(self, value):
        return value.spec if isinstance(value, _BufferValue) else None

    def dynamic_binary(self, left, right, op, node, comparison):
        if isinstance(left, _Runtime) or isinstance(right, _Runtime):
            self.fail(node, _RUNTIME_SCALAR)
        self.fail(node, "numeric expressions require scalar operands")

    def dynamic_unary(self, value, op, node):
        self.fail(node, _RUNTIME_SCALAR)

    def assign_local(self, target, value, node):
        if value is None:
            self.fail(node, "launches do not return source values")
        self.env[target.id] = value

    def assign_element(self, target, value, node):
        self.fail(target, "buffer writes are only valid in kernels")

    def loop(self, node, induction, start, stop, step):
        if type(start) is not int or type(stop) is not int:
            self.fail(node, "program range bounds must be compile-time integers")
        values = range(start, stop, step)
        if len(values) > 1024:
            self.fail(node, "program unrolling is limited to 1024 iterations")

        def unrolled():
            for value in values:
                self.env[induction] = value
                self.walk(node.body)

        self.with_binding(induction, None, unrolled)

    # ---- intrinsics ------------------------------------------------------------------------
    def _coordinate(self, node):
        self.arguments(node)
        self.fail(node, "device coordinates are only valid in kernels")

    intrinsic_global_id = intrinsic_thread_id = intrinsic_block_id = _coordinate
    intrinsic_block_dim = intrinsic_grid_dim = _coordinate

    def _host_math(self, node):
        self.arguments(node)
        self.fail(node, _RUNTIME_SCALAR)

    intrinsic_exp = intrinsic_rsqrt = intrinsic_select = _host_math

    def _temporary(self, spec) -> _BufferValue:
        rid = self._resource("temporary", spec, name=f"alloc{len(self.temporaries)}")
        self.temporaries.append(rid)
        self.events.append(Event("alloc", resource=rid))
        return _BufferValue(rid, spec)

    def intrinsic_empty_like(self, node):
        values, keywords = self.arguments(node)
        if keywords or len(values) != 1 or not isinstance(values[0], _BufferValue):
            self.fail(node, "empty_like requires one buffer")
        return self._temporary(values[0].spec)

    def intrinsic_empty(self, node):
        values, keywords = self.arguments(node)
        if len(values) != 1 or set(keywords) != {"dtype"}:
            self.fail(node, "use empty(shape_tuple, dtype=element_type)")
        try:
            spec = BufferSpec(values[0], keywords["dtype"])
        except (ValueError, TypeError) as error:
            self.fail(node, str(error))
        return self._temporary(spec)

    def intrinsic_subview(self, node):
        values, keywords = self.arguments(node)
        if len(values) != 1 or not isinstance(values[0], _BufferValue) \
                or set(keywords) != {"offset", "shape"}:
            self.fail(node, "use subview(buffer, offset=element_offset, shape=shape_tuple)")
        source, offset = values[0], keywords["offset"]
        try:
            spec = BufferSpec(keywords["shape"], source.spec.dtype)
        except (TypeError, ValueError) as error:
            self.fail(node, str(error))
        if type(offset) is not int or not 0 <= offset < (1 << 63) \
                or offset + spec.elements > source.spec.elements:
            self.fail(node, "subview offset/shape must be constant and within the source")
        parent = self.resources[source.resource]
        rid = self._resource("view", spec, base=parent.root,
                             byte_offset=parent.byte_offset + offset * spec.dtype.bytes,
                             name=f"view{len(self.resources)}")
        return _BufferValue(rid, spec)

    def intrinsic_cast(self, node):
        values, keywords = self.arguments(node)
        if keywords or len(values) != 2 or not isinstance(values[1], ScalarType):
            self.fail(node, "use cast(value, scalar_type)")
        value, dtype = values
        if isinstance(value, _Runtime):
            self.fail(node, _RUNTIME_SCALAR)
        if dtype in (i32, i64, index) and type(value) is float and math.isfinite(value):
            value = int(value)
        return constant(value, dtype, self.definition, node)

    def _geometry(self, node, keywords):
        shape = []
        for name in ("grid", "block"):
            extents = keywords[name]
            if type(extents) is not tuple or len(extents) not in (1, 2, 3) or not all(
                    type(e) is int and 0 < e < (1 << 63) for e in extents):
                self.fail(node, f"{name} requires a tuple of one to three positive compile-time "
                                "integers")
            shape.append(extents + (1,) * (3 - len(extents)))
        shared = keywords.get("shared_memory", 0)
        if type(shared) is not int or not 0 <= shared < (1 << 63):
            self.fail(node, "shared_memory requires nonnegative compile-time bytes")
        return shape[0], shape[1], shared

    def _operand(self, parameter, argument, declared, signature, constants):
        """Classify one launch argument against the kernel parameter it feeds."""
        given = self.evaluate(argument)
        if isinstance(declared, ConstexprType):
            if isinstance(given, (_Runtime, _BufferValue)):
                self.fail(argument, "constexpr launch arguments must be compile-time constants")
            constants[parameter.arg] = given
            return None
        if isinstance(declared, ScalarType):
            signature[parameter.arg] = declared
            if isinstance(given, _BufferValue):
                self.fail(argument, "kernel arguments must be typed buffers or scalars")
            if not isinstance(given, _Runtime):
                return Operand("constant", declared,
                               value=constant(given, declared, self.definition, argument))
            if given.dtype != declared:
                self.fail(argument, f"expected {declared.name}, got {given.dtype.mlir}; use "
                                    "ckl.cast explicitly")
            return Operand("scalar", declared, argument=given.position)
        if not isinstance(given, _BufferValue):
            self.fail(argument, "kernel arguments must be typed buffers or scalars")
        signature[parameter.arg] = given.spec
        return Operand("resource", given.spec, resource=given.resource)

    def intrinsic_launch(self, node):
        if not node.args:
            self.fail(node, "launch requires a kernel definition")
        kernel = self.evaluate(node.args[0])
        if not isinstance(kernel, Definition) or kernel.kind != "kernel":
            self.fail(node, "launch requires a @ckl.kernel definition")
        parameters = kernel.tree.args.args
        if len(node.args) != len(parameters) + 1:
            self.fail(node, "launch argument count does not match kernel signature")
        keywords = {k.arg: self.evaluate(k.value) for k in node.keywords}
        if not {"grid", "block"} <= set(keywords) <= {"grid", "block", "shared_memory"}:
            self.fail(node, "launch requires grid and block; only shared_memory is optional")
        grid, block, shared = self._geometry(node, keywords)
        signature, constants = {}, {}
        operands = [self._operand(p, a, parameter_type(kernel, p), signature, constants)
                    for p, a in zip(parameters, node.args[1:])]
        bound = bind(kernel, signature, constants)
        key = identity(kernel, bound)
        specialization = self.specializations.setdefault(
            key, Specialization("kernel_" + key[:24], key, bound, kernel))
        self.events.append(Event("dispatch", dispatch=Dispatch(
            specialization, [o for o in operands if o is not None], grid, block, shared,
            self.location(node))))
        return None

    def trace(self) -> ProgramTrace:
        self.walk(self.definition.tree.body, top=True)
        self.events.extend(Event("free", resource=rid) for rid in reversed(self.temporaries))
        return ProgramTrace(self.definition.name, self.signature, self.resources, self.events)


def render(trace: ProgramTrace, symbol: str) -> str:
    """A readable, deterministic rendering of a traced program."""
    names = {r.id: r.name for r in trace.resources}
    params = []
    position = 0
    for p in trace.signature.parameters:
        if p.is_constant:
            continue
        spelled = p.dtype.mlir if isinstance(p.dtype, (BufferSpec, ScalarType)) else str(p.dtype)
        params.append(f"%arg{position}: {spelled}")
        position += 1
    lines = [f'ckl.program @{symbol}({", ".join(params)}) {{']
    for r in trace.resources:
        if r.kind == "view":
            lines.append(f"  %{r.name} = ckl.subview %{names[r.base]} bytes {r.byte_offset} : {r.spec.mlir}")
    for event in trace.events:
        if event.kind == "alloc":
            r = trace.resources[event.resource]
            lines.append(f"  %{r.name} = ckl.alloc : {r.spec.mlir}")
        elif event.kind == "free":
            lines.append(f"  ckl.free %{names[event.resource]}")
        else:
            d = event.dispatch
            operands = []
            for op in d.operands:
                if op.kind == "resource":
                    operands.append("%" + names[op.resource])
                elif op.kind == "scalar":
                    operands.append(f"%arg{op.argument}")
                else:
                    operands.append(f"{op.value!r}:{op.dtype.name}")
            lines.append(f"  ckl.dispatch @{d.specialization.symbol}({', '.join(operands)}) "
                         f"grid {list(d.grid)} block {list(d.block)} shared {d.shared_memory}"
                         f"  // {d.specialization.definition.name} at {d.location}")
    lines.append("}")
    return "\n".join(lines) + "\n"


def lower_program(definition: Definition, signature, constants, *, verify=False,
                  ckl_opt=None) -> LoweredProgram:
    bound = bind(definition, signature, constants)
    program_identity = identity(definition, bound)
    tracer = ProgramTracer(definition, bound)
    trace = tracer.trace()
    # Kernel bodies are type-checked when the program is lowered, as the reference's emitter
    # does; the generated source is kept for kernels the library does not implement.
    from ..codegen import generate
    for spec in tracer.specializations.values():
        generate(spec.definition, spec.signature, spec.identity)
    symbol = "program_" + program_identity[:24]
    text = render(trace, symbol)
    for spec in tracer.specializations.values():
        text += f"// @{spec.symbol} = {spec.definition.name} {spec.identity}\n"
    key = hashlib.sha256((program_identity + text).encode()).hexdigest()
    result = LoweredProgram(text, bound, tuple(tracer.specializations.values()), key, (), trace)
    if verify:
        result.verify(ckl_opt=ckl_opt)
    return result
