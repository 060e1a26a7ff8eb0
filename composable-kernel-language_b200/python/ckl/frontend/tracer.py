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

import ast
import hashlib
import json
import math
import operator
from dataclasses import dataclass, field

from ..types import (BufferSpec, ConstexprType, Dimension, NUMERIC_TYPES, ScalarType, bool_,
                     f32, f64, i32, i64, index)
from .checker import BoundSignature, annotation_of, bind, constant
from .source import Definition, Intrinsic, Namespace, UnsupportedBinding, fingerprint


def identity(definition: Definition, signature: BoundSignature) -> str:
    """Specialization identity: definition content plus every bound parameter."""
    payload = [definition.identity, [
        [p.name,
         fingerprint(p.dtype) if isinstance(p.dtype, ScalarType)
         else [list(p.dtype.shape), p.dtype.dtype.name, p.dtype.layout],
         p.value, p.is_constant]
        for p in signature.parameters]]
    return hashlib.sha256(json.dumps(payload, sort_keys=True).encode()).hexdigest()


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


_STATIC_BINARY = {ast.Add: operator.add, ast.Sub: operator.sub, ast.Mult: operator.mul,
                  ast.Div: operator.truediv, ast.Lt: operator.lt, ast.LtE: operator.le,
                  ast.Gt: operator.gt, ast.GtE: operator.ge, ast.Eq: operator.eq,
                  ast.NotEq: operator.ne}


class ProgramTracer:
    def __init__(self, definition: Definition, signature: BoundSignature):
        self.definition = definition
        self.signature = signature
        self.dims = dict(signature.dimensions)
        self.env: dict[str, object] = {}
        self.resources: list[Resource] = []
        self.events: list[Event] = []
        self.temporaries: list[int] = []
        self.specializations: dict[str, Specialization] = {}
        self.local_names = {p.name for p in signature.parameters} | {
            n.id for n in ast.walk(definition.tree)
            if isinstance(n, ast.Name) and isinstance(n.ctx, ast.Store)}
        position = 0
        for parameter in signature.parameters:
            if parameter.is_constant:
                self.env[parameter.name] = parameter.value
                continue
            if isinstance(parameter.dtype, BufferSpec):
                resource = self._resource("argument", parameter.dtype, argument=position,
                                          name=f"arg{position}")
                self.env[parameter.name] = _BufferValue(resource, parameter.dtype)
            else:
                self.env[parameter.name] = _Runtime(position, parameter.dtype)
            position += 1

    def _resource(self, kind, spec, **fields) -> int:
        rid = len(self.resources)
        self.resources.append(Resource(rid, kind, spec, **fields))
        return rid

    def fail(self, node, message):
        raise self.definition.error(node, message)

    def location(self, node) -> str:
        line = self.definition.first_line + getattr(node, "lineno", 1) - 1
        column = self.definition.indentation + getattr(node, "col_offset", 0) + 1
        return f"{self.definition.filename}:{line}:{column}"

    # -- expressions ---------------------------------------------------------------------
    def expression(self, node):
        if isinstance(node, ast.Constant) and type(node.value) in (int, float, bool):
            if type(node.value) is float and not math.isfinite(node.value):
                self.fail(node, "non-finite source constants are unsupported")
            return node.value
        if isinstance(node, ast.Name):
            if node.id in self.env:
                return self.env[node.id]
            if node.id in self.local_names:
                self.fail(node, f"local '{node.id}' is not defined on this path")
            if node.id not in self.definition.bindings:
                self.fail(node, f"unknown name '{node.id}'")
            bound = self.definition.bindings[node.id]
            if isinstance(bound, UnsupportedBinding):
                self.fail(node, f"unsupported captured binding '{node.id}'")
            if isinstance(bound, Dimension):
                if bound.name not in self.dims:
                    self.fail(node, f"unbound dimension '{bound.name}'")
                return self.dims[bound.name]
            return bound
        if isinstance(node, ast.Tuple):
            return tuple(self.expression(item) for item in node.elts)
        if isinstance(node, ast.Attribute):
            base = self.expression(node.value)
            if isinstance(base, Namespace) and node.attr in base.values:
                return base.values[node.attr]
            if isinstance(base, _BufferValue):
                if node.attr == "shape":
                    return base.spec.shape
                if node.attr == "dtype":
                    return base.spec.dtype
            self.fail(node, f"unsupported attribute '{node.attr}'")
        if isinstance(node, ast.Subscript):
            base = self.expression(node.value)
            if isinstance(base, _BufferValue):
                self.fail(node, "buffer contents can only be accessed inside a kernel")
            if type(base) is tuple:
                position = self.expression(node.slice)
                if type(position) is not int or not 0 <= position < len(base):
                    self.fail(node, "tuple/shape axes require an in-range nonnegative "
                                    "compile-time integer")
                return base[position]
            self.fail(node, "unsupported subscript; slices and negative indexing are not supported")
        if isinstance(node, (ast.BinOp, ast.Compare)):
            comparison = isinstance(node, ast.Compare)
            if comparison and len(node.ops) != 1:
                self.fail(node, "chained comparisons are not supported")
            left = self.expression(node.left)
            right = self.expression(node.comparators[0] if comparison else node.right)
            op = node.ops[0] if comparison else node.op
            if type(op) not in _STATIC_BINARY:
                self.fail(node, f"unsupported numeric operator: {type(op).__name__}")
            allowed = (int, float, bool) if comparison else (int, float)
            if type(left) not in allowed or type(right) not in allowed:
                if isinstance(left, _Runtime) or isinstance(right, _Runtime):
                    self.fail(node, "computed runtime host scalars are unsupported; forward the "
                                    "parameter unchanged")
                self.fail(node, "numeric expressions require scalar operands")
            try:
                result = _STATIC_BINARY[type(op)](left, right)
            except (ZeroDivisionError, OverflowError) as error:
                self.fail(node, f"invalid constant expression: {error}")
            if type(result) is float and not math.isfinite(result):
                self.fail(node, "non-finite constant expression")
            return result
        if isinstance(node, ast.UnaryOp) and isinstance(node.op, (ast.USub, ast.UAdd)):
            value = self.expression(node.operand)
            if type(value) in (int, float):
                return -value if isinstance(node.op, ast.USub) else value
            self.fail(node, "computed runtime host scalars are unsupported; forward the "
                            "parameter unchanged")
        if isinstance(node, ast.Call):
            return self.call(node)
        self.fail(node, f"unsupported expression: {type(node).__name__}")

    def call(self, node: ast.Call):
        callee = self.expression(node.func)
        if isinstance(callee, Definition):
            self.fail(node, "kernel definitions are not ordinary calls; use ckl.launch")
        if not isinstance(callee, Intrinsic):
            self.fail(node, "calling arbitrary Python functions is unsupported")
        if any(isinstance(a, ast.Starred) for a in node.args) or any(k.arg is None for k in node.keywords):
            self.fail(node, "argument expansion is unsupported")
        name = callee.name
        if name == "launch":
            return self.launch(node)
        args = [self.expression(a) for a in node.args]
        keywords = {k.arg: self.expression(k.value) for k in node.keywords}
        if len(keywords) != len(node.keywords):
            self.fail(node, "duplicate keyword arguments")
        if name in ("global_id", "thread_id", "block_id", "block_dim", "grid_dim"):
            self.fail(node, "device coordinates are only valid in kernels")
        if name == "cdiv":
            if len(args) != 2 or keywords or any(type(v) is not int for v in args) \
                    or args[0] < 0 or args[1] <= 0:
                self.fail(node, "cdiv requires a nonnegative constant extent and positive "
                                "constant divisor")
            return (args[0] + args[1] - 1) // args[1]
        if name in ("empty", "empty_like"):
            if name == "empty_like":
                if len(args) != 1 or keywords or not isinstance(args[0], _BufferValue):
                    self.fail(node, "empty_like requires one buffer")
                spec = args[0].spec
            else:
                if len(args) != 1 or set(keywords) != {"dtype"}:
                    self.fail(node, "use empty(shape_tuple, dtype=element_type)")
                try:
                    spec = BufferSpec(args[0], keywords["dtype"])
                except (ValueError, TypeError) as error:
                    self.fail(node, str(error))
            rid = self._resource("temporary", spec, name=f"alloc{len(self.temporaries)}")
            self.temporaries.append(rid)
            self.events.append(Event("alloc", resource=rid))
            return _BufferValue(rid, spec)
        if name == "subview":
            if len(args) != 1 or set(keywords) != {"offset", "shape"} \
                    or not isinstance(args[0], _BufferValue):
                self.fail(node, "use subview(buffer, offset=element_offset, shape=shape_tuple)")
            source, offset = args[0], keywords["offset"]
            try:
                spec = BufferSpec(keywords["shape"], source.spec.dtype)
            except (TypeError, ValueError) as error:
                self.fail(node, str(error))
            if type(offset) is not int or offset < 0 or offset >= (1 << 63) \
                    or offset + spec.elements > source.spec.elements:
                self.fail(node, "subview offset/shape must be constant and within the source")
            parent = self.resources[source.resource]
            base = parent.root
            byte_offset = parent.byte_offset + offset * spec.dtype.bytes
            rid = self._resource("view", spec, base=base, byte_offset=byte_offset,
                                 name=f"view{len(self.resources)}")
            return _BufferValue(rid, spec)
        if name == "cast":
            if len(args) != 2 or keywords or not isinstance(args[1], ScalarType):
                self.fail(node, "use cast(value, scalar_type)")
            value, dtype = args
            if isinstance(value, _Runtime):
                self.fail(node, "computed runtime host scalars are unsupported; forward the "
                                "parameter unchanged")
            if dtype in (i32, i64, index) and type(value) is float and math.isfinite(value):
                value = int(value)
            return constant(value, dtype, self.definition, node)
        if name in ("exp", "rsqrt", "select"):
            self.fail(node, "computed runtime host scalars are unsupported; forward the "
                            "parameter unchanged")
        self.fail(node, f"unsupported intrinsic: {name}")

    def launch(self, node: ast.Call):
        if not node.args:
            self.fail(node, "launch requires a kernel definition")
        definition = self.expression(node.args[0])
        if not isinstance(definition, Definition) or definition.kind != "kernel":
            self.fail(node, "launch requires a @ckl.kernel definition")
        parameters = definition.tree.args.args
        if len(node.args) - 1 != len(parameters):
            self.fail(node, "launch argument count does not match kernel signature")
        keywords = {k.arg: self.expression(k.value) for k in node.keywords}
        if set(keywords) - {"grid", "block", "shared_memory"} or not {"grid", "block"} <= set(keywords):
            self.fail(node, "launch requires grid and block; only shared_memory is optional")
        geometry = []
        for name in ("grid", "block"):
            dims = keywords[name]
            if type(dims) is not tuple or not 1 <= len(dims) <= 3 or any(
                    type(d) is not int or not 0 < d < (1 << 63) for d in dims):
                self.fail(node, f"{name} requires a tuple of one to three positive compile-time integers")
            geometry.append(tuple(dims) + (1,) * (3 - len(dims)))
        shared = keywords.get("shared_memory", 0)
        if type(shared) is not int or not 0 <= shared < (1 << 63):
            self.fail(node, "shared_memory requires nonnegative compile-time bytes")
        signature, constants, operands = {}, {}, []
        for parameter, argument in zip(parameters, node.args[1:]):
            annotation = annotation_of(definition, parameter)
            actual = self.expression(argument)
            if isinstance(annotation, ConstexprType):
                if isinstance(actual, (_Runtime, _BufferValue)):
                    self.fail(argument, "constexpr launch arguments must be compile-time constants")
                constants[parameter.arg] = actual
                continue
            if isinstance(annotation, ScalarType):
                if isinstance(actual, _Runtime):
                    if actual.dtype != annotation:
                        self.fail(argument, f"expected {annotation.name}, got "
                                            f"{actual.dtype.mlir}; use ckl.cast explicitly")
                    operands.append(Operand("scalar", annotation, argument=actual.position))
                elif isinstance(actual, _BufferValue):
                    self.fail(argument, "kernel arguments must be typed buffers or scalars")
                else:
                    value = constant(actual, annotation, self.definition, argument)
                    operands.append(Operand("constant", annotation, value=value))
                signature[parameter.arg] = annotation
                continue
            if not isinstance(actual, _BufferValue):
                self.fail(argument, "kernel arguments must be typed buffers or scalars")
            signature[parameter.arg] = actual.spec
            operands.append(Operand("resource", actual.spec, resource=actual.resource))
        bound = bind(definition, signature, constants)
        key = identity(definition, bound)
        if key not in self.specializations:
            self.specializations[key] = Specialization("kernel_" + key[:24], key, bound, definition)
        grid, block = geometry
        self.events.append(Event("dispatch", dispatch=Dispatch(
            self.specializations[key], operands, grid, block, shared, self.location(node))))
        return None

    # -- statements ----------------------------------------------------------------------
    def statements(self, nodes, top=False):
        for position, node in enumerate(nodes):
            if isinstance(node, ast.Return):
                if not top or position != len(nodes) - 1 or node.value is not None:
                    self.fail(node, "only a final bare return is supported; buffers carry outputs")
            elif isinstance(node, ast.Assign):
                if len(node.targets) != 1:
                    self.fail(node, "chained assignment is unsupported")
                target = node.targets[0]
                if isinstance(target, ast.Subscript):
                    self.fail(target, "buffer writes are only valid in kernels")
                if not isinstance(target, ast.Name):
                    self.fail(target, "assignment requires a local name or indexed buffer element")
                value = self.expression(node.value)
                if value is None:
                    self.fail(node, "launches do not return source values")
                self.env[target.id] = value
            elif isinstance(node, ast.If):
                predicate = self.expression(node.test)
                if type(predicate) is not bool:
                    self.fail(node.test, "if requires a boolean predicate; program control flow "
                                         "must be compile-time")
                self.statements(node.body if predicate else node.orelse)
            elif isinstance(node, ast.For):
                self.for_loop(node)
            elif isinstance(node, ast.Expr):
                if isinstance(node.value, ast.Constant) and isinstance(node.value.value, str) \
                        and position == 0 and top:
                    continue
                if not isinstance(node.value, ast.Call) or self.expression(node.value) is not None:
                    self.fail(node, "expression statements must be kernel launches")
            elif isinstance(node, ast.Pass):
                continue
            else:
                self.fail(node, f"unsupported statement: {type(node).__name__}")

    def for_loop(self, node: ast.For):
        if node.orelse or not isinstance(node.target, ast.Name) or not isinstance(node.iter, ast.Call):
            self.fail(node, "for requires a simple induction variable and range without else")
        callee = self.expression(node.iter.func)
        if not isinstance(callee, Intrinsic) or callee.name != "range" or node.iter.keywords:
            self.fail(node, "for requires range(start, stop, positive_constant_step)")
        bounds = [self.expression(a) for a in node.iter.args]
        if not 1 <= len(bounds) <= 3:
            self.fail(node, "range requires one to three bounds")
        start, stop, step = (0, bounds[0], 1) if len(bounds) == 1 else \
            (bounds[0], bounds[1], bounds[2] if len(bounds) == 3 else 1)
        if type(step) is not int or step <= 0:
            self.fail(node, "range step must be a positive compile-time integer")
        if type(start) is not int or type(stop) is not int:
            self.fail(node, "program range bounds must be compile-time integers")
        if len(range(start, stop, step)) > 1024:
            self.fail(node, "program unrolling is limited to 1024 iterations")
        induction = node.target.id
        outer = self.env.get(induction, _MISSING)
        for value in range(start, stop, step):
            self.env[induction] = value
            self.statements(node.body)
        if outer is _MISSING:
            self.env.pop(induction, None)
        else:
            self.env[induction] = outer

    def trace(self) -> ProgramTrace:
        self.statements(self.definition.tree.body, top=True)
        for rid in reversed(self.temporaries):
            self.events.append(Event("free", resource=rid))
        return ProgramTrace(self.definition.name, self.signature, self.resources, self.events)


_MISSING = object()


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
