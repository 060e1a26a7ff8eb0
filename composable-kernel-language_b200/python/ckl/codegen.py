"""CUDA C++ code generation for CKL kernel bodies that the sm_100a library does not implement.

The reference compiles every ``@ckl.kernel`` body through its MLIR emitter
(``python/ckl/frontend/emitter.py:120-726``) and the NVPTX pipeline into naive device code.
Here a kernel specialization whose canonical structure has no library entry (or whose launch
does not cover the library kernel's whole index space) is translated statement by statement
into one ``extern "C" __global__`` function, following the emitter's typing rules:

* Python ``int``/``float``/``bool`` constants and expressions over them stay static and fold;
  a static operand meeting a typed value takes the typed value's type (``typed``), two typed
  operands must have equal types (``binary``), integer division is rejected;
* ``global_id``/``thread_id``/``block_id``/``block_dim``/``grid_dim`` are ``index`` (i64);
  buffer indices are ``index``; buffers are contiguous row-major with static shapes;
* ``cast`` follows ``arith`` conversions (``extf``/``truncf``, ``extsi``/``trunci``,
  ``fptosi``/``sitofp``, ``index_cast``), ``exp``/``rsqrt`` take f32/f64, ``select`` a
  boolean predicate;
* a runtime ``if`` only writes buffers and branch-local names; a runtime ``for`` carries the
  outer names its body reassigns (``scf.for`` iteration arguments; static initial values
  become f32 / i32 / bool).

Floating-point arithmetic is emitted as the round-to-nearest intrinsics (``__fadd_rn``,
``__fmul_rn`` ...), which the compiler never contracts into a fused multiply-add: each
operation rounds once, as ``arith.addf``/``arith.mulf`` without fast-math flags do.  Integer
``+ - *`` wrap (two's complement, as ``arith.addi``); comparisons of floats are ordered except
``!=`` (unordered, ``une``).  Device code is compiled for sm_100a by NVRTC in the native library
(``ckl_cuda_compile``); the CUBIN is the plan's device binary next to the library kernels.
"""
from __future__ import annotations

import ast
import math
import re
import struct
from dataclasses import dataclass

from .frontend.checker import BoundSignature, constant
from .frontend.source import Definition
from .frontend.walker import SPELLINGS, BodyWalker, is_static
from .types import BufferSpec, ScalarType, bool_, f32, f64, i32, i64, index

CTYPE = {f32: "float", f64: "double", i32: "int", i64: "long long", index: "long long",
         bool_: "bool"}
_COORDINATES = {"thread_id": "threadIdx", "block_id": "blockIdx", "block_dim": "blockDim",
                "grid_dim": "gridDim"}
SYMBOL_PREFIX = "ckl_gen_"


@dataclass(frozen=True)
class _Value:
    """A typed device value: a C expression (identifier or literal) and its CKL type."""

    code: str
    dtype: ScalarType


@dataclass(frozen=True)
class _Buffer:
    code: str
    spec: BufferSpec


@dataclass(frozen=True)
class GeneratedKernel:
    """One generated kernel: its C symbol, CUDA source and runtime parameter types."""

    symbol: str
    source: str
    parameters: tuple


def _literal(value, dtype: ScalarType) -> str:
    if dtype == f32:
        bits = struct.unpack("<I", struct.pack("<f", value))[0]
        return f"__int_as_float(0x{bits:08x})"
    if dtype == f64:
        bits = struct.unpack("<Q", struct.pack("<d", value))[0]
        return f"__longlong_as_double(0x{bits:016x}LL)"
    if dtype == bool_:
        return "true" if value else "false"
    if dtype == i32:
        return f"((int)0x{value & 0xFFFFFFFF:08x}u)"
    return f"((long long)0x{value & 0xFFFFFFFFFFFFFFFF:016x}ull)"


_FLOATS, _INTEGERS = (f32, f64), (i32, i64)


def _conversion(source: ScalarType, target: ScalarType, code: str):
    """C expression converting `code` from `source` to `target` as the reference's ``arith``
    casts do (extf/truncf, extsi/trunci, fptosi/sitofp, index_cast), or None if there is no
    direct conversion."""
    integral = _INTEGERS + (index,)
    if source in _FLOATS and target in _FLOATS:
        return f"(double)({code})" if target == f64 else f"__double2float_rn({code})"
    if source in integral and target in integral:
        return f"(long long)({code})" if target in (i64, index) else f"(int)(unsigned)({code})"
    if (source in _FLOATS and target in _INTEGERS) or (source in _INTEGERS and target in _FLOATS):
        return f"({CTYPE[target]})({code})"
    return None


class _Emitter(BodyWalker):
    """Walks a kernel body emitting CUDA C++: typed device values become ``const`` locals,
    runtime branches and loops become C control flow, static values fold."""

    def __init__(self, definition: Definition, signature: BoundSignature):
        super().__init__(definition, signature.dimensions)
        self.lines: list[str] = []
        self.depth = 1
        self.counter = 0
        # Outer names of the innermost runtime branch (their reassignment is rejected).
        self.branch_outer = None
        self.parameters = []
        for parameter in signature.parameters:
            if parameter.is_constant:
                self.env[parameter.name] = parameter.value
                continue
            code = f"p_{parameter.name}"
            kind = _Buffer if isinstance(parameter.dtype, BufferSpec) else _Value
            self.env[parameter.name] = kind(code, parameter.dtype)
            self.parameters.append((code, parameter.dtype))

    # ---- emission helpers ------------------------------------------------------------------
    def line(self, text: str):
        self.lines.append("  " * self.depth + text)

    def fresh(self, prefix: str) -> str:
        self.counter += 1
        return f"{prefix}{self.counter}"

    def temporary(self, expression: str, dtype: ScalarType) -> _Value:
        name = self.fresh("t")
        self.line(f"const {CTYPE[dtype]} {name} = {expression};")
        return _Value(name, dtype)

    def typed(self, value, dtype: ScalarType, node) -> _Value:
        """`value` as a device value of `dtype`: typed values must match, static ones convert."""
        if isinstance(value, _Value):
            if value.dtype != dtype:
                self.fail(node, f"expected {dtype.name}, got {value.dtype.mlir}; use ckl.cast "
                                "explicitly")
            return value
        if not is_static(value):
            self.fail(node, f"expected a {dtype.name} scalar")
        return _Value(_literal(constant(value, dtype, self.definition, node), dtype), dtype)

    def nested(self, body) -> None:
        self.depth += 1
        self.walk(body)
        self.depth -= 1

    def arith(self, left: str, right: str, symbol: str, dtype: ScalarType) -> _Value:
        if dtype in _FLOATS:
            operation = {"+": "add", "-": "sub", "*": "mul", "/": "div"}[symbol]
            return self.temporary(f"__{'f' if dtype == f32 else 'd'}{operation}_rn({left}, {right})",
                                  dtype)
        unsigned = "unsigned" if dtype == i32 else "unsigned long long"
        return self.temporary(f"({CTYPE[dtype]})(({unsigned})({left}) {symbol} "
                              f"({unsigned})({right}))", dtype)

    def linear_index(self, buffer: _Buffer, node: ast.Subscript) -> str:
        indices = node.slice.elts if isinstance(node.slice, ast.Tuple) else [node.slice]
        extents = buffer.spec.shape
        if len(indices) != len(extents):
            self.fail(node, "requires one index per buffer dimension")
        code = None
        for axis, (item, extent) in enumerate(zip(indices, extents)):
            value = self.evaluate(item)
            if type(value) is int and not 0 <= value < extent:
                self.fail(item, f"constant index is out of bounds for dimension {axis}")
            term = self.typed(value, index, item).code
            code = term if code is None else f"({code}) * {extent}LL + {term}"
        return code

    # ---- walker hooks ----------------------------------------------------------------------
    def is_dynamic(self, value) -> bool:
        return isinstance(value, _Value)

    def buffer_spec(self, value):
        return value.spec if isinstance(value, _Buffer) else None

    def read_element(self, buffer, node):
        return self.temporary(f"{buffer.code}[{self.linear_index(buffer, node)}]",
                              buffer.spec.dtype)

    def dynamic_binary(self, left, right, op, node, comparison):
        anchor = left if isinstance(left, _Value) else right
        if not isinstance(anchor, _Value):
            self.fail(node, "numeric expressions require scalar operands")
        symbol = SPELLINGS[type(op)]
        if anchor.dtype == bool_ and symbol not in ("==", "!="):
            self.fail(node, "numeric expressions require compatible scalar types")
        a, b = self.typed(left, anchor.dtype, node), self.typed(right, anchor.dtype, node)
        if comparison:
            return self.temporary(f"{a.code} {symbol} {b.code}", bool_)
        if symbol == "/" and anchor.dtype not in _FLOATS:
            self.fail(node, "division requires floating operands")
        return self.arith(a.code, b.code, symbol, anchor.dtype)

    def dynamic_unary(self, value, op, node):
        if not isinstance(value, _Value) or value.dtype == bool_:
            self.fail(node, "unary arithmetic requires a numeric scalar")
        if isinstance(op, ast.UAdd):
            return value
        if value.dtype in _FLOATS:
            return self.temporary(f"-{value.code}", value.dtype)
        return self.arith(_literal(0, value.dtype), value.code, "-", value.dtype)

    def assign_local(self, target, value, node):
        if self.branch_outer is not None and target.id in self.branch_outer:
            self.fail(target, "runtime branch results are deferred; write buffers or use "
                              "branch-local variables")
        previous = self.env.get(target.id)
        if isinstance(previous, _Value):  # a typed local keeps its type
            value = self.typed(value, previous.dtype, node.value)
        self.env[target.id] = value

    def assign_element(self, target, value_node, node):
        value = self.evaluate(value_node)
        buffer = self.evaluate(target.value)
        if not isinstance(buffer, _Buffer):
            self.fail(target, "expected a typed buffer")
        where = self.linear_index(buffer, target)
        stored = self.typed(value, buffer.spec.dtype, value_node)
        self.line(f"{buffer.code}[{where}] = {stored.code};")

    def runtime_branch(self, node, predicate):
        if not isinstance(predicate, _Value) or predicate.dtype != bool_:
            self.fail(node.test, "if requires a boolean predicate; program control flow must "
                                 "be compile-time")
        saved_env, saved_outer = dict(self.env), self.branch_outer
        self.branch_outer = set(saved_env)
        self.line(f"if ({predicate.code}) {{")
        self.nested(node.body)
        self.env = dict(saved_env)
        if node.orelse:
            self.line("} else {")
            self.nested(node.orelse)
        self.line("}")
        self.env, self.branch_outer = saved_env, saved_outer

    def loop(self, node, induction, start, stop, step):
        reassigned = {n.id for statement in node.body for n in ast.walk(statement)
                      if isinstance(n, ast.Name) and isinstance(n.ctx, ast.Store)}
        if induction in reassigned:
            self.fail(node, "cannot assign to the loop induction variable")
        saved = dict(self.env)
        # Outer names the body reassigns are carried through the loop (scf.for iteration
        # arguments); static initial values take f32 / i32 / bool.
        carried_names = sorted(reassigned & saved.keys())
        initial = []
        for name in carried_names:
            if self.branch_outer is not None and name in self.branch_outer:
                self.fail(node, "runtime branch results are deferred")
            value = saved[name]
            if not isinstance(value, _Value):
                value = self.typed(value, {float: f32, int: i32}.get(type(value), bool_), node)
            initial.append(value)
        low, high = self.typed(start, index, node), self.typed(stop, index, node)
        carried = []
        for value in initial:
            variable = self.fresh("c")
            self.line(f"{CTYPE[value.dtype]} {variable} = {value.code};")
            carried.append(_Value(variable, value.dtype))
        counter = self.fresh("i")
        self.line(f"for (long long {counter} = {low.code}; {counter} < {high.code}; "
                  f"{counter} += {step}LL) {{")
        self.depth += 1
        self.env[induction] = _Value(counter, index)
        self.env.update(zip(carried_names, carried))
        self.walk(node.body)
        results = [self.typed(self.env[name], slot.dtype, node)
                   for name, slot in zip(carried_names, carried)]
        # Stage every new value before any carried variable is overwritten.
        staged = [value if value.code == slot.code else self.temporary(value.code, value.dtype)
                  for value, slot in zip(results, carried)]
        for value, slot in zip(staged, carried):
            if value.code != slot.code:
                self.line(f"{slot.code} = {value.code};")
        self.depth -= 1
        self.line("}")
        self.env = saved
        self.env.update(zip(carried_names, carried))

    # ---- intrinsics ------------------------------------------------------------------------
    def _coordinate(self, node, name):
        values, keywords = self.arguments(node)
        if keywords or len(values) != 1 or type(values[0]) is not int or values[0] not in (0, 1, 2):
            self.fail(node, "device coordinates require one constant axis 0, 1, or 2")
        axis = "xyz"[values[0]]
        if name == "global_id":
            return self.temporary(f"(long long)blockIdx.{axis} * (long long)blockDim.{axis} + "
                                  f"(long long)threadIdx.{axis}", index)
        return self.temporary(f"(long long){_COORDINATES[name]}.{axis}", index)

    def intrinsic_global_id(self, node):
        return self._coordinate(node, "global_id")

    def intrinsic_thread_id(self, node):
        return self._coordinate(node, "thread_id")

    def intrinsic_block_id(self, node):
        return self._coordinate(node, "block_id")

    def intrinsic_block_dim(self, node):
        return self._coordinate(node, "block_dim")

    def intrinsic_grid_dim(self, node):
        return self._coordinate(node, "grid_dim")

    def intrinsic_launch(self, node):
        self.fail(node, "kernels cannot launch other kernels")

    def _program_only(self, node):
        self.arguments(node)
        self.fail(node, "program temporaries cannot be allocated inside kernels")

    intrinsic_empty = intrinsic_empty_like = _program_only

    def intrinsic_subview(self, node):
        self.arguments(node)
        self.fail(node, "subview is currently supported only in programs")

    def intrinsic_cast(self, node):
        values, keywords = self.arguments(node)
        if keywords or len(values) != 2 or not isinstance(values[1], ScalarType):
            self.fail(node, "use cast(value, scalar_type)")
        value, target = values
        if not isinstance(value, _Value):
            if target in (i32, i64, index) and type(value) is float and math.isfinite(value):
                value = int(value)
            return constant(value, target, self.definition, node)
        if value.dtype == target:
            return value
        if bool_ in (value.dtype, target):
            self.fail(node, "boolean/buffer casts are unsupported")
        expression = _conversion(value.dtype, target, value.code)
        if expression is None:
            self.fail(node, "cast through an integer type to convert between index and float")
        return self.temporary(expression, target)

    def _unary_math(self, node, name):
        values, keywords = self.arguments(node)
        if keywords or len(values) != 1 or not isinstance(values[0], _Value) \
                or values[0].dtype not in _FLOATS:
            self.fail(node, f"{name} requires one typed floating-point scalar")
        suffix = "f" if values[0].dtype == f32 else ""
        return self.temporary(f"{name}{suffix}({values[0].code})", values[0].dtype)

    def intrinsic_exp(self, node):
        return self._unary_math(node, "exp")

    def intrinsic_rsqrt(self, node):
        return self._unary_math(node, "rsqrt")

    def intrinsic_select(self, node):
        values, keywords = self.arguments(node)
        if keywords or len(values) != 3:
            self.fail(node, "use select(predicate, true_value, false_value)")
        condition = self.typed(values[0], bool_, node)
        anchor = next((v for v in values[1:] if isinstance(v, _Value)), None)
        if anchor is None:
            self.fail(node, "select requires a typed scalar alternative")
        chosen, other = (self.typed(v, anchor.dtype, node) for v in values[1:])
        return self.temporary(f"{condition.code} ? {chosen.code} : {other.code}", chosen.dtype)


def symbol_for(definition: Definition, identity: str) -> str:
    """The C symbol of a generated kernel specialization."""
    base = re.sub(r"[^A-Za-z0-9_]", "_", definition.name)
    return f"{SYMBOL_PREFIX}{base}_{identity[:16]}"


_GENERATED: dict = {}


def _generate(definition: Definition, signature: BoundSignature, symbol: str) -> GeneratedKernel:
    emitter = _Emitter(definition, signature)
    emitter.walk(definition.tree.body, top=True)
    parameters = []
    for code, dtype in emitter.parameters:
        if isinstance(dtype, BufferSpec):
            parameters.append(f"{CTYPE[dtype.dtype]} *{code}")
        else:
            parameters.append(f"{CTYPE[dtype]} {code}")
    header = (f"// {definition.name} ({definition.filename}:{definition.first_line})\n"
              f"extern \"C\" __global__ void {symbol}({', '.join(parameters)}) {{\n")
    body = "\n".join(emitter.lines)
    source = header + (body + "\n" if body else "") + "}\n"
    types = tuple(d if isinstance(d, ScalarType) else d.dtype for _, d in emitter.parameters)
    return GeneratedKernel(symbol, source, types)


def generate(definition: Definition, signature: BoundSignature, identity: str) -> GeneratedKernel:
    """CUDA source of one kernel specialization; raises FrontendError for invalid bodies."""
    kernel = _GENERATED.get(identity)
    if kernel is None:
        kernel = _GENERATED[identity] = _generate(definition, signature,
                                                  symbol_for(definition, identity))
    return kernel


def translation_unit(kernels) -> str:
    """One NVRTC translation unit holding every generated kernel of a program."""
    parts = ["// Generated by ckl-b200 for sm_100a: one kernel per CKL kernel specialization.\n"]
    seen = set()
    for kernel in kernels:
        if kernel.symbol not in seen:
            seen.add(kernel.symbol)
            parts.append(kernel.source)
    return "\n".join(parts)
