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
from .frontend.source import Definition, Intrinsic, Namespace, UnsupportedBinding
from .types import BufferSpec, Dimension, ScalarType, bool_, f32, f64, i32, i64, index

CTYPE = {f32: "float", f64: "double", i32: "int", i64: "long long", index: "long long",
         bool_: "bool"}
_COORDINATES = {"thread_id": "threadIdx", "block_id": "blockIdx", "block_dim": "blockDim",
                "grid_dim": "gridDim"}
_AXES = "xyz"
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


def _static(value) -> bool:
    return type(value) in (int, float, bool)


class _Emitter:
    def __init__(self, definition: Definition, signature: BoundSignature):
        self.definition = definition
        self.signature = signature
        self.dimensions = dict(signature.dimensions)
        self.lines: list[str] = []
        self.depth = 1
        self.counter = 0
        self.env: dict[str, object] = {}
        self.local_names = {p.name for p in signature.parameters} | {
            n.id for n in ast.walk(definition.tree)
            if isinstance(n, ast.Name) and isinstance(n.ctx, ast.Store)}
        self.parameters = []
        for parameter in signature.parameters:
            if parameter.is_constant:
                self.env[parameter.name] = parameter.value
                continue
            code = f"p_{parameter.name}"
            if isinstance(parameter.dtype, BufferSpec):
                self.env[parameter.name] = _Buffer(code, parameter.dtype)
                self.parameters.append((code, parameter.dtype))
            else:
                self.env[parameter.name] = _Value(code, parameter.dtype)
                self.parameters.append((code, parameter.dtype))

    # -- helpers ---------------------------------------------------------------------------
    def fail(self, node, message):
        raise self.definition.error(node, message)

    def line(self, text: str):
        self.lines.append("  " * self.depth + text)

    def temporary(self, expression: str, dtype: ScalarType) -> _Value:
        self.counter += 1
        name = f"t{self.counter}"
        self.line(f"const {CTYPE[dtype]} {name} = {expression};")
        return _Value(name, dtype)

    def variable(self, prefix: str) -> str:
        self.counter += 1
        return f"{prefix}{self.counter}"

    def typed(self, value, dtype: ScalarType, node) -> _Value:
        if isinstance(value, _Value):
            if value.dtype != dtype:
                self.fail(node, f"expected {dtype.name}, got {value.dtype.mlir}; use ckl.cast "
                                "explicitly")
            return value
        if not _static(value):
            self.fail(node, f"expected a {dtype.name} scalar")
        return _Value(_literal(constant(value, dtype, self.definition, node), dtype), dtype)

    # -- expressions -----------------------------------------------------------------------
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
            captured = self.definition.bindings[node.id]
            if isinstance(captured, UnsupportedBinding):
                self.fail(node, f"unsupported captured binding '{node.id}'")
            if isinstance(captured, Dimension):
                if captured.name not in self.dimensions:
                    self.fail(node, f"unbound dimension '{captured.name}'")
                return self.dimensions[captured.name]
            return captured
        if isinstance(node, ast.Tuple):
            return tuple(self.expression(item) for item in node.elts)
        if isinstance(node, ast.Attribute):
            base = self.expression(node.value)
            if isinstance(base, Namespace) and node.attr in base.values:
                return base.values[node.attr]
            if isinstance(base, _Buffer):
                if node.attr == "shape":
                    return base.spec.shape
                if node.attr == "dtype":
                    return base.spec.dtype
            self.fail(node, f"unsupported attribute '{node.attr}'")
        if isinstance(node, ast.Subscript):
            base = self.expression(node.value)
            if isinstance(base, _Buffer):
                offset = self.offset(base, node)
                return self.temporary(f"{base.code}[{offset}]", base.spec.dtype)
            if type(base) is tuple:
                position = self.expression(node.slice)
                if type(position) is not int or not 0 <= position < len(base):
                    self.fail(node, "tuple/shape axes require an in-range nonnegative "
                                    "compile-time integer")
                return base[position]
            self.fail(node, "unsupported subscript; slices and negative indexing are not "
                            "supported")
        if isinstance(node, ast.BinOp):
            return self.binary(node.left, node.right, node.op, node, comparison=False)
        if isinstance(node, ast.UnaryOp) and isinstance(node.op, (ast.USub, ast.UAdd)):
            value = self.expression(node.operand)
            if type(value) in (int, float):
                return -value if isinstance(node.op, ast.USub) else value
            if not isinstance(value, _Value) or value.dtype == bool_:
                self.fail(node, "unary arithmetic requires a numeric scalar")
            if isinstance(node.op, ast.UAdd):
                return value
            if value.dtype in (f32, f64):
                return self.temporary(f"-{value.code}", value.dtype)
            return self.arith(_literal(0, value.dtype), value.code, "-", value.dtype)
        if isinstance(node, ast.Compare):
            if len(node.ops) != 1:
                self.fail(node, "chained comparisons are not supported")
            return self.binary(node.left, node.comparators[0], node.ops[0], node, comparison=True)
        if isinstance(node, ast.Call):
            return self.call(node)
        self.fail(node, f"unsupported expression: {type(node).__name__}")

    def offset(self, buffer: _Buffer, node: ast.Subscript) -> str:
        items = node.slice.elts if isinstance(node.slice, ast.Tuple) else [node.slice]
        shape = buffer.spec.shape
        if len(items) != len(shape):
            self.fail(node, "requires one index per buffer dimension")
        linear = None
        for axis, item in enumerate(items):
            value = self.expression(item)
            if type(value) is int and not 0 <= value < shape[axis]:
                self.fail(item, f"constant index is out of bounds for dimension {axis}")
            code = self.typed(value, index, item).code
            linear = code if linear is None else f"({linear}) * {shape[axis]}LL + {code}"
        return linear

    def arith(self, left: str, right: str, symbol: str, dtype: ScalarType) -> _Value:
        if dtype in (f32, f64):
            suffix = "f" if dtype == f32 else "d"
            name = {"+": "add", "-": "sub", "*": "mul", "/": "div"}[symbol]
            return self.temporary(f"__{suffix}{name}_rn({left}, {right})", dtype)
        if dtype == i32:
            return self.temporary(f"(int)((unsigned)({left}) {symbol} (unsigned)({right}))", dtype)
        return self.temporary(
            f"(long long)((unsigned long long)({left}) {symbol} (unsigned long long)({right}))",
            dtype)

    def binary(self, left_node, right_node, op, node, *, comparison: bool):
        left, right = self.expression(left_node), self.expression(right_node)
        symbols = {ast.Add: "+", ast.Sub: "-", ast.Mult: "*", ast.Div: "/", ast.Lt: "<",
                   ast.LtE: "<=", ast.Gt: ">", ast.GtE: ">=", ast.Eq: "==", ast.NotEq: "!="}
        if type(op) not in symbols:
            self.fail(node, f"unsupported numeric operator: {type(op).__name__}")
        symbol = symbols[type(op)]
        if not isinstance(left, _Value) and not isinstance(right, _Value):
            allowed = (int, float, bool) if comparison else (int, float)
            if type(left) not in allowed or type(right) not in allowed:
                self.fail(node, "numeric expressions require scalar operands")
            try:
                result = {"+": lambda a, b: a + b, "-": lambda a, b: a - b,
                          "*": lambda a, b: a * b, "/": lambda a, b: a / b,
                          "<": lambda a, b: a < b, "<=": lambda a, b: a <= b,
                          ">": lambda a, b: a > b, ">=": lambda a, b: a >= b,
                          "==": lambda a, b: a == b, "!=": lambda a, b: a != b}[symbol](left, right)
            except (ZeroDivisionError, OverflowError) as error:
                self.fail(node, f"invalid constant expression: {error}")
            if type(result) is float and not math.isfinite(result):
                self.fail(node, "non-finite constant expression")
            return result
        dynamic = left if isinstance(left, _Value) else right
        dtype = dynamic.dtype
        if dtype == bool_ and symbol not in ("==", "!="):
            self.fail(node, "numeric expressions require compatible scalar types")
        left, right = self.typed(left, dtype, node), self.typed(right, dtype, node)
        if comparison:
            return self.temporary(f"{left.code} {symbol} {right.code}", bool_)
        if symbol == "/" and dtype not in (f32, f64):
            self.fail(node, "division requires floating operands")
        return self.arith(left.code, right.code, symbol, dtype)

    def call(self, node: ast.Call):
        callee = self.expression(node.func)
        if isinstance(callee, Definition):
            self.fail(node, "kernel definitions are not ordinary calls; use ckl.launch")
        if not isinstance(callee, Intrinsic):
            self.fail(node, "calling arbitrary Python functions is unsupported")
        if any(isinstance(a, ast.Starred) for a in node.args) or any(k.arg is None
                                                                     for k in node.keywords):
            self.fail(node, "argument expansion is unsupported")
        name = callee.name
        if name == "launch":
            self.fail(node, "kernels cannot launch other kernels")
        args = [self.expression(a) for a in node.args]
        keywords = {k.arg: self.expression(k.value) for k in node.keywords}
        if name in ("global_id",) + tuple(_COORDINATES):
            if len(args) != 1 or keywords or type(args[0]) is not int or not 0 <= args[0] <= 2:
                self.fail(node, "device coordinates require one constant axis 0, 1, or 2")
            axis = _AXES[args[0]]
            if name == "global_id":
                return self.temporary(f"(long long)blockIdx.{axis} * (long long)blockDim.{axis} "
                                      f"+ (long long)threadIdx.{axis}", index)
            return self.temporary(f"(long long){_COORDINATES[name]}.{axis}", index)
        if name == "cdiv":
            if len(args) != 2 or keywords or any(type(v) is not int for v in args) \
                    or args[0] < 0 or args[1] <= 0:
                self.fail(node, "cdiv requires a nonnegative constant extent and positive constant "
                                "divisor")
            return (args[0] + args[1] - 1) // args[1]
        if name in ("empty", "empty_like"):
            self.fail(node, "program temporaries cannot be allocated inside kernels")
        if name == "subview":
            self.fail(node, "subview is currently supported only in programs")
        if name == "cast":
            if len(args) != 2 or keywords or not isinstance(args[1], ScalarType):
                self.fail(node, "use cast(value, scalar_type)")
            return self.cast(args[0], args[1], node)
        if name in ("exp", "rsqrt"):
            if len(args) != 1 or keywords or not isinstance(args[0], _Value) \
                    or args[0].dtype not in (f32, f64):
                self.fail(node, f"{name} requires one typed floating-point scalar")
            suffix = "f" if args[0].dtype == f32 else ""
            return self.temporary(f"{name}{suffix}({args[0].code})", args[0].dtype)
        if name == "select":
            if len(args) != 3 or keywords:
                self.fail(node, "use select(predicate, true_value, false_value)")
            condition = self.typed(args[0], bool_, node)
            dynamic = next((v for v in args[1:] if isinstance(v, _Value)), None)
            if dynamic is None:
                self.fail(node, "select requires a typed scalar alternative")
            lhs, rhs = [self.typed(v, dynamic.dtype, node) for v in args[1:]]
            return self.temporary(f"{condition.code} ? {lhs.code} : {rhs.code}", lhs.dtype)
        self.fail(node, f"unsupported intrinsic: {name}")

    def cast(self, value, dtype: ScalarType, node):
        if not isinstance(value, _Value):
            if dtype in (i32, i64, index) and type(value) is float and math.isfinite(value):
                value = int(value)
            return constant(value, dtype, self.definition, node)
        source = value.dtype
        if source == dtype:
            return value
        if bool_ in (source, dtype):
            self.fail(node, "boolean/buffer casts are unsupported")
        floats, integers = (f32, f64), (i32, i64)
        if source in floats and dtype in floats:
            expression = f"(double)({value.code})" if dtype == f64 \
                else f"__double2float_rn({value.code})"
        elif source in integers and dtype in integers:
            expression = f"(long long)({value.code})" if dtype == i64 \
                else f"(int)(unsigned)({value.code})"
        elif source in floats and dtype in integers:
            expression = f"({CTYPE[dtype]})({value.code})"
        elif source in integers and dtype in floats:
            expression = f"({CTYPE[dtype]})({value.code})"
        elif index in (source, dtype) and (source in integers or dtype in integers):
            expression = f"(long long)({value.code})" if dtype == index or dtype == i64 \
                else f"(int)(unsigned)({value.code})"
        else:
            self.fail(node, "cast through an integer type to convert between index and float")
        return self.temporary(expression, dtype)

    # -- statements ------------------------------------------------------------------------
    def statements(self, nodes, *, top=False, branch_outer=None):
        for position, node in enumerate(nodes):
            if isinstance(node, ast.Return):
                if not top or position != len(nodes) - 1 or node.value is not None:
                    self.fail(node, "only a final bare return is supported; buffers carry outputs")
            elif isinstance(node, ast.Assign):
                if len(node.targets) != 1:
                    self.fail(node, "chained assignment is unsupported")
                target = node.targets[0]
                value = self.expression(node.value)
                if isinstance(target, ast.Name):
                    if branch_outer is not None and target.id in branch_outer:
                        self.fail(target, "runtime branch results are deferred; write buffers or "
                                          "use branch-local variables")
                    old = self.env.get(target.id)
                    if isinstance(old, _Value):
                        value = self.typed(value, old.dtype, node.value)
                    self.env[target.id] = value
                elif isinstance(target, ast.Subscript):
                    buffer = self.expression(target.value)
                    if not isinstance(buffer, _Buffer):
                        self.fail(target, "expected a typed buffer")
                    offset = self.offset(buffer, target)
                    stored = self.typed(value, buffer.spec.dtype, node.value)
                    self.line(f"{buffer.code}[{offset}] = {stored.code};")
                else:
                    self.fail(target, "assignment requires a local name or indexed buffer element")
            elif isinstance(node, ast.If):
                predicate = self.expression(node.test)
                if type(predicate) is bool:
                    self.statements(node.body if predicate else node.orelse,
                                    branch_outer=branch_outer)
                    continue
                if not isinstance(predicate, _Value) or predicate.dtype != bool_:
                    self.fail(node.test, "if requires a boolean predicate; program control flow "
                                         "must be compile-time")
                outer = dict(self.env)
                self.line(f"if ({predicate.code}) {{")
                self.depth += 1
                self.statements(node.body, branch_outer=set(outer))
                self.depth -= 1
                self.env = dict(outer)
                if node.orelse:
                    self.line("} else {")
                    self.depth += 1
                    self.statements(node.orelse, branch_outer=set(outer))
                    self.depth -= 1
                self.line("}")
                self.env = outer
            elif isinstance(node, ast.For):
                self.loop(node, branch_outer)
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

    def loop(self, node: ast.For, branch_outer):
        if node.orelse or not isinstance(node.target, ast.Name) \
                or not isinstance(node.iter, ast.Call):
            self.fail(node, "for requires a simple induction variable and range without else")
        callee = self.expression(node.iter.func)
        if not isinstance(callee, Intrinsic) or callee.name != "range" or node.iter.keywords:
            self.fail(node, "for requires range(start, stop, positive_constant_step)")
        bounds = [self.expression(a) for a in node.iter.args]
        if not 1 <= len(bounds) <= 3:
            self.fail(node, "range requires one to three bounds")
        start, stop, step = (0, bounds[0], 1) if len(bounds) == 1 else (
            bounds[0], bounds[1], bounds[2] if len(bounds) == 3 else 1)
        if type(step) is not int or step <= 0:
            self.fail(node, "range step must be a positive compile-time integer")
        induction = node.target.id
        outer = dict(self.env)
        assignments = {n.id for statement in node.body for n in ast.walk(statement)
                       if isinstance(n, ast.Name) and isinstance(n.ctx, ast.Store)}
        if induction in assignments:
            self.fail(node, "cannot assign to the loop induction variable")
        names = sorted(assignments & outer.keys())
        initials = []
        for name in names:
            if branch_outer is not None and name in branch_outer:
                self.fail(node, "runtime branch results are deferred")
            value = outer[name]
            if not isinstance(value, _Value):
                dtype = f32 if type(value) is float else i32 if type(value) is int else bool_
                value = self.typed(value, dtype, node)
            initials.append(value)
        lower, upper = self.typed(start, index, node), self.typed(stop, index, node)
        carried = []
        for name, initial in zip(names, initials):
            variable = self.variable("c")
            self.line(f"{CTYPE[initial.dtype]} {variable} = {initial.code};")
            carried.append(_Value(variable, initial.dtype))
        counter = self.variable("i")
        self.line(f"for (long long {counter} = {lower.code}; {counter} < {upper.code}; "
                  f"{counter} += {step}LL) {{")
        self.depth += 1
        self.env[induction] = _Value(counter, index)
        for name, value in zip(names, carried):
            self.env[name] = value
        self.statements(node.body, branch_outer=branch_outer)
        yielded = [self.typed(self.env[name], value.dtype, node) for name, value in
                   zip(names, carried)]
        staged = [self.temporary(v.code, v.dtype) if v.code != c.code else v
                  for v, c in zip(yielded, carried)]
        for value, variable in zip(staged, carried):
            if value.code != variable.code:
                self.line(f"{variable.code} = {value.code};")
        self.depth -= 1
        self.line("}")
        self.env = outer
        for name, value in zip(names, carried):
            self.env[name] = value


def symbol_for(definition: Definition, identity: str) -> str:
    """The C symbol of a generated kernel specialization."""
    base = re.sub(r"[^A-Za-z0-9_]", "_", definition.name)
    return f"{SYMBOL_PREFIX}{base}_{identity[:16]}"


_GENERATED: dict = {}


def _generate(definition: Definition, signature: BoundSignature, symbol: str) -> GeneratedKernel:
    emitter = _Emitter(definition, signature)
    emitter.statements(definition.tree.body, top=True)
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
