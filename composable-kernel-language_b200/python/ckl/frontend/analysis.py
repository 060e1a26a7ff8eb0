"""Kernel-body analysis: per-parameter memory effects and a canonical structural key.

Effects follow the reference's effect model (``lib/Analysis/EffectAnalysis.cpp:41-254``,
``lib/Core/MemoryEffects.cpp:204-234``):

* a buffer element read is a ``read`` of that parameter, an element store a ``write``;
* an access whose indices are all compile-time integers within bounds covers exactly that
  element (a ``(byte_offset, byte_length)`` interval); any other access covers the whole
  parameter;
* several accesses to one parameter merge to the enclosing interval, or ``whole``.

The canonical key identifies *what a kernel computes* independently of how its locals,
parameters and dimensions are named: parameters become positional tokens, locals are
numbered by first appearance, named dimensions become (parameter, axis) positions and
``buf.shape[k]`` is folded to the same token.  Two kernels with equal keys perform the same
operations in the same order on the same kinds of operands; the sm_100a kernel library is
indexed by this key.
"""
from __future__ import annotations

import ast
import hashlib
import math
from dataclasses import dataclass, field

from ..types import (BufferSpec, BufferType, ConstexprType, Dimension, ScalarType, f32, f64,
                     i32, i64, index)
from .checker import BoundSignature, parameter_type
from .source import Definition, Intrinsic, ModuleView, Opaque

READ, WRITE, ALLOCATE, FREE = 1, 2, 4, 8
WHOLE = "whole"


class _Dynamic:
    """A value known only on the device."""

    __slots__ = ()


DYNAMIC = _Dynamic()


@dataclass
class _BufferParam:
    position: int          # index among runtime parameters
    spec: BufferSpec


@dataclass
class KernelSummary:
    """Effects of one kernel specialization, indexed by runtime parameter position."""

    bits: list
    regions: list
    accesses: int = 0

    def effects(self):
        """``[(runtime_param_index, bits, region)]`` for parameters that are accessed."""
        return [(i, b, r) for i, (b, r) in enumerate(zip(self.bits, self.regions)) if b]


def _merge(existing, region):
    if existing is None:
        return region
    if existing == WHOLE or region == WHOLE:
        return WHOLE
    start = min(existing[0], region[0])
    end = max(existing[0] + existing[1], region[0] + region[1])
    return (start, end - start)


class _EffectWalker:
    def __init__(self, definition: Definition, signature: BoundSignature):
        self.definition = definition
        self.dims = dict(signature.dimensions)
        runtime = [p for p in signature.parameters if not p.is_constant]
        self.summary = KernelSummary([0] * len(runtime), [None] * len(runtime))
        self.env: dict[str, object] = {}
        position = 0
        for parameter in signature.parameters:
            if parameter.is_constant:
                self.env[parameter.name] = parameter.value
                continue
            if isinstance(parameter.dtype, BufferSpec):
                self.env[parameter.name] = _BufferParam(position, parameter.dtype)
            else:
                self.env[parameter.name] = DYNAMIC
            position += 1

    def fail(self, node, message):
        raise self.definition.error(node, message)

    # -- expressions ---------------------------------------------------------------------
    def value(self, node):
        if isinstance(node, ast.Constant):
            return node.value
        if isinstance(node, ast.Name):
            if node.id in self.env:
                return self.env[node.id]
            bound = self.definition.bindings.get(node.id)
            if bound is None:
                self.fail(node, f"unknown name '{node.id}'")
            if isinstance(bound, Opaque):
                self.fail(node, f"unsupported captured binding '{node.id}'")
            if isinstance(bound, Dimension):
                if bound.name not in self.dims:
                    self.fail(node, f"unbound dimension '{bound.name}'")
                return self.dims[bound.name]
            return bound
        if isinstance(node, ast.Tuple):
            return tuple(self.value(item) for item in node.elts)
        if isinstance(node, ast.Attribute):
            base = self.value(node.value)
            if isinstance(base, ModuleView) and node.attr in base.values:
                return base.values[node.attr]
            if isinstance(base, _BufferParam):
                if node.attr == "shape":
                    return base.spec.shape
                if node.attr == "dtype":
                    return base.spec.dtype
            self.fail(node, f"unsupported attribute '{node.attr}'")
        if isinstance(node, ast.Subscript):
            base = self.value(node.value)
            if isinstance(base, _BufferParam):
                self.access(base, node, READ)
                return DYNAMIC
            if type(base) is tuple:
                position = self.value(node.slice)
                if type(position) is int and 0 <= position < len(base):
                    return base[position]
            self.fail(node, "unsupported subscript")
        if isinstance(node, ast.BinOp):
            left, right = self.value(node.left), self.value(node.right)
            if _static(left) and _static(right):
                return _fold_binary(node.op, left, right)
            return DYNAMIC
        if isinstance(node, ast.UnaryOp):
            operand = self.value(node.operand)
            if _static(operand) and isinstance(node.op, ast.USub):
                return -operand
            if _static(operand) and isinstance(node.op, ast.UAdd):
                return operand
            return DYNAMIC
        if isinstance(node, ast.Compare):
            left, right = self.value(node.left), self.value(node.comparators[0])
            if _static(left) and _static(right) and len(node.ops) == 1:
                return _fold_compare(node.ops[0], left, right)
            return DYNAMIC
        if isinstance(node, ast.Call):
            callee = self.value(node.func)
            arguments = [self.value(a) for a in node.args]
            for keyword in node.keywords:
                self.value(keyword.value)
            if isinstance(callee, Intrinsic):
                if callee.name == "cast" and len(arguments) == 2 and _static(arguments[0]) \
                        and isinstance(arguments[1], ScalarType):
                    value, target = arguments
                    if target in (i32, i64, index) and type(value) is float and math.isfinite(value):
                        return int(value)
                    if target in (f32, f64) and type(value) in (int, float):
                        return float(value)
                    return value
                if callee.name == "cdiv" and all(type(a) is int for a in arguments):
                    return (arguments[0] + arguments[1] - 1) // arguments[1]
                if callee.name == "launch":
                    self.fail(node, "kernels cannot launch other kernels")
            return DYNAMIC
        self.fail(node, f"unsupported expression: {type(node).__name__}")

    def access(self, buffer: _BufferParam, node: ast.Subscript, bit: int):
        items = node.slice.elts if isinstance(node.slice, ast.Tuple) else [node.slice]
        indices = [self.value(item) for item in items]
        if len(indices) != len(buffer.spec.shape):
            self.fail(node, "requires one index per buffer dimension")
        region = WHOLE
        if all(type(i) is int for i in indices):
            linear = 0
            inside = True
            for value, extent in zip(indices, buffer.spec.shape):
                if not 0 <= value < extent:
                    inside = False
                    break
                linear = linear * extent + value
            if inside:
                size = buffer.spec.dtype.bytes
                region = (linear * size, size)
        slot = buffer.position
        self.summary.bits[slot] |= bit
        self.summary.regions[slot] = _merge(self.summary.regions[slot], region)
        self.summary.accesses += 1

    # -- statements ----------------------------------------------------------------------
    def block(self, statements):
        for statement in statements:
            self.statement(statement)

    def statement(self, node):
        if isinstance(node, ast.Assign):
            target = node.targets[0]
            value = self.value(node.value)
            if isinstance(target, ast.Name):
                self.env[target.id] = value
            elif isinstance(target, ast.Subscript):
                buffer = self.value(target.value)
                if not isinstance(buffer, _BufferParam):
                    self.fail(target, "buffer writes require a buffer parameter")
                self.access(buffer, target, WRITE)
            else:
                self.fail(target, "assignment requires a local name or indexed buffer element")
        elif isinstance(node, ast.If):
            test = self.value(node.test)
            if type(test) is bool:
                self.block(node.body if test else node.orelse)
                return
            outer = dict(self.env)
            self.block(node.body)
            self.env = dict(outer)
            self.block(node.orelse)
            self.env = outer
        elif isinstance(node, ast.For):
            for argument in node.iter.args:
                self.value(argument)
            outer = dict(self.env)
            assigned = {n.id for s in node.body for n in ast.walk(s)
                        if isinstance(n, ast.Name) and isinstance(n.ctx, ast.Store)}
            for name in assigned:
                if name in self.env:
                    self.env[name] = DYNAMIC
            self.env[node.target.id] = DYNAMIC
            self.block(node.body)
            self.env = outer
            for name in assigned & set(outer):
                self.env[name] = DYNAMIC
        elif isinstance(node, ast.Expr):
            if isinstance(node.value, ast.Constant) and isinstance(node.value.value, str):
                return
            self.value(node.value)
        elif isinstance(node, (ast.Pass, ast.Return)):
            return
        else:
            self.fail(node, f"unsupported statement: {type(node).__name__}")


def _static(value) -> bool:
    return type(value) in (int, float, bool)


def _fold_binary(op, left, right):
    if isinstance(op, ast.Add):
        return left + right
    if isinstance(op, ast.Sub):
        return left - right
    if isinstance(op, ast.Mult):
        return left * right
    if isinstance(op, ast.Div):
        return left / right if right else DYNAMIC
    return DYNAMIC


def _fold_compare(op, left, right):
    table = {ast.Lt: lambda a, b: a < b, ast.LtE: lambda a, b: a <= b,
             ast.Gt: lambda a, b: a > b, ast.GtE: lambda a, b: a >= b,
             ast.Eq: lambda a, b: a == b, ast.NotEq: lambda a, b: a != b}
    function = table.get(type(op))
    return function(left, right) if function else DYNAMIC


def summarize(definition: Definition, signature: BoundSignature) -> KernelSummary:
    """Memory effects of a kernel specialization."""
    walker = _EffectWalker(definition, signature)
    walker.block(definition.tree.body)
    return walker.summary


# ---------------------------------------------------------------------------------------
# Canonical structural key
# ---------------------------------------------------------------------------------------
_SKIPPED_FIELDS = {"ctx", "type_comment", "lineno", "col_offset", "end_lineno",
                   "end_col_offset", "kind", "type_params", "decorator_list", "returns"}


def _parameter_descriptor(definition: Definition, argument: ast.arg, dims: dict) -> list:
    annotation = parameter_type(definition, argument)
    if isinstance(annotation, BufferType):
        shape = []
        for extent in annotation.shape:
            shape.append(dims[extent.name] if isinstance(extent, Dimension) else extent)
        return ["buffer", annotation.dtype.name, shape]
    if isinstance(annotation, ConstexprType):
        return ["constexpr", annotation.dtype.name]
    if isinstance(annotation, ScalarType):
        return ["scalar", annotation.name]
    return ["unknown", repr(annotation)]


class _Canonicalizer:
    def __init__(self, definition: Definition):
        self.definition = definition
        arguments = definition.tree.args.args
        self.params = {a.arg: f"p{i}" for i, a in enumerate(arguments)}
        self.buffer_dims: dict[str, list] = {}
        self.dims: dict[str, str] = {}
        for i, argument in enumerate(arguments):
            annotation = parameter_type(definition, argument)
            if isinstance(annotation, BufferType):
                tokens = []
                for axis, extent in enumerate(annotation.shape):
                    if isinstance(extent, Dimension):
                        token = self.dims.setdefault(extent.name, f"d{i}.{axis}")
                        tokens.append(token)
                    else:
                        tokens.append(extent)
                self.buffer_dims[argument.arg] = tokens
        self.locals: dict[str, str] = {}
        self.descriptors = [_parameter_descriptor(definition, a, self.dims) for a in arguments]

    def name(self, identifier: str):
        if identifier in self.params:
            return ["param", self.params[identifier]]
        if identifier in self.locals:
            return ["local", self.locals[identifier]]
        bound = self.definition.bindings.get(identifier)
        if isinstance(bound, Dimension):
            return ["dim", self.dims.get(bound.name, "free:" + bound.name)]
        if isinstance(bound, ModuleView):
            return ["ckl"]
        if isinstance(bound, Intrinsic):
            return ["intrinsic", bound.name]
        if isinstance(bound, ScalarType):
            return ["type", bound.name]
        if type(bound) in (int, float, bool):
            return ["constant", repr(bound)]
        # First appearance of a local (stores are visited before later loads).
        token = f"v{len(self.locals)}"
        self.locals[identifier] = token
        return ["local", token]

    def walk(self, node):
        if isinstance(node, ast.Name):
            return self.name(node.id)
        if isinstance(node, ast.Attribute):
            base = node.value
            if isinstance(base, ast.Name) and isinstance(self.definition.bindings.get(base.id),
                                                          ModuleView) and base.id not in self.params:
                bound = self.definition.bindings[base.id].values.get(node.attr)
                if isinstance(bound, Intrinsic):
                    return ["intrinsic", bound.name]
                if isinstance(bound, ScalarType):
                    return ["type", bound.name]
                return ["ckl", node.attr]
        if isinstance(node, ast.Subscript) and isinstance(node.value, ast.Attribute) \
                and node.value.attr == "shape" and isinstance(node.value.value, ast.Name) \
                and node.value.value.id in self.buffer_dims \
                and isinstance(node.slice, ast.Constant) and type(node.slice.value) is int:
            tokens = self.buffer_dims[node.value.value.id]
            axis = node.slice.value
            if 0 <= axis < len(tokens):
                token = tokens[axis]
                return ["dim", token] if isinstance(token, str) else ["constant", repr(token)]
        if isinstance(node, ast.Constant):
            return ["constant", repr(node.value)]
        if isinstance(node, ast.AST):
            # Visit stores of an assignment before its value so a local's number reflects
            # its first definition, not evaluation order of the right-hand side.
            fields = []
            for name, value in ast.iter_fields(node):
                if name in _SKIPPED_FIELDS:
                    continue
                fields.append([name, self.walk(value)])
            return [type(node).__name__, fields]
        if isinstance(node, list):
            return [self.walk(item) for item in node]
        return repr(node)


def canonical_key(definition: Definition) -> str:
    """Name-independent structural key of a kernel definition (hex SHA-256)."""
    canon = _Canonicalizer(definition)
    statements = list(definition.tree.body)
    if statements and isinstance(statements[0], ast.Expr) \
            and isinstance(statements[0].value, ast.Constant) \
            and isinstance(statements[0].value.value, str):
        statements = statements[1:]  # a docstring does not change what the kernel computes
    body = canon.walk(statements)
    payload = repr(["ckl-b200.kernel-key.v1", canon.descriptors, body])
    return hashlib.sha256(payload.encode()).hexdigest()
