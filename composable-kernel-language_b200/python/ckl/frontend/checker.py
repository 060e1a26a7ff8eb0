"""Parameter types of a definition and the binding of one concrete specialization.

Rules (the reference checker's public behaviour, ``python/ckl/frontend/checker.py``): every
parameter is annotated with a CKL type; a ``constexpr[...]`` parameter takes a compile-time
constant from ``constants`` and never appears in the runtime signature; a buffer parameter
takes a :class:`BufferSpec` of the declared element type and rank, whose extents equal the
declared fixed extents and bind each named :class:`Dimension` to one value across all
parameters; a scalar parameter takes exactly its declared scalar type; definitions return
nothing.  Python constants handed to typed slots must fit the type (integers by range, floats
finite after rounding to the target precision).
"""
from __future__ import annotations

import ast
import math
import struct
from collections.abc import Mapping
from dataclasses import dataclass

from ..types import (Buffer, BufferSpec, BufferType, ConstexprType, Dimension, NUMERIC_TYPES,
                     ScalarType, bool_, constexpr, f32, f64, i32, i64, index)
from .source import Definition, ModuleView, Opaque

_UNFIT = object()


class _AnnotationEvaluator(ast.NodeVisitor):
    """Evaluates an annotation expression against a definition's frozen scope: names, ``ckl.``
    attributes, tuples, literals, ``Buffer[...]`` and ``constexpr[...]``."""

    def __init__(self, definition: Definition):
        self.definition = definition

    def generic_visit(self, node):
        raise self.definition.error(node, "unsupported annotation; use CKL types and shape "
                                          "declarations")

    def visit_Expression(self, node):
        return self.visit(node.body)

    def visit_Constant(self, node):
        if isinstance(node.value, str):  # a quoted annotation: evaluate its text
            return self.visit(ast.parse(node.value, mode="eval"))
        if type(node.value) in (int, float, bool) or node.value is None:
            return node.value
        return self.generic_visit(node)

    def visit_Name(self, node):
        scope = self.definition.bindings
        if node.id not in scope:
            raise self.definition.error(node, f"unknown captured name '{node.id}'")
        if isinstance(scope[node.id], Opaque):
            raise self.definition.error(node, f"unsupported captured binding '{node.id}'")
        return scope[node.id]

    def visit_Attribute(self, node):
        owner = self.visit(node.value)
        if isinstance(owner, ModuleView) and node.attr in owner.values:
            return owner.values[node.attr]
        return self.generic_visit(node)

    def visit_Tuple(self, node):
        return tuple(self.visit(item) for item in node.elts)

    def visit_Subscript(self, node):
        constructor = self.visit(node.value)
        if constructor is not Buffer and constructor is not constexpr:
            return self.generic_visit(node)
        arguments = self.visit(node.slice)
        try:
            return constructor[arguments]
        except ValueError as error:
            raise self.definition.error(node, str(error)) from error


def resolve(node: ast.AST, definition: Definition):
    """The value of an annotation expression of `definition`."""
    return _AnnotationEvaluator(definition).visit(node)


def parameter_type(definition: Definition, argument: ast.arg):
    """The CKL type a parameter is annotated with (string annotations resolved here)."""
    declared = definition.annotations.get(argument.arg)
    if declared is not None and not isinstance(declared, str):
        return declared
    if argument.annotation is None:
        raise definition.error(argument, "every CKL parameter requires a type annotation")
    return resolve(argument.annotation, definition)


# ---- constants ---------------------------------------------------------------------------
def _integer_fitter(bits: int):
    low, high = -(1 << (bits - 1)), 1 << (bits - 1)
    return lambda value: value if type(value) is int and low <= value < high else _UNFIT


def _float_fitter(single: bool):
    def fit(value):
        if type(value) not in (int, float):
            return _UNFIT
        try:
            result = float(value)
            if single:  # round to the nearest float32
                result = struct.unpack("<f", struct.pack("<f", result))[0]
        except (OverflowError, struct.error):
            return _UNFIT
        return result if math.isfinite(result) else _UNFIT
    return fit


_FITTERS = {bool_: lambda value: value if type(value) is bool else _UNFIT,
            i32: _integer_fitter(32), i64: _integer_fitter(64), index: _integer_fitter(64),
            f32: _float_fitter(True), f64: _float_fitter(False)}


def constant(value, dtype: ScalarType, definition: Definition, node: ast.AST):
    """`value` as a compile-time constant of `dtype` (f32 values rounded to float32)."""
    fitter = _FITTERS.get(dtype)
    result = fitter(value) if fitter is not None else _UNFIT
    if result is _UNFIT:
        shown = repr(value) if type(value) in (int, float, bool, str) or value is None \
            else f"<{type(value).__name__}>"
        raise definition.error(node, f"constant {shown} does not fit {dtype.name}")
    return result


# ---- binding -----------------------------------------------------------------------------
@dataclass(frozen=True)
class BoundParameter:
    name: str
    dtype: object  # ScalarType | BufferSpec
    value: object = None
    is_constant: bool = False


@dataclass(frozen=True)
class BoundSignature:
    parameters: tuple
    dimensions: tuple

    @property
    def runtime(self) -> tuple:
        return tuple(p for p in self.parameters if not p.is_constant)


class _Binder:
    """Accumulates the bound parameters and dimension extents of one specialization."""

    def __init__(self, definition: Definition, signature: Mapping, constants: Mapping):
        self.definition, self.signature, self.constants = definition, signature, constants
        self.parameters: list = []
        self.extents: dict = {}

    def add(self, argument: ast.arg) -> None:
        declared = parameter_type(self.definition, argument)
        name = argument.arg
        if isinstance(declared, ConstexprType):
            if name in self.signature or name not in self.constants:
                raise self.definition.error(argument, "constexpr parameters require a constants "
                                                      "binding, not a runtime signature")
            value = constant(self.constants[name], declared.dtype, self.definition, argument)
            self.parameters.append(BoundParameter(name, declared.dtype, value, True))
            return
        if name in self.constants or name not in self.signature:
            raise self.definition.error(argument,
                                        f"missing or misplaced runtime signature for '{name}'")
        given = self.signature[name]
        if isinstance(declared, BufferType):
            self._buffer(argument, declared, given)
        elif declared in NUMERIC_TYPES:
            if not (isinstance(given, ScalarType) and given == declared):
                raise self.definition.error(argument, f"scalar type mismatch for '{name}'")
        else:
            raise self.definition.error(argument, "runtime parameters require numeric scalars "
                                                  "or typed buffers")
        self.parameters.append(BoundParameter(name, given))

    def _buffer(self, argument, declared: BufferType, given) -> None:
        if not isinstance(given, BufferSpec) or given.dtype != declared.dtype \
                or len(given.shape) != len(declared.shape):
            raise self.definition.error(argument,
                                        f"buffer type/rank mismatch for '{argument.arg}'")
        for axis_type, extent in zip(declared.shape, given.shape):
            if not isinstance(axis_type, Dimension):
                if axis_type != extent:
                    raise self.definition.error(
                        argument, f"fixed extent {axis_type} does not match {extent}")
                continue
            known = self.extents.setdefault(axis_type.name, extent)
            if known != extent:
                raise self.definition.error(
                    argument, f"dimension {axis_type.name} conflicts: {known} versus {extent}")

    def check_result(self) -> None:
        returns = self.definition.tree.returns
        if returns is None:
            return
        declared = self.definition.annotations.get("return")
        if isinstance(declared, str):
            declared = resolve(returns, self.definition)
        if declared is not None:
            raise self.definition.error(returns, "CKL entry points have no return values")

    def result(self) -> BoundSignature:
        return BoundSignature(tuple(self.parameters), tuple(sorted(self.extents.items())))


def bind(definition: Definition, signature: Mapping, constants: Mapping) -> BoundSignature:
    """Bind `definition` to runtime parameter types (`signature`) and compile-time values
    (`constants`), both keyed by parameter name."""
    if not (isinstance(signature, Mapping) and isinstance(constants, Mapping)):
        raise definition.error(definition.tree, "signature and constants must be mappings")
    spec = definition.tree.args
    if any((spec.posonlyargs, spec.vararg, spec.kwarg, spec.kwonlyargs, spec.defaults,
            spec.kw_defaults)):
        raise definition.error(definition.tree, "CKL definitions require named positional "
                                                "parameters without defaults")
    stray = sorted((set(signature) | set(constants)) - {a.arg for a in spec.args})
    if stray:
        raise definition.error(definition.tree, f"unknown specialization arguments: {stray}")
    binder = _Binder(definition, signature, constants)
    for argument in spec.args:
        binder.add(argument)
    binder.check_result()
    return binder.result()
