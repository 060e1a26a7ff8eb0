"""Resolve restricted annotations and bind a concrete specialization of a definition.

Semantics of the reference checker (``python/ckl/frontend/checker.py:89-142``): every
parameter is annotated; ``constexpr`` parameters take a compile-time constant and never a
runtime signature entry; buffers must match dtype and rank and bind every named dimension
consistently; scalars must match exactly; definitions return nothing.
"""
from __future__ import annotations

import ast
import math
import struct
from collections.abc import Mapping
from dataclasses import dataclass

from ..types import (Buffer, BufferSpec, BufferType, ConstexprType, Dimension, NUMERIC_TYPES,
                     ScalarType, bool_, constexpr, f32, f64, i32, i64, index)
from .source import Definition, Namespace, UnsupportedBinding


def resolve(node: ast.AST, definition: Definition) -> object:
    """Evaluate an annotation expression against the definition's captured bindings."""
    if isinstance(node, ast.Constant) and type(node.value) in (str, int, float, bool, type(None)):
        if isinstance(node.value, str):
            return resolve(ast.parse(node.value, mode="eval").body, definition)
        return node.value
    if isinstance(node, ast.Name):
        if node.id not in definition.bindings:
            raise definition.error(node, f"unknown captured name '{node.id}'")
        value = definition.bindings[node.id]
        if isinstance(value, UnsupportedBinding):
            raise definition.error(node, f"unsupported captured binding '{node.id}'")
        return value
    if isinstance(node, ast.Attribute):
        base = resolve(node.value, definition)
        if isinstance(base, Namespace) and node.attr in base.values:
            return base.values[node.attr]
    if isinstance(node, ast.Tuple):
        return tuple(resolve(item, definition) for item in node.elts)
    if isinstance(node, ast.Subscript):
        base = resolve(node.value, definition)
        arguments = resolve(node.slice, definition)
        try:
            if base is Buffer:
                return Buffer[arguments]
            if base is constexpr:
                return constexpr[arguments]
        except ValueError as error:
            raise definition.error(node, str(error)) from error
    raise definition.error(node, "unsupported annotation; use CKL types and shape declarations")


def constant(value: object, dtype: ScalarType, definition: Definition, node: ast.AST) -> object:
    """Check that a Python constant fits ``dtype``; f32 values are rounded to f32."""
    if dtype == bool_ and type(value) is bool:
        return value
    if dtype in (i32, i64, index) and type(value) is int:
        bits = 32 if dtype == i32 else 64
        if -(1 << (bits - 1)) <= value < (1 << (bits - 1)):
            return value
    if dtype in (f32, f64) and type(value) in (int, float):
        try:
            converted = float(value)
            if dtype == f32:
                converted = struct.unpack("f", struct.pack("f", converted))[0]
            if math.isfinite(converted):
                return converted
        except (OverflowError, struct.error):
            pass
    shown = repr(value) if type(value) in (int, float, bool, str, type(None)) \
        else f"<{type(value).__name__}>"
    raise definition.error(node, f"constant {shown} does not fit {dtype.name}")


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


def annotation_of(definition: Definition, argument: ast.arg) -> object:
    annotation = definition.annotations.get(argument.arg)
    if annotation is None or isinstance(annotation, str):
        if argument.annotation is None:
            raise definition.error(argument, "every CKL parameter requires a type annotation")
        annotation = resolve(argument.annotation, definition)
    return annotation


def bind(definition: Definition, signature: Mapping, constants: Mapping) -> BoundSignature:
    if not isinstance(signature, Mapping) or not isinstance(constants, Mapping):
        raise definition.error(definition.tree, "signature and constants must be mappings")
    args = definition.tree.args
    if args.posonlyargs or args.vararg or args.kwarg or args.kwonlyargs or args.defaults \
            or args.kw_defaults:
        raise definition.error(definition.tree,
                               "CKL definitions require named positional parameters without defaults")
    names = {a.arg for a in args.args}
    extra = (set(signature) | set(constants)) - names
    if extra:
        raise definition.error(definition.tree, f"unknown specialization arguments: {sorted(extra)}")
    parameters, dimensions = [], {}
    for argument in args.args:
        annotation = annotation_of(definition, argument)
        name = argument.arg
        if isinstance(annotation, ConstexprType):
            if name not in constants or name in signature:
                raise definition.error(
                    argument, "constexpr parameters require a constants binding, not a runtime signature")
            value = constant(constants[name], annotation.dtype, definition, argument)
            parameters.append(BoundParameter(name, annotation.dtype, value, True))
            continue
        if name not in signature or name in constants:
            raise definition.error(argument, f"missing or misplaced runtime signature for '{name}'")
        actual = signature[name]
        if isinstance(annotation, BufferType):
            if not isinstance(actual, BufferSpec) or actual.dtype != annotation.dtype \
                    or len(actual.shape) != len(annotation.shape):
                raise definition.error(argument, f"buffer type/rank mismatch for '{name}'")
            for declared, extent in zip(annotation.shape, actual.shape):
                if isinstance(declared, Dimension):
                    previous = dimensions.setdefault(declared.name, extent)
                    if previous != extent:
                        raise definition.error(
                            argument, f"dimension {declared.name} conflicts: {previous} versus {extent}")
                elif declared != extent:
                    raise definition.error(argument, f"fixed extent {declared} does not match {extent}")
        elif annotation in NUMERIC_TYPES:
            if not isinstance(actual, ScalarType) or actual != annotation:
                raise definition.error(argument, f"scalar type mismatch for '{name}'")
        else:
            raise definition.error(argument, "runtime parameters require numeric scalars or typed buffers")
        parameters.append(BoundParameter(name, actual))
    if definition.tree.returns is not None:
        returned = definition.annotations.get("return")
        if isinstance(returned, str):
            returned = resolve(definition.tree.returns, definition)
        if returned is not None:
            raise definition.error(definition.tree.returns, "CKL entry points have no return values")
    return BoundSignature(tuple(parameters), tuple(sorted(dimensions.items())))
