"""Capture ``@ckl.kernel`` / ``@ckl.program`` definitions without executing their bodies.

Behaviour follows the reference frontend (``python/ckl/frontend/source.py:17-236``):
a definition keeps its parsed AST, the values of the free names it uses (immutable
constants and CKL types only; anything else becomes an :class:`UnsupportedBinding` that is
rejected if it is actually used), its annotations and a content identity hash.
"""
from __future__ import annotations

import ast
import hashlib
import inspect
import json
import textwrap
from dataclasses import dataclass
from types import MappingProxyType, ModuleType
from typing import Mapping

from ..types import Buffer, BufferType, ConstexprType, Dimension, ScalarType, constexpr


class FrontendError(ValueError):
    """A diagnostic tied to a source location of a CKL definition."""


@dataclass(frozen=True)
class Intrinsic:
    name: str

    def __call__(self, *args, **kwargs):
        raise FrontendError(f"ckl.{self.name} is only valid inside a CKL source definition")


_INTRINSIC_NAMES = ("global_id", "thread_id", "block_id", "block_dim", "grid_dim", "launch",
                    "empty_like", "empty", "cdiv", "cast", "exp", "rsqrt", "select", "subview")
INTRINSICS = {name: Intrinsic(name) for name in _INTRINSIC_NAMES}


@dataclass(frozen=True)
class Namespace:
    """The subset of the ``ckl`` module a definition may reference (types and intrinsics)."""

    values: Mapping[str, object]


@dataclass(frozen=True)
class UnsupportedBinding:
    name: str


def _immutable(value: object) -> bool:
    if type(value) is tuple:
        return all(_immutable(item) for item in value)
    return type(value) in (int, float, bool, str, type(None))


def capture(value: object, name: str) -> object:
    if value is range:
        return Intrinsic("range")
    if _immutable(value) or value is Buffer or value is constexpr or isinstance(
            value, (ScalarType, BufferType, ConstexprType, Dimension, Definition, Intrinsic)):
        return value
    if isinstance(value, ModuleType) and value.__name__ == "ckl":
        allowed = {key: item for key, item in vars(value).items()
                   if isinstance(item, (ScalarType, Intrinsic)) or item is Buffer
                   or item is constexpr}
        return Namespace(MappingProxyType(allowed))
    return UnsupportedBinding(name)


def fingerprint(value: object) -> object:
    """A JSON-serialisable description of a captured value, for identity hashing."""
    if isinstance(value, Definition):
        return ["definition", value.identity]
    if isinstance(value, Namespace):
        return ["namespace", sorted((key, fingerprint(item)) for key, item in value.values.items())]
    if value is Buffer or value is constexpr:
        return ["type_constructor", value.__name__]
    if isinstance(value, (ScalarType, Dimension, Intrinsic, UnsupportedBinding)):
        return [type(value).__name__, value.name]
    if isinstance(value, BufferType):
        return ["BufferType", fingerprint(value.dtype), fingerprint(value.shape)]
    if isinstance(value, ConstexprType):
        return ["ConstexprType", fingerprint(value.dtype), None]
    if type(value) is tuple:
        return ["tuple", [fingerprint(item) for item in value]]
    return [type(value).__name__, repr(value)]


@dataclass(frozen=True)
class Definition:
    """A captured CKL kernel or program."""

    kind: str
    name: str
    tree: ast.FunctionDef
    source: str
    filename: str
    first_line: int
    indentation: int
    bindings: Mapping[str, object]
    annotations: Mapping[str, object]
    identity: str

    def error(self, node: ast.AST, message: str) -> FrontendError:
        lineno = getattr(node, "lineno", 1)
        offset = getattr(node, "col_offset", 0)
        lines = self.source.splitlines()
        excerpt = lines[lineno - 1] if lineno - 1 < len(lines) else ""
        where = f"{self.filename}:{self.first_line + lineno - 1}:{self.indentation + offset + 1}"
        return FrontendError(f"{where}: {message}\n{excerpt}\n{' ' * offset}^")

    def __call__(self, *args, **kwargs):
        hint = "use ckl.launch inside a program" if self.kind == "kernel" \
            else "use .lower(signature=...)"
        raise self.error(self.tree, f"CKL {self.kind} bodies are not Python callables; {hint}")

    def lower(self, *, signature, constants=None, verify=False, ckl_opt=None):
        """Specialize a program and trace it into a dispatch plan (no device work)."""
        if self.kind != "program":
            raise self.error(self.tree, "lower a @ckl.program entry point")
        from .tracer import lower_program

        return lower_program(self, signature, {} if constants is None else constants,
                             verify=verify, ckl_opt=ckl_opt)


def _annotation_names(annotation: str) -> set[str]:
    return {n.id for n in ast.walk(ast.parse(annotation, mode="eval")) if isinstance(n, ast.Name)}


def decorate(function, kind: str) -> Definition:
    try:
        lines, first_line = inspect.getsourcelines(function)
        filename = inspect.getsourcefile(function) or "<unknown>"
    except (OSError, TypeError) as error:
        raise FrontendError("CKL definitions require retrievable source in a Python file") from error
    source = textwrap.dedent("".join(lines))
    node = next((n for n in ast.parse(source).body if isinstance(n, ast.FunctionDef)), None)
    if node is None:
        raise FrontendError("CKL requires a synchronous function definition")
    environment = dict(function.__globals__)
    environment.setdefault("range", range)
    environment.update(inspect.getclosurevars(function).nonlocals)
    used = {n.id for n in ast.walk(node) if isinstance(n, ast.Name)}
    for annotation in function.__annotations__.values():
        if isinstance(annotation, str):
            used |= _annotation_names(annotation)
    bindings = {name: capture(environment[name], name) for name in sorted(used)
                if name in environment}
    annotations = {name: value if isinstance(value, str) else capture(value, name)
                   for name, value in function.__annotations__.items()}
    payload = ["ckl-b200.frontend.v1", kind, ast.dump(node, include_attributes=False),
               [(name, fingerprint(value)) for name, value in bindings.items()],
               [(name, fingerprint(value)) for name, value in sorted(annotations.items())]]
    identity = hashlib.sha256(json.dumps(payload, sort_keys=True).encode()).hexdigest()
    indentation = len(lines[0]) - len(lines[0].lstrip())
    return Definition(kind, function.__name__, node, source, filename, first_line, indentation,
                      MappingProxyType(bindings), MappingProxyType(annotations), identity)


def kernel(function) -> Definition:
    return decorate(function, "kernel")


def program(function) -> Definition:
    return decorate(function, "program")
