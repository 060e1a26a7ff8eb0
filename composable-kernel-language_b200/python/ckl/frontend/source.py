"""``@ckl.kernel`` / ``@ckl.program``: a parsed function, its frozen scope and its identity.

A decorated function never runs as Python.  Decoration parses its source once and freezes
the values of every free name the body (or a string annotation) mentions, looked up the way
Python would resolve them at that moment: closure cells first, then module globals, then the
builtin ``range``.  A value survives freezing only if the compiler can use it - literals and
tuples of literals, CKL types and dimensions, other definitions, intrinsics, and the ``ckl``
module itself, seen through a :class:`ModuleView` of its types and intrinsics.  Anything else
is kept as an :class:`Opaque` marker that fails only if the body actually evaluates it.

The definition's identity is a SHA-256 digest of a canonical text: the definition kind, the
function's AST without positions, and a stable description of every frozen value and
annotation.  Two definitions with the same identity compile to the same code, which is what
specialization caching keys on.  The reference captures definitions the same way
(``python/ckl/frontend/source.py``); the names, diagnostics and error format below are its
public behaviour.
"""
from __future__ import annotations

import ast
import hashlib
import inspect
import textwrap
from collections import ChainMap
from types import MappingProxyType, ModuleType

from ..types import Buffer, BufferType, ConstexprType, Dimension, ScalarType, constexpr


class FrontendError(ValueError):
    """A diagnostic tied to a source location of a CKL definition."""


class Intrinsic:
    """The placeholder behind ``ckl.<name>``; only meaningful inside a definition's body."""

    __slots__ = ("name",)

    def __init__(self, name: str):
        self.name = name

    def __eq__(self, other):
        return isinstance(other, Intrinsic) and other.name == self.name

    def __hash__(self):
        return hash(("ckl-intrinsic", self.name))

    def __repr__(self):
        return f"Intrinsic({self.name!r})"

    def __call__(self, *args, **kwargs):
        raise FrontendError(f"ckl.{self.name} is only valid inside a CKL source definition")


#: Intrinsics exported as ``ckl.<name>``.
INTRINSIC_NAMES = ("global_id", "thread_id", "block_id", "block_dim", "grid_dim", "launch",
                   "empty_like", "empty", "cdiv", "cast", "exp", "rsqrt", "select", "subview")
INTRINSICS = {name: Intrinsic(name) for name in INTRINSIC_NAMES}


class ModuleView:
    """What a body can reach through the ``ckl`` module: scalar types, intrinsics, ``Buffer``
    and ``constexpr`` (``values`` maps attribute names to them)."""

    __slots__ = ("values",)

    def __init__(self, module: ModuleType):
        reachable = {}
        for attribute, item in vars(module).items():
            if isinstance(item, (ScalarType, Intrinsic)) or item is Buffer or item is constexpr:
                reachable[attribute] = item
        self.values = MappingProxyType(reachable)


class Opaque:
    """A free name whose value CKL cannot use; evaluating it in a body is an error."""

    __slots__ = ("name",)

    def __init__(self, name: str):
        self.name = name


def _is_literal(value) -> bool:
    kind = type(value)
    if kind is tuple:
        return all(_is_literal(item) for item in value)
    return kind in (int, float, bool, str) or value is None


def _is_ckl_object(value) -> bool:
    return value is Buffer or value is constexpr or isinstance(
        value, (ScalarType, BufferType, ConstexprType, Dimension, Definition, Intrinsic))


def freeze(name: str, value):
    """The form in which a free name's value is kept by a definition."""
    if value is range:
        return Intrinsic("range")
    if _is_literal(value) or _is_ckl_object(value):
        return value
    if isinstance(value, ModuleType) and value.__name__ == "ckl":
        return ModuleView(value)
    return Opaque(name)


def describe(value) -> str:
    """A stable one-line description of a frozen value (the input of identities)."""
    if isinstance(value, Definition):
        return f"definition {value.identity}"
    if isinstance(value, ModuleView):
        inner = "; ".join(f"{key}: {describe(item)}" for key, item in sorted(value.values.items()))
        return f"ckl module {{{inner}}}"
    if value is Buffer:
        return "type constructor Buffer"
    if value is constexpr:
        return "type constructor constexpr"
    if isinstance(value, Opaque):
        return f"opaque {value.name}"
    if isinstance(value, (ScalarType, Dimension, Intrinsic)):
        return f"{type(value).__name__} {value.name}"
    if isinstance(value, BufferType):
        return f"buffer of {describe(value.dtype)} shaped {describe(value.shape)}"
    if isinstance(value, ConstexprType):
        return f"constexpr {describe(value.dtype)}"
    if type(value) is tuple:
        return "(" + ", ".join(describe(item) for item in value) + ")"
    return f"{type(value).__name__} {value!r}"


class Definition:
    """A captured kernel or program.

    ``tree`` is the function's AST, ``source`` its dedented text starting at line
    ``first_line`` of ``filename`` (indented by ``indentation`` columns there); ``bindings``
    maps each free name to its frozen value and ``annotations`` each parameter (and
    ``return``) to its annotation (strings are resolved lazily by the checker)."""

    __slots__ = ("kind", "name", "tree", "source", "filename", "first_line", "indentation",
                 "bindings", "annotations", "identity")

    def __init__(self, kind, name, tree, source, filename, first_line, indentation, bindings,
                 annotations):
        self.kind, self.name, self.tree, self.source = kind, name, tree, source
        self.filename, self.first_line, self.indentation = filename, first_line, indentation
        self.bindings = MappingProxyType(dict(bindings))
        self.annotations = MappingProxyType(dict(annotations))
        self.identity = self._digest()

    def _digest(self) -> str:
        lines = ["ckl-b200 definition 2", self.kind, ast.dump(self.tree, include_attributes=False)]
        lines += [f"free {name} = {describe(value)}" for name, value in sorted(self.bindings.items())]
        for name, value in sorted(self.annotations.items()):
            shown = f"text {value!r}" if isinstance(value, str) else describe(value)
            lines.append(f"annotation {name} = {shown}")
        return hashlib.sha256("\n".join(lines).encode()).hexdigest()

    def __eq__(self, other):
        return isinstance(other, Definition) and other.identity == self.identity

    def __hash__(self):
        return hash(self.identity)

    def __repr__(self):
        return f"<ckl {self.kind} {self.name} {self.identity[:12]}>"

    def error(self, node: ast.AST, message: str) -> FrontendError:
        """A diagnostic at `node`: ``file:line:column: message``, the line, a caret."""
        row = getattr(node, "lineno", 1)
        column = getattr(node, "col_offset", 0)
        text = self.source.splitlines()
        shown = text[row - 1] if 0 < row <= len(text) else ""
        place = f"{self.filename}:{self.first_line + row - 1}:{self.indentation + column + 1}"
        return FrontendError("\n".join((f"{place}: {message}", shown, " " * column + "^")))

    def __call__(self, *args, **kwargs):
        advice = ("use ckl.launch inside a program" if self.kind == "kernel"
                  else "use .lower(signature=...)")
        raise self.error(self.tree, f"CKL {self.kind} bodies are not Python callables; {advice}")

    def lower(self, *, signature, constants=None, verify=False, ckl_opt=None):
        """Specialize a program and trace it into a dispatch plan (no device work)."""
        if self.kind != "program":
            raise self.error(self.tree, "lower a @ckl.program entry point")
        from .tracer import lower_program

        return lower_program(self, signature, constants or {}, verify=verify, ckl_opt=ckl_opt)


def _function_source(function):
    """(function AST, dedented text, filename, first line, indentation) of a function."""
    try:
        lines, first_line = inspect.getsourcelines(function)
        filename = inspect.getsourcefile(function) or "<unknown>"
    except (OSError, TypeError) as error:
        raise FrontendError("CKL definitions require retrievable source in a Python file") \
            from error
    text = textwrap.dedent("".join(lines))
    functions = [n for n in ast.parse(text).body if isinstance(n, ast.FunctionDef)]
    if not functions:
        raise FrontendError("CKL requires a synchronous function definition")
    indentation = len(lines[0]) - len(lines[0].lstrip())
    return functions[0], text, filename, first_line, indentation


def _mentioned(tree: ast.AST, annotations) -> set:
    """Every identifier the body mentions, plus those inside string annotations."""
    trees = [tree] + [ast.parse(text, mode="eval") for text in annotations.values()
                      if isinstance(text, str)]
    return {n.id for t in trees for n in ast.walk(t) if isinstance(n, ast.Name)}


def decorate(function, kind: str) -> Definition:
    tree, text, filename, first_line, indentation = _function_source(function)
    raw = function.__annotations__
    scope = ChainMap(inspect.getclosurevars(function).nonlocals, function.__globals__,
                     {"range": range})
    bindings = {name: freeze(name, scope[name]) for name in _mentioned(tree, raw) if name in scope}
    annotations = {name: value if isinstance(value, str) else freeze(name, value)
                   for name, value in raw.items()}
    return Definition(kind, function.__name__, tree, text, filename, first_line, indentation,
                      bindings, annotations)


def kernel(function) -> Definition:
    return decorate(function, "kernel")


def program(function) -> Definition:
    return decorate(function, "program")
