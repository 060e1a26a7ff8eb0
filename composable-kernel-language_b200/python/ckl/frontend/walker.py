"""One evaluator for CKL definition bodies, shared by the program tracer and the kernel
code generator.

A body is a restricted Python function.  Both consumers interpret it the same way up to the
point where a value stops being known at compile time: names resolve through the walker's
locals, then the definition's frozen scope (named dimensions become their bound extents);
literals, tuples, shapes, ``ckl.`` attributes and arithmetic on Python numbers fold at compile
time; calls go to intrinsics only; statements are assignments, ``if``, ``for ... in range``,
launches (expression statements) and a final bare ``return``.  What happens to a value that
is *not* static is the consumer's business, through a small set of hooks:

========================  ==============================  ==================================
hook                      program tracer                  kernel code generator
========================  ==============================  ==================================
``is_dynamic``            a forwarded runtime scalar      a typed device value
``buffer_spec``           a program buffer                a kernel buffer parameter
``read_element``          rejected                        a load
``dynamic_binary/unary``  rejected                        emitted arithmetic
``intrinsic_<name>``      launch, empty, subview, ...     coordinates, cast, exp, select, ...
``assign_local/element``  locals only                     locals, stores
``runtime_branch``        rejected                        emitted ``if``
``loop``                  unrolled                        emitted ``for`` with carried values
========================  ==============================  ==================================

The diagnostics are the reference frontend's (``python/ckl/frontend/emitter.py``), so user
code sees the same messages; the evaluator itself is this module's own design.
"""
from __future__ import annotations

import ast
import math
import operator

from ..types import Dimension
from .source import Definition, Intrinsic, ModuleView, Opaque

#: Compile-time folding of binary operators on Python numbers.
FOLDS = {ast.Add: operator.add, ast.Sub: operator.sub, ast.Mult: operator.mul,
         ast.Div: operator.truediv, ast.Lt: operator.lt, ast.LtE: operator.le,
         ast.Gt: operator.gt, ast.GtE: operator.ge, ast.Eq: operator.eq, ast.NotEq: operator.ne}
#: The same operators as C spellings (for code generators).
SPELLINGS = {ast.Add: "+", ast.Sub: "-", ast.Mult: "*", ast.Div: "/", ast.Lt: "<",
             ast.LtE: "<=", ast.Gt: ">", ast.GtE: ">=", ast.Eq: "==", ast.NotEq: "!="}
COORDINATE_INTRINSICS = ("global_id", "thread_id", "block_id", "block_dim", "grid_dim")

_ABSENT = object()


def is_static(value) -> bool:
    """A compile-time Python number or boolean."""
    return type(value) in (int, float, bool)


class BodyWalker:
    """Evaluates one definition body; subclasses supply the hooks listed in the module
    docstring.  ``env`` maps local names to values; ``dimensions`` maps bound dimension
    names to extents."""

    def __init__(self, definition: Definition, dimensions):
        self.definition = definition
        self.dimensions = dict(dimensions)
        self.env: dict = {}
        # Names the body assigns: reading one before its assignment is a path error, not an
        # unknown name.
        self.assigned = {n.id for n in ast.walk(definition.tree)
                         if isinstance(n, ast.Name) and isinstance(n.ctx, ast.Store)}
        self.assigned |= {a.arg for a in definition.tree.args.args}

    # ---- hooks (defaults reject) ---------------------------------------------------------
    def is_dynamic(self, value) -> bool:
        return False

    def buffer_spec(self, value):
        """The BufferSpec of a buffer value, else None."""
        return None

    def read_element(self, buffer, node):
        self.fail(node, "buffer contents can only be accessed inside a kernel")

    def dynamic_binary(self, left, right, op, node, comparison: bool):
        self.fail(node, "numeric expressions require scalar operands")

    def dynamic_unary(self, value, op, node):
        self.fail(node, "unsupported expression: UnaryOp")

    def assign_local(self, target: ast.Name, value, node: ast.Assign) -> None:
        self.env[target.id] = value

    def assign_element(self, target: ast.Subscript, value, node: ast.Assign) -> None:
        self.fail(target, "assignment requires a local name or indexed buffer element")

    def runtime_branch(self, node: ast.If, predicate) -> None:
        self.fail(node.test, "if requires a boolean predicate; program control flow must be "
                             "compile-time")

    def loop(self, node: ast.For, induction: str, start, stop, step: int) -> None:
        raise NotImplementedError

    def launch_result_ok(self, value) -> bool:
        """Whether an expression statement's value is acceptable (a launch returns None)."""
        return value is None

    # ---- diagnostics -----------------------------------------------------------------------
    def fail(self, node, message):
        raise self.definition.error(node, message)

    def location(self, node) -> str:
        line = self.definition.first_line + getattr(node, "lineno", 1) - 1
        column = self.definition.indentation + getattr(node, "col_offset", 0) + 1
        return f"{self.definition.filename}:{line}:{column}"

    # ---- expressions -----------------------------------------------------------------------
    def evaluate(self, node):
        method = getattr(self, "_expression_" + type(node).__name__, None)
        if method is None:
            self.fail(node, f"unsupported expression: {type(node).__name__}")
        return method(node)

    def _expression_Constant(self, node):
        value = node.value
        if not is_static(value):
            self.fail(node, f"unsupported expression: {type(node).__name__}")
        if type(value) is float and not math.isfinite(value):
            self.fail(node, "non-finite source constants are unsupported")
        return value

    def _expression_Name(self, node):
        found = self.env.get(node.id, _ABSENT)
        if found is not _ABSENT:
            return found
        if node.id in self.assigned:
            self.fail(node, f"local '{node.id}' is not defined on this path")
        frozen = self.definition.bindings.get(node.id, _ABSENT)
        if frozen is _ABSENT:
            self.fail(node, f"unknown name '{node.id}'")
        if isinstance(frozen, Opaque):
            self.fail(node, f"unsupported captured binding '{node.id}'")
        if isinstance(frozen, Dimension):
            if frozen.name not in self.dimensions:
                self.fail(node, f"unbound dimension '{frozen.name}'")
            return self.dimensions[frozen.name]
        return frozen

    def _expression_Tuple(self, node):
        return tuple(self.evaluate(item) for item in node.elts)

    def _expression_Attribute(self, node):
        owner = self.evaluate(node.value)
        if isinstance(owner, ModuleView) and node.attr in owner.values:
            return owner.values[node.attr]
        spec = self.buffer_spec(owner)
        if spec is not None and node.attr in ("shape", "dtype"):
            return spec.shape if node.attr == "shape" else spec.dtype
        self.fail(node, f"unsupported attribute '{node.attr}'")

    def _expression_Subscript(self, node):
        owner = self.evaluate(node.value)
        if self.buffer_spec(owner) is not None:
            return self.read_element(owner, node)
        if type(owner) is not tuple:
            self.fail(node, "unsupported subscript; slices and negative indexing are not "
                            "supported")
        axis = self.evaluate(node.slice)
        if type(axis) is not int or not 0 <= axis < len(owner):
            self.fail(node, "tuple/shape axes require an in-range nonnegative compile-time "
                            "integer")
        return owner[axis]

    def _operate(self, node, op, left_node, right_node, comparison):
        left, right = self.evaluate(left_node), self.evaluate(right_node)
        if type(op) not in FOLDS:
            self.fail(node, f"unsupported numeric operator: {type(op).__name__}")
        if self.is_dynamic(left) or self.is_dynamic(right):
            return self.dynamic_binary(left, right, op, node, comparison)
        kinds = (int, float, bool) if comparison else (int, float)
        if type(left) not in kinds or type(right) not in kinds:
            return self.dynamic_binary(left, right, op, node, comparison)
        try:
            result = FOLDS[type(op)](left, right)
        except (ZeroDivisionError, OverflowError) as error:
            self.fail(node, f"invalid constant expression: {error}")
        if type(result) is float and not math.isfinite(result):
            self.fail(node, "non-finite constant expression")
        return result

    def _expression_BinOp(self, node):
        return self._operate(node, node.op, node.left, node.right, False)

    def _expression_Compare(self, node):
        if len(node.ops) != 1:
            self.fail(node, "chained comparisons are not supported")
        return self._operate(node, node.ops[0], node.left, node.comparators[0], True)

    def _expression_UnaryOp(self, node):
        if not isinstance(node.op, (ast.USub, ast.UAdd)):
            self.fail(node, f"unsupported expression: {type(node).__name__}")
        value = self.evaluate(node.operand)
        if type(value) in (int, float):
            return -value if isinstance(node.op, ast.USub) else value
        return self.dynamic_unary(value, node.op, node)

    def _expression_Call(self, node):
        callee = self.evaluate(node.func)
        if isinstance(callee, Definition):
            self.fail(node, "kernel definitions are not ordinary calls; use ckl.launch")
        if not isinstance(callee, Intrinsic):
            self.fail(node, "calling arbitrary Python functions is unsupported")
        if any(isinstance(a, ast.Starred) for a in node.args) or \
                any(k.arg is None for k in node.keywords):
            self.fail(node, "argument expansion is unsupported")
        handler = getattr(self, "intrinsic_" + callee.name, None)
        if handler is None:
            self.fail(node, f"unsupported intrinsic: {callee.name}")
        return handler(node)

    def arguments(self, node: ast.Call):
        """Evaluated positional and keyword arguments of an intrinsic call."""
        values = [self.evaluate(a) for a in node.args]
        keywords = {}
        for keyword in node.keywords:
            if keyword.arg in keywords:
                self.fail(node, "duplicate keyword arguments")
            keywords[keyword.arg] = self.evaluate(keyword.value)
        return values, keywords

    def intrinsic_cdiv(self, node):
        values, keywords = self.arguments(node)
        if keywords or len(values) != 2 or not all(type(v) is int for v in values) \
                or values[0] < 0 or values[1] <= 0:
            self.fail(node, "cdiv requires a nonnegative constant extent and positive constant "
                            "divisor")
        return -(-values[0] // values[1])

    # ---- statements ------------------------------------------------------------------------
    def walk(self, body, *, top: bool = False) -> None:
        for position, statement in enumerate(body):
            method = getattr(self, "_statement_" + type(statement).__name__, None)
            if method is None:
                self.fail(statement, f"unsupported statement: {type(statement).__name__}")
            method(statement, top and position == len(body) - 1, top and position == 0)

    def _statement_Pass(self, node, last, first):
        return None

    def _statement_Return(self, node, last, first):
        if not last or node.value is not None:
            self.fail(node, "only a final bare return is supported; buffers carry outputs")

    def _statement_Expr(self, node, last, first):
        if first and isinstance(node.value, ast.Constant) and isinstance(node.value.value, str):
            return  # docstring
        if not isinstance(node.value, ast.Call) or \
                not self.launch_result_ok(self.evaluate(node.value)):
            self.fail(node, "expression statements must be kernel launches")

    def _statement_Assign(self, node, last, first):
        if len(node.targets) != 1:
            self.fail(node, "chained assignment is unsupported")
        target = node.targets[0]
        if isinstance(target, ast.Name):
            self.assign_local(target, self.evaluate(node.value), node)
        elif isinstance(target, ast.Subscript):
            self.assign_element(target, node.value, node)
        else:
            self.fail(target, "assignment requires a local name or indexed buffer element")

    def _statement_If(self, node, last, first):
        predicate = self.evaluate(node.test)
        if type(predicate) is bool:
            self.walk(node.body if predicate else node.orelse)
        else:
            self.runtime_branch(node, predicate)

    def _statement_For(self, node, last, first):
        if node.orelse or not isinstance(node.target, ast.Name) or \
                not isinstance(node.iter, ast.Call):
            self.fail(node, "for requires a simple induction variable and range without else")
        callee = self.evaluate(node.iter.func)
        if callee != Intrinsic("range") or node.iter.keywords:
            self.fail(node, "for requires range(start, stop, positive_constant_step)")
        bounds = [self.evaluate(a) for a in node.iter.args]
        if len(bounds) not in (1, 2, 3):
            self.fail(node, "range requires one to three bounds")
        start, stop, step = {1: lambda b: (0, b[0], 1), 2: lambda b: (b[0], b[1], 1),
                             3: lambda b: tuple(b)}[len(bounds)](bounds)
        if type(step) is not int or step <= 0:
            self.fail(node, "range step must be a positive compile-time integer")
        self.loop(node, node.target.id, start, stop, step)

    # ---- helpers for subclasses ------------------------------------------------------------
    def with_binding(self, name: str, value, action) -> None:
        """Run `action()` with `name` bound to `value`, restoring the previous binding."""
        previous = self.env.get(name, _ABSENT)
        self.env[name] = value
        try:
            action()
        finally:
            if previous is _ABSENT:
                self.env.pop(name, None)
            else:
                self.env[name] = previous
