"""Symbolic scalar expressions of the DSL (same public names as the
reference's src/dsl/var.py: Var, ArithmeticExpression, Comparison,
Conditional, Summation, MatMulExpression, InverseExperession).

Expressions are plain trees.  ``evaluate(expr, env)`` computes one on
concrete integers (used to check storage layouts), where ``env`` maps Var
names to values and ``"<name>_data"`` arrays to sequences.
"""
from __future__ import annotations

from typing import Any, Mapping


class Expression:
    """Base of every symbolic node."""

    def _op(self, op, other):
        return ArithmeticExpression(self, op, other)

    def __add__(self, other):
        return self._op("+", other)

    def __radd__(self, other):
        return ArithmeticExpression(other, "+", self)

    def __sub__(self, other):
        return self._op("-", other)

    def __rsub__(self, other):
        return ArithmeticExpression(other, "-", self)

    def __mul__(self, other):
        return self._op("*", other)

    def __rmul__(self, other):
        return ArithmeticExpression(other, "*", self)

    def __truediv__(self, other):
        return self._op("/", other)

    def __neg__(self):
        return ArithmeticExpression(self, "-", None)

    def __getitem__(self, index):
        return ArithmeticExpression(self, "subscript", index)

    def __lt__(self, other):
        return Comparison(self, "<", other)

    def __le__(self, other):
        return Comparison(self, "<=", other)

    def __gt__(self, other):
        return Comparison(self, ">", other)

    def __ge__(self, other):
        return Comparison(self, ">=", other)


class Var(Expression):
    """A named symbol (a dimension such as ``n``, a loop index, or a data
    array ``<matrix>_data``).  As in the reference, ``==`` builds a
    Comparison node; hashing is by name, so Vars of one name collapse in sets."""

    def __init__(self, name):
        self.name = name

    def __repr__(self):
        return str(self.name)

    def __hash__(self):
        return hash(self.name)

    def __eq__(self, other):  # symbolic equality, as in the reference DSL
        return Comparison(self, "==", other)

    def __ne__(self, other):
        return Comparison(self, "!=", other)


class ArithmeticExpression(Expression):
    def __init__(self, left, op, right):
        self.left = left
        self.op = op
        self.right = right

    def __repr__(self):
        if self.op == "subscript":
            return f"{self.left}[{self.right}]"
        if self.right is None:
            return f"{self.op}{self.left}"
        return f"({self.left} {self.op} {self.right})"

    def __eq__(self, other):
        return Comparison(self, "==", other)

    __hash__ = object.__hash__


class Comparison(Expression):
    def __init__(self, left, op, right):
        self.left = left
        self.op = op
        self.right = right

    def __repr__(self):
        return f"({self.left} {self.op} {self.right})"

    def __eq__(self, other):
        return (isinstance(other, Comparison) and self.op == other.op and _same(self.left, other.left)
                and _same(self.right, other.right))

    def __hash__(self):
        return hash((repr(self.left), self.op, repr(self.right)))


class Conditional(Expression):
    def __init__(self, condition, true_value, false_value):
        self.condition = condition
        self.true_value = true_value
        self.false_value = false_value

    def __repr__(self):
        return f"({self.condition} ? {self.true_value} : {self.false_value})"


class Summation(Expression):
    def __init__(self, expression, loop_var, start, end):
        self.expression = expression
        self.loop_var = loop_var
        self.start = start
        self.end = end

    def __repr__(self):
        return f"sum({self.loop_var}={self.start}..{self.end}, {self.expression})"


class MatMulExpression(Expression):
    def __init__(self, left_matrix_expr, right_matrix_expr, k_var, inner_dim_size_var):
        self.left_matrix_expr = left_matrix_expr
        self.right_matrix_expr = right_matrix_expr
        self.k_var = k_var
        self.inner_dim_size_var = inner_dim_size_var

    def __repr__(self):
        return f"MatMulExpression(left={self.left_matrix_expr}, right={self.right_matrix_expr})"


class InverseExperession(Expression):
    """Element (i, j) of the inverse of a matrix (name kept as the reference spells it)."""

    def __init__(self, operand_matrix, i, j):
        self.operand_matrix = operand_matrix
        self.i = i
        self.j = j

    def __repr__(self):
        return f"Inverse({self.operand_matrix.name})[{self.i},{self.j}]"


InverseExpression = InverseExperession


def _same(a, b) -> bool:
    if isinstance(a, Var) and isinstance(b, Var):
        return a.name == b.name
    if isinstance(a, Expression) or isinstance(b, Expression):
        return repr(a) == repr(b)
    return a == b


def evaluate(expr: Any, env: Mapping[str, Any]):
    """Evaluate an index/value expression on concrete values.  Integer
    division is floor division (the generated C divides integers)."""
    if isinstance(expr, (int, float)):
        return expr
    if isinstance(expr, Var):
        return env[expr.name]
    if isinstance(expr, Conditional):
        return evaluate(expr.true_value if evaluate(expr.condition, env) else expr.false_value, env)
    if isinstance(expr, Comparison):
        a, b = evaluate(expr.left, env), evaluate(expr.right, env)
        return {"<": a < b, "<=": a <= b, ">": a > b, ">=": a >= b, "==": a == b, "!=": a != b}[expr.op]
    if isinstance(expr, ArithmeticExpression):
        if expr.op == "subscript":
            return evaluate(expr.left, env)[evaluate(expr.right, env)]
        a = evaluate(expr.left, env)
        if expr.right is None:
            return -a
        b = evaluate(expr.right, env)
        if expr.op == "+":
            return a + b
        if expr.op == "-":
            return a - b
        if expr.op == "*":
            return a * b
        if expr.op == "/":
            return a // b if isinstance(a, int) and isinstance(b, int) else a / b
    raise TypeError(f"cannot evaluate {expr!r}")
