"""Expression-graph nodes of the DSL (same public surface as the reference's
src/dsl/operations.py): an Operation is itself a Matrix whose shape is
inferred from its operands; unnamed operations get the auto names
``intermediate_<operator>_<k>`` the graph runner uses for intermediates."""
from __future__ import annotations

from collections import defaultdict

from .matrix import Matrix
from .var import InverseExperession, MatMulExpression, Var

opcounters = defaultdict(int)


def _dims_conflict(a, b) -> bool:
    return isinstance(a, int) and isinstance(b, int) and a != b


class Operation(Matrix):
    def __init__(self, operator, operands, name=None):
        self.operator = operator
        self.operands = operands
        if name is None:
            key = operator.lower()
            name = f"intermediate_{key}_{opcounters[key]}"
            opcounters[key] += 1
        super().__init__(name=name, shape=self.infer_shape(), dtype=self.infer_dtype())

    def _expect_arity(self, k):
        if len(self.operands) != k:
            word = "one operand" if k == 1 else "exactly two operands"
            raise ValueError(f"{self.operator} operation requires {word}.")

    def infer_shape(self):
        op = self.operator
        if op in ("add", "sub"):
            self._expect_arity(2)
            a, b = self.operands
            if a.shape != b.shape:
                raise ValueError(f"Shapes must match for {op} operation: {a.shape} vs {b.shape}")
            return a.shape
        if op == "matmul":
            self._expect_arity(2)
            (m, k1), (k2, n) = self.operands[0].shape, self.operands[1].shape
            if _dims_conflict(k1, k2):
                raise ValueError(f"Inner dimensions for matrix multiplication must match: {k1} vs {k2}.")
            return (m, n)
        if op == "transpose":
            self._expect_arity(1)
            r, c = self.operands[0].shape
            return (c, r)
        if op == "inverse":
            self._expect_arity(1)
            r, c = self.operands[0].shape
            if _dims_conflict(r, c) or (isinstance(r, Var) and isinstance(c, Var) and r.name != c.name):
                raise ValueError("Matrix must be square to be invertible.")
            return (r, c)
        raise NotImplementedError(f"Shape inference for {op} is not implemented.")

    def infer_dtype(self):
        return "double" if any(getattr(o, "dtype", None) == "double" for o in self.operands) else "float"

    def get_symbolic_expression(self, i, j):
        op = self.operator
        if op in ("add", "sub"):
            from .var import ArithmeticExpression
            sym = "+" if op == "add" else "-"
            return ArithmeticExpression(self.operands[0].get_symbolic_expression(i, j), sym,
                                        self.operands[1].get_symbolic_expression(i, j))
        if op == "matmul":
            k = Var("k")
            return MatMulExpression(self.operands[0].get_symbolic_expression(i, k),
                                    self.operands[1].get_symbolic_expression(k, j), k, self.operands[0].shape[1])
        if op == "transpose":
            return self.operands[0].get_symbolic_expression(j, i)
        if op == "inverse":
            return InverseExperession(self.operands[0], i, j)
        raise ValueError(f"Unsupported operation: {op} for symbolic expression generation.")

    def __repr__(self):
        names = [o.name if isinstance(o, Matrix) else str(o) for o in self.operands]
        return f"Operation(operator='{self.operator}', operands={names}, name='{self.name}')"
