"""Matrix types of the DSL (same class names, constructor signatures and
shape rules as the reference's src/dsl/matrix.py).  The type of each operand
selects the kernel; the layout function documents the storage format the
library expects for it."""
from __future__ import annotations

from .layout_functions import (
    diagonal_layout,
    general_layout,
    lower_triangular_layout,
    symmetric_layout,
    toeplitz_layout,
    upper_triangular_layout,
    vector_layout,
)
from .layout_functions import N as SymbolicN  # noqa: F401  (re-exported like the reference)
from .var import Var


class DType:
    float = "float"
    double = "double"


class Matrix:
    def __init__(self, shape, dtype, name="unnamed"):
        self.shape = shape
        self.dtype = dtype
        self.name = name

    def __repr__(self):
        return f"Matrix(shape={self.shape}, dtype={self.dtype}, name={self.name})"

    def get_symbolic_expression(self, i, j):
        raise NotImplementedError(f"{type(self).__name__} has no symbolic element expression")

    def __add__(self, other):
        from .operations import Operation
        return Operation("add", [self, other])

    def __sub__(self, other):
        from .operations import Operation
        return Operation("sub", [self, other])

    def __matmul__(self, other):
        from .operations import Operation
        return Operation("matmul", [self, other])

    @property
    def T(self):
        from .operations import Operation
        return Operation("transpose", [self])

    def __invert__(self):
        from .operations import Operation
        return Operation("inverse", [self])


class SymbolicMatrix(Matrix):
    def __init__(self, shape, dtype, name="unnamed", layout_function=None):
        super().__init__(shape, dtype, name)
        if not layout_function:
            raise ValueError("SymbolicMatrix must be initialized with a layout_function.")
        self.layout_function = layout_function

    def __repr__(self):
        return f"SymbolicMatrix(shape={self.shape}, dtype={self.dtype}, name={self.name})"

    def get_symbolic_expression(self, i, j):
        if len(self.shape) != 2:
            raise ValueError("Matrix must be 2-dimensional.")
        rows, cols = self.shape
        data = Var(f"{self.name}_data")
        if isinstance(rows, int) and isinstance(cols, int) and rows == cols:
            return self.layout_function(i, j, data, Var(rows))
        return self.layout_function(i, j, data, cols)


def _same_dim(a, b) -> bool:
    if isinstance(a, Var) and isinstance(b, Var):
        return a.name == b.name
    if isinstance(a, Var) or isinstance(b, Var):
        return True  # one symbolic, one concrete: checked when the sizes are bound
    return a == b


def _require_square(kind, shape):
    if not (len(shape) == 2 and _same_dim(shape[0], shape[1])):
        raise ValueError(f"{kind} must be square")


class GeneralMatrix(SymbolicMatrix):
    def __init__(self, shape, name="unnamed", dtype=DType.float):
        super().__init__(shape, dtype, name, general_layout)


class DiagonalMatrix(SymbolicMatrix):
    def __init__(self, shape, name="unnamed", dtype=DType.float):
        _require_square("DiagonalMatrix", shape)
        super().__init__(shape, dtype, name, diagonal_layout)


class UpperTriangularMatrix(SymbolicMatrix):
    def __init__(self, shape, name="unnamed", dtype=DType.float):
        _require_square("UpperTriangularMatrix", shape)
        super().__init__(shape, dtype, name, upper_triangular_layout)


class LowerTriangularMatrix(SymbolicMatrix):
    def __init__(self, shape, name="unnamed", dtype=DType.float):
        _require_square("LowerTriangularMatrix", shape)
        super().__init__(shape, dtype, name, lower_triangular_layout)


class ToeplitzMatrix(SymbolicMatrix):
    def __init__(self, shape, name="unnamed", dtype=DType.float):
        _require_square("ToeplitzMatrix", shape)
        super().__init__(shape, dtype, name, toeplitz_layout)


class SymmetricMatrix(SymbolicMatrix):
    def __init__(self, shape, name="unnamed", dtype=DType.float):
        _require_square("SymmetricMatrix", shape)
        super().__init__(shape, dtype, name, symmetric_layout)


class Vector(SymbolicMatrix):
    def __init__(self, shape, name="unnamed", dtype=DType.float):
        if not (len(shape) == 2 and (shape[1] == 1 or shape[0] == 1)):
            raise ValueError("Vector must have a shape of (N, 1) or (1, N)")
        super().__init__(shape, dtype, name, vector_layout)
