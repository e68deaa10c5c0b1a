"""Storage layouts of the structured matrix types: element (i, j) of an n x n
matrix as an expression over its data array (``data[...]``) or a structural
zero.  Same conventions as the reference (src/dsl/layout_functions.py):

  general            data[i*n + j]
  upper triangular   i <= j ? data[i*n - i*(i-1)/2 + (j-i)] : 0   (row-major packed)
  lower triangular   i >= j ? data[i*(i+1)/2 + j] : 0
  diagonal           i == j ? data[i] : 0
  Toeplitz           data[(j-i) + (n-1)]                           (2n-1 generator)
  symmetric          upper packed, (i, j) and (j, i) share one element
  vector             data[i] for an (n, 1) shape, data[j] for (1, n)
"""
from __future__ import annotations

from .var import ArithmeticExpression as AE
from .var import Comparison, Conditional, Var

N = Var("N")


def _packed_upper_index(r, c, n):
    # r*n - r*(r-1)/2 + (c - r): elements of the rows above r, then the offset in row r
    before = AE(AE(r, "*", n), "-", AE(AE(r, "*", AE(r, "-", 1)), "/", 2))
    return AE(before, "+", AE(c, "-", r))


def general_layout(i, j, data_arr, dim_size_n):
    return data_arr[AE(AE(i, "*", dim_size_n), "+", j)]


def upper_triangular_layout(i, j, data_arr, dim_size_n):
    return Conditional(Comparison(i, "<=", j), data_arr[_packed_upper_index(i, j, dim_size_n)], 0)


def lower_triangular_layout(i, j, data_arr, dim_size_n):
    idx = AE(AE(AE(i, "*", AE(i, "+", 1)), "/", 2), "+", j)
    return Conditional(Comparison(i, ">=", j), data_arr[idx], 0)


def diagonal_layout(i, j, data_arr, dim_size_n):
    return Conditional(Comparison(i, "==", j), data_arr[i], 0)


def toeplitz_layout(i, j, data_arr, dim_size_n):
    return data_arr[AE(AE(j, "-", i), "+", AE(dim_size_n, "-", 1))]


def symmetric_layout(i, j, data_arr, dim_size_n):
    return Conditional(Comparison(i, "<=", j), data_arr[_packed_upper_index(i, j, dim_size_n)],
                       data_arr[_packed_upper_index(j, i, dim_size_n)])


def vector_layout(i, j, data_arr, cols_dim):
    return Conditional(Comparison(cols_dim, "==", Var(1)), data_arr[i], data_arr[j])
