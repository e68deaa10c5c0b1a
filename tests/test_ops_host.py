"""Argument checking of ops.host_product on CPU: bad calls are rejected before
any device work, with the error a Python caller expects."""
import pytest
import torch

from cpp1_b200 import ops


def host(*shape, dtype=torch.float32):
    return torch.zeros(shape, dtype=dtype)


def test_unknown_product_is_rejected():
    with pytest.raises(ValueError, match="unknown host product"):
        ops.host_product("trsm", host(4, 4), host(4, 4))


@pytest.mark.parametrize("op,n", [("gemm", 1), ("upper", 3), ("sandwich", 2)])
def test_wrong_number_of_inputs_is_rejected(op, n):
    with pytest.raises(ValueError, match="takes"):
        ops.host_product(op, *[host(4, 4)] * n)


def test_unknown_mode_is_rejected():
    with pytest.raises(ValueError, match="unknown mode"):
        ops.host_product("gemm", host(4, 4), host(4, 4), mode="fp8")


def test_gemm_inner_dimensions_must_match():
    with pytest.raises(ValueError, match="inner dimensions"):
        ops.host_product("gemm", host(4, 5), host(6, 4))


def test_inputs_must_be_float32():
    with pytest.raises(TypeError, match="float32"):
        ops.host_product("gemm", host(4, 4, dtype=torch.float64), host(4, 4))


@pytest.mark.parametrize("op,left", [("upper", 9), ("symm", 11), ("toeplitz", 6)])
def test_structured_left_operand_size_is_checked(op, left):
    # order 4: packed triangles hold 10 elements, a Toeplitz generator 7
    with pytest.raises(ValueError, match="elements, expected"):
        ops.host_product(op, host(left), host(4, 8))


def test_sandwich_needs_a_square_left_factor():
    with pytest.raises(ValueError, match="square"):
        ops.host_product("sandwich", host(4, 5), host(10), host(4, 4))
