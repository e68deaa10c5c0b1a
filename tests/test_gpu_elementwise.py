"""Elementwise sums and storage converters on the GPU, through the C ABI,
against the oracle: bit-exact (one fp32 add per element, or a copy).

Edge cases: order 1, orders that are not multiples of the 4-float vector or
of the 32 x 128 tile, rows that are not 16-byte aligned (scalar path), a
1-D sum starting at an unaligned offset, rectangular Toeplitz matrices, and
the reference builder's own generator as a golden vector.  At the full
8192 order the checks are size-independent identities against PyTorch's
IEEE fp32 add on the same device."""
import numpy as np
import pytest
import torch

import oracle as O
from cpp1_b200 import _lib, ops

pytestmark = pytest.mark.gpu

FMTS = ["upper", "lower", "symm", "diag", "toeplitz"]
ORDERS = [1, 7, 33, 128, 255, 1000, 2049]


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def rand(shape, seed):
    return np.random.default_rng(seed).uniform(-1, 1, shape).astype(np.float32)


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("n", ORDERS)
def test_add_struct_bitexact(cuda, fmt, n):
    A = rand((n, n), n)
    S = rand(O.struct_numel(fmt, n), n + 1)
    got = ops.add_struct(dev(A), dev(S), fmt).cpu().numpy()
    assert np.array_equal(got, O.add_struct_f32(A, S, fmt))


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("n", ORDERS)
def test_unpack_bitexact(cuda, fmt, n):
    S = rand(O.struct_numel(fmt, n), 2 * n)
    got = ops.unpack(dev(S), fmt, n).cpu().numpy()
    assert np.array_equal(got, O.unpack_f32(S, fmt, n))


@pytest.mark.parametrize("fmt", ["upper", "lower", "symm"])
@pytest.mark.parametrize("n", ORDERS)
def test_pack_bitexact(cuda, fmt, n):
    D = rand((n, n), 3 * n)
    got = ops.pack(dev(D), fmt).cpu().numpy()
    assert np.array_equal(got, O.pack_f32(D, fmt))


@pytest.mark.parametrize("count", [1, 3, 4, 1001, 4096, 1 << 20])
def test_add_bitexact(cuda, count):
    A, B = rand(count, count), rand(count, count + 1)
    assert np.array_equal(ops.add(dev(A), dev(B)).cpu().numpy(), O.add_f32(A, B))


def test_add_unaligned_offsets(cuda):
    # operands starting 4 bytes past a 16-byte boundary take the scalar path
    A, B = rand(5001, 1), rand(5001, 2)
    a, b = dev(A), dev(B)
    c = torch.empty(5001, device="cuda")
    L = _lib.load()
    n = 4999
    _lib.check(L.smm_add(a.data_ptr() + 4, b.data_ptr() + 4, c.data_ptr() + 4, n, None), "smm_add")
    torch.cuda.synchronize()
    assert np.array_equal(c.cpu().numpy()[1:1 + n], A[1:1 + n] + B[1:1 + n])


@pytest.mark.parametrize("shape", [(1, 1), (1, 9), (9, 1), (37, 53), (53, 37), (1024, 2048)])
def test_toeplitz_compact_bitexact(cuda, shape):
    T = rand(shape, shape[0] * 7 + shape[1])
    assert np.array_equal(ops.toeplitz_compact(dev(T)).cpu().numpy(), O.toeplitz_compact_f32(T))


def test_toeplitz_compact_matches_reference_builder_golden(cuda, golden):
    got = ops.toeplitz_compact(dev(golden["tcompact_T"])).cpu().numpy()
    assert np.array_equal(got, golden["tcompact_g"])


def test_pack_unpack_round_trip_full_size(cuda):
    n = 8192
    g = torch.Generator(device="cuda").manual_seed(0)
    S = torch.rand(n * (n + 1) // 2, device="cuda", generator=g) * 2 - 1
    for fmt in ("upper", "lower", "symm"):
        assert torch.equal(ops.pack(ops.unpack(S, fmt, n), fmt), S)


def test_add_struct_full_size_matches_torch_add(cuda):
    n = 8192
    g = torch.Generator(device="cuda").manual_seed(1)
    A = torch.rand(n, n, device="cuda", generator=g) * 2 - 1
    S = torch.rand(n * (n + 1) // 2, device="cuda", generator=g) * 2 - 1
    D = ops.unpack(S, "symm", n)
    assert torch.equal(D, D.T)
    assert torch.equal(ops.add_struct(A, S, "symm"), A + D)
    gen = torch.rand(2 * n - 1, device="cuda", generator=g)
    assert torch.equal(ops.add_struct(A, gen, "toeplitz"), A + ops.unpack(gen, "toeplitz", n))
