"""Host logic of the multi-GPU row-slab partition, on CPU: slab boundaries,
equal-work splits for the triangular operand, and the broadcast + slab
compute + gather sequence run by two gloo ranks (the slab products computed
by the oracle, since there is no GPU here)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cpp1_b200 import multigpu as MG


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_slabs_cover_rows(world):
    for n in (1, 100, 1024, 8192, 16384):
        for tri in (False, True):
            b = MG.row_slabs(n, world, tri)
            assert b[0] == 0 and b[-1] == n and len(b) == world + 1
            assert all(b[i] <= b[i + 1] for i in range(world))
            assert all(x % 256 == 0 or x == n for x in b[1:-1])


def test_triangular_slabs_balance_work():
    n, world = 8192, 8
    b = MG.row_slabs(n, world, triangular=True)
    work = [MG.slab_useful_flops("upper", n, b[i], b[i + 1]) for i in range(world)]
    total = MG.slab_useful_flops("upper", n, 0, n)
    assert sum(work) == total == n * n * (n + 1)
    # the slowest rank sets the time: within 15% of an equal share (the first
    # 256-row tile alone is half a share, so tile granularity costs ~15%; the
    # pair tiles it avoids leaving half empty cost more)
    assert max(work) <= 1.15 * total / world
    uniform = MG.row_slabs(n, world, triangular=False)
    uw = [MG.slab_useful_flops("upper", n, uniform[i], uniform[i + 1]) for i in range(world)]
    assert max(uw) > 1.7 * total / world  # uniform rows would be 1.9x slower


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results):
    import oracle as O
    from cpp1_b200 import workloads as W
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n = 384
        w = W.make_upper(n, 96, seed=3)
        U = w["U"]
        # only rank 0 starts with B; the others hold garbage until the broadcast
        B = torch.from_numpy(w["B"]) if rank == 0 else torch.full((n, 96), float("nan"))

        def compute(r0, r1):
            Bn = B.numpy()
            full = O.upper_left_f32(U, Bn)  # stands in for the GPU slab kernel
            return torch.from_numpy(np.ascontiguousarray(full[r0:r1]))

        bounds = MG.row_slabs(n, world, triangular=True)
        shapes = [bounds[i + 1] - bounds[i] for i in range(world)]
        C = MG.distributed_product(compute, B, rank, world, n, triangular=True,
                                   gather=lambda s: MG.gather_rows(s, world, shapes, 96))
        if rank == 0:
            results["ok"] = bool(np.array_equal(C.numpy(), O.upper_left_f32(U, w["B"])))
            results["bounds"] = bounds
    finally:
        dist.destroy_process_group()


def test_two_rank_broadcast_slab_gather_gloo():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")  # no fork after CUDA or thread start-up
    with ctx.Manager() as m:
        results = m.dict()
        procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        assert results["ok"], results


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_uniform_shares_cover_rows(world):
    for n in (0, 1, 5, 4096, 4099):
        b = MG.uniform_shares(n, world)
        assert b[0] == 0 and b[-1] == n and len(b) == world + 1
        assert all(b[i] <= b[i + 1] for i in range(world))
        assert max(b[i + 1] - b[i] for i in range(world)) <= -(-n // world) if n else True


def _sandwich_worker(rank, world, port, results):
    import oracle as O
    from cpp1_b200 import workloads as W
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n = 97  # not a multiple of the rank count: the last share is short
        w = W.make_sandwich(n, seed=4)
        S = W.unpack_symmetric(w["S"], n).astype(np.float64)
        A, B = w["A"].astype(np.float64), w["B"].astype(np.float64)

        def x_rows(r0, r1):  # stands in for the GPU slab kernel X[r0:r1] = S[r0:r1] B
            return torch.from_numpy((S[r0:r1] @ B).astype(np.float32))

        def c_rows(X, r0, r1):
            return torch.from_numpy((A[r0:r1] @ X.numpy().astype(np.float64)).astype(np.float32))

        C = MG.distributed_sandwich(x_rows, c_rows, rank, world, n)
        b = MG.uniform_shares(n, world)
        Cs = MG.allgather_rows(C, world, n)
        if rank == 0:
            ref = (A @ (S @ B).astype(np.float32).astype(np.float64)).astype(np.float32)
            results["ok"] = bool(np.allclose(Cs.numpy(), ref, rtol=1e-5, atol=1e-4))
            results["rows"] = b
    finally:
        dist.destroy_process_group()


def test_two_rank_sandwich_slabs_gloo():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")  # no fork after CUDA or thread start-up
    with ctx.Manager() as m:
        results = m.dict()
        procs = [ctx.Process(target=_sandwich_worker, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        assert results["ok"], results


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_library_slabs_match_host_partition(world):
    """libsmm's smm_mg_row_slabs and the host restatement agree."""
    for n in (0, 1, 100, 1024, 4096, 8192, 16384, 1000):
        for tri in (False, True):
            assert MG.lib_row_slabs(n, world, tri) == MG.row_slabs(n, world, tri), (n, world, tri)


@pytest.mark.parametrize("ncols,world", [(8192, 8), (16384, 8), (4096, 2), (1000, 2), (300, 4), (8192, 1)])
def test_library_column_blocks(ncols, world):
    cb = MG.lib_chunks(ncols, world)
    assert cb[0] == 0 and cb[-1] == ncols
    assert all(a < b for a, b in zip(cb, cb[1:]))
    assert all(x % 256 == 0 for x in cb[:-1])  # blocks start on whole output tiles
    want = 1 if world == 1 else 4 if world == 2 else 2 if world <= 4 else 1
    assert len(cb) - 1 == min(want, -(-ncols // 256))


@pytest.mark.parametrize("ncols,world", [(8192, 8), (16384, 8), (4096, 2), (1000, 4), (300, 4), (8192, 1)])
def test_library_gather_column_blocks(ncols, world):
    """The copy-engine gather's blocks (smm_mg_gather_chunks): the same
    256-column tiling, 4 blocks at every world size above 1."""
    cb = MG.lib_chunks(ncols, world, copy_engines=True)
    assert cb[0] == 0 and cb[-1] == ncols
    assert all(a < b for a, b in zip(cb, cb[1:]))
    assert all(x % 256 == 0 for x in cb[:-1])
    want = 1 if world == 1 else 4
    assert len(cb) - 1 == min(want, -(-ncols // 256))


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_library_share_rows(world):
    """smm_mg_share_rows agrees with the host rule (ceil(K / world)), and the
    shares [r s, min(K, (r + 1) s)) cover B's rows exactly once."""
    for k in (0, 1, 7, 1000, 2301, 8192, 16384):
        s = MG.lib_share_rows(k, world)
        assert s == MG.share_rows(k, world) == -(-k // world)
        rows = [i for r in range(world) for i in range(min(k, r * s), min(k, (r + 1) * s))]
        assert rows == list(range(k))


def test_packed_order():
    for n in (1, 2, 1000, 8192):
        assert MG.packed_order(n * (n + 1) // 2) == n
    with pytest.raises(ValueError):
        MG.packed_order(4)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_interleaved_row_tiles(world):
    """smm_mg_upper_row_tiles agrees with the host restatement; the ranks'
    tiles cover U's 256-row tiles exactly once, ascending; the work per rank
    is within one tile's work of the others; 32 tiles on 8 ranks give rank r
    the tiles {r, 15 - r, 16 + r, 31 - r}."""
    for n in (1, 255, 256, 1000, 4096, 8192, 8193):
        nt = -(-n // 256)
        own = [MG.lib_upper_row_tiles(n, world, r) for r in range(world)]
        assert own == [MG.upper_row_tiles(n, world, r) for r in range(world)]
        assert sorted(t for o in own for t in o) == list(range(nt))
        assert all(o == sorted(o) for o in own)
        work = [sum(n - i for i in MG.tile_rows_of(n, o)) for o in own]
        assert max(work) - min(work) <= n * 256
    assert [MG.lib_upper_row_tiles(8192, 8, r) for r in range(8)] == \
        [sorted([r, 15 - r, 16 + r, 31 - r]) for r in range(8)]
