"""libsmm's multi-GPU products on two GPUs (skipped with fewer).

Two processes, one per GPU.  B comes from rank 0 (the other rank passes
NaN-filled buffers) or sharded by rows (each rank passes only its share;
gathered by NCCL, then again by the copy engines after
smm_mg_enable_copy_engines), and S for the sandwich from rank 0, so a slab
is right only if the column blocks sent inside the call delivered every
block before the contraction that consumes it.  Each rank checks its own output slab against
an fp64 recomputation of the whole product (torch float64 on its GPU,
test-only), within the mode's bound: 3xTF32 1e-5, TF32 5e-3, bf16 1e-2.
Shapes cover equal-work triangular slabs, a ragged last block (a column
count that is not a multiple of the block width), a short last share (K not
a multiple of the world size), more blocks than internal compute streams
(SMM_MG_CHUNKS=5), and the sandwich's S broadcast.  NVLS is off (NCCL_NVLS_ENABLE=0)
and every rank issues the same calls in the same order."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

TOL = {"3xtf32": 1e-5, "tf32": 5e-3, "bf16": 1e-2}


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _relerr(C, R):
    return float(torch.linalg.vector_norm(C.double() - R) / torch.linalg.vector_norm(R))


def _worker(rank, world, port, results):
    import torch.distributed as dist

    from cpp1_b200 import multigpu as MG
    from cpp1_b200 import ops
    from cpp1_b200 import workloads as W

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    comm = None
    errs = {}
    try:
        comm = MG.Communicator(rank, world)

        def dev(x):
            return torch.from_numpy(np.ascontiguousarray(x)).cuda()

        def recv(x):  # B on the root, a NaN receive buffer elsewhere
            t = dev(x)
            if rank != 0:
                t.fill_(float("nan"))
            return t

        def barg(x, k, placement):
            """B as this rank passes it: the root's whole B (a NaN buffer on
            the other ranks), or this rank's row share."""
            if placement == "root":
                return recv(x)  # "sharded" and "ce" pass this rank's share
            s = MG.share_rows(k, world)
            lo, hi = min(k, rank * s), min(k, (rank + 1) * s)
            return dev(x[lo:hi]) if hi > lo else torch.empty((1, x.shape[1]), device="cuda")

        def plane_need():  # the largest plane set of the shapes below (5 blocks for T B)
            need = 0
            for mode in ("3xtf32", "tf32", "bf16"):
                for k, nc in ((2304, 1024), (2301, 520), (4096, 1024), (1000, 1000), (2048, 2048)):
                    need = max(need, comm.plane_bytes(k, nc, mode))
                os.environ["SMM_MG_CHUNKS"] = "5"
                need = max(need, comm.plane_bytes(4096, 2560, mode))
                del os.environ["SMM_MG_CHUNKS"]
            return need

        for placement in ("root", "sharded", "ce"):
            root = 0 if placement == "root" else MG.SHARDED
            if placement == "ce":
                comm.enable_copy_engines(plane_need())
                assert comm.copy_engines_enabled()
            for mode in ("3xtf32", "tf32", "bf16"):
                tag = f"{placement}_{mode}"
                # GEMM: A row slabs, B (K x N); K = 2301 leaves a short last share
                for M, K, N in ((2048, 2304, 1024), (640, 2301, 520)):
                    w = W.make_gemm(M, N, K, seed=31 + K)
                    b = MG.lib_row_slabs(M, world)
                    r0, r1 = b[rank], b[rank + 1]
                    C = torch.empty((r1 - r0, N), device="cuda")
                    comm.gemm(dev(w["A"][r0:r1]), barg(w["B"], K, placement), C, mode=mode, root=root)
                    torch.cuda.synchronize()
                    R = dev(w["A"][r0:r1]).double() @ dev(w["B"]).double()
                    errs[f"gemm{K}_{tag}"] = _relerr(C, R)

                # U B, packed U on every rank, equal-work slabs; ragged last column block
                for n, ncols in ((4096, 1024), (1000, 1000)):
                    w = W.make_upper(n, ncols, seed=32)
                    b = MG.lib_row_slabs(n, world, triangular=True)
                    r0, r1 = b[rank], b[rank + 1]
                    C = torch.empty((r1 - r0, ncols), device="cuda")
                    comm.upper_left(dev(w["U"]), barg(w["B"], n, placement), C, r0, mode=mode, root=root)
                    torch.cuda.synchronize()
                    Ud = ops.unpack(dev(w["U"]), "upper", n).double()
                    R = Ud[r0:r1] @ dev(w["B"]).double()
                    errs[f"upper{n}_{tag}"] = _relerr(C, R)

                # U B by interleaved row tiles (the balanced partition), ragged
                # last tile at 1000
                for n, ncols in ((4096, 1024), (1000, 1000)):
                    w = W.make_upper(n, ncols, seed=35)
                    tiles = MG.lib_upper_row_tiles(n, world, rank)
                    rows = MG.tile_rows_of(n, tiles)
                    C = torch.empty((max(len(rows), 1), ncols), device="cuda")
                    comm.upper_left_tiles(dev(w["U"]), barg(w["B"], n, placement), C, tiles, mode=mode, root=root)
                    torch.cuda.synchronize()
                    Ud = ops.unpack(dev(w["U"]), "upper", n).double()
                    R = Ud[torch.tensor(rows, device="cuda")] @ dev(w["B"]).double()
                    errs[f"uppertiles{n}_{tag}"] = _relerr(C[:len(rows)], R)

                # T B with 5 column blocks (more than the 4 compute streams)
                os.environ["SMM_MG_CHUNKS"] = "5"
                n, ncols = 4096, 2560
                w = W.make_toeplitz(n, ncols, seed=33)
                b = MG.lib_row_slabs(n, world)
                r0, r1 = b[rank], b[rank + 1]
                C = torch.empty((r1 - r0, ncols), device="cuda")
                comm.toeplitz_left(dev(w["g"]), barg(w["B"], n, placement), C, r0, mode=mode, root=root)
                torch.cuda.synchronize()
                del os.environ["SMM_MG_CHUNKS"]
                T = dev(W.toeplitz_dense(w["g"], n)).double()
                errs[f"toeplitz_{tag}"] = _relerr(C, T[r0:r1] @ dev(w["B"]).double())

                # A S B: A row slabs; S (packed) from rank 0, B from the root or sharded
                n = 2048
                w = W.make_sandwich(n, seed=34)
                b = MG.lib_row_slabs(n, world)
                r0, r1 = b[rank], b[rank + 1]
                C = torch.empty((r1 - r0, n), device="cuda")
                comm.symm_sandwich(dev(w["A"][r0:r1]), recv(w["S"]), barg(w["B"], n, placement), C, mode=mode,
                                   root=root)
                torch.cuda.synchronize()
                Sd = dev(W.unpack_symmetric(w["S"], n)).double()
                R = (dev(w["A"][r0:r1]).double() @ Sd) @ dev(w["B"]).double()
                errs[f"sandwich_{tag}"] = _relerr(C, R)
        # B whole on every rank (nothing travels)
        n, ncols = 2048, 768
        w = W.make_upper(n, ncols, seed=36)
        tiles = MG.lib_upper_row_tiles(n, world, rank)
        rows = MG.tile_rows_of(n, tiles)
        C = torch.empty((len(rows), ncols), device="cuda")
        comm.upper_left_tiles(dev(w["U"]), dev(w["B"]), C, tiles, mode="3xtf32", root=MG.REPLICATED)
        torch.cuda.synchronize()
        Ud = ops.unpack(dev(w["U"]), "upper", n).double()
        errs["uppertiles_replicated_3xtf32"] = _relerr(C, Ud[torch.tensor(rows, device="cuda")] @ dev(w["B"]).double())
        ops.device_status()
        comm.status()
        dist.barrier()
        comm.close()
        comm = None
        results[rank] = errs
    finally:
        if comm is not None:
            comm.abort()
        dist.destroy_process_group()


def test_two_gpu_products_match_fp64(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")  # no fork after CUDA or thread start-up
    with ctx.Manager() as m:
        results = m.dict()
        procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(600)
        for p in procs:
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        res = dict(results)
    assert set(res) == {0, 1}
    for rank, errs in res.items():
        for key, e in errs.items():
            mode = key.split("_")[-1]
            assert e <= TOL[mode], (rank, key, e, errs)


@pytest.mark.parametrize("mode", ["3xtf32", "tf32", "bf16"])
@pytest.mark.parametrize("tiles_env", ["auto", "pairs", "nosplit"])
def test_single_rank_interleaved_row_tiles(cuda, monkeypatch, mode, tiles_env):
    """smm_mg_upper_left_tiles on one rank: rows of U B from arbitrary
    ascending 256-row tiles of U, stacked; each output row tile takes its K
    range from its own U row (the kernels' row-tile map), in the single-CTA
    split, per-tile pair and persistent pair kernels (SMM_PAIR=1 forces pairs,
    SMM_SPLITK=0 the unsplit single-CTA tiles); B in place and replicated."""
    from cpp1_b200 import multigpu as MG
    from cpp1_b200 import ops
    from cpp1_b200 import workloads as W
    if tiles_env == "pairs":  # 256-wide pair tiles: the persistent kernel in the one-pass modes
        monkeypatch.setenv("SMM_PAIR", "1")
        monkeypatch.setenv("SMM_TILE_N", "256")
    elif tiles_env == "nosplit":
        monkeypatch.setenv("SMM_SPLITK", "0")
    comm = MG.Communicator(0, 1)
    try:
        for n, ncols, tiles in ((2048, 1024, [1, 2, 6, 7]), (2048, 520, [0, 5]), (1000, 600, [0, 3]),
                                (1000, 260, [3]), (1024, 512, [0, 1, 2, 3])):
            w = W.make_upper(n, ncols, seed=n + ncols + len(tiles))
            U = torch.from_numpy(w["U"]).cuda()
            B = torch.from_numpy(w["B"]).cuda()
            rows = MG.tile_rows_of(n, tiles)
            R = ops.unpack(U, "upper", n).double()[torch.tensor(rows, device="cuda")] @ B.double()
            for root in (0, MG.REPLICATED):
                C = torch.full((len(rows), ncols), float("nan"), device="cuda")
                comm.upper_left_tiles(U, B, C, tiles, mode=mode, root=root)
                torch.cuda.synchronize()
                assert _relerr(C, R) <= TOL[mode], (n, ncols, tiles, root, _relerr(C, R))
        ops.device_status()
    finally:
        comm.close()


def _leave_worker(rank, world, port, results):
    """Rank 1 leaves between calls (it aborts its communicator and exits);
    rank 0's next copy-engine call sees it at the host barrier, before
    enqueuing any wait on rank 1, and returns SMM_ERR_NCCL within the
    barrier limit; rank 0 then aborts its communicator."""
    import time

    import torch.distributed as dist

    from cpp1_b200 import _lib
    from cpp1_b200 import multigpu as MG
    from cpp1_b200 import workloads as W

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["SMM_MG_BARRIER_MS"] = "2000"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    comm = MG.Communicator(rank, world)
    try:
        M, K, N = 512, 1024, 512
        w = W.make_gemm(M, N, K, seed=41)
        s = MG.share_rows(K, world)
        A = torch.from_numpy(w["A"][rank * (M // 2):(rank + 1) * (M // 2)]).cuda()
        Bs = torch.from_numpy(np.ascontiguousarray(w["B"][rank * s:(rank + 1) * s])).cuda()
        C = torch.empty((M // 2, N), device="cuda")
        comm.enable_copy_engines(comm.plane_bytes(K, N, "3xtf32"))
        comm.gemm(A, Bs, C, "3xtf32", root=MG.SHARDED)  # one good call
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 1:
            comm.abort()
            comm = None
            results[rank] = "left"
            return
        time.sleep(0.5)
        t0 = time.time()
        try:
            comm.gemm(A, Bs, C, "3xtf32", root=MG.SHARDED)
            results[rank] = "no error"
        except _lib.SmmError as e:
            results[rank] = (int(e.status), round(time.time() - t0, 2), str(e))
    finally:
        if comm is not None:
            comm.abort()
        torch.cuda.synchronize()
        dist.destroy_process_group()


def test_rank_leaving_is_seen_at_the_host_barrier(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from cpp1_b200 import _lib
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        procs = [ctx.Process(target=_leave_worker, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
        for p in procs:
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        res = dict(results)
    assert res.get(1) == "left"
    code, seconds, msg = res[0]
    assert code == _lib.SMM_ERR_NCCL and "host barrier" in msg, res[0]
    assert seconds < 30, res[0]
