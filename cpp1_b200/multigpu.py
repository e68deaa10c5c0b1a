"""Row-slab partition of a structured product across the GPUs of one node,
and the host side of libsmm's multi-GPU products (``Communicator``).

One process per GPU (torchrun), torch.distributed over NCCL for the
plumbing.  For C = X B with X one of the library's left operands (dense A,
packed U, Toeplitz generator, packed S):

* every rank owns output rows [r0, r1) and computes them with the slab entry
  point of libsmm (``smm_*_rows``; a row offset of A for the dense GEMM);
* the right operand B is shared: rank 0 holds it and broadcasts it (one
  NCCL broadcast per product); X itself is small (generator, packed
  triangle) or row-sliced, so it is replicated or sliced locally;
* for the triangular operand row i costs N - i, so slab boundaries are
  equal-work: boundary g of G sits at N (1 - sqrt(1 - g/G)), rounded to the
  256-row pair-tile height;
* the diagonal scale shards with no collective at all (rows independent).

``Communicator`` wraps libsmm's own NCCL communicator (``smm_mg_*``): each
product call brings B to every rank in column blocks on a high-priority
stream -- broadcast from a root rank, or all-gathered from row shares when B
is sharded -- and computes this rank's slab block by block as they land, so
the transfer overlaps the tensor-core work inside one call.

No kernel reads another GPU's memory; remote data reaches local HBM through
NCCL before any kernel touches it.

The collective steps take a ``compute`` callable so the host logic runs the
same way under the gloo backend on CPU (tests) and NCCL on GPUs.
"""
from __future__ import annotations

import math
from typing import Callable, List, Optional, Sequence, Tuple

TILE_ROWS = 256  # a CTA-pair tile's height


def _tile_work(n: int, triangular: bool, align: int) -> List[int]:
    tiles = (n + align - 1) // align
    if not triangular:
        return [min(align, n - t * align) for t in range(tiles)]
    # rows [a, b) of U cost sum (n - i)
    return [sum_range_cost(n, t * align, min(n, (t + 1) * align)) for t in range(tiles)]


def sum_range_cost(n: int, a: int, b: int) -> int:
    return (b - a) * n - (b * (b - 1) - a * (a - 1)) // 2


def row_slabs(n: int, world: int, triangular: bool = False, align: int = TILE_ROWS) -> List[int]:
    """Slab boundaries b[0]=0 <= ... <= b[world]=n on tile (align-row)
    granularity, minimising the largest slab's work: uniform rows for dense
    operands, rows of cost (n - i) for the upper-triangular one (the
    continuous optimum is N (1 - sqrt(1 - g/G)); the tile-granular optimum is
    found by binary search on the largest slab).  Slabs may be empty when n
    has fewer tiles than ranks."""
    if world < 1:
        raise ValueError("world must be >= 1")
    if n <= 0:
        return [0] * (world + 1)
    w = _tile_work(n, triangular, align)

    def groups_needed(cap: int) -> int:
        count, acc = 1, 0
        for x in w:
            if acc + x > cap:
                count, acc = count + 1, x
            else:
                acc += x
        return count

    lo, hi = max(w), sum(w)
    while lo < hi:
        mid = (lo + hi) // 2
        if groups_needed(mid) <= world:
            hi = mid
        else:
            lo = mid + 1
    cuts, acc = [0], 0
    for t, x in enumerate(w):
        if acc + x > lo:
            cuts.append(t * align)
            acc = x
        else:
            acc += x
    cuts.append(n)
    while len(cuts) < world + 1:  # fewer non-empty slabs than ranks
        cuts.insert(len(cuts) - 1, n)
    return cuts


def slab_of(n: int, rank: int, world: int, triangular: bool = False) -> Tuple[int, int]:
    b = row_slabs(n, world, triangular)
    return b[rank], b[rank + 1]


def slab_useful_flops(op: str, n: int, r0: int, r1: int, ncols: Optional[int] = None) -> int:
    """Useful FLOPs of output rows [r0, r1) (structural zeros excluded)."""
    ncols = n if ncols is None else ncols
    rows = r1 - r0
    if op in ("gemm", "toeplitz", "symm"):
        return 2 * rows * n * ncols
    if op == "upper":
        # row i of U has n - i nonzeros: 2 * ncols * sum_{i=r0}^{r1-1} (n - i)
        s = rows * n - (r1 * (r1 - 1) - r0 * (r0 - 1)) // 2
        return 2 * ncols * s
    raise ValueError(op)


def distributed_product(compute: Callable[[int, int], object], B, rank: int, world: int, n: int,
                        triangular: bool = False, broadcast: Callable = None, gather: Callable = None):
    """Run one row-slab product on this rank.

    compute(r0, r1) -> C slab (rows [r0, r1) of the product), called after B
    holds rank 0's data.  ``broadcast(tensor, src)`` and ``gather(slab)``
    default to torch.distributed; ``gather`` returning None skips assembly."""
    import torch.distributed as dist
    bcast = broadcast or (lambda t, src: dist.broadcast(t, src=src))
    if world > 1:
        bcast(B, 0)
    r0, r1 = slab_of(n, rank, world, triangular)
    C = compute(r0, r1)
    if gather is not None:
        return gather(C)
    return C


def gather_rows(slab, world: int, shapes: Sequence[int], ncols: int):
    """all_gather of uneven row slabs (pads to the largest slab, then trims)."""
    import torch
    import torch.distributed as dist
    rmax = max(shapes)
    pad = torch.zeros((rmax, ncols), dtype=slab.dtype, device=slab.device)
    pad[: slab.shape[0]] = slab
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad)
    return torch.cat([p[:r] for p, r in zip(parts, shapes)], dim=0)


# ---------------------------------------------------------------- shares and row all-gather
def uniform_shares(n: int, world: int) -> List[int]:
    """Boundaries of `world` equal row shares of n rows (the last ones may be
    short or empty): share g is rows [b[g], b[g+1]), each at most ceil(n/world)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    per = -(-n // world) if n > 0 else 0
    return [min(n, g * per) for g in range(world)] + [n]


def allgather_rows(share, world: int, n: int, out=None):
    """Assemble an n-row matrix from every rank's row share (uniform_shares
    boundaries) over torch.distributed: each rank contributes its share padded
    to ceil(n/world) rows; the result is the first n rows.  `out`, if given,
    must hold world * ceil(n/world) rows (it is filled in place and its first
    n rows are returned).  NCCL gathers straight into `out`; other backends
    (gloo, in the CPU tests) gather a list and copy."""
    import torch
    import torch.distributed as dist
    per = -(-n // world) if n > 0 else 0
    cols = share.shape[1] if share.dim() == 2 else 1
    if share.shape[0] < per:
        pad = torch.zeros((per, cols), dtype=share.dtype, device=share.device)
        pad[: share.shape[0]] = share.view(-1, cols)
        share = pad
    if out is None:
        out = torch.empty((world * per, cols), dtype=share.dtype, device=share.device)
    if dist.get_backend() == "nccl":
        dist.all_gather_into_tensor(out, share.contiguous())
    else:
        parts = list(out.view(world, per, cols).unbind(0))
        gathered = [torch.empty_like(share) for _ in range(world)]
        dist.all_gather(gathered, share.contiguous())
        for p, g in zip(parts, gathered):
            p.copy_(g)
    return out[:n]


def distributed_sandwich(x_rows: Callable[[int, int], object], c_rows: Callable[[object, int, int], object],
                         rank: int, world: int, n: int, x_out=None):
    """C = A S B by row slabs without redundant work: this rank computes rows
    [r0, r1) of X = S B (x_rows(r0, r1)), the X row shares are all-gathered
    (every rank then holds all of X), and this rank computes its rows of
    C = A X (c_rows(X, r0, r1)).  Shares are uniform_shares(n, world); the
    caller has already made S and B available on every rank.  Returns this
    rank's C rows."""
    b = uniform_shares(n, world)
    r0, r1 = b[rank], b[rank + 1]
    X = x_rows(r0, r1)
    X_full = allgather_rows(X, world, n, out=x_out) if world > 1 else X
    return c_rows(X_full, r0, r1)


# ---------------------------------------------------------------- libsmm multi-GPU communicator
class Communicator:
    """This rank's libsmm multi-GPU communicator (NCCL, one process per GPU),
    on the current CUDA device.  Collective: every rank constructs it.  The
    NCCL unique id is made by rank 0 and handed to the others over
    torch.distributed (any initialised backend), or passed in as ``uid``."""

    def __init__(self, rank: int, world: int, uid: Optional[bytes] = None):
        import ctypes
        from . import _lib
        self._lib = _lib
        L = _lib.load()
        self.rank, self.world = rank, world
        idbuf = ctypes.create_string_buffer(128)
        if world > 1:
            if uid is None:
                import torch.distributed as dist
                obj = [None]
                if rank == 0:
                    _lib.check(L.smm_mg_unique_id(idbuf), "smm_mg_unique_id")
                    obj = [bytes(idbuf.raw)]
                dist.broadcast_object_list(obj, src=0)
                uid = obj[0]
            idbuf = ctypes.create_string_buffer(bytes(uid), 128)
        h = ctypes.c_void_p()
        _lib.check(L.smm_mg_comm_init(ctypes.byref(h), rank, world, idbuf), "smm_mg_comm_init")
        self.h = h

    def close(self) -> None:
        if self.h is not None:
            self._lib.check(self._lib.load().smm_mg_comm_destroy(self.h), "smm_mg_comm_destroy")
            self.h = None

    def abort(self) -> None:
        if self.h is not None:
            self._lib.load().smm_mg_comm_abort(self.h)
            self.h = None

    def status(self) -> None:
        self._lib.check(self._lib.load().smm_mg_comm_status(self.h), "smm_mg_comm_status")

    # ---- helpers
    @staticmethod
    def _stream(stream):
        import torch
        s = stream if stream is not None else torch.cuda.current_stream()
        return s.cuda_stream or None

    def _ws(self, nbytes, device):
        from . import ops
        buf = ops.workspace(nbytes, device)
        return (buf.data_ptr(), buf.numel()) if buf is not None else (None, 0)

    # ---- copy-engine gather of a sharded B (collective)
    def plane_bytes(self, k: int, ncols: int, mode: str = "3xtf32") -> int:
        """Plane-buffer bytes a sharded call with a K x ncols B gathers into."""
        return int(self._lib.load().smm_mg_plane_bytes(self.h, k, ncols, self._lib.MODES[mode]))

    def enable_copy_engines(self, plane_bytes: int) -> None:
        """Collective: every rank allocates `plane_bytes` (the same on every
        rank) and maps every peer's buffer; from then on sharded calls whose
        planes fit are gathered by copy engines instead of NCCL."""
        self._lib.check(self._lib.load().smm_mg_enable_copy_engines(self.h, int(plane_bytes)),
                        "smm_mg_enable_copy_engines")

    def copy_engines_enabled(self) -> bool:
        return bool(self._lib.load().smm_mg_copy_engines_enabled(self.h))

    # ---- products (every rank calls them with the same shapes, mode and root)
    # root: the rank holding all of B (broadcast), or SHARDED: B is this
    # rank's share, rows [rank * s, rank * s + s) of B with s = share_rows(K,
    # world) (all-gathered inside the call).
    @staticmethod
    def _root(root) -> int:
        if root in (SHARDED, "sharded"):
            return SHARDED
        if root in (REPLICATED, "replicated"):
            return REPLICATED
        return int(root)

    def gemm(self, A_slab, B, C_slab, mode: str = "3xtf32", root=0, stream=None):
        """C_slab = A_slab @ B.  Broadcast: B is read on the root only (the
        other ranks pass a tensor of the same shape, whose content is not
        used).  Sharded: B is this rank's share of B's rows."""
        L = self._lib.load()
        m = self._lib.MODES[mode]
        nrows, K = A_slab.shape
        N = B.shape[1]
        ws, wsb = self._ws(L.smm_mg_gemm_workspace_size(self.h, nrows, N, K, m), B.device)
        self._lib.check(L.smm_mg_gemm(self.h, A_slab.data_ptr(), B.data_ptr(), C_slab.data_ptr(), nrows, N, K, m,
                                      self._root(root), ws, wsb, self._stream(stream)), "smm_mg_gemm")
        return C_slab

    def upper_left(self, U, B, C_slab, row0: int, mode: str = "3xtf32", root=0, stream=None):
        """C_slab = U[row0:row0+nrows] @ B, U packed upper on every rank (its
        order N from the packed length)."""
        L = self._lib.load()
        m = self._lib.MODES[mode]
        N = packed_order(U.numel())
        ncols = B.shape[1]
        nrows = C_slab.shape[0] if C_slab is not None else 0
        ws, wsb = self._ws(L.smm_mg_upper_left_workspace_size(self.h, N, ncols, nrows, m), B.device)
        cp = C_slab.data_ptr() if nrows else None
        self._lib.check(L.smm_mg_upper_left(self.h, U.data_ptr(), B.data_ptr(), cp, N, ncols, row0, nrows, m,
                                            self._root(root), ws, wsb, self._stream(stream)), "smm_mg_upper_left")
        return C_slab

    def upper_left_tiles(self, U, B, C_rows, tiles, mode: str = "3xtf32", root=0, stream=None):
        """C_rows = the rows of U @ B in `tiles` (ascending indices of 256-row
        tiles of U; upper_row_tiles gives the balanced interleaved share),
        stacked in that order; U packed upper on every rank."""
        import ctypes
        L = self._lib.load()
        m = self._lib.MODES[mode]
        N = packed_order(U.numel())
        ncols = B.shape[1]
        t = (ctypes.c_int * max(1, len(tiles)))(*tiles)
        ws, wsb = self._ws(L.smm_mg_upper_left_tiles_workspace_size(self.h, N, ncols, len(tiles), m), B.device)
        cp = C_rows.data_ptr() if len(tiles) else None
        self._lib.check(L.smm_mg_upper_left_tiles(self.h, U.data_ptr(), B.data_ptr(), cp, N, ncols, t, len(tiles), m,
                                                  self._root(root), ws, wsb, self._stream(stream)),
                        "smm_mg_upper_left_tiles")
        return C_rows

    def toeplitz_left(self, g, B, C_slab, row0: int, mode: str = "3xtf32", root=0, stream=None):
        """C_slab = T[row0:row0+nrows] @ B, T of generator g (2N - 1 values)
        on every rank."""
        L = self._lib.load()
        m = self._lib.MODES[mode]
        N = (g.numel() + 1) // 2
        ncols = B.shape[1]
        nrows = C_slab.shape[0] if C_slab is not None else 0
        ws, wsb = self._ws(L.smm_mg_toeplitz_left_workspace_size(self.h, N, ncols, m), B.device)
        cp = C_slab.data_ptr() if nrows else None
        self._lib.check(L.smm_mg_toeplitz_left(self.h, g.data_ptr(), B.data_ptr(), cp, N, ncols, row0, nrows, m,
                                               self._root(root), ws, wsb, self._stream(stream)),
                        "smm_mg_toeplitz_left")
        return C_slab

    def symm_sandwich(self, A_slab, S, B, C_slab, mode: str = "3xtf32", root=0, stream=None):
        """C_slab = (A_slab @ S) @ B with packed S (from the root; rank 0 when
        B is sharded) and B from the root or sharded."""
        L = self._lib.load()
        m = self._lib.MODES[mode]
        N = packed_order(S.numel())
        nrows = A_slab.shape[0] if A_slab is not None else 0
        ws, wsb = self._ws(L.smm_mg_symm_sandwich_workspace_size(self.h, N, nrows, m), B.device)
        ap = A_slab.data_ptr() if nrows else None
        cp = C_slab.data_ptr() if nrows else None
        self._lib.check(L.smm_mg_symm_sandwich(self.h, ap, S.data_ptr(), B.data_ptr(), cp, N, nrows, m,
                                               self._root(root), ws, wsb, self._stream(stream)),
                        "smm_mg_symm_sandwich")
        return C_slab


SHARDED = -1  # root value of a call whose B is sharded by rows (SMM_MG_SHARDED)
REPLICATED = -2  # root value of a call whose B is whole on every rank (SMM_MG_REPLICATED)
TILE_ROWS_MG = 256  # rows of a tile of U in the interleaved partition


def upper_row_tiles(n: int, world: int, rank: int) -> List[int]:
    """This rank's row tiles of U in the interleaved partition (restatement
    of libsmm's smm_mg_upper_row_tiles): tiles in decreasing order of work
    (row i costs n - i) each to the rank with the least work so far, ties to
    the lower rank."""
    nt = -(-n // TILE_ROWS_MG)
    load = [0] * world
    mine = []
    for t in range(nt):
        a, e = t * TILE_ROWS_MG, min(n, (t + 1) * TILE_ROWS_MG)
        cost = (e - a) * n - (e * (e - 1) - a * (a - 1)) // 2
        g = min(range(world), key=lambda h: (load[h], h))
        load[g] += cost
        if g == rank:
            mine.append(t)
    return mine


def tile_rows_of(n: int, tiles: List[int]) -> List[int]:
    """Rows of U (and of C) that a list of row tiles covers, in stacked order."""
    return [i for t in tiles for i in range(t * TILE_ROWS_MG, min(n, (t + 1) * TILE_ROWS_MG))]


def lib_upper_row_tiles(n: int, world: int, rank: int) -> List[int]:
    """The library's interleaved row tiles (smm_mg_upper_row_tiles)."""
    import ctypes
    from . import _lib
    cap = max(1, -(-n // TILE_ROWS_MG))
    b = (ctypes.c_int * cap)()
    k = ctypes.c_int(0)
    _lib.check(_lib.load().smm_mg_upper_row_tiles(n, world, rank, b, cap, ctypes.byref(k)), "smm_mg_upper_row_tiles")
    return list(b)[:k.value]


def packed_order(length: int) -> int:
    """Order N of a packed triangle of N (N + 1) / 2 values."""
    n = int((math.isqrt(8 * length + 1) - 1) // 2)
    if n * (n + 1) // 2 != length:
        raise ValueError(f"{length} values are not a packed triangle")
    return n


def share_rows(k: int, world: int) -> int:
    """Rows in each rank's share of a K-row B sharded over `world` ranks
    (ceil(K / world), libsmm's smm_mg_share_rows)."""
    if world < 1 or k < 0:
        raise ValueError("bad share arguments")
    return -(-k // world)


def lib_share_rows(k: int, world: int) -> int:
    from . import _lib
    r = _lib.load().smm_mg_share_rows(k, world)
    if r < 0:
        _lib.check(r, "smm_mg_share_rows")
    return r


def lib_row_slabs(n: int, world: int, triangular: bool = False) -> List[int]:
    """The library's own slab boundaries (smm_mg_row_slabs)."""
    import ctypes
    from . import _lib
    b = (ctypes.c_int * (world + 1))()
    _lib.check(_lib.load().smm_mg_row_slabs(n, world, 1 if triangular else 0, b), "smm_mg_row_slabs")
    return list(b)


def lib_chunks(ncols: int, world: int, copy_engines: bool = False) -> List[int]:
    """The column-block boundaries the library's transfers of B use: NCCL
    broadcasts and all-gathers (smm_mg_chunks), or the copy-engine gather
    (smm_mg_gather_chunks)."""
    import ctypes
    from . import _lib
    b = (ctypes.c_int * 17)()
    fn = "smm_mg_gather_chunks" if copy_engines else "smm_mg_chunks"
    nch = getattr(_lib.load(), fn)(ncols, world, b)
    if nch < 1:
        _lib.check(nch if nch else 1, fn)
    return list(b)[: nch + 1]
