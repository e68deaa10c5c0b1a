"""Benchmark of the structured matrix-multiply hot path: one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--op diag|gemm|upper|sandwich|toeplitz|add] [--mode 3xtf32|tf32|bf16]

Default workload (what the metric is quoted on at N = 8192, one GPU, in its
primary unit): upper-triangular x dense, C = U B with U (8192, packed upper,
entries ~ U[-1,1]) and B (8192 x 8192, ~ U[-1,1]) (seeded,
cpp1_b200.workloads), 3xTF32 (fp32 semantics), useful TFLOP/s over the
N^2 (N+1) flops that exclude U's structural zeros.  The other ops are the
remaining configured workloads (GEMM 8192^3, A S B at 4096, T B at 16384,
diag(d) B at 8192^2 in GB/s over 4N + 8N^2 bytes); `add` (general + packed
symmetric at 8192, the DSL's `+`) is reported in GB/s like the diagonal scale.

Before timing, sampled output rows of every rank's slab are checked against
the oracle's fp64 rows (normwise bound of the mode; the run fails loudly
beyond it) and the result is reported under "check".

Multi-GPU (torchrun, one process per GPU, NCCL):
  diag      weak scaling: every rank scales its own 8192 x 8192 row slab;
            no collective on the data path (the rows are independent).
  others    strong scaling: the output is split into row slabs (equal-work
            boundaries for the triangular operand; --partition tiles deals
            U B's rows out as interleaved 256-row tiles instead); each step
            is one libsmm multi-GPU call (smm_mg_*).  By default B arrives
            sharded by rows (--b-placement sharded) and is gathered in column
            blocks inside the call by the copy engines through CUDA IPC
            (--transfer ce) or by NCCL all-gathers (--transfer nccl), as
            default_transfer chooses; --b-placement root keeps B on rank 0
            and broadcasts it by NCCL.  Every rank computes its
            slab's columns block by block as they land, so the transfer
            overlaps the contraction within one product.  A S B computes
            (A_slab S) B per slab.  The line also carries the compute-only
            and transfer-only times and the fused call's roofline (MMA time
            vs the NVLink time of the bytes each rank receives).

Timing: W untimed warm-up steps, then K steps between a barrier +
synchronize on both sides, CUDA events on the launching stream, max over
ranks.  Inputs are larger than L2 (126 MB) for every workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "useful TFLOP/s (GB/s for diag) at N=8192, 1/2/4/8 B200, % of roofline vs CPU"

WORKLOADS = {
    "diag": dict(N=8192, unit="GB/s", bound="hbm", desc="C = diag(d) B, d 8192, B 8192x8192 fp32"),
    "gemm": dict(N=8192, unit="TFLOP/s", bound="tensor", desc="C = A B, 8192^3 fp32"),
    "upper": dict(N=8192, unit="TFLOP/s", bound="tensor", desc="C = U B, U 8192 upper (packed), B 8192x8192"),
    "sandwich": dict(N=4096, unit="TFLOP/s", bound="tensor", desc="C = A S B, 4096, S packed symmetric"),
    "toeplitz": dict(N=16384, unit="TFLOP/s", bound="tensor", desc="C = T B, T from a 32767 generator, B 16384^2"),
    "add": dict(N=8192, unit="GB/s", bound="hbm",
                desc="C = A + S, A 8192x8192, S packed symmetric (the DSL's General + Symmetric)"),
}
HBM_OPS = ("diag", "add")


def hbm_bytes(op: str, n: int) -> int:
    """Bytes an HBM-bound call must move (read the inputs, write C)."""
    if op == "diag":
        return 4 * n + 8 * n * n
    return 8 * n * n + 2 * n * (n + 1)  # A and C dense, S packed


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--op", choices=sorted(WORKLOADS), default="upper")
    ap.add_argument("--mode", choices=["3xtf32", "tf32", "bf16"], default="3xtf32")
    ap.add_argument("--n", "--order", dest="n", type=int, default=None,
                    help="override the problem order (--order under torchrun, whose parser claims --n)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--b-placement", choices=["sharded", "root"], default="sharded",
                    help="G > 1: B arrives sharded by rows (all-gathered inside each call) or whole on rank 0 "
                         "(broadcast inside each call)")
    ap.add_argument("--transfer", choices=["ce", "nccl"], default=None,
                    help="G > 1 with B sharded: gather B's blocks by copy engines (IPC peer copies) or by NCCL "
                         "(default: see default_transfer)")
    ap.add_argument("--partition", choices=["slabs", "tiles"], default="slabs",
                    help="U B at G > 1: one contiguous equal-work slab per rank (smm_mg_row_slabs), or interleaved "
                         "256-row tiles of U per rank (smm_mg_upper_row_tiles)")
    ap.add_argument("--roofline-s", type=float, default=1.0,
                    help="seconds of repeated calls over which the roofline kernel is timed")
    a = ap.parse_args()
    if a.steps is None:
        a.steps = {"diag": 400, "gemm": 20, "upper": 30, "sandwich": 30, "toeplitz": 6, "add": 300}[a.op]
    if a.warmup is None:
        a.warmup = {"diag": 20, "gemm": 3, "upper": 3, "sandwich": 3, "toeplitz": 3, "add": 20}[a.op]
    if a.transfer is None:
        n = a.n or WORKLOADS[a.op]["N"]
        a.transfer = default_transfer(a.op, n, a.mode, int(os.environ.get("WORLD_SIZE", "1")))
    return a


def default_transfer(op: str, n: int, mode: str, world: int) -> str:
    """How a sharded B is gathered by default.  The copy engines use no SM, so
    their transfer overlaps the contractions fully, but from 5 GPUs their
    pushes add up to only ~320 GB/s per rank (512 with one peer); NCCL's
    all-gather moves ~560 GB/s per rank there but competes with the
    contractions for SMs, so it runs as one block before them.  Measured at
    8 GPUs: U B 8192 (MMA time per rank ~ NVLink time) 1.03 ms per call with
    NCCL against 1.11 with copy engines; T B 16384 (MMA time 3x the NVLink
    time) hides the copy-engine gather (5.53 ms, compute alone 4.53).  So:
    copy engines up to 4 GPUs, and above that when the heaviest rank's MMA
    time at the TF32 (bf16) peak is at least twice the time its share of B
    takes at 770 GB/s; NCCL otherwise."""
    if world <= 4 or op in HBM_OPS:
        return "ce"
    from cpp1_b200.multigpu import row_slabs, slab_useful_flops
    b = row_slabs(n, world, triangular=(op == "upper"))
    kind = "gemm" if op in ("sandwich", "toeplitz") else op
    heaviest = max(slab_useful_flops(kind, n, b[g], b[g + 1]) for g in range(world))
    if op == "sandwich":
        heaviest *= 2  # (A_slab S) B: two products per slab
    passes = 3 if mode == "3xtf32" else 1
    peak = measured_peaks()["bf16_tflops"] * 1e12 / (1 if mode == "bf16" else 2)
    t_mma = passes * heaviest / peak
    t_link = (2 if mode == "bf16" else 4) * n * n * (world - 1) / world / 770e9
    return "ce" if t_mma >= 2 * t_link else "nccl"


# ---------------------------------------------------------------- peaks
def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profile_traffic(op: str):
    """DRAM bytes per launch of the op's dominant kernel from the committed
    ncu summary (profiles/ncu_traffic.json), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            t = json.load(f)
        return t.get(op, {}).get("dram_bytes_per_launch")
    except Exception:
        return None


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML in a thread while
    the timed region runs (reading only; no setting is changed)."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, index: int, period_s: float = 0.001):
        self.index = index
        self.period = period_s
        self.samples = []
        self.power = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.power.append(nv.nvmlDeviceGetPowerUsage(self._h) / 1000.0)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"]}
        names = [k for k, v in self.REASONS.items() if self.reasons & v]
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None,
               "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}
        if self.power:
            out["power_w_median"] = round(statistics.median(self.power), 1)
            out["power_w_max"] = round(max(self.power), 1)
        return out


# ---------------------------------------------------------------- distributed
def dist_init(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        # High-priority NCCL streams: the contraction kernels hold every SM
        # with long-running CTAs, and the block scheduler must hand SMs that
        # free up to the broadcast first, or it only creeps along in the gaps
        # (measured at 2 GPUs: exposed broadcast time -33% for GEMM 4096).
        opts = dist.ProcessGroupNCCL.Options(is_high_priority_stream=True)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local), pg_options=opts)
    elif args.impl == "ours":
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- CPU baseline
_REF_INPUTS = {}


def cpu_reference_call(op: str, n: int, sample_n: int):
    """One call of the reference's own CPU kernel (oracle/_ref) on a seeded
    problem of order sample_n; returns (kernel ms, units moved/computed).
    The reference's `+` has no CPU kernel of its own on this path (its CUDA
    backend generates it), so `add` times the oracle's C restatement."""
    import oracle as O
    from cpp1_b200 import workloads as W
    if op == "add":
        key = (op, sample_n)
        if key not in _REF_INPUTS:
            _REF_INPUTS.clear()
            _REF_INPUTS[key] = W.make_add(sample_n, seed=0)
        w = _REF_INPUTS[key]
        t0 = time.perf_counter()
        O.add_struct_f32(w["A"], w["S"], "symm")
        return (time.perf_counter() - t0) * 1e3, hbm_bytes(op, sample_n)
    if not O.ref_available():
        raise RuntimeError("oracle/_ref not built")
    key = (op, sample_n)
    if key not in _REF_INPUTS:
        _REF_INPUTS.clear()
        _REF_INPUTS[key] = {"diag": lambda: W.make_diag(sample_n, sample_n, seed=0),
                            "gemm": lambda: W.make_gemm(sample_n, sample_n, sample_n, seed=0),
                            "upper": lambda: W.make_upper(sample_n, seed=0),
                            "sandwich": lambda: W.make_sandwich(sample_n, seed=0),
                            "toeplitz": lambda: W.make_toeplitz(sample_n, seed=0)}[op]()
    w = _REF_INPUTS[key]
    if op == "diag":
        _, ms = O.ref_diag_rows(w["d"], w["B"])
        return ms, 4 * sample_n + 8 * sample_n * sample_n
    if op == "gemm":
        _, ms = O.ref_gemm(w["A"], w["B"])
        return ms, 2 * sample_n ** 3
    if op == "upper":
        _, ms = O.ref_upper_left(w["U"], w["B"])
        return ms, sample_n * sample_n * (sample_n + 1)
    if op == "sandwich":
        _, ms = O.ref_sandwich(w["A"], w["S"], w["B"])
        return ms, 4 * sample_n ** 3
    if op == "toeplitz":
        _, ms = O.ref_toeplitz_left(w["g"], w["B"])
        return ms, 2 * sample_n ** 3
    raise ValueError(op)


CPU_SAMPLE_N = {"diag": 8192, "gemm": 2048, "upper": 2048, "sandwich": 1024, "toeplitz": 2048, "add": 4096}


def cpu_model() -> str:
    """The host CPU's model name (lscpu's), for the baseline record."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"
CPU_KIND = {"add": "port"}  # every other op runs the reference's own kernel


def cpu_baseline(op: str, n: int, budget_s: float = 12.0):
    cores = int(os.environ.get("OMP_NUM_THREADS", host_threads()))
    sn = min(n, CPU_SAMPLE_N[op])
    rates = []
    t0 = time.time()
    while time.time() - t0 < budget_s or len(rates) < 2:
        ms, units = cpu_reference_call(op, n, sn)
        rates.append(units / (ms * 1e-3))
        if len(rates) >= 50:
            break
    rate = statistics.median(rates)
    scale = 1e9 if op in HBM_OPS else 1e12
    kind = CPU_KIND.get(op, "reference")
    if kind == "port":
        return {"value": rate / scale, "unit": WORKLOADS[op]["unit"], "cores": 1, "kind": "port",
                "cpu": cpu_model(), "host_threads": host_threads(),
                "sample": f"{op} at order {sn} ({len(rates)} calls, median; the oracle's scalar C restatement, "
                          "one thread)"}
    return {"value": rate / scale, "unit": WORKLOADS[op]["unit"], "cores": cores, "kind": "reference",
            "cpu": cpu_model(), "host_threads": host_threads(),
            "sample": f"{op} at order {sn} ({len(rates)} calls, median; the reference's AVX2+OpenMP kernel, "
                      f"its own chrono window, OMP threads = {cores})"}


# ---------------------------------------------------------------- our arm
def run_ours(args, rank, world, local):
    import torch
    import torch.distributed as dist
    from cpp1_b200 import _lib, ops
    from cpp1_b200 import workloads as W

    L = _lib.load()
    op = args.op
    n = args.n or WORKLOADS[op]["N"]
    stream = torch.cuda.current_stream()
    peaks = measured_peaks()
    mode = args.mode

    # ---- inputs (host, seeded) -> device
    if op == "diag":
        w = W.make_diag(n, n, seed=rank)
        h_in = [w["d"], w["B"]]
    elif op == "gemm":
        w = W.make_gemm(n, n, n, seed=0)
        h_in = [w["A"], w["B"]]
    elif op == "upper":
        w = W.make_upper(n, seed=0)
        h_in = [w["U"], w["B"]]
    elif op == "sandwich":
        w = W.make_sandwich(n, seed=0)
        h_in = [w["A"], w["S"], w["B"]]
    elif op == "toeplitz":
        w = W.make_toeplitz(n, seed=0)
        h_in = [w["g"], w["B"]]
    else:
        w = W.make_add(n, seed=rank)
        h_in = [w["A"], w["S"]]
    d_in = [torch.from_numpy(x).cuda() for x in h_in]

    from cpp1_b200 import multigpu as MG
    from cpp1_b200.multigpu import slab_useful_flops
    bounds = None if op in HBM_OPS else MG.lib_row_slabs(n, world, triangular=(op == "upper"))
    r0, r1 = (bounds[rank], bounds[rank + 1]) if bounds else (0, n)
    nrows = r1 - r0
    # U B on several GPUs: interleaved 256-row tiles of U per rank (the
    # partition whose tile schedules come out even) instead of one slab.
    tiles = (MG.lib_upper_row_tiles(n, world, rank)
             if (op == "upper" and world > 1 and args.partition == "tiles") else None)
    row_ids = MG.tile_rows_of(n, tiles) if tiles is not None else list(range(r0, r1))
    nrows = len(row_ids)
    out = torch.empty((nrows, n), dtype=torch.float32, device="cuda")
    m = _lib.MODES[mode]

    def ws_for(nbytes):
        buf = ops.workspace(nbytes, out.device)
        return (buf.data_ptr(), buf.numel()) if buf is not None else (None, 0)

    sp = stream.cuda_stream or None
    if op == "diag":
        d, B = d_in

        def step():
            _lib.check(L.smm_diag_rows(d.data_ptr(), B.data_ptr(), out.data_ptr(), n, n, sp), "diag")
        units_per_rank_call = hbm_bytes(op, n)
    elif op == "add":
        A, S = d_in

        def step():
            _lib.check(L.smm_add_struct(A.data_ptr(), S.data_ptr(), _lib.STRUCTS["symm"], out.data_ptr(), n, sp),
                       "add")
        units_per_rank_call = hbm_bytes(op, n)
    else:
        # Contractions.  One GPU: the single-GPU entry point.  G > 1: one
        # libsmm multi-GPU call per step (smm_mg_*): B reaches every rank in
        # column blocks inside the call (all-gathered from the row shares, or
        # broadcast from rank 0; the sandwich's S from rank 0) and this
        # rank's row slab is computed block by block as they land.
        # slab_local() runs the same slab with the operands already in place (the
        # single-GPU slab entry points), for the compute-only time.
        comm = MG.Communicator(rank, world) if world > 1 else None
        # B as this rank passes it to the call: its row share (sharded
        # placement: rows [rank s, rank s + s) of the resident B) or the
        # whole B (read on rank 0 only).
        root = MG.SHARDED if args.b_placement == "sharded" else 0
        if comm is not None and root == MG.SHARDED and args.transfer == "ce":
            comm.enable_copy_engines(comm.plane_bytes(n, n, mode))
        B_full = d_in[-1]
        if root == MG.SHARDED:
            s_rows = MG.share_rows(n, world)
            lo_b, hi_b = min(n, rank * s_rows), min(n, (rank + 1) * s_rows)
            B_arg = B_full[lo_b:hi_b] if hi_b > lo_b else B_full[:1]
        else:
            B_arg = B_full
        if op == "gemm":
            A, B = d_in
            A_slab = A[r0:r1]
            ws, wsb = ws_for(L.smm_gemm_workspace_size(max(nrows, 1), n, n, m))

            def slab_local():
                if nrows:
                    _lib.check(L.smm_gemm(A_slab.data_ptr(), B.data_ptr(), out.data_ptr(), nrows, n, n, m, ws, wsb,
                                          sp), "gemm")

            def step():
                comm.gemm(A_slab, B_arg, out, mode, root=root) if comm else slab_local()
            units_per_rank_call = 2 * nrows * n * n
        elif op == "upper" and tiles is not None:
            U, B = d_in

            def slab_local():  # the same tiles with B whole on every rank: nothing travels
                comm.upper_left_tiles(U, B_full, out, tiles, mode, root=MG.REPLICATED)

            def step():
                comm.upper_left_tiles(U, B_arg, out, tiles, mode, root=root)
            units_per_rank_call = sum(slab_useful_flops("upper", n, t * MG.TILE_ROWS_MG,
                                                        min(n, (t + 1) * MG.TILE_ROWS_MG)) for t in tiles)
        elif op == "upper":
            U, B = d_in
            ws, wsb = ws_for(L.smm_upper_left_workspace_size(n, n, _lib.FMT_PACKED, m))

            def slab_local():
                _lib.check(L.smm_upper_left_rows(U.data_ptr(), _lib.FMT_PACKED, B.data_ptr(), out.data_ptr(), n, n,
                                                 r0, nrows, m, ws, wsb, sp), "upper")

            def step():
                comm.upper_left(U, B_arg, out, r0, mode, root=root) if comm else slab_local()
            units_per_rank_call = slab_useful_flops("upper", n, r0, r1)
        elif op == "sandwich":
            A, S, B = d_in
            A_slab = A[r0:r1]
            ws, wsb = ws_for(L.smm_symm_sandwich_workspace_size(n, m))

            def slab_local():
                if world == 1:
                    _lib.check(L.smm_symm_sandwich(A.data_ptr(), S.data_ptr(), B.data_ptr(), out.data_ptr(), n, m,
                                                   ws, wsb, sp), "sandwich")
                elif nrows:  # (A_slab S) B, the order the multi-GPU call uses
                    ops.gemm(ops.gen_x_symm(A_slab, S, mode=mode), B, mode=mode, out=out)

            def step():
                comm.symm_sandwich(A_slab, S, B_arg, out, mode, root=root) if comm else slab_local()
            units_per_rank_call = 4 * nrows * n * n
        else:
            g, B = d_in
            ws, wsb = ws_for(L.smm_toeplitz_left_workspace_size(n, n, m))

            def slab_local():
                _lib.check(L.smm_toeplitz_left_rows(g.data_ptr(), B.data_ptr(), out.data_ptr(), n, n, r0, nrows,
                                                    m, ws, wsb, sp), "toeplitz")

            def step():
                comm.toeplitz_left(g, B_arg, out, r0, mode, root=root) if comm else slab_local()
            units_per_rank_call = 2 * nrows * n * n

    # useful FLOPs of the first contraction kernel of one call (the one the
    # roofline times alone): the slab product; for the sandwich its S B part
    if op == "sandwich":
        kernel_useful = 2 * n * n * n  # its first product, S B (one GPU)
    elif op not in HBM_OPS:
        kernel_useful = units_per_rank_call
    else:
        kernel_useful = 0

    # inputs that fit in L2 (126 MB) are flushed out of it between timed steps
    l2_resident = sum(int(t.numel()) * t.element_size() for t in d_in) <= 126 * 10 ** 6

    # correctness of this rank's slab before anything is timed
    step()
    torch.cuda.synchronize()
    ops.device_status()
    check = check_slab(op, w, row_ids, out, mode)
    check["relerr"] = max_over_ranks(check["relerr"], world)
    if not check["relerr"] <= check["tol"]:
        raise RuntimeError(f"{op}: sampled rows differ from the oracle: relerr {check['relerr']:.3e} "
                           f"> {check['tol']:.0e}")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ops.device_status()

    barrier(world)
    torch.cuda.synchronize()
    launches0 = L.smm_launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if l2_resident:
        # inputs that fit in L2: every step timed alone between its own
        # events, after a 256 MiB write that evicts the previous step's data
        flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        with ClockSampler(local) as clk:
            for a0, a1 in evs:
                flush.zero_()
                a0.record(stream)
                step()
                a1.record(stream)
            torch.cuda.synchronize()
        ms_local = sum(a0.elapsed_time(a1) for a0, a1 in evs)
        del flush
    else:
        with ClockSampler(local) as clk:
            ev0.record(stream)
            for _ in range(args.steps):
                step()
            ev1.record(stream)
            torch.cuda.synchronize()
        ms_local = ev0.elapsed_time(ev1)
    barrier(world)
    launches = L.smm_launch_count() - launches0
    ops.device_status()
    ms = max_over_ranks(ms_local, world)
    ms_per_step = ms / args.steps

    # ---- G > 1: the same slabs with the operands already in place (no
    # broadcast), so the line shows compute-only and broadcast-inclusive times
    # side by side, and the roofline of the fused call: the slower of the
    # heaviest slab's MMA work at the TF32 (bf16) peak and the bytes each
    # receiving rank must take in over NVLink at the measured 770 GB/s.
    multi = None
    if world > 1 and op not in HBM_OPS:
        barrier(world)
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for _ in range(args.steps):
            slab_local()
        c1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        ms_c = max_over_ranks(c0.elapsed_time(c1), world) / args.steps
        # B's transfer alone (a zero-row product: every rank receives B's
        # blocks, none computes)
        empty_a = torch.empty((0, n), dtype=torch.float32, device="cuda")
        barrier(world)
        torch.cuda.synchronize()
        c0.record(stream)
        for _ in range(args.steps):
            comm.gemm(empty_a, B_arg, empty_a, mode, root=root)
        c1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        ms_b = max_over_ranks(c0.elapsed_time(c1), world) / args.steps
        b_bytes = (2 if mode == "bf16" else 4) * n * n  # B's blocks travel as bf16 in bf16 mode
        s_bytes = 2 * n * (n + 1) if op == "sandwich" else 0  # packed S, fp32, from rank 0
        # bytes the busiest receiving rank takes in over NVLink per step
        link_in = (b_bytes * (world - 1) // world if root == MG.SHARDED else b_bytes) + s_bytes
        passes = {"3xtf32": 3, "tf32": 1, "bf16": 1}[mode]
        peak = peaks["bf16_tflops"] / (1 if mode == "bf16" else 2)
        heaviest = max_over_ranks(float(units_per_rank_call), world)
        t_mma = passes * heaviest / (peak * 1e12) * 1e3
        t_link = link_in / 770e9 * 1e3
        how = ((f"gathered from every rank's row share by "
                f"{'copy engines (IPC peer copies, no SM)' if comm.copy_engines_enabled() else 'NCCL all-gather'}")
               if root == MG.SHARDED else "broadcast from rank 0 (NCCL)")
        multi = {"compute_only_ms_per_step": round(ms_c, 4), "transfer_inclusive_ms_per_step": round(ms_per_step, 4),
                 "transfer_only_ms_per_step": round(ms_b, 4),
                 "b_placement": args.b_placement,
                 "b_transfer_gbs": round(b_bytes / (ms_b * 1e-3) / 1e9, 1),
                 "b_bytes_per_step": int(b_bytes),
                 "nvlink_in_bytes_per_rank": int(link_in),
                 "column_blocks": MG.lib_chunks(n, world, comm.copy_engines_enabled() and root == MG.SHARDED),
                 "transfer": "copy engines" if comm.copy_engines_enabled() else "nccl",
                 "overlap": f"B {how} in column blocks inside each call (libsmm smm_mg_*); each block's columns of "
                            "the slab are computed as soon as it lands, on internal compute streams",
                 "slab_rows": [bounds[g + 1] - bounds[g] for g in range(world)] if tiles is None else None,
                 "row_tiles_of_rank0": MG.lib_upper_row_tiles(n, world, 0) if tiles is not None else None,
                 "roofline": {"bound": "tensor" if t_mma >= t_link else "nvlink",
                              "t_mma_ms": round(t_mma, 4), "t_nvlink_ms": round(t_link, 4),
                              "target_ms": round(max(t_mma, t_link), 4),
                              "frac": round(max(t_mma, t_link) / ms_per_step, 4),
                              "basis": f"heaviest slab's {passes}-pass MMA FLOPs at {peak:.1f} TFLOP/s; the bytes "
                                       "the busiest rank receives over NVLink at the measured 770 GB/s peer "
                                       "bandwidth"}}
        comm.close()

    total_units = units_per_rank_call * world if op in HBM_OPS else (
        n * n * (n + 1) if op == "upper" else (4 * n ** 3 if op == "sandwich" else 2 * n ** 3))
    scale = 1e9 if op in HBM_OPS else 1e12
    value = total_units / (ms_per_step * 1e-3) / scale

    # ---- roofline of the dominant kernel, timed on its own on this rank
    roof = roofline(op, n, mode, step, stream, peaks, kernel_useful, ms_per_step, world, L, local, args.roofline_s)

    res = {
        "metric": METRIC, "value": round(value, 3), "unit": WORKLOADS[op]["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak" if op in HBM_OPS else "strong", "vs_baseline": None,
        "dtype": "f32" if op in HBM_OPS else {"3xtf32": "f32 (3xTF32 tensor cores)", "tf32": "tf32",
                                             "bf16": "bf16 (fp32 accumulate)"}[mode],
        "data": "synthetic (seeded numpy PCG64, cpp1_b200.workloads)",
        "config": {"workload": WORKLOADS[op]["desc"], "op": op, "N": n, "mode": mode if op not in HBM_OPS else "f32",
                   "parallelism": (f"{'interleaved row tiles' if tiles is not None else 'row-slabs'} x{world}, "
                                   f"B {args.b_placement}"
                                   + (f" ({'copy engines' if args.transfer == 'ce' else 'NCCL'})"
                                      if args.b_placement == "sharded" else " (NCCL)")
                                   if world > 1 and op not in HBM_OPS
                                   else (f"row-slabs x{world}" if world > 1 else "single GPU")),
                   "l2": ("inputs smaller than L2: a 256 MiB write flushes it before every step, each step "
                          "timed alone between its own CUDA events" if l2_resident
                          else "inputs larger than L2 (126 MB): no flush needed")},
        "roofline": roof,
        "check": check,
        "gpu_launches": int(launches),
        **({"multi_gpu": multi} if multi else {}),
        "clocks": clk.summary(),
    }
    return res, d_in, h_in


def check_slab(op, w, row_ids, out, mode):
    """Normwise relative error of sampled rows of this rank's output (global
    rows row_ids, stacked in out) against the oracle's fp64 rows (diag and
    add: bit-exact against the oracle's fp32 result, reported as 0 or inf).
    The first and last rows are always among them."""
    import oracle as O
    nr = len(row_ids)
    if nr == 0:
        return {"relerr": 0.0, "rows": 0, "tol": 0.0, "against": "no rows on this rank"}
    rng = np.random.default_rng(int(row_ids[0]) + 7)
    k = min(nr, 8)
    local = np.unique(np.concatenate([[0, nr - 1], rng.integers(0, nr, size=max(k - 2, 0))])).astype(np.int64)
    rows = np.asarray(row_ids, dtype=np.int32)[local]
    got = out[local.tolist()].cpu().numpy()
    if op == "diag":
        ref = w["d"][rows, None] * w["B"][rows]
        return {"relerr": 0.0 if np.array_equal(got, ref) else float("inf"), "rows": len(rows), "tol": 0.0,
                "against": "oracle fp32 (bit-exact)"}
    if op == "add":
        S = w["S"]
        n = w["A"].shape[1]
        ref = np.empty_like(got)
        for t, i in enumerate(rows):
            srow = np.array([S[O_packed(min(i, j), max(i, j), n)] for j in range(n)], np.float32)
            ref[t] = w["A"][i] + srow
        return {"relerr": 0.0 if np.array_equal(got, ref) else float("inf"), "rows": len(rows), "tol": 0.0,
                "against": "oracle fp32 (bit-exact)"}
    if op == "gemm":
        R = O.gemm_rows_f64(w["A"], w["B"], rows)
    elif op == "upper":
        R = O.upper_left_rows_f64(w["U"], w["B"], rows)
    elif op == "sandwich":
        R = O.sandwich_rows_f64(w["A"], w["S"], w["B"], rows)
    else:
        R = O.toeplitz_left_rows_f64(w["g"], w["B"], rows)
    tol = {"3xtf32": 1e-5, "tf32": 5e-3, "bf16": 1e-2}[mode]
    return {"relerr": float(O.relerr(got, R)), "rows": len(rows), "tol": tol, "against": "oracle fp64 rows"}


def O_packed(i, j, n):
    """Packed-upper index of (i, j), i <= j."""
    return i * n - i * (i - 1) // 2 + (j - i)


def roofline(op, n, mode, step, stream, peaks, kernel_useful, call_ms, world, L, local, seconds=1.0):
    """Roofline of the dominant kernel, timed on the launching stream with
    CUDA events.  HBM-bound ops: the kernel is the whole call.  Contractions:
    the library brackets its first contraction kernel of each call with the
    caller's events (smm_debug_time_next), so the time excludes operand
    staging and packed-operand expansion; the whole call's time is reported
    beside it.  Two runs: a burst of about 50 ms right after the timed region
    (against the burst peaks: the kernel timed alone) and `seconds` of
    back-to-back calls (against the sustained peak, under the power cap)."""
    import torch
    if world > 1:
        return {"bound": WORKLOADS[op]["bound"], "note": "reported at n_gpus = 1"}

    def run(reps):
        torch.cuda.synchronize()
        if op in HBM_OPS:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(local) as clk:
                ev0.record(stream)
                for _ in range(reps):
                    step()
                ev1.record(stream)
                torch.cuda.synchronize()
            t = ev0.elapsed_time(ev1) / reps
            return t, t, clk.summary()
        pairs = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)  # creates the events; the library records them again around its kernel
            e1.record(stream)
            pairs.append((e0, e1))
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            c0.record(stream)
            for e0, e1 in pairs:
                _lib_check(L.smm_debug_time_next(e0.cuda_event, e1.cuda_event), "smm_debug_time_next")
                step()
            c1.record(stream)
            torch.cuda.synchronize()
        return (statistics.fmean(e0.elapsed_time(e1) for e0, e1 in pairs), c0.elapsed_time(c1) / reps,
                clk.summary())

    burst_reps = int(min(200, max(3, math.ceil(50.0 / max(call_ms, 1e-3)))))
    time.sleep(1.0)  # idle first: the burst runs at the clocks of a rested GPU, not under the power cap
    sus_reps = int(min(4000, max(3, math.ceil(1000.0 * seconds / max(call_ms, 1e-3)))))
    launch_ms, whole_ms, clocks = run(burst_reps)
    s_launch_ms, s_whole_ms, s_clocks = run(sus_reps) if seconds > 0 else (None, None, None)
    if op in HBM_OPS:
        bytes_launch = hbm_bytes(op, n)
        achieved = bytes_launch / (launch_ms * 1e-3) / 1e9
        peak = peaks["hbm_gbs"]
        out = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
               "frac": round(achieved / peak, 4), "traffic": profile_traffic(op),
               "algorithmic_bytes_per_launch": bytes_launch, "launch_ms": round(launch_ms, 4), "reps": burst_reps,
               "peak_source": f"{peaks['source']} HBM copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
               "clocks": clocks}
        if s_launch_ms:
            a = bytes_launch / (s_launch_ms * 1e-3) / 1e9
            out["sustained"] = {"seconds": seconds, "reps": sus_reps, "launch_ms": round(s_launch_ms, 4),
                                "achieved": round(a, 1), "frac": round(a / peak, 4), "clocks": s_clocks}
        return out
    passes = {"3xtf32": 3, "tf32": 1, "bf16": 1}[mode]
    mma_flops = passes * kernel_useful
    achieved = mma_flops / (launch_ms * 1e-3) / 1e12
    if mode == "bf16":
        peak, peak_s = peaks["bf16_tflops"], peaks["bf16_tflops_sustained"]
        src = f"{peaks['source']} cuBLAS bf16 burst (sustained: the {peaks['source']} sustained figure)"
    else:
        peak, peak_s = peaks["bf16_tflops"] / 2, peaks["bf16_tflops_sustained"] / 2
        src = (f"TF32 = half the {peaks['source']} cuBLAS bf16 burst (sustained: half the sustained figure); "
               "datasheet TF32 dense 1100 TFLOP/s")
    out = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
           "frac": round(achieved / peak, 4), "frac_of_datasheet_tf32": (round(achieved / 1100.0, 4)
                                                                        if mode != "bf16" else None),
           "traffic": profile_traffic(op),
           "algorithmic_flops_per_launch": mma_flops, "launch_ms": round(launch_ms, 4),
           "call_ms": round(whole_ms, 4), "reps": burst_reps,
           "launch_covers": "the contraction kernel alone (CUDA events recorded by the library right before and "
                            "after its launch, on its stream); call_ms is the whole product call"
                            + (" (the sandwich: its first product, S B)" if op == "sandwich" else ""),
           "peak_source": src + f"; {passes} MMA pass(es) per useful FLOP",
           "clocks": clocks}
    if s_launch_ms:
        a = mma_flops / (s_launch_ms * 1e-3) / 1e12
        out["sustained"] = {"seconds": seconds, "reps": sus_reps, "launch_ms": round(s_launch_ms, 4),
                            "call_ms": round(s_whole_ms, 4), "achieved": round(a, 1), "peak": peak_s,
                            "frac": round(a / peak_s, 4), "clocks": s_clocks}
    return out


def _lib_check(rc, what):
    from cpp1_b200 import _lib
    _lib.check(rc, what)


# The public call each op's e2e goes through.
E2E_API = {"diag": " (smm_diag_rows_host)", "add": " via cpp1_b200.ops.add_struct",
           "gemm": " (smm_gemm_host)", "upper": " (smm_upper_left_host)",
           "toeplitz": " (smm_toeplitz_left_host)", "sandwich": " (smm_symm_sandwich_host)"}


def e2e_ours(args, h_in, n):
    """The same metric through the C ABI with HOST buffers: copy-in, compute
    and copy-out of each step inside the timed region."""
    import torch
    from cpp1_b200 import _lib, ops
    L = _lib.load()
    op = args.op
    if op == "diag":
        d = torch.from_numpy(h_in[0]).pin_memory()
        B = torch.from_numpy(h_in[1]).pin_memory()
        C = torch.empty_like(B).pin_memory()
        need = L.smm_diag_rows_host_workspace_size(n, n)
        ws = ops.workspace(need, torch.device("cuda", torch.cuda.current_device()))

        def step():
            _lib.check(L.smm_diag_rows_host(d.data_ptr(), B.data_ptr(), C.data_ptr(), n, n, ws.data_ptr(),
                                            ws.numel()), "smm_diag_rows_host")
        h2d = 4 * n + 4 * n * n
        d2h = 4 * n * n
        units = 4 * n + 8 * n * n
        steps = max(5, min(args.steps // 20, 30))
    elif op == "add":
        hp = [torch.from_numpy(x).pin_memory() for x in h_in]
        C = torch.empty((n, n), dtype=torch.float32).pin_memory()

        def step():
            A, S = [x.cuda(non_blocking=True) for x in hp]
            C.copy_(ops.add_struct(A, S, "symm"), non_blocking=True)
            torch.cuda.current_stream().synchronize()
        h2d = sum(x.nbytes for x in h_in)
        d2h = C.numel() * 4
        units = hbm_bytes(op, n)
        steps = 10
    else:
        # smm_*_host: the left operand(s) cross PCIe once, B streams through
        # in column chunks whose copies overlap the products
        hp = [torch.from_numpy(x).pin_memory() for x in h_in]
        C = torch.empty((n, n), dtype=torch.float32).pin_memory()

        def step():
            ops.host_product(op, *hp, mode=args.mode, out=C)
        h2d = sum(x.nbytes for x in h_in)
        d2h = C.numel() * 4
        units = {"gemm": 2 * n ** 3, "upper": n * n * (n + 1), "sandwich": 4 * n ** 3, "toeplitz": 2 * n ** 3}[op]
        steps = 2 if op == "toeplitz" else 5
    step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    torch.cuda.synchronize()
    dt = (time.perf_counter() - t0) / steps
    scale = 1e9 if op in HBM_OPS else 1e12
    return {"value": round(units / dt / scale, 3), "unit": WORKLOADS[op]["unit"], "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "steps": steps, "ms_per_step": round(dt * 1e3, 3),
            "api": "C ABI with pinned host buffers" + E2E_API[op]}


def e2e_dist(args, h_in, n, rank, world):
    """Host-buffer end to end at G > 1 for the contractions, through the
    library's multi-GPU calls.  Every rank copies only its share of the host
    inputs over its own PCIe link -- its row slab of the left operand (the
    whole 128 KiB generator for T B; packed S on rank 0 for the sandwich)
    and its row share of B -- then one smm_mg_* call all-gathers B's column
    blocks over NVLink and computes the slab, and the rank copies its rows of
    C back to the host.  Wall time per step, max over ranks."""
    import torch
    from cpp1_b200 import _lib
    from cpp1_b200 import multigpu as MG
    op = args.op
    mode = args.mode
    stream = torch.cuda.current_stream()
    dev = torch.device("cuda", torch.cuda.current_device())
    bounds = MG.lib_row_slabs(n, world, triangular=(op == "upper"))
    r0, r1 = bounds[rank], bounds[rank + 1]
    nrows = r1 - r0
    tiles = (MG.lib_upper_row_tiles(n, world, rank)  # interleaved rows of U B
             if (op == "upper" and args.partition == "tiles") else None)
    if tiles is not None:
        nrows = len(MG.tile_rows_of(n, tiles))
    per = MG.share_rows(n, world)
    s0, s1 = min(n, rank * per), min(n, (rank + 1) * per)

    def pin(x):
        return torch.from_numpy(np.ascontiguousarray(x)).pin_memory()

    comm = MG.Communicator(rank, world)
    if args.transfer == "ce":
        comm.enable_copy_engines(comm.plane_bytes(n, n, mode))
    Bh = h_in[-1]  # B is the last input of every contraction
    hB = pin(Bh[s0:s1])
    B_share = torch.zeros((max(s1 - s0, 1), n), dtype=torch.float32, device=dev)
    C = torch.empty((max(nrows, 1), n), dtype=torch.float32, device=dev)
    hC = torch.empty((nrows, n), dtype=torch.float32).pin_memory()
    h2d = Bh.nbytes
    if op in ("gemm", "sandwich"):
        hA = pin(h_in[0][r0:r1])
        A = torch.empty((nrows, n), dtype=torch.float32, device=dev)
        h2d += h_in[0].nbytes
    if op == "gemm":
        def load():
            A.copy_(hA, non_blocking=True)

        def comp():
            comm.gemm(A, B_share, C[:nrows], mode, root=MG.SHARDED)
    elif op == "upper" and tiles is None:
        Up = h_in[0]
        lo, hi = r0 * n - r0 * (r0 - 1) // 2, r1 * n - r1 * (r1 - 1) // 2  # packed rows [r0, r1)
        hU = pin(Up[lo:hi])
        U = torch.zeros(Up.size, dtype=torch.float32, device=dev)
        h2d += Up.nbytes

        def load():
            U[lo:hi].copy_(hU, non_blocking=True)

        def comp():
            comm.upper_left(U, B_share, C[:nrows], r0, mode, root=MG.SHARDED)
    elif op == "upper":
        Up = h_in[0]
        segs = []  # the packed rows of each of this rank's row tiles
        for t in tiles:
            a, e = t * MG.TILE_ROWS_MG, min(n, (t + 1) * MG.TILE_ROWS_MG)
            lo, hi = a * n - a * (a - 1) // 2, e * n - e * (e - 1) // 2
            segs.append((lo, hi, pin(Up[lo:hi])))
        U = torch.zeros(Up.size, dtype=torch.float32, device=dev)
        h2d += Up.nbytes

        def load():
            for lo, hi, hU in segs:
                U[lo:hi].copy_(hU, non_blocking=True)

        def comp():
            comm.upper_left_tiles(U, B_share, C[:nrows], tiles, mode, root=MG.SHARDED)
    elif op == "toeplitz":
        hg = pin(h_in[0])
        g = torch.empty(h_in[0].size, dtype=torch.float32, device=dev)
        h2d += world * h_in[0].nbytes

        def load():
            g.copy_(hg, non_blocking=True)

        def comp():
            comm.toeplitz_left(g, B_share, C[:nrows], r0, mode, root=MG.SHARDED)
    else:
        Sh = h_in[1]
        hS = pin(Sh) if rank == 0 else None
        S = torch.empty(Sh.size, dtype=torch.float32, device=dev)
        h2d += Sh.nbytes  # rank 0 alone copies packed S; the call broadcasts it

        def load():
            A.copy_(hA, non_blocking=True)
            if hS is not None:
                S.copy_(hS, non_blocking=True)

        def comp():
            comm.symm_sandwich(A, S, B_share, C[:nrows], mode, root=MG.SHARDED)

    def step():
        load()
        if s1 > s0:
            B_share[:s1 - s0].copy_(hB, non_blocking=True)
        comp()
        if nrows > 0:
            hC.copy_(C[:nrows], non_blocking=True)
        stream.synchronize()

    steps = 2 if op == "toeplitz" else 5
    step()
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    torch.cuda.synchronize()
    dt = max_over_ranks(time.perf_counter() - t0, world) / steps
    barrier(world)
    comm.close()
    units = {"gemm": 2 * n ** 3, "upper": n * n * (n + 1), "sandwich": 4 * n ** 3, "toeplitz": 2 * n ** 3}[op]
    return {"value": round(units / dt / 1e12, 3), "unit": WORKLOADS[op]["unit"], "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(n * n * 4), "steps": steps, "ms_per_step": round(dt * 1e3, 3),
            "api": "libsmm smm_mg_* (B sharded) with pinned host buffers: per-rank input shares over each GPU's "
                   "PCIe link, B's column blocks gathered over NVLink inside the call "
                   f"({'copy engines' if args.transfer == 'ce' else 'NCCL'}; whole-job bytes)"}


# ---------------------------------------------------------------- reference arm
def host_threads() -> int:
    """Host cores this process may use (its CPU affinity)."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def use_all_host_threads() -> int:
    """torchrun sets OMP_NUM_THREADS=1 per rank; the CPU kernels of the
    reference arm and the CPU baseline run alone on the host and get every
    core.  Must run before the OpenMP runtime is loaded."""
    n = host_threads()
    os.environ["OMP_NUM_THREADS"] = str(n)
    return n


def run_reference(args, rank, world):
    """The reference's own CPU implementation of the path (oracle/_ref: its
    AVX2+OpenMP kernels compiled from its sources) on this host's cores, same
    config, metric and unit.  Rank 0 only."""
    op = args.op
    n = args.n or WORKLOADS[op]["N"]
    use_all_host_threads()
    import oracle as O
    kind = CPU_KIND.get(op, "reference")
    if kind == "reference" and not O.ref_available():
        return {"impl": "reference", "unavailable": "oracle/_ref (the reference CPU kernels) was not built"}
    sn = min(n, CPU_SAMPLE_N[op])
    for _ in range(max(0, min(args.warmup, 2))):
        cpu_reference_call(op, n, sn)
    times, units = [], 0
    for _ in range(args.steps if op == "diag" else min(args.steps, 3)):
        ms, units = cpu_reference_call(op, n, sn)
        times.append(ms)
    ms = statistics.median(times)
    scale = 1e9 if op in HBM_OPS else 1e12
    value = units / (ms * 1e-3) / scale
    cores = 1 if kind == "port" else int(os.environ.get("OMP_NUM_THREADS", host_threads()))
    how = ("the oracle's scalar C restatement (the reference's `+` is generated CUDA only), one thread"
           if kind == "port" else "the reference's AVX2+OpenMP kernel, its own chrono window")
    sample = f"{op} at order {sn}" + ("" if sn == n else f" (bounded sample of the order-{n} workload)")
    return {
        "metric": METRIC, "value": round(value, 3), "unit": WORKLOADS[op]["unit"], "n_gpus": world,
        "steps": len(times), "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "weak" if op in HBM_OPS else "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded numpy PCG64, cpp1_b200.workloads)",
        "config": {"workload": WORKLOADS[op]["desc"], "op": op, "N": n, "sample_N": sn},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 3), "unit": WORKLOADS[op]["unit"], "cores": cores, "kind": kind,
                         "cpu": cpu_model(), "host_threads": host_threads(),
                         "sample": sample + "; " + how},
        "e2e": {"value": round(value, 3), "unit": WORKLOADS[op]["unit"], "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    args = parse_args()
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return 0
        print(json.dumps(run_reference(args, rank, world)), flush=True)
        return 0

    if int(os.environ.get("WORLD_SIZE", "1")) == 1:
        use_all_host_threads()  # the CPU baseline leg runs at N = 1 only
    rank, world, local = dist_init(args)
    res, d_in, h_in = run_ours(args, rank, world, local)
    n = args.n or WORKLOADS[args.op]["N"]
    if not args.no_e2e:
        # HBM-bound ops (weak scaling): every rank runs the single-GPU
        # host-buffer path on its own problem and the whole job is the
        # slowest rank's rate times the rank count.  Contractions at G > 1:
        # one distributed product over per-rank input shares (e2e_dist).
        del d_in
        if world > 1 and args.op not in HBM_OPS:
            e2e = e2e_dist(args, h_in, n, rank, world)
        else:
            e2e = e2e_ours(args, h_in, n)
        if world > 1 and args.op in HBM_OPS:
            e2e["value"] = round(max_over_ranks(-e2e["value"], world) * -1 * world, 3)
        res["e2e"] = e2e
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            res["cpu_baseline"] = cpu_baseline(args.op, n)
        except Exception as e:  # the baseline is reported, not required
            res["cpu_baseline"] = {"value": None, "unavailable": str(e)}
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
