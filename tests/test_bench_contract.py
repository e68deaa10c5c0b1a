"""bench.py's static contract on CPU: every workload has the tables the timed
and end-to-end paths index, and the reference arm runs to its JSON line."""
import importlib.util
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_every_workload_has_its_tables():
    b = load_bench()
    ops = set(b.WORKLOADS)
    assert ops == set(b.E2E_API)
    assert "diag" in ops and set(b.HBM_OPS) <= ops
    for op, w in b.WORKLOADS.items():
        assert {"unit", "desc", "bound", "N"} <= set(w), op


def test_reference_arm_prints_one_json_line():
    """`bench.py --impl reference` times the reference's CPU kernels (or the
    oracle port) on a bounded sample; at a small order it finishes in seconds."""
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0",
                        "--order", "256"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    if "unavailable" not in line:
        assert line["value"] > 0 and line["e2e"]["h2d_bytes_per_step"] == 0


def test_default_transfer_follows_the_compute_to_link_balance():
    """Copy engines up to 4 GPUs; above, copy engines only where the MMA time
    hides their slower gather (T B 16384), NCCL where the transfer dominates
    (U B and GEMM at 8192)."""
    b = load_bench()
    for op in ("upper", "gemm", "toeplitz", "sandwich"):
        n = b.WORKLOADS[op]["N"]
        assert [b.default_transfer(op, n, "3xtf32", w) for w in (1, 2, 4)] == ["ce"] * 3
    assert b.default_transfer("toeplitz", 16384, "3xtf32", 8) == "ce"
    assert b.default_transfer("upper", 8192, "3xtf32", 8) == "nccl"
    assert b.default_transfer("gemm", 8192, "3xtf32", 8) == "nccl"
    assert b.default_transfer("diag", 8192, "3xtf32", 8) == "ce"
