"""CPU checks of the benchmark's output contract.

The reference arm (``bench.py --impl reference``) times the CPU reference
path and needs no GPU, so its JSON line is checked here key by key; under
torchrun only rank 0 runs it and the other ranks exit 0 without work.  The
GPU arm's line carries the same keys plus ``roofline``, ``clocks`` and
``gpu_launches`` (exercised by the GPU runs, not here).
"""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def run_bench(*args, env=None):
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True,
                          text=True, timeout=600, env={**os.environ, **(env or {})}, cwd=ROOT)
    lines = [line for line in proc.stdout.splitlines() if line.startswith("{")]
    return proc.returncode, lines, proc.stderr


def test_reference_arm_prints_one_contract_line():
    rc, lines, err = run_bench("--impl", "reference", "--steps", "1", "--warmup", "1")
    assert rc == 0, err[-2000:]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["config"]["workload"] == "cfg4"
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == line["value"]
    assert cpu["blas"] and cpu["blas_threads_per_worker"] == 1 and cpu["workers"] == cpu["cores"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"],
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only():
    rc, lines, err = run_bench("--impl", "reference", "--steps", "1", "--warmup", "1",
                               env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert rc == 0 and lines == [], err[-2000:]


def test_exchange_micro_needs_several_ranks():
    rc, lines, _ = run_bench("--exchange-micro")
    assert rc == 0 and json.loads(lines[0]) == {
        "exchange_micro": "needs torchrun with 2 or more ranks"}


def test_default_workload_and_modes():
    """N=1 runs config 4 alone; N>1 splits one batch (strong scaling): by rows
    by default, by context for config 5."""
    sys.path.insert(0, str(ROOT))
    import bench
    args = bench.parse_args([])
    assert args.config == "cfg4" and args.mode == "auto"
    assert bench.resolve_mode(args, 1) == "single"
    assert bench.resolve_mode(args, 8) == "batch"
    assert bench.resolve_mode(bench.parse_args(["--config", "cfg5"]), 4) == "context"
    assert bench.resolve_mode(bench.parse_args(["--mode", "head"]), 2) == "head"
    assert bench.resolve_mode(bench.parse_args(["--mode", "replica"]), 2) == "replica"


def test_committed_traffic_is_scaled_to_the_launch_kv_bytes():
    """The per-launch DRAM bytes come from the ncu summaries under profiles/
    (``traffic[config][kernel]: BYTES of KV_BYTES``) and are scaled by the KV
    bytes of the launch the bench measured."""
    sys.path.insert(0, str(ROOT))
    import importlib
    bench = importlib.import_module("bench")
    traffic, src = bench.committed_traffic("cfg4", "mma", 3074609152)
    assert traffic == 3119899360 and "profiles/" in src and "scaled" not in src
    half, src = bench.committed_traffic("cfg4", "mma", 3074609152 // 2)
    assert abs(half - 3119899360 // 2) <= 1 and "scaled" in src
    assert bench.committed_traffic("cfg1", "mma", 1) == (None, None)
