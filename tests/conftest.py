"""Shared pytest setup: the ``gpu`` marker and import paths.

CPU tests (``-m "not gpu"``) cover the oracle against golden vectors, the
host-side logic and the C-ABI symbol table; ``-m gpu`` tests are the parity
tests proper and call the CUDA path through the C-ABI.
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT, ROOT / "paged-decode-lab_b200", ROOT / "tests" / "golden"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_sessionstart(session):
    """Bring the sm_100a library up to date before any test loads it: the
    build recompiles only sources newer than their objects (nvcc
    cross-compiles without a GPU), so a library older than csrc/ is never
    tested as it is."""
    csrc = ROOT / "paged-decode-lab_b200" / "csrc"
    sys.path.insert(0, str(csrc))
    import importlib
    importlib.import_module("build").build()


def pytest_terminal_summary(terminalreporter):
    """Worst observed error / bound ratios of the parity checks in this run."""
    gpu_util = sys.modules.get("gpu_util")
    if gpu_util is None or not gpu_util.WORST["lse_checked"] and not gpu_util.WORST["output_ratio"]:
        return
    w = gpu_util.WORST
    terminalreporter.write_line(
        "parity worst: output max abs err %.3e (%.3f of 2^-7); LSE error/bound %.3f over %d "
        "values, largest relative LSE error where |ref| >= 1e-3: %.3e; %d values needed the "
        "FP32 score allowance" % (w["output_abs_err"], w["output_ratio"], w["lse_ratio"],
                                  w["lse_checked"], w["lse_rel_err_strict"],
                                  w["lse_needing_score_allowance"]))
