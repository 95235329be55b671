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
    """Build the sm_100a library once if this checkout has none yet (nvcc
    cross-compiles without a GPU); an existing build is left as it is."""
    library = ROOT / "paged-decode-lab_b200" / "paged_decode" / "libpdl_b200.so"
    if not library.exists():
        csrc = ROOT / "paged-decode-lab_b200" / "csrc"
        sys.path.insert(0, str(csrc))
        import importlib
        importlib.import_module("build").build()
