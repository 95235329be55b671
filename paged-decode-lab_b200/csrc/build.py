"""Build the sm_100a shared library ``paged_decode/libpdl_b200.so`` in-tree.

    python paged-decode-lab_b200/csrc/build.py [-v] [--force]

Every ``.cu`` file here is compiled by nvcc for ``sm_100a`` only
(``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``) into
``csrc/_build/`` and linked into one shared object with the CUDA runtime
linked statically, so the library loads without a GPU and exports the
plain-C symbols declared in ``include/pdl_b200.h``.
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent / "paged_decode"
INCLUDE = CSRC.parents[1] / "include"
OBJDIR = CSRC / "_build"
TARGET = PKG / "libpdl_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required")
    return path


def _stale(obj, src, headers):
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *headers])


def build(verbose=False, force=False, ptxas_info=False):
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    OBJDIR.mkdir(exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    jobs = []
    for src in sources:
        obj = OBJDIR / (src.stem + ".o")
        if force or ptxas_info or _stale(obj, src, headers):
            jobs.append([nvcc(), *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)])
    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        for cmd, r in pool.map(run, jobs):
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
            if verbose or ptxas_info:
                sys.stdout.write(r.stdout + r.stderr)
    objs = [str(OBJDIR / (src.stem + ".o")) for src in sources]
    if force or jobs or not TARGET.exists():
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(TARGET), *objs]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return TARGET


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills (-Xptxas -v)")
    args = ap.parse_args()
    print(build(args.verbose, args.force, args.ptxas_info))
