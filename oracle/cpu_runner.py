"""Timed CPU baseline: the oracle port run over host cores (TEST/BASELINE ONLY).

Used by ``bench.py`` for its ``cpu_baseline`` leg and its ``--impl reference``
arm.  It builds a seeded, BF16-valued sample of a BASELINE config on the host
(NumPy only -- no GPU is touched), places K/V/q/table/lengths in POSIX shared
memory, and times ``streaming_reference(split=True)`` (the reference's CPU
path, reference.py:74-88) with rows spread over a ``spawn`` process pool, one
single-threaded BLAS per worker.
"""
import math
import os
import time
from dataclasses import dataclass
from multiprocessing import get_context, shared_memory

import numpy as np

from .reference import round_bf16, streaming_reference

PAGE = 256

# (batch, Hq, Hkv, D, per-row lengths or None, capacity, partition) of each config.
CONFIGS = {
    "cfg1": (4, 8, 2, 128, None, 1024, 1024),
    "cfg2": (64, 32, 32, 64, None, 2048, 1024),
    "cfg3": (32, 16, 4, 256, None, 2064, 1024),
    "cfg4": (128, 32, 8, 128, "lognormal", 32768, 1024),
    "cfg5": (2, 64, 8, 128, None, 524288, 1024),
}


@dataclass
class Sample:
    names: dict          # shared-memory block names
    shapes: dict
    rows: int
    hq: int
    hkv: int
    dim: int
    kv_bytes: int        # algorithmic KV bytes (BF16) of one pass over the sample
    partition: int
    description: str


def _cfg4_lengths():
    rng = np.random.default_rng(20261201)
    x = rng.lognormal(mean=math.log(4096), sigma=1.0, size=128)
    lengths = np.clip(np.round(x), 1, 32768).astype(np.int32)
    lengths[::32] = 0
    return lengths


def build_sample(config, rows, max_tokens=None, seed=0):
    """Seeded sample of `rows` rows of `config` in shared memory.

    ``max_tokens`` caps each row's length (cfg5 rows of 524288 tokens are
    sampled as their first ``max_tokens`` tokens); the description says so.
    """
    batch, hq, hkv, dim, lens_kind, cap, partition = CONFIGS[config]
    if lens_kind == "lognormal":
        all_lengths = _cfg4_lengths()
        pick = np.random.default_rng(seed + 1).choice(batch, size=min(rows, batch), replace=False)
        lengths = all_lengths[np.sort(pick)]
    else:
        lengths = np.full(min(rows, batch), cap, dtype=np.int32)
    if max_tokens is not None:
        lengths = np.minimum(lengths, max_tokens).astype(np.int32)
    rows = len(lengths)
    need = [max(1, -(-int(n) // PAGE)) for n in lengths]
    width = max(need)
    pages = sum(need)
    rng = np.random.default_rng(seed)
    perm = rng.permutation(pages).astype(np.int32)
    table = np.full((rows, width), -1, dtype=np.int32)
    off = 0
    for r, n in enumerate(need):
        table[r, :n] = perm[off:off + n]
        off += n
    arrays = {
        "k": round_bf16(rng.standard_normal((pages, PAGE, hkv, dim), dtype=np.float32)),
        "v": round_bf16(rng.standard_normal((pages, PAGE, hkv, dim), dtype=np.float32)),
        "q": round_bf16(rng.standard_normal((rows, hq, dim), dtype=np.float32)),
        "table": table,
        "lengths": lengths.astype(np.int32),
    }
    names, shapes = {}, {}
    for key, arr in arrays.items():
        shm = shared_memory.SharedMemory(create=True, size=max(1, arr.nbytes))
        np.ndarray(arr.shape, arr.dtype, buffer=shm.buf)[...] = arr
        names[key] = shm.name
        shapes[key] = (arr.shape, arr.dtype.str)
        _KEEP.append(shm)
    kv_bytes = int(lengths.sum()) * hkv * dim * 2 * 2
    desc = (f"{config}: {rows} of {batch} rows, {int(lengths.sum())} tokens"
            + (f" (rows capped at {max_tokens} tokens)" if max_tokens else ""))
    return Sample(names, shapes, rows, hq, hkv, dim, kv_bytes, partition, desc)


_KEEP = []  # parent-side handles, released by release()


def release():
    while _KEEP:
        shm = _KEEP.pop()
        shm.close()
        shm.unlink()


def _attach(sample):
    handles, views = [], {}
    for key, name in sample.names.items():
        shm = shared_memory.SharedMemory(name=name)
        shape, dtype = sample.shapes[key]
        views[key] = np.ndarray(shape, np.dtype(dtype), buffer=shm.buf)
        handles.append(shm)
    return handles, views


def _work(job):
    sample, lo, hi = job
    handles, a = _attach(sample)
    try:
        t0 = time.perf_counter()
        streaming_reference(a["q"][lo:hi], a["k"], a["v"], a["table"][lo:hi],
                            a["lengths"][lo:hi], split=True, partition=sample.partition)
        return time.perf_counter() - t0
    finally:
        for h in handles:
            h.close()


def _init_worker():
    for var in ("OPENBLAS_NUM_THREADS", "OMP_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = "1"


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class Runner:
    """A spawn pool that runs one pass of the oracle over a sample per call."""

    def __init__(self, sample, workers=None):
        self.sample = sample
        self.workers = max(1, min(workers or host_cores(), sample.rows))
        self.pool = get_context("spawn").Pool(self.workers, initializer=_init_worker)
        bounds = np.linspace(0, sample.rows, self.workers + 1).astype(int)
        self.jobs = [(sample, int(a), int(b)) for a, b in zip(bounds[:-1], bounds[1:]) if b > a]

    def run_once(self):
        t0 = time.perf_counter()
        self.pool.map(_work, self.jobs, chunksize=1)
        return time.perf_counter() - t0

    def close(self):
        self.pool.close()
        self.pool.join()
