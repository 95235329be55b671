"""Seeded, BF16-exact input cases shared by the golden generator and the tests.

Inputs are drawn as float32 N(0,1) with NumPy's PCG64, rounded to BF16 by
round-to-nearest-even on the bits, and kept as uint16 patterns.  The GPU gets
those patterns as ``torch.bfloat16``; the oracle gets the float32 values they
denote.  Fixtures store only seeds and outputs; each case is rebuilt here and
its input checksum is compared against the one recorded by the generator.
"""
from dataclasses import dataclass
import hashlib

import numpy as np

PAGE = 256


def _bf16_bits(x):
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _f32(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


@dataclass
class Case:
    q_bits: np.ndarray      # [B, Hq, D] uint16
    k_bits: np.ndarray      # [P, 256, Hkv, D] uint16
    v_bits: np.ndarray      # [P, 256, Hkv, D] uint16
    table: np.ndarray       # [B, W] int32
    lengths: np.ndarray     # [B] int32
    capacity: int           # max_context_len the case was built for

    @property
    def q(self):
        return _f32(self.q_bits)

    @property
    def k(self):
        return _f32(self.k_bits)

    @property
    def v(self):
        return _f32(self.v_bits)

    def arrays(self):
        """(q, k, v, table, lengths) as the oracle takes them."""
        return self.q, self.k, self.v, self.table, self.lengths

    def checksum(self):
        h = hashlib.sha256()
        for a in (self.q_bits, self.k_bits, self.v_bits, self.table, self.lengths):
            h.update(np.ascontiguousarray(a).tobytes())
        return h.hexdigest()


def make_case(lengths, hq=4, hkv=1, dim=64, seed=9, capacity=None, pool_factor=1.0):
    """Random pages, a permuted block table and N(0,1) BF16 q/K/V.

    Mirrors the shape of the reference's ``make_case`` helper
    (tests/test_reference.py:8-17): ``ceil(capacity/256)`` table columns per
    row, physical pages drawn as a permutation of the pool.
    """
    rng = np.random.default_rng(seed)
    lengths = np.asarray(lengths, dtype=np.int32)
    capacity = max(int(lengths.max(initial=0)), 1) if capacity is None else capacity
    width = -(-capacity // PAGE)
    need = len(lengths) * width
    pages = max(need, int(round(need * pool_factor)))
    table = rng.permutation(pages)[:need].reshape(len(lengths), width).astype(np.int32)
    k = _bf16_bits(rng.standard_normal((pages, PAGE, hkv, dim), dtype=np.float32))
    v = _bf16_bits(rng.standard_normal((pages, PAGE, hkv, dim), dtype=np.float32))
    q = _bf16_bits(rng.standard_normal((len(lengths), hq, dim), dtype=np.float32))
    return Case(q, k, v, table, lengths, capacity)


def poison_tails(case):
    """Set -1 past each row's live pages and NaN in dead slots of the last live page.

    Follows the reference GPU tests (tests/test_gpu.py:55-63): padding table
    entries are -1 and the unused slots of a partly filled page hold NaN; a
    correct kernel never reads either.
    """
    nan = np.uint16(0x7FC0)
    for b, n in enumerate(case.lengths.tolist()):
        live = -(-n // PAGE)
        case.table[b, live:] = -1
        if n % PAGE:
            page = case.table[b, n // PAGE]
            case.k_bits[page, n % PAGE:] = nan
            case.v_bits[page, n % PAGE:] = nan
    return case


def config1(seed=20261201):
    """B=4, Hq=8, Hkv=2, D=128, pool 64 pages, len U[0,1024].

    The table is a seeded permutation of the 64-page pool; one length is
    forced to 0 and one to exactly 1024.
    """
    rng = np.random.default_rng(seed)
    batch, hq, hkv, dim, pool, capacity = 4, 8, 2, 128, 64, 1024
    width = capacity // PAGE
    table = rng.permutation(pool)[:batch * width].reshape(batch, width).astype(np.int32)
    lengths = rng.integers(0, capacity, size=batch, endpoint=True).astype(np.int32)
    lengths[0], lengths[1] = 0, capacity
    k = _bf16_bits(rng.standard_normal((pool, PAGE, hkv, dim), dtype=np.float32))
    v = _bf16_bits(rng.standard_normal((pool, PAGE, hkv, dim), dtype=np.float32))
    q = _bf16_bits(rng.standard_normal((batch, hq, dim), dtype=np.float32))
    return Case(q, k, v, table, lengths, capacity)


# The reference's oracle sweep (tests/test_reference.py:20-28).
SWEEP_LENGTHS = (0, 1, 255, 256, 257, 1023, 1024, 1025, 2051)
SWEEP_GEOMETRIES = ((64, 4, 1), (128, 4, 2), (64, 2, 2), (256, 8, 2))


def sweep_case(length, dim, hq, hkv):
    return make_case([length, 1], hq, hkv, dim)
