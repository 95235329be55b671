"""Restatement of the reference's geometry and static split-KV plan (oracle only).

TEST INFRASTRUCTURE: see ``oracle/__init__.py`` for who may import this.
The product computes the same plan natively (``pdl_splitkv_plan`` in the
C-ABI library); tests compare the two with each other and with golden values
that the reference's own ``make_splitkv_plan`` produced.
"""
from dataclasses import dataclass
import math
import struct


def _f32(x):
    """Round a Python float to float32 (reference splitkv_plan.py:11-12)."""
    return struct.unpack("f", struct.pack("f", x))[0]


@dataclass(frozen=True)
class OraclePlan:
    splits: int
    tile_tokens: int
    tokens_per_split: int
    table_capacity_tokens: int
    lse_lanes: int
    sm_count: int
    policy: str


def spec_geometry(max_batch, num_heads, num_kv_heads, head_dim, max_context_len, page_size=256):
    """partitions, table_width, split_workspace_bytes (reference spec.py:32-42)."""
    partitions = -(-max_context_len // 1024)
    table_width = -(-max_context_len // page_size)
    workspace = max_batch * num_heads * partitions * (head_dim + 2) * 4
    return partitions, table_width, workspace


def make_splitkv_plan(max_batch, num_heads, num_kv_heads, head_dim, max_context_len,
                      sm_count, num_splits=0):
    """Static split count and partition size (reference splitkv_plan.py:26-56).

    tile = 256/128/64 tokens for D = 64/128/256; capacity = table_width*256;
    blocks = ceil(capacity/tile).  With num_splits = 0 the count is chosen by
    wave efficiency on 2*sm_count virtual SMs: 1 if batch*Hkv >= 0.8*virtual
    (float32 arithmetic), else the first eligible n whose efficiency reaches
    0.85 of the best.  tokens_per_split = ceil(blocks/splits)*tile.
    """
    if type(sm_count) is not int or sm_count < 1:
        raise ValueError("positive SM count required")
    if type(num_splits) is not int or not 0 <= num_splits <= 128:
        raise ValueError("num_splits must be an integer in [0,128]")
    if num_heads // num_kv_heads > 16:
        raise ValueError("matched split-KV requires at most 16 query heads per KV head")
    tile = {64: 256, 128: 128}.get(head_dim, 64)
    capacity = -(-max_context_len // 256) * 256
    blocks = -(-capacity // tile)
    splits = num_splits
    if splits == 0:
        work = max_batch * num_kv_heads
        virtual = 2 * sm_count
        if work >= _f32(_f32(0.8) * virtual):
            splits = 1
        else:
            best, scores = 0.0, []
            for n in range(1, min(128, virtual, blocks) + 1):
                if n > 1 and -(-blocks // n) == -(-blocks // (n - 1)):
                    continue
                waves = _f32(_f32(work * n) / virtual)
                eff = _f32(waves / math.ceil(waves))
                scores.append((n, eff))
                best = max(best, eff)
            splits = next(n for n, eff in scores if eff >= 0.85 * best)
    padded = 1 << (splits - 1).bit_length()
    merge_rows = 4 if head_dim % 128 == 0 else 8
    return OraclePlan(splits, tile, -(-blocks // splits) * tile, capacity,
                      min(padded, 128 // merge_rows), sm_count,
                      "explicit" if num_splits else "pinned_geometry")
