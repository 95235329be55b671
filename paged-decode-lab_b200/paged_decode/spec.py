"""Host-side geometry contract; no CUDA calls or device synchronisation.

Same names, fields, properties and error messages as the reference's
``src/paged_decode/spec.py`` so engine code written against it keeps working.
"""
from dataclasses import dataclass

BACKENDS = ("flash_attn", "triton_base", "triton_splitk", "triton_tc", "triton_tc_splitk")
PAGE_SIZE = 256
PARTITION_SIZE = 1024
TILE_SIZE = 64


@dataclass(frozen=True)
class DecodeSpec:
    """Capacity of one decode geometry (reference spec.py:11-42).

    ``partitions = ceil(max_context_len / 1024)``,
    ``table_width = ceil(max_context_len / 256)`` and
    ``split_workspace_bytes = max_batch * num_heads * partitions * (head_dim + 2) * 4``;
    the same numbers come from ``pdl_spec_geometry`` in the C ABI.
    """
    max_batch: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    max_context_len: int
    page_size: int = PAGE_SIZE

    def __post_init__(self):
        for name in ("max_batch", "num_heads", "num_kv_heads", "max_context_len"):
            value = getattr(self, name)
            if type(value) is not int or value <= 0:
                raise ValueError(f"{name} must be a positive integer")
        if self.head_dim not in (64, 128, 256):
            raise ValueError("custom decode supports head_dim 64, 128, or 256")
        if self.page_size != PAGE_SIZE:
            raise ValueError("custom decode supports page_size=256 only")
        if self.num_heads % self.num_kv_heads:
            raise ValueError("query heads must be divisible by KV heads")

    @property
    def group(self):
        return self.num_heads // self.num_kv_heads

    @property
    def partitions(self):
        return -(-self.max_context_len // PARTITION_SIZE)

    @property
    def table_width(self):
        return -(-self.max_context_len // self.page_size)

    @property
    def split_workspace_bytes(self):
        return self.max_batch * self.num_heads * self.partitions * (self.head_dim + 2) * 4


def validate_engine_options(backend, tp, page_size, max_batch, max_context_len):
    """Engine-option check of the reference (spec.py:45-54)."""
    if backend not in BACKENDS:
        raise ValueError(f"unknown decode_backend {backend!r}; choose {BACKENDS}")
    if max_batch <= 0 or max_context_len <= 0:
        raise ValueError("batch and context limits must be positive")
    if backend != "flash_attn":
        if tp != 1:
            raise ValueError("custom decode supports tensor_parallel_size=1 only")
        if page_size != PAGE_SIZE:
            raise ValueError("custom decode requires kvcache_block_size=256")
