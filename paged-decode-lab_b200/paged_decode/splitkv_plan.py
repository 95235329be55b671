"""Static split-KV plan, computed natively by ``pdl_splitkv_plan``.

``make_splitkv_plan`` keeps the reference's signature, fields and errors
(src/paged_decode/splitkv_plan.py:15-56): tile = 256/128/64 tokens for
D = 64/128/256, partitions are whole tiles of the table capacity, and with
``num_splits=0`` the count comes from the wave-efficiency heuristic on
``2 * sm_count`` virtual SMs.  The arithmetic itself runs in the C library.
"""
from dataclasses import dataclass
import ctypes

from . import _lib


@dataclass(frozen=True)
class SplitKVPlan:
    splits: int
    tile_tokens: int
    tokens_per_split: int
    table_capacity_tokens: int
    lse_lanes: int
    sm_count: int
    policy: str
    # Not in the reference: the B200 plan may recommend partitions that follow
    # each row's length (PDL_FLAG_BALANCED, granule tile_tokens); see
    # launch_partitioning.
    balanced: bool = False


def launch_partitioning(plan):
    """(tokens_per_split, flags) to launch ``plan`` with: the fixed partitions
    of ``plan.tokens_per_split`` tokens, or -- when the plan recommends it --
    balanced partitions of whole ``tile_tokens`` granules with
    ``PDL_FLAG_BALANCED``."""
    if plan.balanced:
        return plan.tile_tokens, _lib.FLAG_BALANCED
    return plan.tokens_per_split, 0


def make_splitkv_plan(spec, sm_count, *, num_splits=0):
    if type(sm_count) is not int or sm_count < 1:
        raise ValueError("positive SM count required")
    if type(num_splits) is not int or not 0 <= num_splits <= 128:
        raise ValueError("num_splits must be an integer in [0,128]")
    if spec.num_heads // spec.num_kv_heads > 16:
        raise ValueError("matched split-KV requires at most 16 query heads per KV head")
    plan = _lib.PdlPlan()
    status = _lib.load().pdl_splitkv_plan(ctypes.byref(_lib.make_spec(spec)), sm_count,
                                          num_splits, ctypes.byref(plan))
    if status != _lib.PDL_OK:
        raise ValueError(f"invalid split-KV plan request: {_lib.status_text(status)}")
    return SplitKVPlan(plan.splits, plan.tile_tokens, plan.tokens_per_split,
                       plan.table_capacity_tokens, plan.lse_lanes, plan.sm_count,
                       "explicit" if plan.explicit_splits else "pinned_geometry")


def make_b200_plan(spec, sm_count):
    """Split plan for this library's persistent kernels (``pdl_b200_plan``).

    About one work item per CTA slot (two CTAs per SM), items of at most
    4096 tokens so variable-length batches balance under dynamic scheduling,
    partitions a multiple of the reference plan's tile.  For one wave of long
    D = 256 items ``balanced`` is set: launch it as ``launch_partitioning``
    says (``matched_decode`` does).  Use it through
    ``allocate_matched_resources(spec, device, plan=make_b200_plan(spec, sms))``:
    ``num_splits=plan.splits`` would recompute ``tokens_per_split`` with the
    reference heuristic's rounding, which can give other partition bounds.
    """
    if type(sm_count) is not int or sm_count < 1:
        raise ValueError("positive SM count required")
    plan = _lib.PdlPlan()
    status = _lib.load().pdl_b200_plan(ctypes.byref(_lib.make_spec(spec)), sm_count,
                                       ctypes.byref(plan))
    if status != _lib.PDL_OK:
        raise ValueError(f"invalid plan request: {_lib.status_text(status)}")
    return SplitKVPlan(plan.splits, plan.tile_tokens, plan.tokens_per_split,
                       plan.table_capacity_tokens, plan.lse_lanes, plan.sm_count, "b200",
                       bool(plan.balanced))
