"""Capacity-aligned split-KV with normalised FP32 partials + LSE.

Drop-in for the reference's ``src/paged_decode/matched_splitkv.py`` (the
``triton_matched`` slot): ``allocate_matched_resources`` sizes the workspace
from the static plan for this device's SM count, and ``matched_decode``
launches the sm_100a partition kernel (partial = acc / l, lse = m + ln l per
partition, -inf / 0 for empty partitions) and the stable LSE merge.  The
fixed-geometry contract and error messages are the reference's.
"""
from dataclasses import dataclass
import math

import torch

from . import ops
from .runtime import _validate
from .splitkv_plan import launch_partitioning, make_splitkv_plan


@dataclass
class MatchedResources:
    spec: object
    plan: object
    out: torch.Tensor
    partials: torch.Tensor
    lse: torch.Tensor
    # The two scheduler words of the dynamically scheduled partition kernel;
    # zeroed, left zeroed by the kernels.  None selects static scheduling.
    counters: torch.Tensor | None = None


def allocate_matched_resources(spec, device, *, num_splits=0, plan=None):
    """out bf16 [B,Hq,D]; partials f32 [B,Hq,S,D]; lse f32 [B,Hq,S] (matched_splitkv.py:24-34).

    ``plan`` (optional, not in the reference) supplies a ready split plan, e.g.
    ``make_b200_plan(spec, sm_count)``; otherwise the reference heuristic runs
    for this device's SM count with ``num_splits``.
    """
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("matched resources require CUDA")
    if plan is None:
        plan = make_splitkv_plan(spec, ops.sm_count(device), num_splits=num_splits)
    elif plan.splits * plan.tokens_per_split < spec.table_width * 256:
        raise ValueError("plan does not cover the table capacity")
    shape = (spec.max_batch, spec.num_heads, plan.splits)
    return MatchedResources(
        spec, plan,
        torch.empty((spec.max_batch, spec.num_heads, spec.head_dim), device=device,
                    dtype=torch.bfloat16),
        torch.empty((*shape, spec.head_dim), device=device, dtype=torch.float32),
        torch.empty(shape, device=device, dtype=torch.float32),
        torch.zeros(2, device=device, dtype=torch.int32))


def matched_decode(q, k, v, tables, lengths, *, resources, scale=None, kernel="auto"):
    """Partition + LSE merge for the fixed plan; returns ``resources.out``.

    ``kernel`` picks the partition kernel: "auto" (CUDA cores when a KV head
    serves 1 or 2 query heads, tensor cores from 3), "simt" or "mma".
    """
    scale = q.shape[-1] ** -.5 if scale is None else float(scale)
    cache = resources.__dict__.setdefault("_launches", ops.LaunchCache())
    key = ((kernel, scale, q.device) + ops.tensor_key(q, k, v, tables, lengths)
           + ops.buffers_key(resources.out, resources.partials, resources.lse,
                             resources.counters))
    args = cache.get(key)
    if args is not None:
        ops.paged_decode(args, q.device)
        return resources.out
    _validate(q, k, v, tables, lengths, resources, "triton_base", scale)
    if scale <= 0 or not math.isfinite(scale):
        raise ValueError("positive finite scale required")
    spec, plan = resources.spec, resources.plan
    if q.shape[0] != spec.max_batch or tables.shape[1] != spec.table_width:
        raise ValueError("matched plan requires its fixed batch and table capacity")
    shape = (spec.max_batch, spec.num_heads, plan.splits)
    for tensor, geometry in ((resources.lse, shape),
                             (resources.partials, (*shape, spec.head_dim))):
        if (tensor.shape != geometry or tensor.device != q.device
                or tensor.dtype != torch.float32 or not tensor.is_contiguous()):
            raise ValueError("invalid matched workspace")
    tokens, bounds = launch_partitioning(plan)
    args = ops.decode_args(q, k, v, tables, lengths, scale=scale,
                           tokens_per_split=tokens, splits=plan.splits,
                           protocol=ops.PROTOCOL_LSE, kernel=kernel, out=resources.out,
                           partial=resources.partials, lse=resources.lse,
                           counters=resources.counters,
                           flags=bounds | (0 if resources.counters is None else ops.FLAG_DYNAMIC))
    ops.paged_decode(args, q.device)
    cache.put(key, args)
    return resources.out
