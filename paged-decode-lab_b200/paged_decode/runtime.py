"""Validated launches and reusable output / split workspace.

Drop-in for the reference's ``src/paged_decode/runtime.py``: the same
``Resources`` / ``allocate_resources`` / ``paged_decode`` /
``validate_device_metadata`` surface, backend names and ``ValueError``
messages, with every backend served by the sm_100a kernels of this package:

  triton_base       one output per row, no exposed workspace (CUDA-core kernel,
                    tensor cores from 3 query heads per KV head); rows longer
                    than this library's plan allows per CTA are split into
                    internal scratch and merged (see allocate_resources)
  triton_splitk     1024-token partitions, (m, l, acc) workspace + merge (kernel
                    chosen as for triton_base)
  triton_tc         as triton_base, BF16 tensor-core kernel
  triton_tc_splitk  1024-token partitions, (m, l, acc) workspace + merge, tensor cores

Tensor CONTENTS are trusted on the hot path (live table entries must be valid
pages; 0 <= length <= table width * 256).  Call ``validate_device_metadata``
once for externally supplied tables.  No host synchronisation, allocation or
device-scalar read happens inside ``paged_decode``, so it can be captured in
a CUDA graph after warm-up.
"""
from dataclasses import dataclass
import math

import torch

from . import ops
from .spec import DecodeSpec, PAGE_SIZE, PARTITION_SIZE  # noqa: F401

_CUSTOM = ("triton_base", "triton_splitk", "triton_tc", "triton_tc_splitk")


@dataclass
class Resources:
    spec: DecodeSpec
    out: torch.Tensor
    maxima: torch.Tensor | None = None
    denoms: torch.Tensor | None = None
    accums: torch.Tensor | None = None
    # The two scheduler words of the dynamically scheduled partition kernel;
    # zeroed, left zeroed by the kernels.
    counters: torch.Tensor | None = None
    # Not in the reference: the single-pass backends' split plan and scratch
    # (partial + LSE per partition), or None where one pass per row is used.
    split_plan: object | None = None
    split_partials: torch.Tensor | None = None
    split_lse: torch.Tensor | None = None


def allocate_resources(spec, device, backend="triton_splitk"):
    """Output buffer plus, for split backends, the (m, l, acc) workspace.

    Shapes follow the reference (runtime.py:24-35): out bf16 [B,Hq,D];
    maxima / denoms f32 [B,Hq,partitions]; accums f32 [B,Hq,partitions,D].
    The single-pass backends additionally get this library's split plan for
    the device and, when it splits rows, partial + LSE scratch for it: one
    CTA per (row, KV head) leaves most of a B200 idle or streams a long row
    alone (config 4: 634 us in one pass against 459 us split).
    """
    if backend not in _CUSTOM:
        raise ValueError("resources require a custom backend")
    out = torch.empty((spec.max_batch, spec.num_heads, spec.head_dim),
                      dtype=torch.bfloat16, device=device)
    result = Resources(spec, out)
    if backend in ("triton_splitk", "triton_tc_splitk"):
        shape = (spec.max_batch, spec.num_heads, spec.partitions)
        result.maxima = torch.empty(shape, device=device, dtype=torch.float32)
        result.denoms = torch.empty(shape, device=device, dtype=torch.float32)
        result.accums = torch.empty((*shape, spec.head_dim), device=device, dtype=torch.float32)
        result.counters = torch.zeros(2, device=device, dtype=torch.int32)
    elif torch.device(device).type == "cuda":
        from .splitkv_plan import make_b200_plan
        plan = make_b200_plan(spec, ops.sm_count(device))
        if plan.splits > 1:
            shape = (spec.max_batch, spec.num_heads, plan.splits)
            result.split_plan = plan
            result.split_partials = torch.empty((*shape, spec.head_dim), device=device,
                                                dtype=torch.float32)
            result.split_lse = torch.empty(shape, device=device, dtype=torch.float32)
            result.counters = torch.zeros(2, device=device, dtype=torch.int32)
    return result


def check_metadata(table, lengths, num_pages, max_context_len, page_size=PAGE_SIZE):
    """Host check of the metadata contract (reference reference.py:10-21)."""
    table = table.to(torch.int64)
    lengths = lengths.to(torch.int64)
    if table.ndim != 2 or lengths.ndim != 1 or table.shape[0] != lengths.shape[0]:
        raise ValueError("metadata batch dimensions differ")
    if lengths.numel() and (int(lengths.min()) < 0 or int(lengths.max()) > max_context_len):
        raise ValueError("context length outside configured capacity")
    for b in range(table.shape[0]):
        live = -(-int(lengths[b]) // page_size)
        if live > table.shape[1]:
            raise ValueError("invalid live page mapping")
        if live:
            pages = table[b, :live]
            if int(pages.min()) < 0 or int(pages.max()) >= num_pages:
                raise ValueError("invalid live page mapping")


def validate_device_metadata(table, lengths, num_pages, max_context_len):
    """Debug check: deliberately synchronises; NEVER call in capture/hot path."""
    if torch.cuda.is_current_stream_capturing():
        raise RuntimeError("metadata content validation cannot run during graph capture")
    if table.dtype not in (torch.int32, torch.int64) or lengths.dtype not in (torch.int32, torch.int64):
        raise ValueError("metadata must be integral")
    check_metadata(table.cpu(), lengths.cpu(), num_pages, max_context_len)


def _validate(q, k, v, tables, lengths, resources, backend, scale):
    """Tensor contract with the reference's messages (runtime.py:46-84)."""
    if backend not in ("triton_base", "triton_splitk"):
        raise ValueError("unknown custom backend")
    spec = resources.spec
    tensors = (q, k, v, tables, lengths, resources.out)
    if not all(t.is_cuda and t.device == q.device for t in tensors):
        raise ValueError("all tensors must be on the same CUDA device")
    if q.dtype != torch.bfloat16 or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("custom decode supports BF16 Q/K/V only")
    if q.ndim != 3 or q.shape[1:] != (spec.num_heads, spec.head_dim):
        raise ValueError("Q must have shape [batch, query_heads, head_dim]")
    batch = q.shape[0]
    if not 0 < batch <= spec.max_batch or q.stride(-1) != 1:
        raise ValueError("Q batch exceeds capacity or innermost dimension is not contiguous")
    if k.ndim != 4 or k.shape[1:] != (256, spec.num_kv_heads, spec.head_dim):
        raise ValueError("KV must use NHD pages [pages,256,kv_heads,head_dim]")
    if k.shape != v.shape or not k.is_contiguous() or not v.is_contiguous() or k.shape[0] == 0:
        raise ValueError("K/V must have matching nonempty contiguous storage")
    if tables.ndim != 2 or tables.shape[0] != batch or tables.stride(1) != 1:
        raise ValueError("block table must have shape [batch,capacity] and contiguous rows")
    # During eager execution the scheduler provides only the live table width.
    if not 0 < tables.shape[1] <= spec.table_width:
        raise ValueError("block table width outside configured capacity")
    if lengths.shape != (batch,) or not lengths.is_contiguous():
        raise ValueError("context lengths must be a contiguous [batch] tensor")
    if tables.dtype != torch.int32 or lengths.dtype != torch.int32:
        raise ValueError("block tables and context lengths must be int32")
    if not math.isfinite(scale):
        raise ValueError("scale must be finite")
    if (resources.out.shape != (spec.max_batch, spec.num_heads, spec.head_dim)
            or resources.out.dtype != q.dtype or not resources.out.is_contiguous()):
        raise ValueError("invalid output buffer")
    if backend == "triton_splitk":
        shape = (spec.max_batch, spec.num_heads, spec.partitions)
        for tensor, expected in ((resources.maxima, shape), (resources.denoms, shape),
                                 (resources.accums, (*shape, spec.head_dim))):
            if (tensor is None or tensor.shape != expected or tensor.device != q.device
                    or tensor.dtype != torch.float32 or not tensor.is_contiguous()):
                raise ValueError("invalid or missing preallocated split-K workspace")


def paged_decode(q, k, v, tables, lengths, *, resources, backend="triton_base", scale=None):
    """Return borrowed [B,H,D] output. Next launch using resources overwrites it.

    Resources must not overlap live inputs or be used concurrently across
    streams.  Live table entries must be valid pages;
    0 <= lengths <= max_context_len and ceil(length/256) <= table width.
    Padding table entries may contain -1 (never read).
    """
    scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    cache = resources.__dict__.setdefault("_launches", ops.LaunchCache())
    key = ((backend, scale, q.device) + ops.tensor_key(q, k, v, tables, lengths)
           + ops.buffers_key(resources.out, resources.maxima, resources.denoms, resources.accums,
                             resources.counters, resources.split_partials))
    args = cache.get(key)
    if args is not None:
        ops.paged_decode(args, q.device)
        return resources.out[:q.shape[0]]
    if backend not in _CUSTOM:
        raise ValueError("unknown custom backend")
    split = backend in ("triton_splitk", "triton_tc_splitk")
    tensor_cores = backend in ("triton_tc", "triton_tc_splitk")
    _validate(q, k, v, tables, lengths, resources, "triton_splitk" if split else "triton_base",
              scale)
    spec = resources.spec
    if tensor_cores:
        # Reference contracts of tc_splitk.py:63-72 and experimental_precision.py:110-121.
        if scale <= 0:
            raise ValueError("Tensor Core split-K requires a positive softmax scale" if split
                             else "BF16-exp paths require a positive softmax scale")
        if q.shape[1] // spec.num_kv_heads > 16:
            raise ValueError("Tensor Core split-K supports at most 16 query heads per KV head"
                             if split else "experimental Tensor Core path supports at most 16 "
                             "query heads per KV head")
    # The CUDA-core backends take the tensor-core kernel once 3 or more query
    # heads share a KV head (the library's AUTO choice): measured on B200 the
    # CUDA-core kernel turns issue-bound there (0.19-0.69 of copy bandwidth at
    # 4-16 heads per KV head) while the tensor-core kernel stays HBM-bound.
    # Backend names fix the workspace protocol and the reference's contract
    # checks, not the instructions that compute the result.
    kernel = "mma" if tensor_cores else "auto"
    if split:
        # The (m, l, acc) workspace is this call's scratch: the merge reads the
        # ceil(length / 1024) live partitions of each row only, so partitions
        # past a row's length are not written (the reference stores -inf, 0, 0
        # there for its merge, which reads all of them).  Writing them costs
        # about 9% at config 4's 32 partitions: 55 MB of stores per call,
        # 486 vs 447 us measured on B200.
        flags = ops.FLAG_SKIP_EMPTY | (0 if resources.counters is None else ops.FLAG_DYNAMIC)
        args = ops.decode_args(q, k, v, tables, lengths, scale=scale,
                               tokens_per_split=PARTITION_SIZE, splits=spec.partitions,
                               protocol=ops.PROTOCOL_MLA, kernel=kernel, out=resources.out,
                               maxima=resources.maxima, denoms=resources.denoms,
                               accums=resources.accums, counters=resources.counters,
                               flags=flags)
    elif resources.split_plan is not None:
        # One output per row, computed in partitions of this library's plan
        # (scratch only: partitions past a row's length are not stored).
        from .splitkv_plan import launch_partitioning
        plan = resources.split_plan
        tokens, bounds = launch_partitioning(plan)
        args = ops.decode_args(q, k, v, tables, lengths, scale=scale,
                               tokens_per_split=tokens, splits=plan.splits,
                               protocol=ops.PROTOCOL_LSE, kernel=kernel, out=resources.out,
                               partial=resources.split_partials, lse=resources.split_lse,
                               counters=resources.counters,
                               flags=bounds | ops.FLAG_SKIP_EMPTY | ops.FLAG_DYNAMIC)
    else:
        args = ops.decode_args(q, k, v, tables, lengths, scale=scale, kernel=kernel,
                               out=resources.out)
    ops.paged_decode(args, q.device)
    cache.put(key, args)
    return resources.out[:q.shape[0]]
