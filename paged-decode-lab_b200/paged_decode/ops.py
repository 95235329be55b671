"""Tensor-level wrappers over the C ABI (no validation beyond the library's).

These take torch tensors that already satisfy the contract (device, dtype,
layout), fill one ``PdlDecodeArgs`` and enqueue on the current CUDA stream
of the tensors' device.  ``runtime.paged_decode`` and
``matched_splitkv.matched_decode`` validate with the reference's messages
first and then call these.
"""
import ctypes

import torch

from . import _lib

PROTOCOL_LSE = _lib.PROTOCOL_LSE
PROTOCOL_MLA = _lib.PROTOCOL_MLA
KERNEL_AUTO = _lib.KERNEL_AUTO
KERNEL_SIMT = _lib.KERNEL_SIMT
KERNEL_MMA = _lib.KERNEL_MMA
FLAG_SKIP_EMPTY = _lib.FLAG_SKIP_EMPTY
FLAG_DIRECT_SINGLE = _lib.FLAG_DIRECT_SINGLE
FLAG_FUSED_MERGE = _lib.FLAG_FUSED_MERGE
FLAG_DYNAMIC = _lib.FLAG_DYNAMIC

_KERNELS = {"auto": KERNEL_AUTO, "simt": KERNEL_SIMT, "mma": KERNEL_MMA}


def _addr(t):
    return None if t is None else t.data_ptr()


def decode_args(q, k, v, tables, lengths, *, scale, tokens_per_split=0, splits=1,
                protocol=PROTOCOL_LSE, kernel="auto", flags=0, out=None, partial=None,
                lse=None, maxima=None, denoms=None, accums=None, counters=None):
    """Fill a ``PdlDecodeArgs`` from tensors (element strides, raw addresses)."""
    a = _lib.PdlDecodeArgs()
    a.q = q.data_ptr()
    a.q_stride_batch = q.stride(0)
    a.q_stride_head = q.stride(1)
    a.k_cache = k.data_ptr()
    a.v_cache = v.data_ptr()
    a.num_pages = k.shape[0]
    a.block_table = tables.data_ptr()
    a.table_stride = tables.stride(0)
    a.table_width = tables.shape[1]
    a.lengths = lengths.data_ptr()
    a.batch = q.shape[0]
    a.num_heads = q.shape[1]
    a.num_kv_heads = k.shape[2]
    a.head_dim = q.shape[2]
    a.scale = float(scale)
    a.tokens_per_split = int(tokens_per_split)
    a.splits = int(splits)
    a.protocol = protocol
    a.kernel = _KERNELS[kernel] if isinstance(kernel, str) else int(kernel)
    a.flags = int(flags)
    a.out = _addr(out)
    a.partial = _addr(partial)
    a.lse = _addr(lse)
    a.maxima = _addr(maxima)
    a.denoms = _addr(denoms)
    a.accums = _addr(accums)
    a.counters = _addr(counters)
    return a


def _call(name, args, device):
    fn = getattr(_lib.load(), name)
    index = device.index if device.index is not None else torch.cuda.current_device()
    if torch.cuda.current_device() == index:
        status = fn(ctypes.byref(args), torch.cuda.current_stream().cuda_stream)
    else:
        with torch.cuda.device(index):
            status = fn(ctypes.byref(args), torch.cuda.current_stream().cuda_stream)
    if status != _lib.PDL_OK:
        raise RuntimeError(f"{name} failed: {_lib.status_text(status)}")


def tensor_key(*tensors):
    """Metadata that fixes a launch: addresses, shapes, strides and dtypes.

    Validation depends only on these, never on tensor contents, so a launch
    whose key was validated once may reuse its filled ``PdlDecodeArgs``.
    """
    key = []
    for t in tensors:
        key.extend((t.data_ptr(), t.shape, t.stride(), t.dtype))
    return tuple(key)


def buffers_key(*tensors):
    """Addresses of output / workspace buffers (None where absent)."""
    return tuple(None if t is None else t.data_ptr() for t in tensors)


class LaunchCache(dict):
    """Bounded map from launch keys to validated ``PdlDecodeArgs``."""

    LIMIT = 64

    def put(self, key, args):
        if len(self) >= self.LIMIT:
            self.clear()
        self[key] = args
        return args


def partition(args, device):
    """Launch the partition kernel (``pdl_partition``)."""
    _call("pdl_partition", args, device)


def merge(args, device):
    """Launch the merge kernel (``pdl_merge``)."""
    _call("pdl_merge", args, device)


def paged_decode(args, device):
    """Partition + merge, or the single-pass kernel (``pdl_paged_decode``)."""
    _call("pdl_paged_decode", args, device)


def paged_decode_static_scratch(args, device):
    """``pdl_paged_decode_static_scratch``: decode without a caller workspace.

    For callers that cannot allocate device memory (an engine that reserved
    nearly all HBM for its KV pool, or a path that must not call
    cudaMalloc/cudaFree); the workspace is the library's 4 MiB device array,
    shared by every call on the device.  Larger requests raise.
    """
    _call("pdl_paged_decode_static_scratch", args, device)


def merge_args(partial, lse, *, rows, parts, head_dim, row_stride, part_stride, lse_row_stride,
               lse_part_stride, out=None, out_partial=None, out_lse=None):
    """Fill a ``PdlMergeArgs`` (strides in floats; tensors give base addresses)."""
    m = _lib.PdlMergeArgs()
    m.partial = partial.data_ptr()
    m.lse = lse.data_ptr()
    m.row_stride, m.part_stride = int(row_stride), int(part_stride)
    m.lse_row_stride, m.lse_part_stride = int(lse_row_stride), int(lse_part_stride)
    m.rows, m.parts, m.head_dim = int(rows), int(parts), int(head_dim)
    m.out = _addr(out)
    m.out_partial = _addr(out_partial)
    m.out_lse = _addr(out_lse)
    return m


def lse_merge(margs, device):
    """Strided LSE merge (``pdl_lse_merge``)."""
    fn = _lib.load().pdl_lse_merge
    index = device.index if device.index is not None else torch.cuda.current_device()
    with torch.cuda.device(index):
        status = fn(ctypes.byref(margs), torch.cuda.current_stream().cuda_stream)
    if status != _lib.PDL_OK:
        raise RuntimeError(f"pdl_lse_merge failed: {_lib.status_text(status)}")


def read_fault(clear=False):
    """Device-side fault word (bounded waits that gave up); synchronises."""
    return _lib.read_fault(clear)


def sm_count(device):
    return torch.cuda.get_device_properties(torch.device(device)).multi_processor_count
