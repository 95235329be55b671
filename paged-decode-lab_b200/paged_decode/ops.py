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
FLAG_DYNAMIC = _lib.FLAG_DYNAMIC
FLAG_BALANCED = _lib.FLAG_BALANCED

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


FAULT_BITS = {1: "producer waited too long for a free stage",
              2: "consumer waited too long for a tile",
              4: "copies in flight did not land at exit",
              8: "dynamic shared memory misaligned",
              16: "exchange peer did not arrive in time"}


def check_fault(clear=True):
    """Raise if a bounded device-side wait gave up since the last clear: the
    outputs of those launches are undefined.  Synchronises; not for hot paths."""
    word = _lib.read_fault(clear)
    if word:
        names = [name for bit, name in FAULT_BITS.items() if word & bit]
        raise RuntimeError(f"device fault word {word:#x}: {'; '.join(names)} -- outputs of the "
                           "launches since the last clear are undefined")


def read_fault(clear=False):
    """Device-side fault word (bounded waits that gave up); synchronises."""
    return _lib.read_fault(clear)


def sm_count(device):
    return torch.cuda.get_device_properties(torch.device(device)).multi_processor_count


# ------------------------------------------------------------ peer exchange
def exchange_plan(rows, head_dim, world, sm_count, emulate=False):
    """``pdl_exchange_plan``: CTAs per rank, rank-block floats, buffer bytes."""
    plan = _lib.PdlExchangePlan()
    status = _lib.load().pdl_exchange_plan(int(rows), int(head_dim), int(world), int(sm_count),
                                           int(bool(emulate)), ctypes.byref(plan))
    if status != _lib.PDL_OK:
        raise ValueError(f"invalid exchange plan request: {_lib.status_text(status)}")
    return plan


def _on_device(device, fn):
    index = device.index if device.index is not None else torch.cuda.current_device()
    with torch.cuda.device(index):
        return fn()


class PeerBuffer:
    """Zeroed device memory owned by this process, exportable over CUDA IPC."""

    def __init__(self, nbytes, device):
        self.device = torch.device(device)
        self.nbytes = int(nbytes)
        ptr, handle = ctypes.c_void_p(), _lib.PdlIpcHandle()
        status = _on_device(self.device, lambda: _lib.load().pdl_peer_buffer_create(
            self.nbytes, ctypes.byref(ptr), ctypes.byref(handle)))
        if status != _lib.PDL_OK:
            raise RuntimeError(f"pdl_peer_buffer_create failed: {_lib.status_text(status)}")
        self.ptr = ptr.value
        self.handle = bytes(handle.bytes)

    def free(self):
        if self.ptr:
            ptr, self.ptr = self.ptr, None
            status = _on_device(self.device, lambda: _lib.load().pdl_peer_buffer_free(ptr))
            if status != _lib.PDL_OK:
                raise RuntimeError(f"pdl_peer_buffer_free failed: {_lib.status_text(status)}")


def open_peer_buffer(handle, device):
    """Map another process's PeerBuffer (64-byte handle) into this one."""
    h = _lib.PdlIpcHandle()
    ctypes.memmove(h.bytes, bytes(handle), 64)
    ptr = ctypes.c_void_p()
    status = _on_device(torch.device(device), lambda: _lib.load().pdl_peer_buffer_open(
        ctypes.byref(h), ctypes.byref(ptr)))
    if status != _lib.PDL_OK:
        raise RuntimeError(f"pdl_peer_buffer_open failed: {_lib.status_text(status)}")
    return ptr.value


def close_peer_buffer(ptr, device):
    status = _on_device(torch.device(device), lambda: _lib.load().pdl_peer_buffer_close(ptr))
    if status != _lib.PDL_OK:
        raise RuntimeError(f"pdl_peer_buffer_close failed: {_lib.status_text(status)}")


def exchange_args(partial, lse, *, rows, parts, head_dim, world, buffers, out, rank=0,
                  lengths=None, num_heads=0, tokens_per_split=0, emulate=False, timeout_us=0):
    """Fill a ``PdlExchangeArgs``; ``buffers`` are raw device addresses (one per rank)."""
    if len(buffers) != world or world > _lib.MAX_PEERS:
        raise ValueError("one exchange buffer per rank, at most 8 ranks")
    a = _lib.PdlExchangeArgs()
    a.partial, a.lse, a.lengths = partial.data_ptr(), lse.data_ptr(), _addr(lengths)
    a.num_heads, a.tokens_per_split = int(num_heads), int(tokens_per_split)
    a.rows, a.parts, a.head_dim = int(rows), int(parts), int(head_dim)
    a.rank, a.world, a.emulate_ranks = int(rank), int(world), int(bool(emulate))
    a.timeout_us = int(timeout_us)
    for q, ptr in enumerate(buffers):
        a.buffers[q] = int(ptr)
    a.out = out.data_ptr()
    return a


def exchange_merge(args, device):
    """Local merge + peer exchange + merge in one kernel (``pdl_exchange_merge``)."""
    _call("pdl_exchange_merge", args, device)
