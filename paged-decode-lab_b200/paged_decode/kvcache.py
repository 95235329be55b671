"""Paged KV append: write the new token's K/V rows before decode.

``store_kvcache`` keeps nano-vLLM's signature and semantics (reference overlay
``nanovllm/layers/attention.py:10-40``): token i goes to physical slot
``slot_mapping[i]`` (page * 256 + offset) and -1 skips it.
``append_decode_kv`` is the decode-loop form of the Qwen3.5 runner's paged
update (reference ``src/paged_decode/hybrid.py:63-72``): row b's token goes to
position ``lengths[b]`` through the block table, and ``lengths[b] += 1`` on the
device, so append + decode steps can be captured in one CUDA graph.
"""
import ctypes

import torch

from . import _lib


def _common(key, value, k_cache, v_cache):
    for t in (key, value):
        if t.dtype != torch.bfloat16 or t.ndim != 3 or t.stride(-1) != 1:
            raise ValueError("key/value must be BF16 [tokens, kv_heads, head_dim] with "
                             "contiguous head_dim")
    if k_cache.shape != v_cache.shape or k_cache.ndim != 4 or k_cache.shape[1] != 256:
        raise ValueError("KV must use NHD pages [pages,256,kv_heads,head_dim]")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("K/V caches must be contiguous")
    if key.shape != value.shape or key.shape[1:] != k_cache.shape[2:]:
        raise ValueError("key/value rows must match the cache's [kv_heads, head_dim]")
    a = _lib.PdlAppendArgs()
    a.key, a.value = key.data_ptr(), value.data_ptr()
    a.key_stride_token, a.key_stride_head = key.stride(0), key.stride(1)
    a.value_stride_token, a.value_stride_head = value.stride(0), value.stride(1)
    a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    a.num_pages = k_cache.shape[0]
    a.n_tokens = key.shape[0]
    a.num_kv_heads, a.head_dim = key.shape[1], key.shape[2]
    return a


def _launch(args, device):
    lib = _lib.load()
    with torch.cuda.device(device):
        status = lib.pdl_append_kv(ctypes.byref(args), torch.cuda.current_stream().cuda_stream)
    if status != _lib.PDL_OK:
        raise RuntimeError(f"pdl_append_kv failed: {_lib.status_text(status)}")


def store_kvcache(key, value, k_cache, v_cache, slot_mapping):
    """Write key[i]/value[i] into slot slot_mapping[i] of the caches (-1: skip)."""
    if slot_mapping.dtype != torch.int32 or slot_mapping.numel() != key.shape[0]:
        raise ValueError("slot_mapping must be int32 with one entry per token")
    a = _common(key, value, k_cache, v_cache)
    a.slot_mapping = slot_mapping.data_ptr()
    _launch(a, key.device)


def append_decode_kv(key, value, k_cache, v_cache, tables, lengths, increment=True):
    """Row b's new token -> position lengths[b] via the block table; then lengths[b] += 1.

    Rows whose table is already full are skipped (and keep their length).
    """
    if tables.dtype != torch.int32 or lengths.dtype != torch.int32:
        raise ValueError("block tables and context lengths must be int32")
    if tables.ndim != 2 or tables.stride(1) != 1 or lengths.shape != (key.shape[0],):
        raise ValueError("need one table row and one length per token")
    a = _common(key, value, k_cache, v_cache)
    a.block_table = tables.data_ptr()
    a.table_stride, a.table_width = tables.stride(0), tables.shape[1]
    a.lengths = lengths.data_ptr()
    a.increment_lengths = 1 if increment else 0
    _launch(a, key.device)
