"""The decode attention slot of a hybrid (Qwen3.5-style) fixed-batch runner.

The reference's runner (``src/paged_decode/hybrid.py``) keeps its
full-attention layers' KV in a paged pool and calls this operator for decode.
These are the places where it touches the operator, with the same
names, arguments and errors; the model, its Transformers blocks and the
linear-attention state are not part of this package:

* ``HYBRID_BACKENDS`` / ``validate_hybrid_options`` -- the runner's option
  check (reference ``hybrid_options.py:1-19``): the engine backends plus the
  fixed-geometry ``triton_matched``;
* ``allocate_hybrid_resources`` -- reference ``hybrid.py:15-21``;
* ``paged_update`` -- the paged write of ``PagedHybridCache.update``
  (``hybrid.py:63-72``): the chunk's K/V rows go to
  ``tables[b, pos // 256] * 256 + pos % 256`` and every row's length becomes
  ``position[-1] + 1``.  The write runs through this package's append kernel
  (``pdl_append_kv``, slot mode) instead of ``index_copy_``;
* ``decode_attention`` -- the decode branch of ``_attention``
  (``hybrid.py:80-95``) for the custom backends.  ``flash_attn`` is not
  served here (no FlashAttention dispatch); it raises instead of falling back.
"""
import torch

from .kvcache import store_kvcache
from .runtime import allocate_resources, paged_decode
from .spec import BACKENDS, PAGE_SIZE

# The engine's scheduler may change batch and table geometry between steps,
# so its backend list leaves out the capacity-aligned fixed-plan path, which
# only the fixed-batch runner offers.
HYBRID_BACKENDS = (*BACKENDS, "triton_matched")


def validate_hybrid_options(backend, mode, batch, max_context):
    """Reject runner options before anything is loaded (same messages as the reference)."""
    if backend not in HYBRID_BACKENDS:
        raise ValueError(f"unknown Qwen3.5 backend {backend!r}; choose {HYBRID_BACKENDS}")
    if mode not in ("eager", "graph"):
        raise ValueError("execution mode must be eager or graph")
    if type(batch) is not int or batch < 1:
        raise ValueError("batch must be a positive integer")
    if type(max_context) is not int or max_context < 1:
        raise ValueError("max_context must be a positive integer")
    if mode == "graph" and max_context < 3:
        raise ValueError("Graph warmup needs context capacity >=3")


def allocate_hybrid_resources(spec, device, backend):
    """None for ``flash_attn``; the matched workspace for ``triton_matched``;
    otherwise the backend's ``Resources``."""
    if backend == "flash_attn":
        return None
    if backend == "triton_matched":
        from .matched_splitkv import allocate_matched_resources
        return allocate_matched_resources(spec, device)
    return allocate_resources(spec, device, backend)


def paged_update(k_pages, v_pages, tables, lengths, key, value, position):
    """Write a chunk of K/V for every row into the paged pool.

    key, value: [batch, kv_heads, len(position), head_dim] (the layout the
    attention blocks produce); position: int64 [len(position)], the same for
    every row.  Afterwards ``lengths[:] = position[-1] + 1`` (on the device).
    """
    batch, hkv, steps, dim = key.shape
    if value.shape != key.shape or position.shape != (steps,):
        raise ValueError("key, value and position must describe the same chunk")
    if tables.dtype != torch.int32 or lengths.dtype != torch.int32:
        raise ValueError("block tables and context lengths must be int32")
    page = tables[:, position // PAGE_SIZE].long()                 # [batch, steps]
    slots = (page * PAGE_SIZE + (position % PAGE_SIZE)[None, :]).to(torch.int32).flatten()
    rows_k = key.transpose(1, 2).reshape(batch * steps, hkv, dim)
    rows_v = value.transpose(1, 2).reshape(batch * steps, hkv, dim)
    store_kvcache(rows_k, rows_v, k_pages, v_pages, slots)
    lengths.copy_((position[-1] + 1).expand(batch))


def decode_attention(q, k_pages, v_pages, tables, lengths, *, backend, resources, scale):
    """[batch, num_heads, head_dim] decode output (borrowed from ``resources``)."""
    if backend == "flash_attn":
        raise ValueError("flash_attn decode is not served by this operator")
    if backend == "triton_matched":
        from .matched_splitkv import matched_decode
        return matched_decode(q, k_pages, v_pages, tables, lengths, resources=resources,
                              scale=scale)
    return paged_decode(q, k_pages, v_pages, tables, lengths, resources=resources,
                        backend=backend, scale=scale)
