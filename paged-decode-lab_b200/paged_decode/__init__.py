"""B200 (sm_100a) paged decode attention behind the reference's backend surface.

Module layout mirrors the reference package ``paged_decode`` so engine code
that imports ``paged_decode.runtime`` / ``paged_decode.matched_splitkv`` /
``paged_decode.spec`` keeps working when this directory is on ``sys.path``:

  spec              DecodeSpec, backend names, engine-option checks
  splitkv_plan      static split-KV plan (computed by the C library)
  runtime           Resources, allocate_resources, paged_decode
  matched_splitkv   MatchedResources, allocate_matched_resources, matched_decode
  integration       configure_model (nano-vLLM hook)
  ops               tensor-level calls into the C ABI
  parallel          batch / KV-head / context sharding over NCCL
  kvcache           paged KV append (store_kvcache)

GPU modules import torch lazily so the geometry contract works on CPU hosts.
"""
from .spec import DecodeSpec

__all__ = ["DecodeSpec"]
