"""CPU tests of the callers' set-up hooks (no kernel runs).

``configure_model`` follows the reference's nano-vLLM hook
(src/paged_decode/integration.py:8-26): layers of equal geometry share one
resource set, ``flash_attn`` leaves the model alone, non-BF16 caches and
models without attention layers are rejected.  ``allocate_hybrid_resources``
and ``decode_attention`` follow the Qwen3.5 runner's slot
(src/paged_decode/hybrid.py:15-21, 80-95), ``validate_hybrid_options`` its
option check (src/paged_decode/hybrid_options.py:1-19, tests
tests/test_hybrid_options.py:8-25).
"""
from types import SimpleNamespace

import pytest
import torch

from paged_decode.hybrid import (HYBRID_BACKENDS, allocate_hybrid_resources, decode_attention,
                                 validate_hybrid_options)
from paged_decode.integration import configure_model
from paged_decode.runtime import Resources
from paged_decode.spec import BACKENDS, DecodeSpec, validate_engine_options


class FakeAttention(torch.nn.Module):
    def __init__(self, hq, hkv, d, dtype=torch.bfloat16):
        super().__init__()
        self.num_heads, self.num_kv_heads, self.head_dim = hq, hkv, d
        self.k_cache = torch.zeros(2, 256, hkv, d, dtype=dtype)
        self.v_cache = torch.zeros(2, 256, hkv, d, dtype=dtype)
        self.decode_backend = "flash_attn"
        self.decode_resources = None


def config(backend="triton_splitk"):
    return SimpleNamespace(decode_backend=backend, max_num_seqs=4, max_model_len=2048,
                           kvcache_block_size=256)


def test_layers_of_equal_geometry_share_one_resource_set():
    model = torch.nn.ModuleList([FakeAttention(8, 2, 128), FakeAttention(8, 2, 128),
                                 FakeAttention(16, 4, 256)])
    configure_model(model, config())
    a, b, c = model
    assert a.decode_backend == b.decode_backend == c.decode_backend == "triton_splitk"
    assert a.decode_resources is b.decode_resources
    assert c.decode_resources is not a.decode_resources
    assert a.decode_resources.out.shape == (4, 8, 128)
    assert c.decode_resources.accums.shape == (4, 16, 2, 256)  # 2048 tokens = 2 partitions


def test_flash_attn_leaves_the_model_alone_and_bad_models_are_rejected():
    model = torch.nn.ModuleList([FakeAttention(8, 2, 128)])
    configure_model(model, config("flash_attn"))
    assert model[0].decode_backend == "flash_attn" and model[0].decode_resources is None
    with pytest.raises(ValueError, match="BF16"):
        configure_model(torch.nn.ModuleList([FakeAttention(8, 2, 128, torch.float16)]), config())
    with pytest.raises(ValueError, match="no compatible attention layers"):
        configure_model(torch.nn.ModuleList([torch.nn.Linear(2, 2)]), config())


def test_hybrid_slot_resources_and_dispatch():
    spec = DecodeSpec(2, 8, 2, 256, 1024)
    assert allocate_hybrid_resources(spec, "cpu", "flash_attn") is None
    res = allocate_hybrid_resources(spec, "cpu", "triton_base")
    assert isinstance(res, Resources) and res.out.shape == (2, 8, 256)
    with pytest.raises(ValueError, match="flash_attn"):
        decode_attention(None, None, None, None, None, backend="flash_attn", resources=None,
                         scale=0.0625)


def test_matched_backend_belongs_to_the_fixed_batch_runner_only():
    assert "triton_matched" in HYBRID_BACKENDS and "triton_matched" not in BACKENDS
    with pytest.raises(ValueError, match="unknown decode_backend"):
        validate_engine_options("triton_matched", 1, 256, 1, 1024)
    validate_hybrid_options("triton_matched", "graph", 8, 2176)


@pytest.mark.parametrize("options", [
    ("unknown", "eager", 1, 1024), ("triton_matched", "unknown", 1, 1024),
    ("triton_matched", "eager", 0, 1024), ("triton_matched", "eager", True, 1024),
    ("triton_matched", "eager", 1, 0), ("triton_matched", "graph", 1, 2)])
def test_invalid_runner_options(options):
    with pytest.raises(ValueError):
        validate_hybrid_options(*options)
