"""The operator inside its two callers' call sequences, on the GPU.

* nano-vLLM (reference overlays/nano-vllm/nanovllm/layers/attention.py:60-77):
  ``configure_model`` hands every attention layer a backend and a shared
  resource set; a decode step stores the new token with ``store_kvcache``
  through ``context.slot_mapping`` and calls ``paged_decode`` with the
  scheduler's -1-padded live-width block tables and ``context_lens``.  Every
  custom backend is checked against the NumPy oracle on the caches as
  written, and the step (store + decode, full-width tables as the runner's
  graph buffers hold them) is replayed from a CUDA graph with new inputs.
* the Qwen3.5 runner's slot (reference src/paged_decode/hybrid.py:15-21,
  63-95): ``paged_update`` writes a prefill chunk and decode positions into
  random pages (checked bit for bit against plain indexing) and sets the
  lengths; ``decode_attention`` with ``triton_matched`` matches the oracle,
  eagerly and replayed from a graph that also holds the paged write.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import oracle
from gpu_util import assert_out_close, requires_cuda
from paged_decode.hybrid import allocate_hybrid_resources, decode_attention, paged_update
from paged_decode.integration import configure_model
from paged_decode.kvcache import store_kvcache
from paged_decode.runtime import paged_decode

pytestmark = [pytest.mark.gpu, requires_cuda]

DEV = torch.device("cuda", 0)


def expected(q, k, v, table, lengths, scale):
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    return oracle.dense_reference(f(q), f(k), f(v), table.cpu().numpy(),
                                  lengths.cpu().numpy(), scale=scale)


class Attention(torch.nn.Module):
    """The attributes nano-vLLM's Attention layer exposes to configure_model."""

    def __init__(self, hq, hkv, d, pages, gen):
        super().__init__()
        self.num_heads, self.num_kv_heads, self.head_dim = hq, hkv, d
        self.scale = d ** -0.5
        shape = (pages, 256, hkv, d)
        self.k_cache = torch.randn(shape, generator=gen, device=DEV).to(torch.bfloat16)
        self.v_cache = torch.randn(shape, generator=gen, device=DEV).to(torch.bfloat16)
        self.decode_backend = "flash_attn"
        self.decode_resources = None


def scheduler_tables(pool_perm, lens_after, width):
    """-1-padded tables, one row per sequence, `width` columns."""
    rows = []
    off = 0
    for n in lens_after:
        live = -(-n // 256)
        rows.append(pool_perm[off:off + live] + [-1] * (width - live))
        off += live
    return torch.tensor(rows, dtype=torch.int32, device=DEV)


def slots_of(tables, positions):
    pages = tables[torch.arange(len(positions), device=DEV), positions // 256].long()
    return (pages * 256 + positions % 256).to(torch.int32)


@pytest.mark.parametrize("backend", ["triton_base", "triton_splitk", "triton_tc",
                                     "triton_tc_splitk"])
def test_nanovllm_decode_step(backend):
    gen = torch.Generator(device=DEV).manual_seed(5)
    b, hq, hkv, d, pages = 3, 8, 2, 128, 24
    model = torch.nn.ModuleList([Attention(hq, hkv, d, pages, gen) for _ in range(2)])
    configure_model(model, SimpleNamespace(decode_backend=backend, max_num_seqs=4,
                                           max_model_len=2048, kvcache_block_size=256))
    assert model[0].decode_resources is model[1].decode_resources
    lens_before = torch.tensor([300, 0, 1023], device=DEV)
    lens_after = (lens_before + 1).to(torch.int32)
    perm = torch.randperm(pages, generator=gen, device=DEV).tolist()
    width = max(-(-int(n) // 256) for n in lens_after)       # live width, as the scheduler pads
    tables = scheduler_tables(perm, lens_after.tolist(), width)
    slot_mapping = slots_of(tables, lens_before)
    for layer in model:
        q = torch.randn(b, hq, d, generator=gen, device=DEV).to(torch.bfloat16)
        k_new = torch.randn(b, hkv, d, generator=gen, device=DEV).to(torch.bfloat16)
        v_new = torch.randn(b, hkv, d, generator=gen, device=DEV).to(torch.bfloat16)
        store_kvcache(k_new, v_new, layer.k_cache, layer.v_cache, slot_mapping)
        o = paged_decode(q, layer.k_cache, layer.v_cache, tables, lens_after,
                         resources=layer.decode_resources, backend=layer.decode_backend,
                         scale=layer.scale).unsqueeze(1)
        assert o.shape == (b, 1, hq, d)
        want = expected(q, layer.k_cache, layer.v_cache, tables, lens_after, layer.scale)
        assert_out_close(o[:, 0], want, what=backend)


def test_nanovllm_decode_step_replayed_from_a_cuda_graph():
    gen = torch.Generator(device=DEV).manual_seed(6)
    b, hq, hkv, d, pages, width = 4, 16, 4, 128, 40, 8
    layer = Attention(hq, hkv, d, pages, gen)
    configure_model(torch.nn.ModuleList([layer]),
                    SimpleNamespace(decode_backend="triton_splitk", max_num_seqs=b,
                                    max_model_len=width * 256, kvcache_block_size=256))
    # Stable graph buffers, as the runner keeps them (full-width tables).
    q = torch.empty(b, hq, d, device=DEV, dtype=torch.bfloat16)
    k_new = torch.empty(b, hkv, d, device=DEV, dtype=torch.bfloat16)
    v_new = torch.empty_like(k_new)
    tables = torch.full((b, width), -1, dtype=torch.int32, device=DEV)
    lens = torch.zeros(b, dtype=torch.int32, device=DEV)
    slots = torch.zeros(b, dtype=torch.int32, device=DEV)

    def fill(lens_before):
        lens_after = [n + 1 for n in lens_before]
        perm = torch.randperm(pages, generator=gen, device=DEV).tolist()
        tables.copy_(scheduler_tables(perm, lens_after, width))
        lens.copy_(torch.tensor(lens_after, dtype=torch.int32, device=DEV))
        slots.copy_(slots_of(tables, torch.tensor(lens_before, device=DEV)))
        q.copy_(torch.randn(q.shape, generator=gen, device=DEV).to(torch.bfloat16))
        k_new.copy_(torch.randn(k_new.shape, generator=gen, device=DEV).to(torch.bfloat16))
        v_new.copy_(torch.randn(v_new.shape, generator=gen, device=DEV).to(torch.bfloat16))

    def step():
        store_kvcache(k_new, v_new, layer.k_cache, layer.v_cache, slots)
        return paged_decode(q, layer.k_cache, layer.v_cache, tables, lens,
                            resources=layer.decode_resources, backend=layer.decode_backend,
                            scale=layer.scale)

    fill([10, 500, 0, 2000])
    side = torch.cuda.Stream(DEV)
    side.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(side):
        for _ in range(3):
            step()
    torch.cuda.current_stream(DEV).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    for lens_before in ([10, 500, 0, 2000], [1, 1023, 1024, 255], [2046, 0, 77, 300]):
        fill(lens_before)
        graph.replay()
        torch.cuda.synchronize(DEV)
        want = expected(q, layer.k_cache, layer.v_cache, tables, lens, layer.scale)
        assert_out_close(out, want, what=f"graph {lens_before}")
    del graph


def test_qwen35_slot_paged_update_and_matched_decode():
    from paged_decode.spec import DecodeSpec
    gen = torch.Generator(device=DEV).manual_seed(7)
    b, hq, hkv, d, cap = 2, 8, 2, 256, 1025
    width = -(-cap // 256)
    tables = torch.randperm(b * width, generator=gen, device=DEV).to(torch.int32).view(b, width)
    shape = (b * width, 256, hkv, d)
    # Every slot holds a finite value: decode positions skip over unwritten ones.
    k = torch.randn(shape, generator=gen, device=DEV).to(torch.bfloat16)
    v = torch.randn(shape, generator=gen, device=DEV).to(torch.bfloat16)
    lengths = torch.zeros(b, dtype=torch.int32, device=DEV)

    # Prefill chunk of 257 positions, then one decode position.
    key = torch.randn(b, hkv, 257, d, generator=gen, device=DEV).to(torch.bfloat16)
    value = torch.randn_like(key)
    position = torch.arange(257, device=DEV)
    paged_update(k, v, tables, lengths, key, value, position)
    for row in range(b):
        phys = tables[row, position // 256].long()
        assert torch.equal(k[phys, position % 256], key[row].transpose(0, 1))
        assert torch.equal(v[phys, position % 256], value[row].transpose(0, 1))
    assert lengths.tolist() == [257, 257]
    new = torch.randn(b, hkv, 1, d, generator=gen, device=DEV).to(torch.bfloat16)
    paged_update(k, v, tables, lengths, new, new, torch.tensor([257], device=DEV))
    assert lengths.tolist() == [258, 258]
    for row in range(b):
        assert torch.equal(k[tables[row, 1].long(), 1], new[row, :, 0])

    spec = DecodeSpec(b, hq, hkv, d, cap)
    res = allocate_hybrid_resources(spec, DEV, "triton_matched")
    q = torch.randn(b, hq, d, generator=gen, device=DEV).to(torch.bfloat16)
    out = decode_attention(q, k, v, tables, lengths, backend="triton_matched", resources=res,
                           scale=0.0625)
    assert_out_close(out, expected(q, k, v, tables, lengths, 0.0625), what="matched eager")

    # Decode loop in a graph: paged write of position p, then decode.
    pos = torch.tensor([258], device=DEV)
    step_k = torch.empty(b, hkv, 1, d, device=DEV, dtype=torch.bfloat16)
    step_v = torch.empty_like(step_k)

    def step():
        paged_update(k, v, tables, lengths, step_k, step_v, pos)
        return decode_attention(q, k, v, tables, lengths, backend="triton_matched",
                                resources=res, scale=0.0625)

    side = torch.cuda.Stream(DEV)
    side.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(side):
        for _ in range(3):
            step()
    torch.cuda.current_stream(DEV).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    for p in (258, 259, 700, 1024):
        pos.fill_(p)
        step_k.copy_(torch.randn(step_k.shape, generator=gen, device=DEV).to(torch.bfloat16))
        step_v.copy_(torch.randn(step_v.shape, generator=gen, device=DEV).to(torch.bfloat16))
        graph.replay()
        torch.cuda.synchronize(DEV)
        assert lengths.tolist() == [p + 1] * b
        for row in range(b):
            assert torch.equal(k[tables[row, p // 256].long(), p % 256], step_k[row, :, 0])
        assert_out_close(out, expected(q, k, v, tables, lengths, 0.0625), what=f"graph p={p}")
    del graph
    assert np.isfinite(out.float().cpu().numpy()).all()


@pytest.mark.filterwarnings("ignore:The CUDA Graph is empty")
def test_metadata_validation_refuses_to_run_inside_a_capture():
    """The debug check synchronises, so during stream capture it raises
    RuntimeError instead (reference runtime.py:38-43)."""
    from paged_decode.runtime import validate_device_metadata
    table = torch.zeros(1, 4, dtype=torch.int32, device=DEV)
    lens = torch.ones(1, dtype=torch.int32, device=DEV)
    validate_device_metadata(table, lens, 1, 1024)  # eager: fine
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(DEV)
    with pytest.raises(RuntimeError, match="capture"):
        with torch.cuda.graph(graph, stream=side):
            validate_device_metadata(table, lens, 1, 1024)
    del graph
