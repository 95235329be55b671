"""GPU tests of the paged KV append and of a graph-captured decode loop.

Append parity is bit-exact against a NumPy scatter (byte work).  The loop test
follows BASELINE config 3's protocol at a reduced size: each step appends one
token per row at its current length (lengths += 1 on the device) and decodes;
the whole multi-step loop is captured once in a CUDA graph and replayed.
"""
import numpy as np
import pytest
import torch

import cases
import oracle
from gpu_util import assert_out_close, device_case, requires_cuda
from paged_decode.kvcache import append_decode_kv, store_kvcache
from paged_decode.matched_splitkv import allocate_matched_resources, matched_decode
from paged_decode.spec import DecodeSpec

pytestmark = [pytest.mark.gpu, requires_cuda]


def bits(t):
    return t.view(torch.int16).cpu().numpy()


@pytest.mark.parametrize("hkv,dim", [(1, 64), (2, 128), (4, 256), (8, 128)])
def test_store_kvcache_slot_mapping(hkv, dim):
    gen = torch.Generator(device="cuda").manual_seed(3)
    pages, n = 6, 40
    k = torch.randn(pages, 256, hkv, dim, generator=gen, device="cuda").to(torch.bfloat16)
    v = torch.randn_like(k)
    # Strided source rows (a slice of a wider buffer) exercise the stride path.
    wide = torch.randn(n, hkv, dim * 2, generator=gen, device="cuda").to(torch.bfloat16)
    key, value = wide[:, :, :dim], wide[:, :, dim:]
    slots = torch.randperm(pages * 256, generator=gen, device="cuda")[:n].to(torch.int32)
    slots[::7] = -1
    ek, ev = bits(k).copy(), bits(v).copy()
    s = slots.cpu().numpy()
    for i in range(n):
        if s[i] >= 0:
            ek[s[i] // 256, s[i] % 256] = bits(key[i])
            ev[s[i] // 256, s[i] % 256] = bits(value[i])
    store_kvcache(key, value, k, v, slots)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(k), ek)
    np.testing.assert_array_equal(bits(v), ev)


def test_append_decode_kv_table_mode_and_full_rows():
    gen = torch.Generator(device="cuda").manual_seed(4)
    b, hkv, dim, width = 5, 2, 128, 3
    k = torch.randn(b * width, 256, hkv, dim, generator=gen, device="cuda").to(torch.bfloat16)
    v = torch.randn_like(k)
    table = torch.randperm(b * width, generator=gen, device="cuda").view(b, width).to(torch.int32)
    lens = torch.tensor([0, 255, 256, 767, 768], dtype=torch.int32, device="cuda")  # last is full
    key = torch.randn(b, hkv, dim, generator=gen, device="cuda").to(torch.bfloat16)
    value = torch.randn_like(key)
    ek, ev, t = bits(k).copy(), bits(v).copy(), table.cpu().numpy()
    for row, n in enumerate(lens.tolist()):
        if n < width * 256:
            ek[t[row, n // 256], n % 256] = bits(key[row])
            ev[t[row, n // 256], n % 256] = bits(value[row])
    append_decode_kv(key, value, k, v, table, lens)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(k), ek)
    np.testing.assert_array_equal(bits(v), ev)
    assert lens.tolist() == [1, 256, 257, 768, 768]


def test_graph_captured_decode_loop_with_device_lengths():
    """Config 3 shape (Hq=16, Hkv=4, D=256, 2% of K channels x8), 4 rows, 24 steps in one graph."""
    steps, b, hq, hkv, dim, start = 24, 4, 16, 4, 256, 500
    case = cases.make_case([start] * b, hq, hkv, dim, seed=41, capacity=start + steps)
    q, k, v, table, lens = device_case(case)
    gen = torch.Generator(device="cuda").manual_seed(9)
    outlier = torch.ones(hkv * dim, device="cuda")
    outlier[torch.randperm(hkv * dim, generator=gen, device="cuda")[:round(0.02 * hkv * dim)]] = 8
    k.copy_((k.float() * outlier.view(1, 1, hkv, dim)).to(torch.bfloat16))
    new_k = torch.randn(steps, b, hkv, dim, generator=gen, device="cuda").to(torch.bfloat16)
    new_v = torch.randn_like(new_k)
    new_q = torch.randn(steps, b, hq, dim, generator=gen, device="cuda").to(torch.bfloat16)
    res = allocate_matched_resources(DecodeSpec(b, hq, hkv, dim, start + steps), "cuda")
    outs = torch.empty(steps, b, hq, dim, dtype=torch.bfloat16, device="cuda")

    def loop():
        for s in range(steps):
            append_decode_kv(new_k[s], new_v[s], k, v, table, lens)
            outs[s].copy_(matched_decode(new_q[s], k, v, table, lens, resources=res))

    k0, v0, lens0 = k.clone(), v.clone(), lens.clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        loop()  # warm-up (also appends); restore the state before capture
    torch.cuda.current_stream().wait_stream(side)
    k.copy_(k0), v.copy_(v0), lens.copy_(lens0)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        loop()
    k.copy_(k0), v.copy_(v0), lens.copy_(lens0)
    graph.replay()
    torch.cuda.synchronize()
    assert lens.tolist() == [start + steps] * b
    kh, vh, th = k.float().cpu().numpy(), v.float().cpu().numpy(), table.cpu().numpy()
    for s in (0, steps // 2, steps - 1):
        n = np.full(b, start + s + 1, dtype=np.int32)
        expected = oracle.dense_reference(new_q[s].float().cpu().numpy(), kh, vh, th, n)
        assert_out_close(outs[s], expected, f"step {s}")
    del graph


def test_config3_decode_loop_of_256_steps_in_one_graph():
    """BASELINE config 3's protocol at its full shape: B=32, Hq=16, Hkv=4,
    D=256 (2% of K channels x8), context 528 -> 784.  Every step appends each
    row's new K/V token at its length (lengths += 1 on the device) and
    decodes; the 256 steps are captured once in a CUDA graph and replayed.
    Steps 0, 128 and 255 of sampled rows match the FP64 reference (outputs
    max-abs 2^-7), and the graph's outputs equal an eager run's bit for bit."""
    from oracle.torch_reference import chunked_reference_rows
    from paged_decode import ops
    from paged_decode.splitkv_plan import make_b200_plan
    from paged_decode.workloads import make_workload
    w = make_workload("cfg3", device="cuda", batch=32, context=528)
    steps, rows = 256, [0, 13, 31]
    gen = torch.Generator(device="cuda").manual_seed(31)
    new_k = torch.randn(steps, 32, 4, 256, generator=gen, device="cuda").to(torch.bfloat16)
    new_v = torch.randn_like(new_k)
    res = allocate_matched_resources(w.spec, "cuda",
                                     plan=make_b200_plan(w.spec, ops.sm_count("cuda")))
    k0, v0, len0 = w.k.clone(), w.v.clone(), w.lengths.clone()

    def restore():
        w.k.copy_(k0)
        w.v.copy_(v0)
        w.lengths.copy_(len0)

    def loop(hist, n):
        for i in range(n):
            append_decode_kv(new_k[i], new_v[i], w.k, w.v, w.table, w.lengths)
            hist[i].copy_(matched_decode(w.q, w.k, w.v, w.table, w.lengths, resources=res,
                                         scale=w.scale))

    eager = torch.empty(steps, 32, 16, 256, dtype=torch.bfloat16, device="cuda")
    loop(eager, steps)
    restore()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        warm = torch.empty(3, 32, 16, 256, dtype=torch.bfloat16, device="cuda")
        loop(warm, 3)
    torch.cuda.current_stream().wait_stream(side)
    restore()
    replayed = torch.empty_like(eager)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        loop(replayed, steps)
    restore()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(w.lengths, len0 + steps)
    assert torch.equal(replayed, eager)
    for i in (0, 128, 255):
        # The cache as step i sees it: the original pages plus tokens 0..i.
        k, v = k0.clone(), v0.clone()
        for j in range(i + 1):
            pos = len0 + j
            pages = w.table[torch.arange(32, device="cuda"), (pos // 256).long()].long()
            k[pages, (pos % 256).long()] = new_k[j]
            v[pages, (pos % 256).long()] = new_v[j]
        want = chunked_reference_rows(w.q, k, v, w.table, len0 + i + 1, rows, scale=w.scale)
        assert_out_close(replayed[i][rows], want.float(), what=f"step {i} rows {rows}")
    del graph
