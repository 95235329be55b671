"""GPU parity of ``paged_decode`` (all four backends) against the NumPy oracle.

Ports the reference's operator tests (tests/test_gpu.py:51-128) to the
oracle-pinned tolerances of ``gpu_util`` and adds the golden sweep: every
case of the reference's oracle sweep (tests/test_reference.py:20-28) is run
on the GPU and compared with the output the reference's own NumPy code
produced for the same BF16 bits.
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import cases
import oracle
from gpu_util import assert_out_close, device_case, requires_cuda
from paged_decode.runtime import allocate_resources, paged_decode, validate_device_metadata
from paged_decode.spec import DecodeSpec

pytestmark = [pytest.mark.gpu, requires_cuda]

GOLDEN = Path(__file__).resolve().parent / "golden"
BACKENDS = ["triton_base", "triton_splitk", "triton_tc", "triton_tc_splitk"]


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "golden_cases.npz")


@pytest.mark.parametrize("backend", BACKENDS)
@pytest.mark.parametrize("dim,hq,hkv", cases.SWEEP_GEOMETRIES)
def test_golden_sweep(golden, backend, dim, hq, hkv):
    for length in cases.SWEEP_LENGTHS:
        case = cases.sweep_case(length, dim, hq, hkv)
        q, k, v, table, lens = device_case(case)
        spec = DecodeSpec(2, hq, hkv, dim, case.capacity)
        res = allocate_resources(spec, "cuda", backend)
        out = paged_decode(q, k, v, table, lens, resources=res, backend=backend)
        assert_out_close(out, golden[f"sweep_{length}_{dim}_{hq}_{hkv}/dense"],
                         f"{backend} len={length}")


def poisoned_case(lengths, hq, hkv, dim, capacity):
    """Reference tests/test_gpu.py:55-63: -1 padding, NaN in dead slots, row 0 empty."""
    case = cases.make_case(lengths, hq, hkv, dim, seed=19, capacity=capacity)
    return cases.poison_tails(case)


@pytest.mark.parametrize("backend", BACKENDS)
@pytest.mark.parametrize("dim,hq,hkv", [(64, 4, 1), (128, 4, 2), (64, 2, 2), (256, 8, 2)])
def test_boundaries_gqa_and_padding(backend, dim, hq, hkv):
    lengths = [0, 1, 255, 256, 257, 1023, 1024, 1025]
    case = poisoned_case(lengths, hq, hkv, dim, 1025)
    args = device_case(case)
    validate_device_metadata(args[3], args[4], args[1].shape[0], 1025)
    res = allocate_resources(DecodeSpec(len(lengths), hq, hkv, dim, 1025), "cuda", backend)
    out = paged_decode(*args, resources=res, backend=backend).clone()
    assert_out_close(out, oracle.dense_reference(*case.arrays()))
    assert torch.count_nonzero(out[0]) == 0


@pytest.mark.parametrize("backend", BACKENDS)
@pytest.mark.parametrize("dim", [64, 256])
def test_graph_replay_changes_lengths_pages_and_kv(backend, dim):
    """Reference tests/test_gpu.py:71-95: capture once, replay with new metadata and data."""
    case = cases.make_case([255, 1023, 0], 4, 1, dim, seed=19, capacity=2048)
    q, k, v, table, lens = device_case(case)
    res = allocate_resources(DecodeSpec(3, 4, 1, dim, 2048), "cuda", backend)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(3):
            paged_decode(q, k, v, table, lens, resources=res, backend=backend)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        output = paged_decode(q, k, v, table, lens, resources=res, backend=backend)
    gen = torch.Generator(device="cuda").manual_seed(5)
    for lengths in ([256, 1024, 0], [257, 1025, 1], [1, 0, 1025], [0, 0, 0]):
        lens.copy_(torch.tensor(lengths, device="cuda", dtype=torch.int32))
        q.copy_(torch.randn(q.shape, generator=gen, device="cuda"))
        k.copy_(torch.randn(k.shape, generator=gen, device="cuda"))
        v.copy_(torch.randn(v.shape, generator=gen, device="cuda"))
        table.copy_(table.flip(1))
        graph.replay()
        host = [t.cpu() for t in (q, k, v, table, lens)]
        expected = oracle.dense_reference(host[0].float().numpy(), host[1].float().numpy(),
                                          host[2].float().numpy(), host[3].numpy(),
                                          host[4].numpy())
        assert_out_close(output, expected)
        eager = paged_decode(q, k, v, table, lens, resources=res, backend=backend).clone()
        torch.testing.assert_close(eager, output, atol=0, rtol=0)
    del graph


def test_public_contract_rejects_bad_dtype_and_missing_workspace():
    args = device_case(cases.make_case([2], 4, 1, 64, seed=19, capacity=2048))
    r = allocate_resources(DecodeSpec(1, 4, 1, 64, 2048), "cuda", "triton_base")
    for backend in ("triton_splitk", "triton_tc_splitk"):
        with pytest.raises(ValueError, match="workspace"):
            paged_decode(*args, resources=r, backend=backend)
    with pytest.raises(ValueError, match="BF16"):
        paged_decode(args[0].float(), *args[1:], resources=r)
    for backend in ("triton_tc", "triton_tc_splitk"):
        rr = allocate_resources(DecodeSpec(1, 4, 1, 64, 2048), "cuda", backend)
        with pytest.raises(ValueError, match="positive"):
            paged_decode(*args, resources=rr, backend=backend, scale=-1.0)


@pytest.mark.parametrize("backend", ["triton_splitk", "triton_tc_splitk"])
@pytest.mark.parametrize("dim", [64, 256])
def test_non_power_of_two_split_count(dim, backend):
    """Reference tests/test_gpu.py:121-128: three partitions, padded merge."""
    case = cases.make_case([0, 2051, 2049, 1025], 4, 1, dim, seed=19, capacity=2051)
    res = allocate_resources(DecodeSpec(4, 4, 1, dim, 2051), "cuda", backend)
    out = paged_decode(*device_case(case), resources=res, backend=backend)
    assert_out_close(out, oracle.dense_reference(*case.arrays()))


@pytest.mark.parametrize("backend", ["triton_base", "triton_splitk"])
def test_signed_and_zero_scales(backend):
    """The CUDA-core backends accept any finite scale, as the reference's do."""
    case = cases.make_case([700, 33], 8, 2, 128, seed=3, capacity=1024)
    args = device_case(case)
    res = allocate_resources(DecodeSpec(2, 8, 2, 128, 1024), "cuda", backend)
    for scale in (0.0, -0.3, 0.5):
        out = paged_decode(*args, resources=res, backend=backend, scale=scale)
        assert_out_close(out, oracle.dense_reference(*case.arrays(), scale=scale))


@pytest.mark.parametrize("backend", BACKENDS)
def test_page_relocation_is_bit_exact(backend):
    """Moving pages and rewriting the table must not change a single output bit."""
    case = cases.make_case([1500, 0, 257, 1024], 8, 2, 128, seed=11, capacity=2048,
                           pool_factor=2.0)
    q, k, v, table, lens = device_case(case)
    res = allocate_resources(DecodeSpec(4, 8, 2, 128, 2048), "cuda", backend)
    first = paged_decode(q, k, v, table, lens, resources=res, backend=backend).clone()
    perm = torch.randperm(k.shape[0], generator=torch.Generator().manual_seed(1)).cuda()
    inverse = torch.empty_like(perm)
    inverse[perm] = torch.arange(perm.numel(), device="cuda")
    k2, v2 = torch.empty_like(k), torch.empty_like(v)
    k2[inverse] = k
    v2[inverse] = v
    table2 = inverse[table.long()].to(torch.int32)
    second = paged_decode(q, k2, v2, table2, lens, resources=res, backend=backend)
    assert torch.equal(first.view(torch.int16), second.view(torch.int16))


def test_config1_all_backends_against_golden(golden):
    """BASELINE config 1 (B=4, Hq=8, Hkv=2, D=128, lengths in [0,1024])."""
    case = cases.config1()
    args = device_case(case)
    for backend in BACKENDS:
        res = allocate_resources(DecodeSpec(4, 8, 2, 128, 1024), "cuda", backend)
        out = paged_decode(*args, resources=res, backend=backend)
        assert_out_close(out, golden["cfg1/dense"], backend)
        assert_out_close(out, golden["cfg1/split"], backend)
        assert torch.count_nonzero(out[0]) == 0


@pytest.mark.parametrize("backend", ["triton_base", "triton_tc"])
@pytest.mark.parametrize("spec_args,lengths", [
    ((8, 16, 4, 256, 2320), [2064, 528, 0, 1, 2320, 1031, 64, 700]),     # balanced partitions
    ((6, 8, 2, 128, 9000), [9000, 0, 4096, 4097, 17, 8191]),            # fixed partitions
])
def test_single_pass_backends_split_like_the_b200_plan(backend, spec_args, lengths):
    """The single-pass backends compute rows in this library's plan (internal
    scratch, empty partitions not stored) when it has more than one partition:
    the output is the one of matched_decode with that plan, bit for bit, and
    within the output tolerance of the dense softmax."""
    from paged_decode import ops
    from paged_decode.matched_splitkv import allocate_matched_resources, matched_decode
    from paged_decode.splitkv_plan import make_b200_plan
    spec = DecodeSpec(*spec_args)
    case = cases.make_case(lengths, spec.num_heads, spec.num_kv_heads, spec.head_dim, seed=41,
                           capacity=spec.max_context_len)
    args = device_case(case)
    res = allocate_resources(spec, "cuda", backend)
    assert res.split_plan is not None and res.split_plan.splits > 1
    out = paged_decode(*args, resources=res, backend=backend).clone()
    plan = make_b200_plan(spec, ops.sm_count(torch.device("cuda")))
    mres = allocate_matched_resources(spec, "cuda", plan=plan)
    want = matched_decode(*args, resources=mres, kernel="mma" if backend == "triton_tc" else "auto")
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    assert_out_close(out, oracle.dense_reference(*case.arrays()))
