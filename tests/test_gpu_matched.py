"""GPU parity of the partition -> partial + LSE -> LSE merge path.

Ports the reference's matched tests (tests/test_matched_splitkv.py:20-69)
and replaces its FlashAttention LSE pin (which is not our contract) with the
oracle: per-partition LSE within 1e-5 relative, normalised partials and the
merged output within the output tolerance, partition bounds exact.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

import cases
import oracle
from gpu_util import assert_lse_close, assert_out_close, device_case, requires_cuda
from paged_decode import ops
from paged_decode.matched_splitkv import allocate_matched_resources, matched_decode
from paged_decode.spec import DecodeSpec

pytestmark = [pytest.mark.gpu, requires_cuda]

GOLDEN = Path(__file__).resolve().parent / "golden"
KERNELS = ["simt", "mma"]


def poisoned(lengths, hq, hkv, dim, capacity, seed=19):
    return cases.poison_tails(cases.make_case(lengths, hq, hkv, dim, seed=seed,
                                              capacity=capacity))


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("splits", [3, 6])
@pytest.mark.parametrize("dim,hq,hkv", [(64, 4, 1), (128, 4, 2), (256, 8, 2), (128, 16, 2)])
def test_explicit_cross_page_boundaries(kernel, splits, dim, hq, hkv):
    lengths = [0, 1, 255, 256, 257, 1023, 1024, 2051]
    case = poisoned(lengths, hq, hkv, dim, 2051)
    args = device_case(case)
    res = allocate_matched_resources(DecodeSpec(8, hq, hkv, dim, 2051), "cuda", num_splits=splits)
    out = matched_decode(*args, resources=res, kernel=kernel)
    ref_out, ref_partials, ref_lse = oracle.matched_reference(
        *case.arrays(), res.plan.tokens_per_split, res.plan.splits)
    assert_out_close(out, ref_out)
    mags = oracle.score_magnitudes(case.q, case.k, case.table, case.lengths,
                                   res.plan.tokens_per_split, res.plan.splits)
    assert_lse_close(res.lse, ref_lse, score_mag=mags)
    assert_out_close(res.partials, ref_partials, "partials")
    assert torch.count_nonzero(out[0]) == 0


@pytest.mark.parametrize("kernel", KERNELS)
def test_graph_replay_and_empty_partitions(kernel):
    case = cases.make_case([255, 1023, 0], 8, 2, 256, seed=19, capacity=2051)
    q, k, v, table, lengths = device_case(case)
    res = allocate_matched_resources(DecodeSpec(3, 8, 2, 256, 2051), "cuda")
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(3):
            matched_decode(q, k, v, table, lengths, resources=res, kernel=kernel)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = matched_decode(q, k, v, table, lengths, resources=res, kernel=kernel)
    gen = torch.Generator(device="cuda").manual_seed(7)
    for values in ([257, 1025, 0], [2051, 1, 0], [0, 0, 0]):
        lengths.copy_(torch.tensor(values, dtype=torch.int32, device="cuda"))
        q.copy_(torch.randn(q.shape, generator=gen, device="cuda"))
        k.copy_(torch.randn(k.shape, generator=gen, device="cuda"))
        v.copy_(torch.randn(v.shape, generator=gen, device="cuda"))
        table.copy_(table.flip(1))
        graph.replay()
        captured = out.clone()
        host = [t.cpu() for t in (q, k, v, table, lengths)]
        expected = oracle.dense_reference(host[0].float().numpy(), host[1].float().numpy(),
                                          host[2].float().numpy(), host[3].numpy(),
                                          host[4].numpy())
        assert_out_close(captured, expected)
        eager = matched_decode(q, k, v, table, lengths, resources=res, kernel=kernel)
        torch.testing.assert_close(captured, eager, atol=0, rtol=0)
    del graph


def test_fixed_plan_contract():
    args = device_case(cases.make_case([1, 2, 0], 8, 2, 256, seed=19, capacity=2051))
    res = allocate_matched_resources(DecodeSpec(3, 8, 2, 256, 2051), "cuda")
    q, k, v, table, lengths = args
    with pytest.raises(ValueError, match="fixed batch"):
        matched_decode(q[:1], k, v, table[:1], lengths[:1], resources=res)
    with pytest.raises(ValueError, match="fixed batch"):
        matched_decode(q, k, v, table[:, :8], lengths, resources=res)
    with pytest.raises(ValueError, match="positive"):
        matched_decode(*args, resources=res, scale=0)


@pytest.mark.parametrize("kernel", KERNELS)
def test_config1_partitions_against_reference_golden(kernel):
    """Per-partition LSE / partials of config 1 vs the reference's own NumPy outputs."""
    golden = np.load(GOLDEN / "golden_cases.npz")
    case = cases.config1()
    q, k, v, table, lens = device_case(case)
    for tokens in (512, 1024):
        splits = 1024 // tokens
        out = torch.empty(4, 8, 128, dtype=torch.bfloat16, device="cuda")
        partial = torch.empty(4, 8, splits, 128, device="cuda")
        lse = torch.empty(4, 8, splits, device="cuda")
        ops.paged_decode(ops.decode_args(q, k, v, table, lens, scale=128 ** -0.5,
                                         tokens_per_split=tokens, splits=splits,
                                         protocol=ops.PROTOCOL_LSE, kernel=kernel, out=out,
                                         partial=partial, lse=lse), q.device)
        key = f"cfg1/p{tokens}"
        mags = oracle.score_magnitudes(case.q, case.k, case.table, case.lengths, tokens, splits,
                                       128 ** -0.5)
        assert_lse_close(lse, golden[f"{key}/lse"], score_mag=mags)
        assert_out_close(partial, golden[f"{key}/partial"], "partial")
        assert_out_close(out, golden["cfg1/dense"])
        # Same run, unnormalised protocol: (m, l, acc) of the reference's _split.
        maxima = torch.empty(4, 8, splits, device="cuda")
        denoms = torch.empty(4, 8, splits, device="cuda")
        accums = torch.empty(4, 8, splits, 128, device="cuda")
        ops.paged_decode(ops.decode_args(q, k, v, table, lens, scale=128 ** -0.5,
                                         tokens_per_split=tokens, splits=splits,
                                         protocol=ops.PROTOCOL_MLA, kernel=kernel, out=out,
                                         maxima=maxima, denoms=denoms, accums=accums), q.device)
        assert_lse_close(maxima, golden[f"{key}/m"], "maxima", score_mag=mags)
        ref_l = golden[f"{key}/l"]
        got_l = denoms.cpu().numpy()
        np.testing.assert_allclose(got_l, ref_l, rtol=2e-5, atol=0)
        np.testing.assert_allclose(accums.cpu().numpy(), golden[f"{key}/acc"], rtol=2e-4, atol=2e-3)
        assert_out_close(out, golden["cfg1/dense"])


@pytest.mark.parametrize("kernel", KERNELS)
def test_skip_empty_flag_matches_full_store(kernel):
    """Not storing empty partitions changes nothing the merge can see."""
    case = cases.make_case([3000, 0, 100, 4096], 8, 2, 128, seed=5, capacity=4096)
    q, k, v, table, lens = device_case(case)
    outs = []
    for flags in (0, ops.FLAG_SKIP_EMPTY):
        out = torch.empty(4, 8, 128, dtype=torch.bfloat16, device="cuda")
        partial = torch.full((4, 8, 8, 128), float("nan"), device="cuda")
        lse = torch.full((4, 8, 8), float("nan"), device="cuda")
        ops.paged_decode(ops.decode_args(q, k, v, table, lens, scale=0.1, tokens_per_split=512,
                                         splits=8, protocol=ops.PROTOCOL_LSE, kernel=kernel,
                                         flags=flags, out=out, partial=partial, lse=lse), q.device)
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
    assert_out_close(outs[0], oracle.dense_reference(*case.arrays(), scale=0.1))


@pytest.mark.parametrize("kernel", KERNELS)
def test_split_layout_invariance(kernel):
    """512-token splits of a row and one 4096-token split agree within tolerance."""
    case = cases.make_case([4096, 3333], 16, 2, 128, seed=8, capacity=4096)
    args = device_case(case)
    res_a = allocate_matched_resources(DecodeSpec(2, 16, 2, 128, 4096), "cuda", num_splits=8)
    res_b = allocate_matched_resources(DecodeSpec(2, 16, 2, 128, 4096), "cuda", num_splits=1)
    a = matched_decode(*args, resources=res_a, kernel=kernel).clone()
    b = matched_decode(*args, resources=res_b, kernel=kernel).clone()
    ref = oracle.dense_reference(*case.arrays())
    assert_out_close(a, ref)
    assert_out_close(b, ref)
    assert (a.float() - b.float()).abs().max().item() <= 2 ** -7


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("protocol", ["lse", "mla"])
@pytest.mark.parametrize("flags", [0, "dynamic", "skip", "dynamic+skip"])
@pytest.mark.parametrize("hq,hkv,d,tps,splits", [(8, 2, 128, 512, 8), (16, 4, 256, 128, 33)])
def test_every_partition_slot_follows_the_workspace_contract(kernel, protocol, flags, hq, hkv,
                                                            d, tps, splits):
    """Live partitions hold the oracle's values; empty ones are stored as empty
    (partial 0 / LSE -inf, or (-inf, 0, 0)) unless PDL_FLAG_SKIP_EMPTY, which
    leaves them untouched.  The workspace starts NaN-poisoned.  The first
    geometry runs several work items per CTA (the live schedule) and stores
    several empty partitions per fill item, the second one per item."""
    lengths = [3000, 0, 1, 4096, 257, 2048, 2049, 0]
    rows = len(lengths)
    case = cases.make_case(lengths, hq, hkv, d, seed=12, capacity=4096)
    q, k, v, table, lens = device_case(case)
    bits = {"dynamic": ops.FLAG_DYNAMIC, "skip": ops.FLAG_SKIP_EMPTY,
            "dynamic+skip": ops.FLAG_DYNAMIC | ops.FLAG_SKIP_EMPTY}.get(flags, 0)
    counters = torch.zeros(2, dtype=torch.int32, device="cuda")
    nan = dict(device="cuda", dtype=torch.float32)
    out = torch.empty(rows, hq, d, dtype=torch.bfloat16, device="cuda")
    if protocol == "lse":
        ws = dict(partial=torch.full((rows, hq, splits, d), float("nan"), **nan),
                  lse=torch.full((rows, hq, splits), float("nan"), **nan))
    else:
        ws = dict(maxima=torch.full((rows, hq, splits), float("nan"), **nan),
                  denoms=torch.full((rows, hq, splits), float("nan"), **nan),
                  accums=torch.full((rows, hq, splits, d), float("nan"), **nan))
    args = ops.decode_args(q, k, v, table, lens, scale=0.09, tokens_per_split=tps, splits=splits,
                           protocol=ops.PROTOCOL_LSE if protocol == "lse" else ops.PROTOCOL_MLA,
                           kernel=kernel, flags=bits, out=out, counters=counters, **ws)
    for _ in range(2):  # the scheduler words reset themselves between launches
        ops.paged_decode(args, q.device)
    torch.cuda.synchronize()
    assert not counters.any() and ops.read_fault() == 0
    assert_out_close(out, oracle.dense_reference(*case.arrays(), scale=0.09))
    live = torch.tensor([[p * tps < n for p in range(splits)] for n in lengths], device="cuda")
    live = live[:, None, :].expand(rows, hq, splits)
    skip = bool(bits & ops.FLAG_SKIP_EMPTY)
    if protocol == "lse":
        ref_p, ref_l = oracle.normalized_partitions(*case.arrays(), tps, splits, scale=0.09)
        got_l = ws["lse"].clone()
        mags = oracle.score_magnitudes(*case.arrays()[:2], case.table, case.lengths, tps, splits,
                                       0.09)
        assert_lse_close(got_l[live], ref_l[live.cpu().numpy()],
                         score_mag=mags[live.cpu().numpy()])
        assert_out_close(ws["partial"][live], ref_p[live.cpu().numpy()], "live partials")
        empty_l, empty_p = ws["lse"][~live], ws["partial"][~live]
        if skip:
            assert torch.isnan(empty_l).all() and torch.isnan(empty_p).all()
        else:
            assert torch.isneginf(empty_l).all() and not empty_p.any()
    else:
        ref_m, ref_d, ref_a = oracle.unnormalized_partitions(*case.arrays(), tps, splits,
                                                             scale=0.09)
        m = live.cpu().numpy()
        mags = oracle.score_magnitudes(*case.arrays()[:2], case.table, case.lengths, tps, splits,
                                       0.09)
        assert_lse_close(ws["maxima"][live], ref_m[m], "maxima", score_mag=mags[m])
        assert np.allclose(ws["denoms"][live].cpu().numpy(), ref_d[m], rtol=1e-5)
        empty = [ws["maxima"][~live], ws["denoms"][~live], ws["accums"][~live]]
        if skip:
            assert all(torch.isnan(t).all() for t in empty)
        else:
            assert torch.isneginf(empty[0]).all() and not empty[1].any() and not empty[2].any()


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("rows", [512, 513, 700])
def test_batches_past_the_register_schedule(kernel, rows):
    """Up to 512 rows the producer keeps every length in registers and hands out
    live items only; larger batches enumerate every partition.  Both must give
    the oracle's outputs and identical bits under static and dynamic scheduling,
    with empty partitions stored or skipped (a skipped item moves the CTA on to
    its next item)."""
    gen = np.random.default_rng(rows)
    lengths = gen.integers(0, 600, size=rows)
    lengths[::7] = 0
    case = cases.make_case(lengths, 4, 1, 64, seed=rows, capacity=768)
    q, k, v, table, lens = device_case(case)
    counters = torch.zeros(2, dtype=torch.int32, device="cuda")
    outs = []
    for flags in (0, ops.FLAG_DYNAMIC, ops.FLAG_SKIP_EMPTY, ops.FLAG_DYNAMIC | ops.FLAG_SKIP_EMPTY):
        out = torch.empty(rows, 4, 64, dtype=torch.bfloat16, device="cuda")
        partial = torch.full((rows, 4, 3, 64), float("nan"), device="cuda")
        lse = torch.full((rows, 4, 3), float("nan"), device="cuda")
        args = ops.decode_args(q, k, v, table, lens, scale=0.125, tokens_per_split=256, splits=3,
                               protocol=ops.PROTOCOL_LSE, kernel=kernel, flags=flags, out=out,
                               partial=partial, lse=lse, counters=counters)
        ops.paged_decode(args, q.device)
        outs.append((out, partial, lse))
    torch.cuda.synchronize()
    assert not counters.any() and ops.read_fault() == 0
    empty = torch.tensor([[p * 256 >= n for p in range(3)] for n in lengths], device="cuda")
    empty = empty[:, None, :].expand(rows, 4, 3)
    assert torch.equal(outs[0][2], outs[1][2])
    for out, partial, lse in outs[1:]:
        assert torch.equal(outs[0][0], out)
        assert torch.equal(outs[0][2][~empty], lse[~empty])
        assert torch.equal(outs[0][1][~empty], partial[~empty])
    for out, partial, lse in outs[2:]:
        assert torch.isnan(lse[empty]).all()  # skipped: never written
    few = list(range(0, rows, max(1, rows // 12)))
    want = oracle.dense_reference(case.q[few], case.k, case.v, case.table[few],
                                  case.lengths[few], scale=0.125)
    assert_out_close(outs[1][0][few], want)
    assert torch.count_nonzero(outs[1][0][lens == 0]) == 0
    assert torch.isneginf(outs[1][2][empty]).all()


@pytest.mark.parametrize("kernel", KERNELS)
def test_dynamic_scheduling_is_bit_identical_to_static(kernel):
    """Atomic, partition-major item hand-out changes which CTA does what, not a bit."""
    lengths = [0, 32768, 1, 4000, 9999, 257, 0, 20000]  # 512 items: > 2 per CTA slot
    rows = len(lengths)
    case = cases.make_case(lengths, 8, 2, 128, seed=13, capacity=32768, pool_factor=1.0)
    q, k, v, table, lens = device_case(case)
    counters = torch.zeros(2, dtype=torch.int32, device="cuda")
    outs = []
    for flags in (0, ops.FLAG_DYNAMIC, ops.FLAG_DYNAMIC | ops.FLAG_SKIP_EMPTY):
        out = torch.empty(rows, 8, 128, dtype=torch.bfloat16, device="cuda")
        partial = torch.empty(rows, 8, 32, 128, device="cuda")
        lse = torch.empty(rows, 8, 32, device="cuda")
        args = ops.decode_args(q, k, v, table, lens, scale=0.088, tokens_per_split=1024,
                               splits=32, protocol=ops.PROTOCOL_LSE, kernel=kernel, flags=flags,
                               out=out, partial=partial, lse=lse, counters=counters)
        for _ in range(2):  # the scheduler words reset themselves between launches
            ops.paged_decode(args, q.device)
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    assert not counters.any()
    few = [0, 1, 2, 3]
    sub = oracle.dense_reference(case.q[few], case.k, case.v, case.table[few], case.lengths[few],
                                 scale=0.088)
    assert_out_close(outs[1][few], sub)


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("protocol", ["lse", "mla"])
@pytest.mark.parametrize("flags", [0, "dynamic+skip"])
@pytest.mark.parametrize("hq,hkv,d,granule,splits", [(16, 4, 256, 64, 3), (8, 2, 128, 64, 5),
                                                     (4, 1, 64, 128, 2), (8, 2, 256, 32, 40)])
def test_balanced_partitions_follow_each_rows_length(kernel, protocol, flags, hq, hkv, d,
                                                     granule, splits):
    """PDL_FLAG_BALANCED: partition p of a row covers [p*c, (p+1)*c) with
    c = granule * ceil(ceil(len / splits) / granule).  Live partitions hold
    the oracle's values for exactly those bounds, the others are stored empty
    (or untouched with PDL_FLAG_SKIP_EMPTY), and the merge, which derives
    the same bounds, gives the dense softmax."""
    lengths = [3000, 0, 1, 4096, 257, 2048, 2049, 65]
    rows = len(lengths)
    case = cases.make_case(lengths, hq, hkv, d, seed=21, capacity=4096)
    q, k, v, table, lens = device_case(case)
    bits = ops.FLAG_BALANCED | {"dynamic+skip": ops.FLAG_DYNAMIC | ops.FLAG_SKIP_EMPTY}.get(flags, 0)
    counters = torch.zeros(2, dtype=torch.int32, device="cuda")
    nan = dict(device="cuda", dtype=torch.float32)
    out = torch.empty(rows, hq, d, dtype=torch.bfloat16, device="cuda")
    if protocol == "lse":
        ws = dict(partial=torch.full((rows, hq, splits, d), float("nan"), **nan),
                  lse=torch.full((rows, hq, splits), float("nan"), **nan))
    else:
        ws = dict(maxima=torch.full((rows, hq, splits), float("nan"), **nan),
                  denoms=torch.full((rows, hq, splits), float("nan"), **nan),
                  accums=torch.full((rows, hq, splits, d), float("nan"), **nan))
    args = ops.decode_args(q, k, v, table, lens, scale=0.09, tokens_per_split=granule,
                           splits=splits,
                           protocol=ops.PROTOCOL_LSE if protocol == "lse" else ops.PROTOCOL_MLA,
                           kernel=kernel, flags=bits, out=out, counters=counters, **ws)
    for _ in range(2):
        ops.paged_decode(args, q.device)
    torch.cuda.synchronize()
    assert not counters.any() and ops.read_fault() == 0
    assert_out_close(out, oracle.dense_reference(*case.arrays(), scale=0.09))
    bounds = [oracle.partition_bounds(n, granule, splits, balanced=True) for n in lengths]
    live = torch.tensor([[e > s for s, e in b] for b in bounds], device="cuda")
    live = live[:, None, :].expand(rows, hq, splits)
    m = live.cpu().numpy()
    skip = bool(bits & ops.FLAG_SKIP_EMPTY)
    mags = oracle.score_magnitudes(*case.arrays()[:2], case.table, case.lengths, granule, splits,
                                   0.09, balanced=True)
    if protocol == "lse":
        ref_p, ref_l = oracle.normalized_partitions(*case.arrays(), granule, splits, scale=0.09,
                                                    balanced=True)
        assert_lse_close(ws["lse"][live], ref_l[m], score_mag=mags[m])
        assert_out_close(ws["partial"][live], ref_p[m], "live partials")
        empty_l, empty_p = ws["lse"][~live], ws["partial"][~live]
        if skip:
            assert torch.isnan(empty_l).all() and torch.isnan(empty_p).all()
        else:
            assert torch.isneginf(empty_l).all() and not empty_p.any()
    else:
        ref_m, ref_d, _ = oracle.unnormalized_partitions(*case.arrays(), granule, splits,
                                                         scale=0.09, balanced=True)
        assert_lse_close(ws["maxima"][live], ref_m[m], "maxima", score_mag=mags[m])
        assert np.allclose(ws["denoms"][live].cpu().numpy(), ref_d[m], rtol=1e-5)
        empty = [ws["maxima"][~live], ws["denoms"][~live], ws["accums"][~live]]
        if skip:
            assert all(torch.isnan(t).all() for t in empty)
        else:
            assert torch.isneginf(empty[0]).all() and not empty[1].any() and not empty[2].any()


@pytest.mark.parametrize("kernel", KERNELS)
def test_balanced_partitions_over_several_waves(kernel):
    """More balanced items than CTA slots (dense enumeration, several waves):
    static and dynamic scheduling give the same bits and the oracle's output."""
    gen = np.random.default_rng(5)
    lengths = gen.integers(0, 1500, size=300)
    lengths[::9] = 0
    case = cases.make_case(lengths, 8, 2, 128, seed=31, capacity=1536)
    q, k, v, table, lens = device_case(case)
    counters = torch.zeros(2, dtype=torch.int32, device="cuda")
    outs = []
    for flags in (ops.FLAG_BALANCED, ops.FLAG_BALANCED | ops.FLAG_DYNAMIC):
        out = torch.empty(300, 8, 128, dtype=torch.bfloat16, device="cuda")
        lse = torch.full((300, 8, 4), float("nan"), device="cuda")
        partial = torch.full((300, 8, 4, 128), float("nan"), device="cuda")
        args = ops.decode_args(q, k, v, table, lens, scale=0.09, tokens_per_split=64, splits=4,
                               protocol=ops.PROTOCOL_LSE, kernel=kernel, flags=flags, out=out,
                               partial=partial, lse=lse, counters=counters)
        ops.paged_decode(args, q.device)
        outs.append((out, lse))
    torch.cuda.synchronize()
    assert not counters.any() and ops.read_fault() == 0
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    few = list(range(0, 300, 23))
    want = oracle.dense_reference(case.q[few], case.k, case.v, case.table[few], case.lengths[few],
                                  scale=0.09)
    assert_out_close(outs[1][0][few], want)
